"""Batched BERT embedding attention on the GPU against fast/vdb.cpp:189-212 (per sequence, no mask
inside a sequence).  fp32 SIMT: <= 1e-4 of the output scale; bf16 tensor cores: <= 2e-2."""
import json
import os

import numpy as np
import pytest

import cases
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def gpu_bert(c, mode):
    from ligguf_b200 import CudaBertAttention
    h = CudaBertAttention(c["H"], c["D"], len(c["lens"]), c["max_len"])
    out = h.attn(c["lens"], c["q"], c["k"], c["v"], mode)
    h.close()
    return out


@pytest.mark.parametrize("mode,tol", [(0, 1e-4), (1, 2e-2)])
@pytest.mark.parametrize("key", ["bert_bert_small", "bert_bert_empty_and_full"])
def test_bert_vs_reference_golden(gpu, key, mode, tol):
    spec = dict(json.load(open(os.path.join(GOLDEN, "golden.json")))[key])
    gold = np.load(os.path.join(GOLDEN, key + ".npz"))
    out = gpu_bert(cases.bert_case(**spec), mode)
    assert cases.rel_err(out, gold["out"]) <= tol
    for b, n in enumerate(spec["lens"]):
        assert not np.any(out[b, n:])  # padded rows are zeros


@pytest.mark.parametrize("mode,tol", [(0, 1e-4), (1, 2e-2)])
@pytest.mark.parametrize("lens,max_len", [((16, 512, 100, 1), 512), ((65, 64, 63, 129, 200), 200), ((3,), 8)])
def test_bert_sweep(gpu, lens, max_len, mode, tol):
    c = cases.bert_case(H=12, D=64, lens=lens, max_len=max_len, scale=0.125, seed=sum(lens))
    out = gpu_bert(c, mode)
    ref = cases.run_bert(orc.Checker("port"), c)
    assert cases.rel_err(out, ref) <= tol


@pytest.mark.parametrize("mode,tol", [(0, 1e-4), (1, 2e-2)])
def test_bert_full_config_layer(gpu, mode, tol):
    """bert_base_attn at full size (64 sequences, lengths U[16,512], one layer)."""
    from ligguf_b200.workloads import BERT_BASE as w
    c = cases.bert_case(H=w.n_heads, D=w.head_dim, lens=tuple(w.lens()), max_len=w.max_len, scale=w.scale,
                        seed=w.seed)
    out = gpu_bert(c, mode)
    ref = cases.run_bert(orc.Checker("port"), c)
    assert cases.rel_err(out, ref) <= tol
