"""Causal prefill on the GPU against the reference's token-by-token loop
(fast/ligguf_fast_qk.cpp:340-356: one inference() per prompt token).

fp32 SIMT path: max |gpu - ref| <= 1e-4 * max |ref|.  bf16 tensor-core path: <= 2e-2 * max |ref|.
"""
import json
import os

import numpy as np
import pytest

import cases
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL_SIMT = 1e-4
TOL_TC = 2e-2
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def gpu_prefill(c, mode, h=None):
    from ligguf_b200 import AttnConfig, CudaAttention
    if h is None:
        cfg = AttnConfig(n_layers=c["layer"] + 1, n_heads=c["H"], n_kv_heads=c["Hk"], head_dim=c["D"],
                         n_context=c["n_ctx"], rope_dim=c["rope_dim"], rope_base=c["theta"], rms_epsilon=c["eps"],
                         qk_norm=bool(c["qk_norm"]), kv_type=c["kv_type"], scale_mode=c["scale_mode"])
        h = CudaAttention(cfg)
    if c["qk_norm"]:
        h.set_qk_norm(c["layer"], c["qg"], c["kg"])
    if c["pos0"] > 0:
        h.kv_synth(c["layer"], 1, 0, c["pos0"], c["seed"], c["scale"])
    out = h.prefill(c["layer"], c["pos0"], c["q"], c["k"], c["v"], mode)
    return out, h


@pytest.mark.parametrize("key", ["prefill_f32_p0", "prefill_f32_qwen3_p5"])
def test_prefill_simt_vs_reference_golden(gpu, key):
    spec = dict(json.load(open(os.path.join(GOLDEN, "golden.json")))[key])
    gold = np.load(os.path.join(GOLDEN, key + ".npz"))
    out, h = gpu_prefill(cases.prefill_case(**spec), 0)
    assert cases.rel_err(out, gold["out"]) <= TOL_SIMT
    h.close()


@pytest.mark.parametrize("shape", [(32, 4, 64), (32, 8, 128), (8, 8, 64)])
@pytest.mark.parametrize("pos0,n", [(0, 1), (0, 70), (37, 100), (128, 64)])
def test_prefill_simt_sweep(gpu, shape, pos0, n):
    H, Hk, D = shape
    c = cases.prefill_case(H=H, Hk=Hk, D=D, n_ctx=256, theta=1e6, qk_norm=int(D == 128), pos0=pos0, n=n,
                           scale=1.0 if D == 128 else 0.125, seed=pos0 * 1000 + n)
    out, h = gpu_prefill(c, 0)
    ref, kc, vc = cases.run_prefill(orc.Checker("port"), c)
    assert cases.rel_err(out, ref) <= TOL_SIMT
    # the prefill appended rows [pos0, pos0+n) to the cache exactly as the token loop does
    k, v = h.kv_download(0, pos0, n)
    assert np.array_equal(v, vc[pos0:pos0 + n])
    assert np.abs(k - kc[pos0:pos0 + n]).max() <= 4e-6 * np.abs(kc[pos0:pos0 + n]).max()
    h.close()


def test_prefill_simt_fp16_cache(gpu):
    """fp16 cache: the token loop reads the current position's k, v unrounded (fp32) and every earlier
    one from the fp16 cache; the batched kernel reads all of them from the cache, so the diagonal term
    differs by one fp16 rounding - bounded here by 2e-3 of the output scale."""
    c = cases.prefill_case(H=8, Hk=2, D=128, n_ctx=256, theta=1e6, qk_norm=1, pos0=20, n=90, kv_type=1, seed=5)
    out, h = gpu_prefill(c, 0)
    ref, _, _ = cases.run_prefill(orc.Checker("port"), c)
    assert cases.rel_err(out, ref) <= 2e-3
    h.close()


@pytest.mark.parametrize("shape", [(32, 8, 128), (32, 4, 64), (12, 12, 64)])
@pytest.mark.parametrize("pos0,n", [(0, 128), (0, 300), (64, 200), (0, 1)])
def test_prefill_tc_sweep(gpu, shape, pos0, n):
    H, Hk, D = shape
    c = cases.prefill_case(H=H, Hk=Hk, D=D, n_ctx=512, theta=1e6, qk_norm=int(D == 128), pos0=pos0, n=n,
                           scale=1.0 if D == 128 else 0.125, seed=77 + n)
    out, h = gpu_prefill(c, 1)
    ref, _, _ = cases.run_prefill(orc.Checker("port"), c)
    assert cases.rel_err(out, ref) <= TOL_TC
    h.close()


def test_prefill_full_size_vs_reference(gpu):
    """qwen3_8b_prefill_2048 at full size (one layer, 2048 tokens from position 0): every row of the
    SIMT and the tensor-core prefill against the C restatement of the reference's token loop (about
    34 GFLOP on the CPU), and sampled rows against the decode kernel replaying that loop."""
    from ligguf_b200 import AttnConfig, CudaAttention
    from ligguf_b200.workloads import QWEN3_PREFILL as w
    c = cases.prefill_case(H=w.n_heads, Hk=w.n_kv_heads, D=w.head_dim, n_ctx=w.n_context, theta=w.rope_base,
                           qk_norm=1, eps=w.eps, pos0=0, n=w.n_tokens, scale=w.scale, seed=w.seed)
    port = orc.Checker("port")
    port.set_threads(os.cpu_count() or 1)
    ref, _, _ = cases.run_prefill(port, c)
    simt, h = gpu_prefill(c, 0)
    assert cases.rel_err(simt, ref) <= TOL_SIMT
    tc, _ = gpu_prefill(c, 1, h)
    assert cases.rel_err(tc, ref) <= TOL_TC
    cfg = AttnConfig(n_layers=1, n_heads=w.n_heads, n_kv_heads=w.n_kv_heads, head_dim=w.head_dim,
                     n_context=w.n_context, rope_dim=w.head_dim, rope_base=w.rope_base, rms_epsilon=w.eps,
                     qk_norm=True)
    d = CudaAttention(cfg)
    d.set_qk_norm(0, c["qg"], c["kg"])
    for i in range(w.n_tokens):  # replay the token loop on the decode kernel
        o = d.decode(0, i, c["q"][i], c["k"][i], c["v"][i])
        if i in (0, 1, 127, 128, 1000, w.n_tokens - 1):
            assert cases.rel_err(o, ref[i]) <= TOL_SIMT, i
    d.close()
    h.close()


def test_prefill_tc_chunks_reuse_and_refresh_the_bf16_shadow(gpu):
    """The tensor-core path keeps a bf16 copy of each layer's cache and converts only the rows written
    since it last matched: a prompt prefilled in chunks equals the one-call result, and every other
    writer of the cache (a decode at an earlier position, a host upload, a SIMT prefill) makes the next
    tensor-core call see the new rows.  The SIMT path on the same handle reads the cache itself and is
    the yardstick."""
    from ligguf_b200 import AttnConfig, CudaAttention
    H, Hk, D, n_ctx = 16, 4, 128, 512
    c = cases.prefill_case(H=H, Hk=Hk, D=D, n_ctx=n_ctx, theta=1e6, qk_norm=1, pos0=0, n=300, seed=91)
    ref, _, _ = cases.run_prefill(orc.Checker("port"), c)
    cfg = AttnConfig(n_layers=1, n_heads=H, n_kv_heads=Hk, head_dim=D, n_context=n_ctx, rope_dim=D,
                     rope_base=c["theta"], rms_epsilon=c["eps"], qk_norm=True)
    h = CudaAttention(cfg)
    h.set_qk_norm(0, c["qg"], c["kg"])
    outs = [h.prefill(0, p, c["q"][p:p + 100], c["k"][p:p + 100], c["v"][p:p + 100], 1) for p in (0, 100, 200)]
    assert cases.rel_err(np.concatenate(outs), ref) <= TOL_TC

    rng = np.random.default_rng(3)
    kv_dim = Hk * D

    def tc_vs_simt(p, n):
        q = rng.standard_normal((n, H * D)).astype(np.float32)
        k = rng.standard_normal((n, kv_dim)).astype(np.float32)
        v = rng.standard_normal((n, kv_dim)).astype(np.float32)
        tc = h.prefill(0, p, q, k, v, 1)
        simt = h.prefill(0, p, q, k, v, 0)  # rewrites the same rows with the same values
        return cases.rel_err(tc, simt)

    # a decode at an earlier position (a backtrack) with a value row that dominates the sums
    q1 = rng.standard_normal(H * D).astype(np.float32)
    k1 = rng.standard_normal(kv_dim).astype(np.float32)
    h.decode(0, 120, q1, k1, 1e3 * rng.standard_normal(kv_dim).astype(np.float32))
    assert tc_vs_simt(300, 40) <= TOL_TC
    # a host upload of earlier rows
    kk, vv = h.kv_download(0, 10, 50)
    h.kv_upload(0, 10, kk * 3, vv * 50)
    assert tc_vs_simt(340, 40) <= TOL_TC
    # a SIMT prefill over earlier rows, then a tensor-core call behind it
    q2 = rng.standard_normal((30, H * D)).astype(np.float32)
    k2 = rng.standard_normal((30, kv_dim)).astype(np.float32)
    h.prefill(0, 200, q2, k2, 30 * rng.standard_normal((30, kv_dim)).astype(np.float32), 0)
    assert tc_vs_simt(380, 40) <= TOL_TC
    h.close()
