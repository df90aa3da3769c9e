"""SARA attn_output projection + reduce (ligguf_cuda_qmat_init_cols, ligguf_cuda_matmul_reduce_async,
ligguf_cuda_reduce_wait_async) on one GPU: a one-rank group, the rank storing its partial rows into
its own buffer.  Against the C restatement: x + matmul_partial_cols(att_out, quantize_q8_0(xb), cols)
(cpp/ligguf_distrib.cpp:587-605,749-750; the residual add of the forward pass), within 1e-4 of the
output scale.  Calls issued directly, then captured in a CUDA graph and replayed (the epochs advance on
the device).  The multi-GPU form is tested in test_multigpu_gpu.py."""
import numpy as np
import pytest

from oracle import oracle as orc
from ligguf_b200.qmat import NvlReduce, QuantMatrix, synthetic_rows

pytestmark = pytest.mark.gpu
TOL = 1e-4


def test_one_rank_reduce_direct_and_replayed(gpu):
    import torch
    n_embed, col0, ncols = 2048, 512, 1024        # this rank's heads: columns [512, 1536)
    rows = synthetic_rows(8, n_embed, n_embed, seed=5)
    w = QuantMatrix(8, n_embed, rows, cols=(col0, ncols))
    red = NvlReduce(n_embed, 1, 0)
    red.open([red.ipc_handle()])
    rng = np.random.default_rng(3)
    xb = [rng.standard_normal(ncols).astype(np.float32) for _ in range(3)]
    res0 = rng.standard_normal(n_embed).astype(np.float32)
    dev = torch.device("cuda", 0)
    d_xb = [torch.from_numpy(v).to(dev) for v in xb]
    x = torch.from_numpy(res0).to(dev)
    out = torch.full((n_embed,), float("nan"), device=dev)
    sub = rows[:, col0 // 32 * 34:(col0 + ncols) // 32 * 34]

    def refs_after(k):
        r = res0.copy()
        for i in range(k):
            r = r + orc.matmul(8, sub, ncols, xb[i % 3], "port")
        return r

    def step(i):
        red.project_async(w, d_xb[i % 3])
        red.wait_async(x_inout=x, out=out)

    for i in range(3):
        step(i)
        torch.cuda.synchronize()
        red.status()
        part = orc.matmul(8, sub, ncols, xb[i], "port")
        assert np.abs(out.cpu().numpy() - part).max() <= TOL * np.abs(part).max()
    ref = refs_after(3)
    assert np.abs(x.cpu().numpy() - ref).max() <= TOL * np.abs(ref).max()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(3):
            step(i)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    red.status()
    ref = refs_after(9)
    assert np.abs(x.cpu().numpy() - ref).max() <= TOL * np.abs(ref).max()
    del g
    red.close()
    w.close()
