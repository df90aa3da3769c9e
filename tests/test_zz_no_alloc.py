"""The allocation-free BERT attention entry point (ligguf_cuda_bert_attn_tc_noalloc).

Some callers may not allocate device memory at all: a host that hands every byte of the GPU to its
own memory pool and forbids libraries from calling cudaMalloc, or a latency-critical loop where a
cudaMalloc (which synchronises the whole device and has unbounded cost) is not allowed.  For them the
library keeps the tensor-core path's scratch (bf16 copies of q, k, v) in a fixed array of its own.

This file checks, through the C ABI, that two calls in a row give the same result as the regular
handle-based entry point (ligguf_cuda_bert_attn_async, tensor-core mode) within the tensor-core
tolerance (2e-2 of the output scale), that the second call is not disturbed by what the first left
in the shared array, and that an oversized call is refused.  It is collected last so that a run
stopping at the first failure has already run everything else; it also passes on its own.
"""
import ctypes

import numpy as np
import pytest

import cases
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL_TC = 2e-2


def _run_both(lib, c):
    import torch
    from ligguf_b200 import CudaBertAttention
    dev = torch.device("cuda", torch.cuda.current_device())
    H, D, lens, max_len = c["H"], c["D"], c["lens"], c["max_len"]
    q, k, v = (torch.from_numpy(np.ascontiguousarray(c[x])).to(dev) for x in ("q", "k", "v"))
    d_lens = torch.from_numpy(np.asarray(lens, dtype=np.int32)).to(dev)
    batch = len(lens)
    ref_out = torch.full_like(q, float("nan"))
    h = CudaBertAttention(H, D, batch, max_len, dev.index)
    h.attn_async(batch, max_len, d_lens, q, k, v, ref_out, mode=1)
    torch.cuda.synchronize()
    h.close()
    out = torch.full_like(q, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ligguf_cuda_bert_attn_tc_noalloc(H, D, batch, max_len, d_lens.data_ptr(), q.data_ptr(), k.data_ptr(),
                                              v.data_ptr(), out.data_ptr(), stream)
    assert rc == 0, lib.ligguf_cuda_attn_last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy(), ref_out.cpu().numpy()


def test_noalloc_matches_handle_path_on_two_calls(gpu):
    lib = gpu
    first = cases.bert_case(H=12, D=64, lens=(5, 100, 37), max_len=128, scale=0.125, seed=901)
    second = cases.bert_case(H=8, D=128, lens=(64, 1), max_len=200, scale=0.125, seed=902)
    for c in (first, second):
        out, ref = _run_both(lib, c)
        assert np.isfinite(out).all()
        assert cases.rel_err(out, ref) <= TOL_TC
        cpu = cases.run_bert(orc.Checker("port"), c)  # and the reference restatement
        assert cases.rel_err(out, cpu) <= TOL_TC


def test_noalloc_refuses_sizes_beyond_its_array(gpu):
    from ligguf_b200 import _lib
    lib = gpu
    too_many = _lib.NOALLOC_MAX_ELEMS // (12 * 64) + 1  # one token row over the limit
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    rc = lib.ligguf_cuda_bert_attn_tc_noalloc(12, 64, 1, too_many, dummy, dummy, dummy, dummy, dummy, None)
    assert rc == _lib.EINVAL
    assert b"no-allocation limit" in lib.ligguf_cuda_attn_last_error()
