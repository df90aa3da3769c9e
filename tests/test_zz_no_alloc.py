"""The allocation-free BERT attention entry point (ligguf_cuda_bert_attn_tc_noalloc).

Some callers may not allocate device memory at all: a host that hands every byte of the GPU to its
own memory pool and forbids libraries from calling cudaMalloc, or a latency-critical loop where a
cudaMalloc (which synchronises the whole device and has unbounded cost) is not allowed.  For them the
library keeps the tensor-core path's scratch (bf16 copies of q, k, v) in a fixed array of its own.

This file checks, through the C ABI:
  - two calls in a row, the larger first, each against the regular handle-based entry point
    (ligguf_cuda_bert_attn_async, tensor-core mode) and the CPU restatement of the reference, within
    the tensor-core tolerance (2e-2 of the output scale);
  - that what one call leaves in the shared array cannot reach the next: a call whose inputs are all
    NaN fills the array, then a smaller call whose first sequence's last key tile runs into the rows
    of an empty second sequence must still be finite and correct;
  - that a call allocates nothing (free device memory does not drop across it);
  - that the status query reports no failure after normal calls, and that an oversized call is
    refused.
It is collected last so that a run stopping at the first failure has already run everything else;
it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import cases
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL_TC = 2e-2


def _dev_inputs(c):
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    q, k, v = (torch.from_numpy(np.ascontiguousarray(c[x])).to(dev) for x in ("q", "k", "v"))
    d_lens = torch.from_numpy(np.asarray(c["lens"], dtype=np.int32)).to(dev)
    return q, k, v, d_lens


def _noalloc(lib, c, q, k, v, d_lens, out):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ligguf_cuda_bert_attn_tc_noalloc(c["H"], c["D"], len(c["lens"]), c["max_len"], d_lens.data_ptr(),
                                              q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), stream)
    assert rc == 0, lib.ligguf_cuda_attn_last_error()


def _handle_path(c, q, k, v, d_lens):
    import torch
    from ligguf_b200 import CudaBertAttention
    ref_out = torch.full_like(q, float("nan"))
    h = CudaBertAttention(c["H"], c["D"], len(c["lens"]), c["max_len"], q.device.index)
    h.attn_async(len(c["lens"]), c["max_len"], d_lens, q, k, v, ref_out, mode=1)
    torch.cuda.synchronize()
    h.close()
    return ref_out.cpu().numpy()


def _check(lib, c, measure_alloc=False):
    import torch
    q, k, v, d_lens = _dev_inputs(c)
    ref = _handle_path(c, q, k, v, d_lens)
    out = torch.full_like(q, float("nan"))
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    _noalloc(lib, c, q, k, v, d_lens, out)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    if measure_alloc:
        assert free1 >= free0, f"device memory dropped by {free0 - free1} bytes across the call"
    assert lib.ligguf_cuda_bert_attn_tc_noalloc_status(None) == 0, lib.ligguf_cuda_attn_last_error()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert cases.rel_err(got, ref) <= TOL_TC
    cpu = cases.run_bert(orc.Checker("port"), c)  # and the reference restatement
    assert cases.rel_err(got, cpu) <= TOL_TC


def test_noalloc_matches_handle_path_on_two_calls(gpu):
    lib = gpu
    # larger first, then smaller: the second call runs over what the first left in the array
    _check(lib, cases.bert_case(H=8, D=128, lens=(64, 1, 200), max_len=200, scale=0.125, seed=902))
    _check(lib, cases.bert_case(H=12, D=64, lens=(5, 100, 37), max_len=128, scale=0.125, seed=901),
           measure_alloc=True)


def test_noalloc_leftovers_cannot_poison_the_next_call(gpu):
    """A call whose q, k and v are all NaN leaves NaN in every operand row of the array.  The next
    call has lens (200, 0) at max_len 200: the first sequence's second key tile (rows 128..255)
    runs 56 rows into the empty second sequence, whose rows must therefore be zero, not stale."""
    import torch
    lib = gpu
    poison = cases.bert_case(H=12, D=64, lens=(512, 512), max_len=512, scale=0.125, seed=903)
    for x in ("q", "k", "v"):
        poison[x] = np.full_like(poison[x], np.nan)
    q, k, v, d_lens = _dev_inputs(poison)
    _noalloc(lib, poison, q, k, v, d_lens, torch.empty_like(q))
    torch.cuda.synchronize()
    _check(lib, cases.bert_case(H=8, D=128, lens=(200, 0), max_len=200, scale=0.125, seed=904))


def test_noalloc_refuses_sizes_beyond_its_array(gpu):
    from ligguf_b200 import _lib
    lib = gpu
    too_many = _lib.NOALLOC_MAX_ELEMS // (12 * 64) + 1  # one token row over the limit
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    rc = lib.ligguf_cuda_bert_attn_tc_noalloc(12, 64, 1, too_many, dummy, dummy, dummy, dummy, dummy, None)
    assert rc == _lib.EINVAL
    assert b"no-allocation limit" in lib.ligguf_cuda_attn_last_error()
