"""Quantized projections: GGUF weight matrices resident in HBM and the matmul / matmul2 / matmul3 of
the FAST forward pass on them (fast/lil_math.cpp:757-899), for one token or a batch of prompt tokens,
plus seeded synthetic weight rows.

No GGUF models are available here, so benchmarks and tests use ``synthetic_rows``: random blocks of
the reference's layouts (fast/lil_gguf.h:64-119) whose fp16 scale fields hold finite values of a
size that keeps the outputs O(1) for O(1) activations, and whose Q8_0 values stay in the quantizer's
range [-127, 127] (the reference's AVX2 dot, fast/arch_avx2.h:20-27, mis-multiplies -128, a value
its own quantizer never produces).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import check

__all__ = ["QT", "BLOCK", "row_bytes", "synthetic_rows", "QuantMatrix", "matmul3_async", "matmul3",
           "matmul3_batch_async", "matmul3_batch", "NvlReduce"]

# gguf_type numbers (fast/lil_gguf.h:26-44) of the supported weight types
QT = {"F32": 0, "F16": 1, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "Q1_0": 40,
      "Q1_G": 41}
# (bytes, elements) per block
BLOCK = {0: (4, 1), 1: (2, 1), 8: (34, 32), 40: (6, 32), 41: (18, 128), 10: (84, 256), 11: (110, 256),
         12: (144, 256), 13: (176, 256), 14: (210, 256)}
# byte offsets of the fp16 scale fields inside a block
_SCALES = {8: (0,), 40: (0,), 41: (0,), 10: (80, 82), 11: (108,), 12: (0, 2), 13: (0, 2), 14: (208,)}


def row_bytes(t: int, n: int) -> int:
    bb, be = BLOCK[t]
    return n // be * bb


def synthetic_rows(t: int, n: int, d: int, seed: int) -> np.ndarray:
    """[d][row_bytes] uint8: seeded random blocks of type t with finite fp16 scales."""
    rng = np.random.default_rng(seed)
    rb = row_bytes(t, n)
    if t == 0:
        return (rng.standard_normal((d, n)) / np.sqrt(n)).astype(np.float32).view(np.uint8).reshape(d, rb)
    if t == 1:
        return (rng.standard_normal((d, n)) / np.sqrt(n)).astype(np.float16).view(np.uint8).reshape(d, rb)
    bb, be = BLOCK[t]
    nb = n // be
    blocks = rng.integers(0, 256, size=(d, nb, bb), dtype=np.uint8)
    if t == 8:  # Q8_0 values come from a quantizer whose range is [-127, 127]
        blocks[:, :, 2:] = rng.integers(-127, 128, size=(d, nb, 32), dtype=np.int8).view(np.uint8)
    # scale magnitude ~ 1 / (sqrt(n) * typical |q|) keeps the dot products O(1)
    qmag = {8: 64.0, 40: 1.0, 41: 1.0, 10: 1.5 * 8, 11: 3.0 * 16, 12: 7.5 * 32, 13: 15.0 * 32, 14: 32.0 * 64}[t]
    for off in _SCALES[t]:
        v = (np.abs(rng.standard_normal((d, nb))) + 0.1) / (np.sqrt(n) * qmag)
        blocks[:, :, off:off + 2] = v.astype(np.float16).view(np.uint8).reshape(d, nb, 2)
    return blocks.reshape(d, rb)


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    return x.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


class QuantMatrix:
    """A d x n weight matrix of GGUF type ``t`` copied to HBM once (ligguf_cuda_qmat_init)."""

    def __init__(self, t: int, n: int, rows, device: int = 0, cols=None):
        """cols = (col0, ncols): keep only those columns of every row (ligguf_cuda_qmat_init_cols)."""
        self.lib = _lib.load()
        self.type, self.n = t, n
        self._h = ctypes.c_void_p()
        if cols is not None:
            rows = np.ascontiguousarray(rows, dtype=np.uint8)
            self.d, self.n = rows.shape[0], cols[1]
            check(self.lib.ligguf_cuda_qmat_init_cols(t, n, self.d, rows.ctypes.data, cols[0], cols[1], 0, device,
                                                      ctypes.byref(self._h)), "ligguf_cuda_qmat_init_cols")
        elif isinstance(rows, np.ndarray):
            rows = np.ascontiguousarray(rows, dtype=np.uint8)
            self.d = rows.shape[0]
            check(self.lib.ligguf_cuda_qmat_init(t, n, self.d, rows.ctypes.data, 0, device, ctypes.byref(self._h)),
                  "ligguf_cuda_qmat_init")
        else:  # a device tensor of d * row_bytes bytes
            self.d = rows.numel() * rows.element_size() // row_bytes(t, n)
            check(self.lib.ligguf_cuda_qmat_init(t, n, self.d, rows.data_ptr(), 1, device, ctypes.byref(self._h)),
                  "ligguf_cuda_qmat_init")

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            self.lib.ligguf_cuda_qmat_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


def _h(w):
    return w.handle if w is not None else None


def matmul3_async(w0: QuantMatrix, w1, w2, x, out0, out1=None, out2=None, stream=None):
    """One token, device tensors; w1/w2 may be None (matmul2 / matmul)."""
    check(_lib.load().ligguf_cuda_matmul3_async(_h(w0), _h(w1), _h(w2), _ptr(x), _ptr(out0), _ptr(out1), _ptr(out2),
                                                _stream(stream)), "ligguf_cuda_matmul3_async")


def matmul3_batch_async(w0: QuantMatrix, w1, w2, x, n_tok: int, out0, out1=None, out2=None, stream=None):
    """n_tok tokens: x [n_tok][n] -> out_i [n_tok][d_i], device tensors."""
    check(_lib.load().ligguf_cuda_matmul3_batch_async(_h(w0), _h(w1), _h(w2), _ptr(x), n_tok, _ptr(out0),
                                                      _ptr(out1), _ptr(out2), _stream(stream)),
          "ligguf_cuda_matmul3_batch_async")


def matmul3_batch(w0: QuantMatrix, w1, w2, x):
    """Host arrays: x [n_tok][n] (or [n]) -> the outputs of the given matrices (synchronous)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n_tok = x.size // w0.n
    outs = [np.empty((n_tok, w.d), dtype=np.float32) if w is not None else None for w in (w0, w1, w2)]
    check(_lib.load().ligguf_cuda_matmul3_batch(_h(w0), _h(w1), _h(w2), x.ctypes.data, n_tok, _ptr(outs[0]),
                                                _ptr(outs[1]), _ptr(outs[2])), "ligguf_cuda_matmul3_batch")
    return [o for o in outs if o is not None]


def matmul3(w0: QuantMatrix, w1, w2, x):
    """One token, host arrays in and out (synchronous)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    outs = [np.empty(w.d, dtype=np.float32) if w is not None else None for w in (w0, w1, w2)]
    check(_lib.load().ligguf_cuda_matmul3(_h(w0), _h(w1), _h(w2), x.ctypes.data, _ptr(outs[0]), _ptr(outs[1]),
                                          _ptr(outs[2])), "ligguf_cuda_matmul3")
    return [o for o in outs if o is not None]


class NvlReduce:
    """One rank of a SARA reduce group (ligguf_cuda_reduce_*): the attn_output partial projection of
    this rank's heads stored into every rank's buffer over NVLink, summed in rank order on every rank
    (cpp/ligguf_distrib.cpp:749-750,1025-1047)."""

    def __init__(self, rows: int, nranks: int, rank: int, device: int = 0):
        self.lib = _lib.load()
        self.rows, self.nranks, self.rank = rows, nranks, rank
        self._h = ctypes.c_void_p()
        check(self.lib.ligguf_cuda_reduce_init(rows, nranks, rank, device, ctypes.byref(self._h)),
              "ligguf_cuda_reduce_init")

    def ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        check(self.lib.ligguf_cuda_reduce_ipc_handle(self._h, buf, 64), "ligguf_cuda_reduce_ipc_handle")
        return buf.raw

    def open(self, handles):
        blob = b"".join(handles)
        check(self.lib.ligguf_cuda_reduce_open(self._h, blob, 64), "ligguf_cuda_reduce_open")

    def project_async(self, w: QuantMatrix, x, stream=None):
        check(self.lib.ligguf_cuda_matmul_reduce_async(w.handle, self._h, _ptr(x), _stream(stream)),
              "ligguf_cuda_matmul_reduce_async")

    def wait_async(self, x_inout=None, out=None, stream=None):
        check(self.lib.ligguf_cuda_reduce_wait_async(self._h, _ptr(x_inout), _ptr(out), _stream(stream)),
              "ligguf_cuda_reduce_wait_async")

    def status(self, stream=None):
        check(self.lib.ligguf_cuda_reduce_status(self._h, _stream(stream)), "ligguf_cuda_reduce_status")

    def close(self):
        if self._h:
            self.lib.ligguf_cuda_reduce_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
