"""ctypes binding of libligguf_cuda_attn.so (the C ABI in include/ligguf_cuda_attn.h).

The library is loaded from this package directory only; there is no CPU fallback.  A missing or
unloadable library raises immediately.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libligguf_cuda_attn.so")

OK, EINVAL, ECUDA, ENOMEM, ETIMEDOUT, EUNSUPPORTED, ESTATE = 0, -1, -2, -3, -4, -5, -6
KV_F32, KV_F16, KV_BF16 = 0, 1, 2
SCALE_MUL, SCALE_DIV = 0, 1
MODE_SIMT, MODE_TC = 0, 1
SYNTH_K, SYNTH_V, SYNTH_Q, SYNTH_KNEW, SYNTH_VNEW, SYNTH_QGAMMA, SYNTH_KGAMMA = 1, 2, 3, 4, 5, 6, 7
NOALLOC_MAX_ELEMS = 1 << 22  # LIGGUF_NOALLOC_MAX_ELEMS

_i, _f, _u64, _sz, _vp, _cp = ctypes.c_int, ctypes.c_float, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p


class AttnCfg(ctypes.Structure):
    """Mirror of ``ligguf_attn_cfg``."""

    _fields_ = [
        ("n_layers", _i),
        ("n_heads", _i),
        ("n_kv_heads", _i),
        ("head_dim", _i),
        ("n_context", _i),
        ("rope_dim", _i),
        ("rope_base", _f),
        ("rope_freq", ctypes.POINTER(_f)),
        ("rms_epsilon", _f),
        ("qk_norm", _i),
        ("kv_type", _i),
        ("scale_mode", _i),
        ("device", _i),
        ("kv_head0", _i),
        ("kv_headn", _i),
    ]


class LigGufAttnError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str):
        super().__init__(f"{where}: status {status} ({detail})")
        self.status = status


_PROTOS = {
    "ligguf_cuda_attn_init": [ctypes.POINTER(AttnCfg), ctypes.POINTER(_vp)],
    "ligguf_cuda_attn_free": [_vp],
    "ligguf_cuda_attn_strerror": [_i],
    "ligguf_cuda_attn_last_error": [],
    "ligguf_cuda_attn_set_qk_norm": [_vp, _i, _vp, _vp],
    "ligguf_cuda_attn_decode": [_vp, _i, _i, _vp, _vp, _vp, _vp],
    "ligguf_cuda_attn_decode_async": [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp],
    "ligguf_cuda_attn_prefill": [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _i],
    "ligguf_cuda_attn_prefill_async": [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _i, _vp],
    "ligguf_cuda_attn_kv_download": [_vp, _i, _i, _i, _vp, _vp],
    "ligguf_cuda_attn_kv_upload": [_vp, _i, _i, _i, _vp, _vp],
    "ligguf_cuda_attn_state_save": [_vp, _cp, _i, _vp, _u64],
    "ligguf_cuda_attn_state_load": [_vp, _cp, ctypes.POINTER(_i), ctypes.POINTER(_i), _vp, _u64],
    "ligguf_cuda_attn_kv_synth": [_vp, _i, _i, _i, _i, _u64, _f],
    "ligguf_cuda_attn_sync": [_vp],
    "ligguf_cuda_attn_gather_ipc_handle": [_vp, _vp, _sz],
    "ligguf_cuda_attn_gather_open": [_vp, _i, _i, _vp, _sz],
    "ligguf_cuda_attn_decode_gather_async": [_vp, _i, _i, _vp, _vp, _vp, _vp],
    "ligguf_cuda_attn_gather_wait_async": [_vp, _i, _vp, _vp],
    "ligguf_cuda_bert_init": [_i, _i, _i, _i, _i, ctypes.POINTER(_vp)],
    "ligguf_cuda_bert_free": [_vp],
    "ligguf_cuda_bert_attn": [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _i],
    "ligguf_cuda_bert_attn_async": [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "ligguf_cuda_bert_attn_tc_noalloc": [_i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp],
    "ligguf_cuda_bert_attn_tc_noalloc_status": [_vp],
    "ligguf_cuda_qmat_row_bytes": [_i, _i],
    "ligguf_cuda_qmat_init": [_i, _i, _i, _vp, _i, _i, ctypes.POINTER(_vp)],
    "ligguf_cuda_qmat_init_cols": [_i, _i, _i, _vp, _i, _i, _i, _i, ctypes.POINTER(_vp)],
    "ligguf_cuda_qmat_free": [_vp],
    "ligguf_cuda_reduce_init": [_i, _i, _i, _i, ctypes.POINTER(_vp)],
    "ligguf_cuda_reduce_free": [_vp],
    "ligguf_cuda_reduce_ipc_handle": [_vp, _vp, _sz],
    "ligguf_cuda_reduce_open": [_vp, _vp, _sz],
    "ligguf_cuda_matmul_reduce_async": [_vp, _vp, _vp, _vp],
    "ligguf_cuda_reduce_wait_async": [_vp, _vp, _vp, _vp],
    "ligguf_cuda_reduce_status": [_vp, _vp],
    "ligguf_cuda_matmul3_async": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "ligguf_cuda_matmul3": [_vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "ligguf_cuda_matmul3_batch_async": [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp],
    "ligguf_cuda_matmul3_batch": [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp],
    "ligguf_cuda_quantize_q8_K_async": [_vp, _i, _vp, _vp],
    "ligguf_cuda_quantize_q8_0_async": [_vp, _i, _vp, _vp],
    "ligguf_cuda_synth_fill": [_vp, _i, _sz, _u64, _u64, _u64, _f, _f, _vp],
}

_lib = None


def load(path: str = LIB_PATH):
    """Loads the CUDA library (raises if it is missing: there is no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with `python -m ligguf_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(path)
    for name, argtypes in _PROTOS.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = (_cp if name in ("ligguf_cuda_attn_strerror", "ligguf_cuda_attn_last_error")
                      else _sz if name == "ligguf_cuda_qmat_row_bytes" else _i)
    _lib = lib
    return lib


def exported_names():
    return list(_PROTOS)


def check(status: int, where: str) -> None:
    if status != OK:
        lib = load()
        detail = lib.ligguf_cuda_attn_last_error().decode(errors="replace") or \
            lib.ligguf_cuda_attn_strerror(status).decode()
        raise LigGufAttnError(status, where, detail)
