"""ctypes access to the CPU checkers.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, never by the product package.  Two libraries with the same entry points:

* ``liboracle_port.so`` - attn_oracle.c, the C restatement of the reference's attention loops
  (fast/ligguf_fast_qk.cpp:42-105, cpp/ligguf.cpp:674-718, fast/vdb.cpp:189-212), plus the seeded
  synthetic generator that the CUDA library reproduces bit for bit.
* ``_ref/libligguf_ref.so`` - the reference's own fast/lil_math.cpp compiled from source
  (oracle/Makefile) driven by ref_harness.cpp.  Present only where it was built (it is built in the
  container that holds the reference tree and travels to the GPU box as a prebuilt file).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(HERE, "liboracle_port.so")
REF_PATH = os.path.join(HERE, "_ref", "libligguf_ref.so")

KV_F32, KV_F16, KV_BF16 = 0, 1, 2
SYNTH_K, SYNTH_V, SYNTH_Q, SYNTH_KNEW, SYNTH_VNEW, SYNTH_QGAMMA, SYNTH_KGAMMA = 1, 2, 3, 4, 5, 6, 7
SYNTH_SD = 37837.227241611614  # sd of the sum of four uniforms on {0..65535}

_c_int, _c_float, _c_u64 = ctypes.c_int, ctypes.c_float, ctypes.c_uint64
_vp = ctypes.c_void_p


class LoCfg(ctypes.Structure):
    """Mirror of ``lo_cfg`` (attn_oracle.c) / ``rf_cfg`` (ref_harness.cpp)."""

    _fields_ = [
        ("n_heads", _c_int),
        ("n_kv_heads", _c_int),
        ("head_dim", _c_int),
        ("n_context", _c_int),
        ("rope_dim", _c_int),
        ("eps", _c_float),
        ("qk_norm", _c_int),
        ("kv_type", _c_int),
        ("scale_mode", _c_int),
    ]


def build(quiet: bool = True) -> None:
    """Runs oracle/Makefile (port always; the reference build when its tree is present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def _ptr(a):
    return a.ctypes.data_as(_vp) if a is not None else None


_port = None
_ref = None


def port_lib():
    global _port
    if _port is None:
        if not os.path.exists(PORT_PATH):
            build()
        lib = ctypes.CDLL(PORT_PATH)
        lib.lo_splitmix64.restype = _c_u64
        lib.lo_splitmix64.argtypes = [_c_u64]
        lib.lo_synth_mul.restype = _c_float
        lib.lo_synth_mul.argtypes = [_c_float]
        lib.lo_synth_fill_f32.argtypes = [_vp, ctypes.c_size_t, _c_u64, _c_u64, _c_u64, _c_float, _c_float]
        lib.lo_f32_to_f16.restype = ctypes.c_uint16
        lib.lo_f32_to_f16.argtypes = [_c_float]
        lib.lo_f16_to_f32.restype = _c_float
        lib.lo_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.lo_f32_to_bf16.restype = ctypes.c_uint16
        lib.lo_f32_to_bf16.argtypes = [_c_float]
        lib.lo_convert_from_f32.argtypes = [_vp, _c_int, _vp, ctypes.c_size_t]
        lib.lo_convert_to_f32.argtypes = [_vp, _vp, _c_int, ctypes.c_size_t]
        lib.lo_rope_table.argtypes = [_vp, _c_int, _c_float]
        lib.lo_rope.argtypes = [_vp, _c_int, _c_int, _c_int, _c_int, _vp]
        lib.lo_rmsnorm_inplace.argtypes = [_vp, _vp, _c_int, _c_float]
        lib.lo_softmax.argtypes = [_vp, _c_int]
        lib.lo_decode_layer.argtypes = [ctypes.POINTER(LoCfg), _vp, _vp, _vp, _vp, _vp, _c_int, _vp, _vp, _vp, _vp]
        lib.lo_prefill_layer.argtypes = [ctypes.POINTER(LoCfg), _vp, _vp, _vp, _vp, _vp, _c_int, _c_int,
                                         _vp, _vp, _vp, _vp]
        lib.lo_bert_attn.argtypes = [_c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp]
        lib.lo_split_even.argtypes = [_c_int, _c_int, _c_int, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]
        lib.lo_kv_synth.argtypes = [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                    _c_u64, _c_float]
        lib.lo_set_threads.argtypes = [_c_int]
        lib.lo_quantize_q8_K.argtypes = [_vp, _c_int, _vp]
        lib.lo_quantize_q8_0.argtypes = [_vp, _c_int, _vp]
        lib.lo_matmul.argtypes = [_vp, _vp, _c_int, _c_int, _vp, _c_int, _c_int, _vp, _vp]
        _port = lib
    return _port


def ref_lib():
    """The reference-compiled checker, or None where it was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        lib = ctypes.CDLL(REF_PATH)
        lib.rf_init.argtypes = []
        lib.rf_f32_to_f16_row.argtypes = [_vp, _vp, _c_int]
        lib.rf_fp16_to_fp32.restype = _c_float
        lib.rf_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        lib.rf_softmax.argtypes = [_vp, _c_int]
        lib.rf_rmsnorm_inplace.argtypes = [_vp, _vp, _c_int, _c_float]
        lib.rf_rope.argtypes = [_vp, _c_int, _c_int, _c_int, _c_int, _vp]
        lib.rf_decode_layer.argtypes = [ctypes.POINTER(LoCfg), _vp, _vp, _vp, _vp, _vp, _c_int, _vp, _vp, _vp, _vp]
        lib.rf_prefill_layer.argtypes = [ctypes.POINTER(LoCfg), _vp, _vp, _vp, _vp, _vp, _c_int, _c_int,
                                         _vp, _vp, _vp, _vp]
        lib.rf_bert_attn.argtypes = [_c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp]
        lib.rf_init()
        _ref = lib
    return _ref


# ------------------------------------------------------------------ synthetic inputs --------
def synth_f32(n: int, seed: int, stream: int, idx0: int = 0, scale: float = 1.0, add: float = 0.0):
    out = np.empty(int(n), dtype=np.float32)
    port_lib().lo_synth_fill_f32(_ptr(out), int(n), seed, stream, idx0, scale, add)
    return out


def stream_id(tensor: int, layer: int) -> int:
    return (tensor << 32) | (layer & 0xFFFFFFFF)


def synth_numpy(n: int, seed: int, stream: int, idx0: int = 0, scale: float = 1.0, add: float = 0.0):
    """Pure-numpy restatement of the generator (cross-checks the C and CUDA versions)."""
    m64 = np.uint64(0xFFFFFFFFFFFFFFFF)

    def sm(x):
        with np.errstate(over="ignore"):
            z = (x + np.uint64(0x9E3779B97F4A7C15)) & m64
            z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & m64
            z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & m64
            return z ^ (z >> np.uint64(31))

    with np.errstate(over="ignore"):
        base = sm(np.uint64(seed) ^ (np.uint64(stream) * np.uint64(0xD1B54A32D192ED03)))
        r = sm(base + np.arange(idx0, idx0 + n, dtype=np.uint64))
    s = sum(((r >> np.uint64(sh)) & np.uint64(0xFFFF)).astype(np.int64) for sh in (0, 16, 32, 48)) - 131070
    mul = np.float32(scale / SYNTH_SD)
    return (s.astype(np.float32) * mul + np.float32(add)).astype(np.float32)


def kv_dtype(kv_type: int):
    return np.float32 if kv_type == KV_F32 else np.uint16


def kv_synth(cache, kv_type, kv_dim_shard, kv_dim_full, kv_off, layer, tensor, pos0, n, seed, scale):
    port_lib().lo_kv_synth(_ptr(cache), kv_type, kv_dim_shard, kv_dim_full, kv_off, layer, tensor,
                           pos0, n, seed, scale)


def to_f32(a, kv_type):
    if kv_type == KV_F32:
        return np.asarray(a, dtype=np.float32)
    out = np.empty(a.size, dtype=np.float32)
    port_lib().lo_convert_to_f32(_ptr(out), _ptr(np.ascontiguousarray(a)), kv_type, a.size)
    return out.reshape(a.shape)


def from_f32(a, kv_type):
    a = np.ascontiguousarray(a, dtype=np.float32)
    if kv_type == KV_F32:
        return a.copy()
    out = np.empty(a.size, dtype=np.uint16)
    port_lib().lo_convert_from_f32(_ptr(out), kv_type, _ptr(a), a.size)
    return out.reshape(a.shape)


def rope_table(rope_dim: int, base: float):
    t = np.zeros(max(rope_dim // 2, 1), dtype=np.float32)
    if rope_dim > 0:
        port_lib().lo_rope_table(_ptr(t), rope_dim, base)
    return t


def split_even(total: int, idx: int, parts: int):
    off, cnt = _c_int(), _c_int()
    port_lib().lo_split_even(total, idx, parts, ctypes.byref(off), ctypes.byref(cnt))
    return off.value, cnt.value


# ------------------------------------------------------------------ attention ---------------
class Checker:
    """decode / prefill / BERT attention through one of the two CPU libraries."""

    def __init__(self, which: str = "port"):
        self.which = which
        if which == "port":
            self.lib, self.p = port_lib(), "lo_"
        elif which == "ref":
            self.lib, self.p = ref_lib(), "rf_"
            if self.lib is None:
                raise FileNotFoundError(REF_PATH)
        else:
            raise ValueError(which)

    def _f(self, name):
        return getattr(self.lib, self.p + name)

    def set_threads(self, n: int) -> int:
        """OpenMP threads of this library's loops (independent of OMP_NUM_THREADS); returns the count."""
        f = self._f("set_threads")
        f.argtypes = [_c_int]
        return int(f(int(n)))

    @staticmethod
    def cfg(n_heads, n_kv_heads, head_dim, n_context, rope_dim, eps=1e-6, qk_norm=0, kv_type=KV_F32,
            scale_mode=0):
        return LoCfg(n_heads, n_kv_heads, head_dim, n_context, rope_dim, eps, qk_norm, kv_type, scale_mode)

    def decode_layer(self, cfg, kc, vc, freq, qg, kg, pos, q, k, v):
        out = np.zeros(cfg.n_heads * cfg.head_dim, dtype=np.float32)
        q, k, v = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v))
        rc = self._f("decode_layer")(ctypes.byref(cfg), _ptr(kc), _ptr(vc), _ptr(freq), _ptr(qg), _ptr(kg),
                                     pos, _ptr(q), _ptr(k), _ptr(v), _ptr(out))
        if rc:
            raise ValueError(f"{self.p}decode_layer failed ({rc})")
        return out

    def prefill_layer(self, cfg, kc, vc, freq, qg, kg, pos0, n, q, k, v):
        out = np.zeros(n * cfg.n_heads * cfg.head_dim, dtype=np.float32)
        q, k, v = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v))
        rc = self._f("prefill_layer")(ctypes.byref(cfg), _ptr(kc), _ptr(vc), _ptr(freq), _ptr(qg), _ptr(kg),
                                      pos0, n, _ptr(q), _ptr(k), _ptr(v), _ptr(out))
        if rc:
            raise ValueError(f"{self.p}prefill_layer failed ({rc})")
        return out.reshape(n, -1)

    def bert_attn(self, n_heads, head_dim, lens, max_len, q, k, v):
        lens = np.ascontiguousarray(lens, dtype=np.int32)
        batch = lens.size
        out = np.zeros(batch * max_len * n_heads * head_dim, dtype=np.float32)
        q, k, v = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v))
        rc = self._f("bert_attn")(n_heads, head_dim, batch, max_len, _ptr(lens), _ptr(q), _ptr(k), _ptr(v),
                                  _ptr(out))
        if rc:
            raise ValueError(f"{self.p}bert_attn failed ({rc})")
        return out.reshape(batch, max_len, n_heads * head_dim)


# ------------------------------------------------------------------ quantized projections ---------
Q8K_BYTES, Q80_BYTES = 292, 34


def quantize_q8_K(x, which: str = "port"):
    """quantize_q8_K (fast/lil_math.cpp:352-385) of x (n % 256 == 0): n/256 blocks as raw bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 256 * Q8K_BYTES, dtype=np.uint8)
    if which == "port":
        port_lib().lo_quantize_q8_K(_ptr(x), x.size, _ptr(out))
    else:
        lib = ref_lib()
        lib.rf_quantize_q8_K.argtypes = [_vp, _c_int, _vp]
        lib.rf_quantize_q8_K(_ptr(x), x.size, _ptr(out))
    return out


def quantize_q8_0(x, which: str = "port"):
    """quantize_q8_0 (fast/lil_math.cpp:329-350) of x (n % 32 == 0): n/32 blocks as raw bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 32 * Q80_BYTES, dtype=np.uint8)
    if which == "port":
        port_lib().lo_quantize_q8_0(_ptr(x), x.size, _ptr(out))
    else:
        lib = ref_lib()
        lib.rf_quantize_q8_0.argtypes = [_vp, _c_int, _vp]
        lib.rf_quantize_q8_0(_ptr(x), x.size, _ptr(out))
    return out


def matmul(w_type: int, w_rows, n: int, x, which: str = "port"):
    """matmul (fast/lil_math.cpp:757-778): out[r] = row r of the GGUF weight rows `w_rows` ([d][rb]
    uint8) against x, with x quantized as the engine does (Q8_K for K-quants, Q8_0 for Q8_0/Q1_*)."""
    w = np.ascontiguousarray(w_rows, dtype=np.uint8)
    d, rb = w.shape
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(d, dtype=np.float32)
    if which == "port":
        sk = np.zeros(max(1, n // 256) * Q8K_BYTES, dtype=np.uint8)
        s0 = np.zeros(max(1, n // 32) * Q80_BYTES, dtype=np.uint8)
        port_lib().lo_matmul(_ptr(out), _ptr(x), n, w_type, _ptr(w), rb, d, _ptr(sk), _ptr(s0))
    else:
        lib = ref_lib()
        lib.rf_matmul.argtypes = [_vp, _vp, _c_int, _c_int, _vp, _c_int, _c_int]
        lib.rf_matmul(_ptr(out), _ptr(x), n, w_type, _ptr(w), rb, d)
    return out


def matmul3(ws, n: int, x):
    """The engine's QKV step (fast/ligguf_fast_qk.cpp:39-40) through the reference build:
    quantize_q8_K, then matmul3 over ws = [(type, rows), (type, rows), (type, rows)]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    (t0, w0), (t1, w1), (t2, w2) = [(t, np.ascontiguousarray(w, dtype=np.uint8)) for t, w in ws]
    outs = [np.zeros(w.shape[0], dtype=np.float32) for w in (w0, w1, w2)]
    lib = ref_lib()
    lib.rf_matmul3.argtypes = [_vp, _vp, _vp, _vp, _c_int] + [_c_int, _vp, _c_int, _c_int] * 3
    lib.rf_matmul3(_ptr(outs[0]), _ptr(outs[1]), _ptr(outs[2]), _ptr(x), n,
                   t0, _ptr(w0), w0.shape[1], w0.shape[0], t1, _ptr(w1), w1.shape[1], w1.shape[0],
                   t2, _ptr(w2), w2.shape[1], w2.shape[0])
    return outs
