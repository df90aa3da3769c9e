"""Python face of the B200 attention block (thin wrappers over the C ABI).

Mirrors what the FAST engine does around its attention (fast/ligguf_fast_qk.cpp:24-105):
``model_state::allocate()`` sizes the KV cache (fast/common.cpp:11-40) -> ``CudaAttention(...)``;
the per-layer block at fast/ligguf_fast_qk.cpp:42-105 -> ``decode(layer, pos, q, k, v)``;
``feed_text`` token loop (fast/ligguf_fast_qk.cpp:340-356) -> ``prefill(layer, pos0, q, k, v)``;
state save/load of the cache rows (fast/ligguf_fast_qk.cpp:236-247,288-295) -> ``kv_download`` /
``kv_upload``; BERT's attention in ``bert_embed`` (fast/vdb.cpp:189-212) -> ``CudaBertAttention``.

Host arrays are numpy; device tensors are anything with ``data_ptr()`` (torch) or raw ints.
Errors raise ``LigGufAttnError`` carrying the library's status code and reason.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import AttnCfg, check

__all__ = ["AttnConfig", "CudaAttention", "CudaBertAttention", "synth_fill", "split_even", "shard_of"]


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
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:  # pragma: no cover - no torch
            return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def split_even(total: int, idx: int, parts: int):
    """SARA's split_even (cpp/ligguf_distrib.cpp:657-663): (offset, count) of part ``idx``."""
    base, rem = divmod(total, parts)
    count = base + (idx < rem)
    off = idx * base + (idx if idx < rem else rem)
    return off, count


def shard_of(n_kv_heads: int, n_heads: int, rank: int, nranks: int):
    """SARA build_shards (cpp/ligguf_distrib.cpp:665-679) for the attention part: the KV heads
    [kv0, kv0+kvn) of ``rank`` and its q heads [kv0*nrep, (kv0+kvn)*nrep)."""
    if nranks > n_kv_heads:  # SARA asserts nranks <= n_kv_heads (cpp/ligguf_distrib.cpp:1203,1219)
        raise ValueError(f"{nranks} ranks for {n_kv_heads} KV heads")
    kv0, kvn = split_even(n_kv_heads, rank, nranks)
    nrep = n_heads // n_kv_heads
    return {"kv_head0": kv0, "kv_headn": kvn, "q_head0": kv0 * nrep, "q_headn": kvn * nrep}


@dataclass
class AttnConfig:
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    n_context: int
    rope_dim: int
    rope_base: float = 10000.0
    rms_epsilon: float = 1e-6
    qk_norm: bool = False
    kv_type: int = _lib.KV_F32
    scale_mode: int = _lib.SCALE_MUL
    device: int = 0
    kv_head0: int = 0
    kv_headn: int = 0  # 0 = all

    @property
    def nrep(self):
        return self.n_heads // self.n_kv_heads

    @property
    def kv_heads_owned(self):
        return self.kv_headn or self.n_kv_heads

    @property
    def q_heads_owned(self):
        return self.kv_heads_owned * self.nrep

    def to_c(self, rope_freq=None):
        c = AttnCfg()
        for f, _ in AttnCfg._fields_:
            if f != "rope_freq":
                setattr(c, f, int(getattr(self, f)) if f not in ("rope_base", "rms_epsilon") else getattr(self, f))
        c.rope_freq = rope_freq.ctypes.data_as(ctypes.POINTER(ctypes.c_float)) if rope_freq is not None else None
        return c


class CudaAttention:
    """One HBM-resident KV cache plus the decode / prefill kernels for one model (or one SARA
    shard of it).  Not thread-safe: one host thread per instance, like ``inference()``."""

    def __init__(self, cfg: AttnConfig, rope_freq: np.ndarray | None = None):
        self.cfg = cfg
        self.lib = _lib.load()
        self._h = ctypes.c_void_p()
        freq = None if rope_freq is None else np.ascontiguousarray(rope_freq, dtype=np.float32)
        c = cfg.to_c(freq)
        check(self.lib.ligguf_cuda_attn_init(ctypes.byref(c), ctypes.byref(self._h)), "ligguf_cuda_attn_init")
        self.q_dim = cfg.q_heads_owned * cfg.head_dim
        self.kv_dim = cfg.kv_heads_owned * cfg.head_dim

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            self.lib.ligguf_cuda_attn_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ weights
    def set_qk_norm(self, layer: int, q_gamma, k_gamma):
        qg = np.ascontiguousarray(q_gamma, dtype=np.float32)
        kg = np.ascontiguousarray(k_gamma, dtype=np.float32)
        check(self.lib.ligguf_cuda_attn_set_qk_norm(self._h, layer, qg.ctypes.data, kg.ctypes.data),
              "ligguf_cuda_attn_set_qk_norm")

    # ------------------------------------------------------------------ decode
    def decode(self, layer: int, pos: int, q, k, v, out: np.ndarray | None = None):
        """Host arrays in, host array out (synchronous)."""
        q = np.ascontiguousarray(q, dtype=np.float32)
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        if q.size != self.q_dim or k.size != self.kv_dim or v.size != self.kv_dim:
            raise ValueError("q/k/v sizes do not match the configuration")
        if out is None:
            out = np.empty(self.q_dim, dtype=np.float32)
        check(self.lib.ligguf_cuda_attn_decode(self._h, layer, pos, q.ctypes.data, k.ctypes.data, v.ctypes.data,
                                               out.ctypes.data), "ligguf_cuda_attn_decode")
        return out

    def decode_async(self, layer: int, pos: int, q, k, v, out, stream=None):
        """Device tensors; enqueued on ``stream`` (default: torch's current stream)."""
        check(self.lib.ligguf_cuda_attn_decode_async(self._h, layer, pos, _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                                     _stream(stream)), "ligguf_cuda_attn_decode_async")

    # ------------------------------------------------------------------ prefill
    def prefill(self, layer: int, pos0: int, q, k, v, mode: int = _lib.MODE_SIMT):
        q = np.ascontiguousarray(q, dtype=np.float32)
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        n = q.size // self.q_dim
        if n * self.q_dim != q.size or k.size != n * self.kv_dim or v.size != n * self.kv_dim:
            raise ValueError("q/k/v sizes do not match the configuration")
        out = np.empty((n, self.q_dim), dtype=np.float32)
        check(self.lib.ligguf_cuda_attn_prefill(self._h, layer, pos0, n, q.ctypes.data, k.ctypes.data,
                                                v.ctypes.data, out.ctypes.data, mode), "ligguf_cuda_attn_prefill")
        return out

    def prefill_async(self, layer: int, pos0: int, n: int, q, k, v, out, mode: int = _lib.MODE_SIMT, stream=None):
        check(self.lib.ligguf_cuda_attn_prefill_async(self._h, layer, pos0, n, _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                                      mode, _stream(stream)), "ligguf_cuda_attn_prefill_async")

    # ------------------------------------------------------------------ cache
    def _kv_np_dtype(self):
        return np.float32 if self.cfg.kv_type == _lib.KV_F32 else np.uint16

    def kv_download(self, layer: int, pos0: int, n: int):
        k = np.empty((n, self.kv_dim), dtype=self._kv_np_dtype())
        v = np.empty_like(k)
        check(self.lib.ligguf_cuda_attn_kv_download(self._h, layer, pos0, n, k.ctypes.data, v.ctypes.data),
              "ligguf_cuda_attn_kv_download")
        return k, v

    def kv_upload(self, layer: int, pos0: int, k, v):
        k = np.ascontiguousarray(k, dtype=self._kv_np_dtype())
        v = np.ascontiguousarray(v, dtype=self._kv_np_dtype())
        n = k.size // self.kv_dim
        check(self.lib.ligguf_cuda_attn_kv_upload(self._h, layer, pos0, n, k.ctypes.data, v.ctypes.data),
              "ligguf_cuda_attn_kv_upload")

    def state_save(self, path: str, pos: int, logits) -> None:
        """The engine's state file (save_model_state, fast/ligguf_fast_qk.cpp:266-302) from the HBM
        cache: header, fp16 K rows [0, pos) per layer, V rows, then ``logits``."""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        check(self.lib.ligguf_cuda_attn_state_save(self._h, os.fsencode(path), pos, lg.ctypes.data, lg.size),
              "ligguf_cuda_attn_state_save")

    def state_load(self, path: str, n_logits: int):
        """load_model_state (fast/ligguf_fast_qk.cpp:216-264) into the HBM cache; returns
        (pos, n_context, logits) from the file."""
        lg = np.empty(n_logits, dtype=np.float32)
        pos, n_ctx = ctypes.c_int(), ctypes.c_int()
        check(self.lib.ligguf_cuda_attn_state_load(self._h, os.fsencode(path), ctypes.byref(pos), ctypes.byref(n_ctx),
                                                   lg.ctypes.data, n_logits), "ligguf_cuda_attn_state_load")
        return pos.value, n_ctx.value, lg

    def kv_synth(self, layer0: int, n_layers: int, pos0: int, n: int, seed: int, scale: float):
        check(self.lib.ligguf_cuda_attn_kv_synth(self._h, layer0, n_layers, pos0, n, seed, scale),
              "ligguf_cuda_attn_kv_synth")

    def sync(self):
        check(self.lib.ligguf_cuda_attn_sync(self._h), "ligguf_cuda_attn_sync")

    # ------------------------------------------------------------------ SARA gather (multi-GPU)
    def gather_ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        check(self.lib.ligguf_cuda_attn_gather_ipc_handle(self._h, buf, 64), "ligguf_cuda_attn_gather_ipc_handle")
        return buf.raw

    def gather_open(self, rank: int, handles: list[bytes]):
        blob = b"".join(handles)
        check(self.lib.ligguf_cuda_attn_gather_open(self._h, len(handles), rank, blob, 64),
              "ligguf_cuda_attn_gather_open")

    def decode_gather_async(self, layer: int, pos: int, q, k, v, stream=None):
        check(self.lib.ligguf_cuda_attn_decode_gather_async(self._h, layer, pos, _ptr(q), _ptr(k), _ptr(v),
                                                            _stream(stream)), "ligguf_cuda_attn_decode_gather_async")

    def gather_wait_async(self, layer: int, out, stream=None):
        check(self.lib.ligguf_cuda_attn_gather_wait_async(self._h, layer, _ptr(out), _stream(stream)),
              "ligguf_cuda_attn_gather_wait_async")


class CudaBertAttention:
    """Batched replacement of bert_embed's attention loop (fast/vdb.cpp:189-212)."""

    def __init__(self, n_heads: int, head_dim: int, max_batch: int, max_len: int, device: int = 0):
        self.lib = _lib.load()
        self._h = ctypes.c_void_p()
        self.n_heads, self.head_dim, self.max_batch, self.max_len = n_heads, head_dim, max_batch, max_len
        check(self.lib.ligguf_cuda_bert_init(n_heads, head_dim, max_batch, max_len, device, ctypes.byref(self._h)),
              "ligguf_cuda_bert_init")

    def close(self):
        if self._h:
            self.lib.ligguf_cuda_bert_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def attn(self, lens, q, k, v, mode: int = _lib.MODE_SIMT):
        lens = np.ascontiguousarray(lens, dtype=np.int32)
        batch = lens.size
        q = np.ascontiguousarray(q, dtype=np.float32)
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        E = self.n_heads * self.head_dim
        max_len = q.size // (batch * E)
        out = np.empty((batch, max_len, E), dtype=np.float32)
        check(self.lib.ligguf_cuda_bert_attn(self._h, batch, max_len, lens.ctypes.data, q.ctypes.data, k.ctypes.data,
                                             v.ctypes.data, out.ctypes.data, mode), "ligguf_cuda_bert_attn")
        return out

    def attn_async(self, batch: int, max_len: int, lens, q, k, v, out, mode: int = _lib.MODE_SIMT, stream=None):
        check(self.lib.ligguf_cuda_bert_attn_async(self._h, batch, max_len, _ptr(lens), _ptr(q), _ptr(k), _ptr(v),
                                                   _ptr(out), mode, _stream(stream)), "ligguf_cuda_bert_attn_async")


def synth_fill(dst, n: int, seed: int, stream_id: int, idx0: int = 0, scale: float = 1.0, add: float = 0.0,
               dtype: int = _lib.KV_F32, stream=None):
    """Fills a device buffer with the seeded generator (bit-identical to the host restatement)."""
    lib = _lib.load()
    check(lib.ligguf_cuda_synth_fill(_ptr(dst), dtype, n, seed, stream_id, idx0, scale, add, _stream(stream)),
          "ligguf_cuda_synth_fill")
