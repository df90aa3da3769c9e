"""The benchmark configurations and their seeded synthetic inputs.

Five configurations of the attention block (no GGUF models are available, so every tensor comes from
the library's seeded generator; values approximate N(0, scale^2), see ligguf_cuda_synth_fill):

  tinyllama_decode_512   22 layers, 32 q / 4 kv heads, head_dim 64, RoPE theta 1e4, cache 0..511,
                         query at 512, inputs ~ N(0,1)/8
  qwen3_8b_decode_4k     36 layers, 32 / 8 heads, head_dim 128, QK RMSNorm (eps 1e-6,
                         gamma 1+N(0,0.02)), theta 1e6, cache 0..4095, query at 4096, N(0,1)
  qwen3_8b_prefill_2048  same layout, causal prefill of 2048 tokens from position 0
  qwen3_8b_decode_32k    as the 4k decode with cache 0..32767, query at 32768; KV heads sharded
                         over 1/2/4/8 GPUs
  bert_base_attn         12 layers, 12 heads, head_dim 64, no RoPE, 64 sequences of length
                         U[16,512] padded to 512, N(0,1)/8

Tensor ids / stream numbering (shared with the host restatement in oracle/attn_oracle.c):
  stream = (tensor_id << 32) | layer; element index = position * full_width + column, where
  full_width is the unsharded width (n_heads*head_dim for q, n_kv_heads*head_dim for k, v).
"""
from __future__ import annotations

from dataclasses import dataclass, field

from ._lib import (KV_F32, SYNTH_K, SYNTH_KGAMMA, SYNTH_KNEW, SYNTH_Q, SYNTH_QGAMMA, SYNTH_V,
                   SYNTH_VNEW)

GAMMA_SCALE, GAMMA_ADD = 0.02, 1.0


def stream_id(tensor: int, layer: int) -> int:
    return (tensor << 32) | (layer & 0xFFFFFFFF)


@dataclass(frozen=True)
class DecodeWorkload:
    name: str
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    rope_base: float
    qk_norm: bool
    eps: float
    pos: int          # query position; cache rows [0, pos) are pre-filled
    scale: float      # input standard deviation
    kv_type: int = KV_F32
    seed: int = 0x5EED0001

    @property
    def n_context(self) -> int:  # room for the query row, rounded up to 64
        return ((self.pos + 1 + 63) // 64) * 64

    @property
    def rope_dim(self) -> int:
        return self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    def kv_bytes_per_token(self, elem_bytes: int = 4) -> int:
        """Algorithmic HBM bytes of one decode step: K and V rows [0, pos] of every layer."""
        return 2 * (self.pos + 1) * self.kv_dim * elem_bytes * self.n_layers

    def flops_per_token(self) -> int:
        return 4 * self.n_heads * self.head_dim * (self.pos + 1) * self.n_layers


@dataclass(frozen=True)
class PrefillWorkload:
    name: str
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    rope_base: float
    qk_norm: bool
    eps: float
    n_tokens: int
    pos0: int
    scale: float
    kv_type: int = KV_F32
    seed: int = 0x5EED0003

    @property
    def n_context(self) -> int:
        return ((self.pos0 + self.n_tokens + 63) // 64) * 64

    @property
    def rope_dim(self) -> int:
        return self.head_dim

    def causal_flops_per_layer(self) -> int:
        """4*D FLOPs per (query, visible key) pair, causal triangle only."""
        n, p0 = self.n_tokens, self.pos0
        pairs = n * p0 + n * (n + 1) // 2
        return 4 * self.head_dim * pairs * self.n_heads


def _splitmix64(x: int) -> int:
    m = (1 << 64) - 1
    z = (x + 0x9E3779B97F4A7C15) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    return z ^ (z >> 31)


@dataclass(frozen=True)
class BertWorkload:
    name: str
    n_layers: int
    n_heads: int
    head_dim: int
    batch: int
    max_len: int
    min_len: int
    scale: float
    seed: int = 0x5EED0005
    lens_override: tuple = field(default=())

    def lens(self):
        """Per-sequence lengths, uniform in [min_len, max_len], seeded (or the override)."""
        if self.lens_override:
            return list(self.lens_override)
        span = self.max_len - self.min_len + 1
        return [self.min_len + _splitmix64(self.seed ^ (0xBE27 << 20) ^ b) % span for b in range(self.batch)]

    def flops_per_layer(self) -> int:
        """4*D FLOPs per (query, key) pair of valid tokens, all heads."""
        return sum(4 * n * n * self.head_dim * self.n_heads for n in self.lens())


TINYLLAMA_DECODE = DecodeWorkload("tinyllama_decode_512", 22, 32, 4, 64, 1e4, False, 1e-5, 512, 0.125)
QWEN3_DECODE_4K = DecodeWorkload("qwen3_8b_decode_4k", 36, 32, 8, 128, 1e6, True, 1e-6, 4096, 1.0)
QWEN3_DECODE_32K = DecodeWorkload("qwen3_8b_decode_32k", 36, 32, 8, 128, 1e6, True, 1e-6, 32768, 1.0)
QWEN3_PREFILL = PrefillWorkload("qwen3_8b_prefill_2048", 36, 32, 8, 128, 1e6, True, 1e-6, 2048, 0, 1.0)
BERT_BASE = BertWorkload("bert_base_attn", 12, 12, 64, 64, 512, 16, 0.125)

DECODE_WORKLOADS = {w.name: w for w in (TINYLLAMA_DECODE, QWEN3_DECODE_4K, QWEN3_DECODE_32K)}

__all__ = [
    "DecodeWorkload", "PrefillWorkload", "BertWorkload", "stream_id", "TINYLLAMA_DECODE",
    "QWEN3_DECODE_4K", "QWEN3_DECODE_32K", "QWEN3_PREFILL", "BERT_BASE", "DECODE_WORKLOADS", "GAMMA_SCALE",
    "GAMMA_ADD", "SYNTH_K", "SYNTH_V", "SYNTH_Q", "SYNTH_KNEW", "SYNTH_VNEW", "SYNTH_QGAMMA", "SYNTH_KGAMMA",
]
