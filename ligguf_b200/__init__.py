"""B200-native (sm_100a) attention block for LiGGUF's FAST engine.

The compute lives in libligguf_cuda_attn.so (hand-written CUDA, C ABI in include/ligguf_cuda_attn.h);
this package is the Python face of that ABI plus the workload definitions used by the benchmark.
"""
from ._lib import (KV_BF16, KV_F16, KV_F32, MODE_SIMT, MODE_TC, SCALE_DIV, SCALE_MUL, LigGufAttnError,
                   load)
from .attn import AttnConfig, CudaAttention, CudaBertAttention, shard_of, split_even, synth_fill

__all__ = [
    "AttnConfig", "CudaAttention", "CudaBertAttention", "LigGufAttnError", "load", "shard_of", "split_even",
    "synth_fill", "KV_F32", "KV_F16", "KV_BF16", "MODE_SIMT", "MODE_TC", "SCALE_MUL", "SCALE_DIV",
]
