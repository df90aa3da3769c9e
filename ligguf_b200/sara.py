"""SARA-style KV-head sharding of decode attention over several GPUs (one process per GPU).

The reference's distributed example splits attention by KV head (cpp/ligguf_distrib.cpp:657-679:
split_even over n_kv_heads, q heads follow x nrep); each rank keeps only its heads' slice of the KV
cache (:705-706) and computes its heads' attention (:730-747).  The reference then projects the
partial through its columns of attn_output and star-reduces over TCP (:749-750, :1025-1047); here
every rank all-gathers the per-head attention outputs instead, so each rank holds the full
[n_heads*head_dim] vector that the (unsharded) output projection consumes.

Gather backends:
  "nccl"  torch.distributed all_gather over NVLink (any backend torch supports: gloo on CPU);
  "p2p"   the library's fused path: the decode kernel stores its head outputs straight into every
          peer's buffer through CUDA IPC mappings and raises a flag; a bounded wait kernel collects.
Ranks must issue the same layers in the same order (one collective per layer).
"""
from __future__ import annotations

from dataclasses import replace

from .attn import AttnConfig, shard_of


class SaraAttention:
    def __init__(self, cfg: AttnConfig, rank: int, world: int, dist=None, compute=None, gather: str = "nccl",
                 group=None):
        """`dist` is torch.distributed (or None for world == 1); `compute(layer, pos, q, k, v, out)` runs
        this rank's shard (default: a CudaAttention on the shard); tensors are torch tensors."""
        self.rank, self.world, self.dist, self.group = rank, world, dist, group
        self.full_cfg = cfg
        self.shards = [shard_of(cfg.n_kv_heads, cfg.n_heads, r, world) for r in range(world)]
        self.shard = self.shards[rank]
        self.D = cfg.head_dim
        self.q_max = max(s["q_headn"] for s in self.shards) * self.D
        self.even = all(s["q_headn"] == self.shard["q_headn"] for s in self.shards)
        self.gather = gather
        self.attn = None
        if compute is None:
            from .attn import CudaAttention
            shard_cfg = replace(cfg, kv_head0=self.shard["kv_head0"],
                                kv_headn=self.shard["kv_headn"] if world > 1 else 0)
            self.attn = CudaAttention(shard_cfg)
            compute = self.attn.decode_async
        self.compute = compute
        if gather == "p2p":
            if self.attn is None:
                raise ValueError("the p2p gather needs the CUDA compute path")
            mine = self.attn.gather_ipc_handle()
            handles = [None] * world
            dist.all_gather_object(handles, mine, group=group)
            self.attn.gather_open(rank, handles)

    # slices of the unsharded vectors owned by this rank
    def q_slice(self):
        s = self.shard
        return slice(s["q_head0"] * self.D, (s["q_head0"] + s["q_headn"]) * self.D)

    def kv_slice(self):
        s = self.shard
        return slice(s["kv_head0"] * self.D, (s["kv_head0"] + s["kv_headn"]) * self.D)

    def decode_layer(self, layer: int, pos: int, q, k, v, out_full, local_out=None):
        """q [q_headn*D], k, v [kv_headn*D]: this rank's slices (device or host tensors of the compute
        path); out_full [n_heads*D] receives every rank's heads in head order."""
        import torch
        if self.gather == "p2p":
            self.attn.decode_gather_async(layer, pos, q, k, v)
            self.attn.gather_wait_async(layer, out_full)
            return out_full
        if local_out is None:
            local_out = torch.empty(self.q_max, dtype=out_full.dtype, device=out_full.device)
        n_mine = self.shard["q_headn"] * self.D
        self.compute(layer, pos, q, k, v, local_out[:n_mine])
        if self.world == 1:
            out_full.copy_(local_out[:n_mine])
            return out_full
        if self.even:
            self.dist.all_gather_into_tensor(out_full, local_out[:n_mine], group=self.group)
            return out_full
        # uneven split_even shards: gather padded blocks, then keep each rank's valid prefix
        buf = torch.empty(self.world * self.q_max, dtype=out_full.dtype, device=out_full.device)
        if n_mine < self.q_max:
            local_out[n_mine:].zero_()
        self.dist.all_gather_into_tensor(buf, local_out, group=self.group)
        o = 0
        for r, s in enumerate(self.shards):
            n = s["q_headn"] * self.D
            out_full[o:o + n].copy_(buf[r * self.q_max:r * self.q_max + n])
            o += n
        return out_full

    def close(self):
        if self.attn is not None:
            self.attn.close()
            self.attn = None
