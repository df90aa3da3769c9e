"""SARA KV-head sharding across GPUs (one process per GPU, NCCL), both gather paths:
NCCL all-gather of head outputs, and the fused path where the decode kernel stores its head outputs
into every peer's buffer over NVLink as epoch-tagged words (bounded wait on the reader).

Needs at least 2 GPUs; every rank has its own GPU (kernels that wait on one another never share
one).  Checked against the CPU restatement of the reference (unsharded) at 1e-4 of the output scale.
"""
import datetime
import multiprocessing as mp
import os
import socket
import sys
import traceback

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _ngpu():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# (H, Hk, D, n_ctx, layers, positions): Qwen3-8B heads split 4 + 4; and 12 heads over 3 KV heads,
# split 2 + 1, so the ranks decode different numbers of splits and merge groups into the same slots.
SHAPES = {"even": (32, 8, 128, 2200, 3, (2049, 2050)), "uneven": (12, 3, 128, 6500, 2, (6400, 6401))}


def _worker(rank, world, port, gather, q, shape="even"):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        import cases
        from oracle import oracle as orc
        from ligguf_b200 import AttnConfig
        from ligguf_b200.sara import SaraAttention
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        H, Hk, D, n_ctx, L, positions = SHAPES[shape]
        cfg = AttnConfig(n_layers=L, n_heads=H, n_kv_heads=Hk, head_dim=D, n_context=n_ctx, rope_dim=D,
                         rope_base=1e6, rms_epsilon=1e-6, qk_norm=True, device=rank)
        sara = SaraAttention(cfg, rank, world, dist, gather=gather)
        s = sara.shard
        dev = torch.device("cuda", rank)
        errs = []
        for step, pos in enumerate(positions):
            for layer in range(L):
                c = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=n_ctx, theta=1e6, qk_norm=1, pos=pos, seed=40 + layer,
                                      layer=layer, kv_head0=s["kv_head0"], kv_headn=s["kv_headn"])
                sara.attn.set_qk_norm(layer, c["qg"], c["kg"])
                if step == 0:
                    sara.attn.kv_synth(layer, 1, 0, pos, c["seed"], 1.0)
                qd = torch.from_numpy(c["q"]).to(dev)
                kd = torch.from_numpy(c["k"]).to(dev)
                vd = torch.from_numpy(c["v"]).to(dev)
                out = torch.empty(H * D, device=dev)
                sara.decode_layer(layer, pos, qd, kd, vd, out)
                torch.cuda.synchronize()
                if rank == 0:
                    full = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=n_ctx, theta=1e6, qk_norm=1, pos=pos,
                                             seed=40 + layer, layer=layer)
                    if step == 1:  # the cache now also holds the row step 0 wrote
                        p0 = positions[0]
                        prev = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=n_ctx, theta=1e6, qk_norm=1, pos=p0,
                                                 seed=40 + layer, layer=layer)
                        _, krow, vrow = cases.run_decode(orc.Checker("port"), prev)
                        full["kc"][p0], full["vc"][p0] = krow, vrow
                    ref, _, _ = cases.run_decode(orc.Checker("port"), full)
                    errs.append(float(np.abs(out.cpu().numpy() - ref).max() / np.abs(ref).max()))
        sara.attn.sync()
        dist.barrier()
        sara.close()
        dist.destroy_process_group()
        q.put((rank, max(errs) if errs else "ok"))
    except Exception:
        q.put((rank, "exception:\n" + traceback.format_exc()))


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("gather,shape", [("nccl", "even"), ("p2p", "even"), ("nccl", "uneven"), ("p2p", "uneven")])
def test_sara_two_gpus(gather, shape):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    ps = [ctx.Process(target=_worker, args=(r, world, port, gather, q, shape)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        r, v = q.get(timeout=300)
        res[r] = v
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert isinstance(res[0], float), res
    assert res[0] <= 1e-4, res
    assert res[1] == "ok", res


def _layer_worker(rank, world, port, q):
    """One SARA attention layer: the rank's KV-head shard decodes (no gather), projects its heads'
    output through its columns of attn_output, and the partial rows are reduced over NVLink into every
    rank's residual (cpp/ligguf_distrib.cpp:709-750,1025-1047)."""
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        import cases
        from oracle import oracle as orc
        from ligguf_b200 import AttnConfig, CudaAttention, shard_of
        from ligguf_b200.qmat import NvlReduce, QuantMatrix, synthetic_rows
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        H, Hk, D, n_ctx, pos = 32, 8, 128, 1100, 1000
        n_embed = H * D
        s = shard_of(Hk, H, rank, world)
        c = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=n_ctx, theta=1e6, qk_norm=1, pos=pos, seed=71, layer=0,
                              kv_head0=s["kv_head0"], kv_headn=s["kv_headn"])
        h = CudaAttention(AttnConfig(n_layers=1, n_heads=H, n_kv_heads=Hk, head_dim=D, n_context=n_ctx, rope_dim=D,
                                     rope_base=1e6, rms_epsilon=1e-6, qk_norm=True, device=rank,
                                     kv_head0=s["kv_head0"], kv_headn=s["kv_headn"]))
        h.set_qk_norm(0, c["qg"], c["kg"])
        h.kv_synth(0, 1, 0, pos, c["seed"], 1.0)
        rows = synthetic_rows(8, n_embed, n_embed, seed=9)   # attn_output, Q8_0, the same on every rank
        col0, ncols = s["q_head0"] * D, s["q_headn"] * D
        w = QuantMatrix(8, n_embed, rows, device=rank, cols=(col0, ncols))
        red = NvlReduce(n_embed, world, rank, device=rank)
        handles = [None] * world
        dist.all_gather_object(handles, red.ipc_handle())
        red.open(handles)
        dev = torch.device("cuda", rank)
        qd, kd, vd = (torch.from_numpy(c[x]).to(dev) for x in ("q", "k", "v"))
        xb = torch.empty(ncols, device=dev)
        res0 = np.random.default_rng(17).standard_normal(n_embed).astype(np.float32)
        x = torch.from_numpy(res0).to(dev)
        for _ in range(2):  # two layers' worth: the epochs advance
            h.decode_async(0, pos, qd, kd, vd, xb)
            red.project_async(w, xb)
            red.wait_async(x_inout=x)
        torch.cuda.synchronize()
        red.status()
        got = x.cpu().numpy()
        dist.barrier()
        result = "ok"
        if rank == 0:
            full = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=n_ctx, theta=1e6, qk_norm=1, pos=pos, seed=71, layer=0)
            att, _, _ = cases.run_decode(orc.Checker("port"), full)
            total = None
            for r in range(world):  # the master's order: rank 0's partial, then += each worker's
                sr = shard_of(Hk, H, r, world)
                c0, nc = sr["q_head0"] * D, sr["q_headn"] * D
                part = orc.matmul(8, rows[:, c0 // 32 * 34:(c0 + nc) // 32 * 34], nc, att[c0:c0 + nc], "port")
                total = part if total is None else total + part
            ref = res0 + 2 * total
            result = float(np.abs(got - ref).max() / np.abs(ref).max())
        dist.barrier()
        red.close()
        w.close()
        h.close()
        dist.destroy_process_group()
        q.put((rank, result))
    except Exception:
        q.put((rank, "exception:\n" + traceback.format_exc()))


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_sara_layer_projection_reduce_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    ps = [ctx.Process(target=_layer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        r, v = q.get(timeout=300)
        res[r] = v
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert isinstance(res[0], float), res
    assert res[0] <= 1e-4, res
    assert res[1] == "ok", res
