"""SARA host logic on CPU ranks (gloo): the shard map, the per-layer all-gather in head order
(uneven split_even shards included) and failure behaviour when a rank never joins.

The per-rank attention here is the CPU restatement of the reference run on that rank's KV-head
slice, so the test checks that sharding + gather reproduce the unsharded attention exactly as
SARA's build_shards/att_partial split it (cpp/ligguf_distrib.cpp:657-679,709-747)."""
import datetime
import multiprocessing as mp
import os
import socket
import sys
import traceback

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        import cases
        from oracle import oracle as orc
        from ligguf_b200 import AttnConfig, shard_of
        from ligguf_b200.sara import SaraAttention
        timeout = datetime.timedelta(seconds=4 if mode == "fail" else 120)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
        H, Hk, D = 32, 8, 64
        cfg = AttnConfig(n_layers=1, n_heads=H, n_kv_heads=Hk, head_dim=D, n_context=160, rope_dim=D, rope_base=1e4)
        s = shard_of(Hk, H, rank, world)
        c = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=160, pos=150, seed=9, scale=0.125,
                              kv_head0=s["kv_head0"], kv_headn=s["kv_headn"])
        port = orc.Checker("port")

        def compute(layer, pos, qq, kk, vv, out):
            o, _, _ = cases.run_decode(port, c)
            out.copy_(torch.from_numpy(o))

        sara = SaraAttention(cfg, rank, world, dist, compute=compute)
        out = torch.empty(H * D)
        if mode == "fail" and rank == world - 1:
            q.put((rank, "left"))  # this rank leaves between steps, never joining the collective
            return
        try:
            sara.decode_layer(0, 150, None, None, None, out)
        except Exception as e:  # the peer never arrived: the collective must fail, not hang
            q.put((rank, f"error: {type(e).__name__}"))
            return
        if rank == 0:
            full = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=160, pos=150, seed=9, scale=0.125)
            ref, _, _ = cases.run_decode(port, full)
            q.put((rank, float(np.abs(out.numpy() - ref).max() / np.abs(ref).max())))
        else:
            q.put((rank, "ok"))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "exception:\n" + traceback.format_exc()))


def _run(world, mode="ok", timeout=180):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        r, v = q.get(timeout=timeout)
        res[r] = v
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_decode_gathers_unsharded_result(world):
    res = _run(world)
    assert isinstance(res[0], float), res
    assert res[0] == 0.0 or res[0] <= 1e-6, res  # shards compute the same heads: the gather is exact
    for r in range(1, world):
        assert res[r] == "ok", res


def test_rank_that_never_joins_fails_the_collective():
    res = _run(2, mode="fail", timeout=120)
    assert res[1] == "left"
    assert str(res[0]).startswith("error"), res
