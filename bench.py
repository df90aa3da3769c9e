"""Benchmark of the B200 attention block (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extra]

Workload (every N): qwen3_8b_decode_32k - Qwen3-8B-shaped single-stream decode at context 32768,
36 layers, 32 q / 8 KV heads, head_dim 128, fp32 KV cache, QK norm and RoPE.  A step is one token:
36 per-layer launches of the decode kernel (the real forward's order: layer l+1 starts after layer
l), each streaming that layer's K and V rows [0, 32768] (268 MB) from HBM.  With N > 1 the KV heads
are split over the ranks as SARA does (cpp/ligguf_distrib.cpp:665-679) and every layer's head
outputs are all-gathered over NVLink by the decode kernel's own peer stores (NCCL all-gather is
timed alongside) - strong scaling of one stream.  Inputs are larger than L2 (9.66 GB of KV per
step), so no L2 flush is needed between steps.

At N == 1 the line also carries the other configurations as `extra`: the 4K-context decode, the
causal 2048-token prefill (fp32 SIMT and bf16 tensor cores) and the BERT attention.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = "qwen3_8b_decode_32k"
METRIC = "decode attn tokens/s (ctx 32K, 36 layers, fp32 KV)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extra", action="store_true", help="skip the other configurations at N=1")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--gather", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: all-gather of head outputs by the decode kernel's peer stores (p2p, default) or NCCL")
    ap.add_argument("--case", choices=["decode-layer", "decode-4k-layer", "prefill-layer", "bert-layer", "qkv-layer"],
                    default=None,
                    help="run one small case a few times and exit (the command the ncu summaries use)")
    return ap.parse_args()


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_profile_traffic(kernel: str):
    """dram read+write bytes per launch of `kernel` from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel)
    except Exception:
        return None


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"ligguf_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


# ------------------------------------------------------------------------------ CPU side
def host_cores() -> int:
    """Cores this process may run on (the reference arm and the CPU baseline use all of them,
    whatever OMP_NUM_THREADS a launcher such as torchrun exported)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def bench_config(w, world: int, gather: str) -> dict:
    """The `config` of the JSON line, identical in both arms."""
    return {"workload": WORKLOAD, "layers": w.n_layers, "ctx": w.pos + 1, "kv": "fp32",
            "heads": [w.n_heads, w.n_kv_heads, w.head_dim],
            "parallelism": (f"kv-head shards x{world} + per-layer all-gather of head outputs "
                            f"({'decode-kernel NVLink peer stores' if gather == 'p2p' else 'NCCL'})")
            if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (KV bytes per step >> 126 MB); no flush",
            "step": "one token through all layers"}


def cpu_step_runner(w):
    """The reference's CPU attention (oracle/_ref: its fast/lil_math.cpp built from source with its
    flags, AVX2 dots, `omp parallel for` over the heads as its MULTITHREAD) set up for full decode
    steps of workload `w`: every layer's fp32 cache [0, pos) in host memory (9.66 GB at 32K), the
    step's q, k, v and QK-norm weights.  Falls back to the C restatement when the reference build is
    absent.  Returns (run_one_step, info)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle import oracle as orc
    try:
        chk, kind = orc.Checker("ref"), "reference"
    except FileNotFoundError:
        chk, kind = orc.Checker("port"), "port"
    cores = host_cores()
    threads = chk.set_threads(min(cores, w.n_heads))  # the loop is over the heads: more threads idle
    kv_dim = w.n_kv_heads * w.head_dim
    cfg = orc.Checker.cfg(w.n_heads, w.n_kv_heads, w.head_dim, w.n_context, w.rope_dim, w.eps, int(w.qk_norm),
                          0, 0)
    freq = orc.rope_table(w.rope_dim, w.rope_base)
    layers = []
    for l in range(w.n_layers):
        kc = np.empty((w.n_context, kv_dim), dtype=np.float32)
        vc = np.empty_like(kc)
        orc.kv_synth(kc, 0, kv_dim, kv_dim, 0, l, 1, 0, w.pos, w.seed, w.scale)
        orc.kv_synth(vc, 0, kv_dim, kv_dim, 0, l, 2, 0, w.pos, w.seed, w.scale)
        sid = lambda t: (t << 32) | l  # noqa: E731
        q = orc.synth_f32(w.n_heads * w.head_dim, w.seed, sid(3), 0, w.scale)
        k = orc.synth_f32(kv_dim, w.seed, sid(4), 0, w.scale)
        v = orc.synth_f32(kv_dim, w.seed, sid(5), 0, w.scale)
        qg = orc.synth_f32(w.head_dim, w.seed, sid(6), 0, 0.02, 1.0)
        kg = orc.synth_f32(w.head_dim, w.seed, sid(7), 0, 0.02, 1.0)
        layers.append((kc, vc, q, k, v, qg, kg))

    def step():
        for (kc, vc, q, k, v, qg, kg) in layers:
            chk.decode_layer(cfg, kc, vc, freq, qg, kg, w.pos, q, k, v)

    return step, {"kind": kind, "cores": threads, "cores_available": cores}


def cpu_timed_steps(w, steps: int, warmup: int):
    """`warmup` untimed, then `steps` timed full decode steps (all layers) of the reference's CPU path."""
    step, info = cpu_step_runner(w)
    for _ in range(warmup):
        step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    info.update(value=steps / total, ms_per_step=1e3 * total / steps, steps=steps, warmup=warmup,
                sample=f"{steps} timed full decode steps ({w.n_layers} layers, {w.pos + 1}-position fp32 cache "
                       f"each) after {warmup} untimed; OpenMP over the {w.n_heads} heads (the reference's "
                       f"MULTITHREAD) on {info['cores']} threads of {info['cores_available']} host cores")
    return info


def cpu_baseline(w, target_s: float = 10.0):
    """The CPU baseline beside the GPU line: full decode steps of the reference's CPU path for about
    `target_s` seconds (after one warm-up step)."""
    step, info = cpu_step_runner(w)
    step()
    times = []
    t_end = time.perf_counter() + target_s
    while time.perf_counter() < t_end or not times:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    tok_s = len(times) / total
    info.update(value=tok_s, unit="tokens/s",
                sample=f"{len(times)} full decode steps ({w.n_layers} layers, {w.pos + 1}-position fp32 cache "
                       f"each, {1e3 * total / len(times):.0f} ms per step) after one untimed; OpenMP over the "
                       f"{w.n_heads} heads (the reference's MULTITHREAD) on {info['cores']} threads of "
                       f"{info['cores_available']} host cores",
                gbs=w.kv_bytes_per_token() * tok_s / 1e9)
    return info


def run_reference_arm(args):
    from ligguf_b200.workloads import DECODE_WORKLOADS
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w = DECODE_WORKLOADS[WORKLOAD]
    r = cpu_timed_steps(w, args.steps, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded generator, ~N(0,1)); random-init "
                                                         "QK-norm weights",
            "config": bench_config(w, world, args.gather),
            "cpu_baseline": {"value": r["value"], "unit": "tokens/s", "cores": r["cores"], "kind": r["kind"],
                             "sample": r["sample"]},
            "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------ GPU side
def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    return rank, world, local, pg


def decode_setup(w, rank, world, local):
    import torch
    from ligguf_b200 import AttnConfig, CudaAttention, shard_of, synth_fill
    from ligguf_b200.workloads import (GAMMA_ADD, GAMMA_SCALE, SYNTH_KGAMMA, SYNTH_KNEW, SYNTH_Q, SYNTH_QGAMMA,
                                       SYNTH_VNEW, stream_id)
    s = shard_of(w.n_kv_heads, w.n_heads, rank, world)
    cfg = AttnConfig(n_layers=w.n_layers, n_heads=w.n_heads, n_kv_heads=w.n_kv_heads, head_dim=w.head_dim,
                     n_context=w.n_context, rope_dim=w.rope_dim, rope_base=w.rope_base, rms_epsilon=w.eps,
                     qk_norm=w.qk_norm, kv_type=w.kv_type, device=local,
                     kv_head0=s["kv_head0"], kv_headn=s["kv_headn"] if world > 1 else 0)
    h = CudaAttention(cfg)
    dev = torch.device("cuda", local)
    D = w.head_dim
    qd, kd = s["q_headn"] * D, s["kv_headn"] * D
    q = torch.empty(w.n_layers, qd, device=dev)
    k = torch.empty(w.n_layers, kd, device=dev)
    v = torch.empty(w.n_layers, kd, device=dev)
    gam = torch.empty(2, D, device=dev)
    for l in range(w.n_layers):
        synth_fill(q[l], qd, w.seed, stream_id(SYNTH_Q, l), s["q_head0"] * D, w.scale)
        synth_fill(k[l], kd, w.seed, stream_id(SYNTH_KNEW, l), s["kv_head0"] * D, w.scale)
        synth_fill(v[l], kd, w.seed, stream_id(SYNTH_VNEW, l), s["kv_head0"] * D, w.scale)
        if w.qk_norm:
            synth_fill(gam[0], D, w.seed, stream_id(SYNTH_QGAMMA, l), 0, GAMMA_SCALE, GAMMA_ADD)
            synth_fill(gam[1], D, w.seed, stream_id(SYNTH_KGAMMA, l), 0, GAMMA_SCALE, GAMMA_ADD)
            g = gam.cpu().numpy()
            h.set_qk_norm(l, g[0], g[1])
    h.kv_synth(0, w.n_layers, 0, w.pos, w.seed, w.scale)
    torch.cuda.synchronize()
    return h, s, q, k, v


def port_decode_layer(w, layer: int):
    """The C restatement of the reference's decode (oracle, port) of one whole layer of workload `w`,
    unsharded: the checker for the parity line."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle import oracle as orc
    chk = orc.Checker("port")
    chk.set_threads(host_cores())
    kv_dim = w.n_kv_heads * w.head_dim
    kc = np.empty((w.n_context, kv_dim), dtype=np.float32)
    vc = np.empty_like(kc)
    orc.kv_synth(kc, 0, kv_dim, kv_dim, 0, layer, 1, 0, w.pos, w.seed, w.scale)
    orc.kv_synth(vc, 0, kv_dim, kv_dim, 0, layer, 2, 0, w.pos, w.seed, w.scale)
    sid = lambda t: (t << 32) | layer  # noqa: E731
    q = orc.synth_f32(w.n_heads * w.head_dim, w.seed, sid(3), 0, w.scale)
    k = orc.synth_f32(kv_dim, w.seed, sid(4), 0, w.scale)
    v = orc.synth_f32(kv_dim, w.seed, sid(5), 0, w.scale)
    qg = orc.synth_f32(w.head_dim, w.seed, sid(6), 0, 0.02, 1.0) if w.qk_norm else None
    kg = orc.synth_f32(w.head_dim, w.seed, sid(7), 0, 0.02, 1.0) if w.qk_norm else None
    cfg = orc.Checker.cfg(w.n_heads, w.n_kv_heads, w.head_dim, w.n_context, w.rope_dim, w.eps, int(w.qk_norm),
                          0, 0)
    return chk.decode_layer(cfg, kc, vc, orc.rope_table(w.rope_dim, w.rope_base), qg, kg, w.pos, q, k, v)


def decode_parity(args, w, h, q, k, v, out, full, rank, world, pg, layer: int = 0):
    """Untimed, before the timed region: one layer through the same path as the timed steps (at N > 1
    the same sharded decode and the same gather), then rank 0's whole [n_heads*head_dim] output against
    the unsharded decode of the C restatement of the reference.  Every rank takes the same steps."""
    import numpy as np
    import torch
    if world > 1 and args.gather == "p2p":
        h.decode_gather_async(layer, w.pos, q[layer], k[layer], v[layer])
        h.gather_wait_async(layer, full[layer])
    else:
        h.decode_async(layer, w.pos, q[layer], k[layer], v[layer], out[layer])
        if world > 1:
            pg.all_gather_into_tensor(full[layer], out[layer])
    torch.cuda.synchronize()
    h.sync()
    res = None
    if rank == 0:
        got = full[layer].cpu().numpy()
        ref = port_decode_layer(w, layer)
        err = float(np.abs(got.astype(np.float64) - ref).max() / max(float(np.abs(ref).max()), 1e-30))
        res = {"max_rel_err": err, "tol": 1e-4, "ok": bool(err <= 1e-4), "layer": layer,
               "checked": f"the whole {w.n_heads}x{w.head_dim} output of layer {layer} on rank 0"
                          + (f" after the {'peer-store' if args.gather == 'p2p' else 'NCCL'} gather of {world} "
                             f"shards" if world > 1 else ""),
               "against": "oracle port (C restatement of the reference), unsharded"}
    if world > 1:
        pg.barrier()
    return res


def bench_decode(args, w, rank, world, local, pg, peaks):
    import torch
    h, s, q, k, v = decode_setup(w, rank, world, local)
    dev = torch.device("cuda", local)
    D = w.head_dim
    out = torch.empty(w.n_layers, s["q_headn"] * D, device=dev)
    full = torch.empty(w.n_layers, w.n_heads * D, device=dev) if world > 1 else out
    L = w.n_layers
    if world > 1:  # the fused gather: decode epilogues store into every peer's buffer (CUDA IPC)
        mine = h.gather_ipc_handle()
        handles = [None] * world
        pg.all_gather_object(handles, mine)
        h.gather_open(rank, handles)
    parity = decode_parity(args, w, h, q, k, v, out, full, rank, world, pg)

    def step(gather=args.gather):
        for l in range(L):
            if world > 1 and gather == "p2p":
                h.decode_gather_async(l, w.pos, q[l], k[l], v[l])
            else:
                h.decode_async(l, w.pos, q[l], k[l], v[l], out[l])
            if world > 1:
                if gather == "p2p":
                    h.gather_wait_async(l, full[l])
                else:
                    pg.all_gather_into_tensor(full[l], out[l])

    def timed(n, gather):
        # One step (36 layers, decode plus gather at N > 1) captured in a CUDA graph and replayed: the
        # kernels carry no per-call host state (the gather epoch lives on the device), and the host
        # would otherwise have to issue two launches per ~18 us layer at N = 8.  The NCCL gather runs
        # as a host loop.
        run = lambda: step(gather=gather)  # noqa: E731
        graph = None
        if world == 1 or gather == "p2p":
            step(gather=gather)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step(gather=gather)
            run = graph.replay
        for _ in range(args.warmup):
            run()
        torch.cuda.synchronize()
        h.sync()
        if world > 1:
            pg.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(n):
            run()
        t1.record()
        torch.cuda.synchronize()
        if world > 1:
            pg.barrier()
            torch.cuda.synchronize()
        h.sync()
        del graph
        ms = t0.elapsed_time(t1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t.item())
        return ms / n

    clk = ClockSampler(local)
    clk.start()
    time.sleep(0.3)
    ms_per_step = timed(args.steps, args.gather)
    clocks = clk.stop()
    tok_s = 1e3 / ms_per_step
    # Average decode-kernel launch duration: the CUDA-event time of the timed region over the decode
    # launches in it (no events between launches: they would serialise the programmatic launches
    # that let consecutive layers overlap).  Gaps between launches count against the kernel.
    kern_avg_ms = ms_per_step / L
    bytes_launch = 2 * (w.pos + 1) * s["kv_headn"] * D * 4 + (s["q_headn"] * 2 + s["kv_headn"] * 2) * D * 4
    achieved = bytes_launch / (kern_avg_ms * 1e-3) / 1e9
    other = None
    if world > 1:  # the other gather, for comparison
        alt = "nccl" if args.gather == "p2p" else "p2p"
        other = {"gather": alt, "tokens_s": 1e3 / timed(max(3, args.steps // 2), alt)}

    sara = bench_sara_layer(args, w, h, s, q, k, v, rank, world, local, pg)

    # end to end through the public API (pinned host buffers, copies inside the timed region)
    e2e = bench_decode_e2e(args, w, h, s, q, k, v, world, local, pg)
    h.close()
    traffic = load_profile_traffic("decode_kernel")
    per_layer = 2 if (world > 1 and args.gather == "p2p") else 1
    return {
        "value": tok_s, "ms_per_step": ms_per_step, "clocks": clocks,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                     "kernel": "decode_kernel<float,128,4>", "kernel_avg_us": kern_avg_ms * 1e3,
                     "algorithmic_bytes_per_launch": bytes_launch,
                     "peak_source": f"{peaks['source']} hbm_gbs (copy)"},
        "hbm_gbs_step": w.kv_bytes_per_token() * tok_s / 1e9,
        "e2e": e2e, "gpu_launches": args.steps * L * per_layer, "other_gather": other, "parity": parity,
        "sara_layer": sara,
    }


def bench_sara_layer(args, w, h, s, q, k, v, rank, world, local, pg):
    """The SARA attention step with its output projection (cpp/ligguf_distrib.cpp:709-750,1025-1047):
    per layer, the rank's shard decodes (no gather), projects its heads' output through its columns of
    a Q8_0 attn_output (synthetic, 4096 x 4096) and the partial rows are reduced over NVLink into
    every rank's residual.  36 layers in a CUDA graph; the same timing rules as the headline."""
    import numpy as np
    import torch
    from ligguf_b200.qmat import NvlReduce, QuantMatrix, synthetic_rows
    D, L = w.head_dim, w.n_layers
    n_embed = w.n_heads * D
    dev = torch.device("cuda", local)
    col0, ncols = s["q_head0"] * D, s["q_headn"] * D
    rows = synthetic_rows(8, n_embed, n_embed, seed=1234)
    n_distinct = 6  # distinct attn_output matrices used in turn (the whole set exceeds L2 at N = 1)
    mats = [QuantMatrix(8, n_embed, synthetic_rows(8, n_embed, n_embed, seed=1234 + i), local, cols=(col0, ncols))
            for i in range(n_distinct)]
    del rows
    red = NvlReduce(n_embed, world, rank, local)
    if world > 1:
        handles = [None] * world
        pg.all_gather_object(handles, red.ipc_handle())
    else:
        handles = [red.ipc_handle()]
    red.open(handles)
    xb = torch.empty(L, ncols, device=dev)
    x = torch.zeros(n_embed, device=dev)

    def step():
        for l in range(L):
            h.decode_async(l, w.pos, q[l], k[l], v[l], xb[l])
            red.project_async(mats[l % n_distinct], xb[l])
            red.wait_async(x_inout=x)
    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        pg.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(3, args.steps // 2)
    t0.record()
    for _ in range(n):
        g.replay()
    t1.record()
    torch.cuda.synchronize()
    red.status()
    ms = t0.elapsed_time(t1) / n
    if world > 1:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
        pg.barrier()
    del g
    red.close()
    for m in mats:
        m.close()
    return {"tokens_s": 1e3 / ms, "ms_per_step": ms, "us_per_layer": ms * 1e3 / L,
            "note": "per layer: sharded decode + Q8_0 attn_output column-slice projection with its partial rows "
                    "stored into every rank's buffer over NVLink + reduce wait adding the rank-ordered sum to the "
                    f"residual; CUDA-graph replay, {n} steps, max over ranks"}


def bench_decode_e2e(args, w, h, s, q, k, v, world, local, pg):
    import torch
    D = w.head_dim
    L = w.n_layers
    qh = q.cpu().pin_memory()
    kh = k.cpu().pin_memory()
    vh = v.cpu().pin_memory()
    lib = h.lib
    steps = max(3, args.steps // 3)
    if world == 1:
        outh = torch.empty(L, s["q_headn"] * D).pin_memory()
        # Host pointers of each layer's rows, taken once: the engine passes its own buffers' pointers,
        # so the timed loop holds only the C-ABI calls.
        fn, hd = lib.ligguf_cuda_attn_decode, h.handle
        rows = [(l, qh[l].data_ptr(), kh[l].data_ptr(), vh[l].data_ptr(), outh[l].data_ptr()) for l in range(L)]

        def step():
            for l, pq, pk, pv, po in rows:
                rc = fn(hd, l, w.pos, pq, pk, pv, po)
                if rc:
                    raise RuntimeError(f"decode failed {rc}")
        h2d = L * (qh.shape[1] + 2 * kh.shape[1]) * 4
        d2h = L * outh.shape[1] * 4
    else:
        dev = torch.device("cuda", local)
        qd, kd, od = torch.empty_like(q[0]), torch.empty_like(k[0]), torch.empty_like(q[0])
        vd = torch.empty_like(v[0])
        full = torch.empty(w.n_heads * D, device=dev)
        outh = torch.empty(L, w.n_heads * D).pin_memory()

        def step():
            for l in range(L):
                qd.copy_(qh[l], non_blocking=True)
                kd.copy_(kh[l], non_blocking=True)
                vd.copy_(vh[l], non_blocking=True)
                if args.gather == "p2p":
                    h.decode_gather_async(l, w.pos, qd, kd, vd)
                    h.gather_wait_async(l, full)
                else:
                    h.decode_async(l, w.pos, qd, kd, vd, od)
                    pg.all_gather_into_tensor(full, od)
                outh[l].copy_(full, non_blocking=True)
            torch.cuda.current_stream().synchronize()
        h2d = L * (qh.shape[1] + 2 * kh.shape[1]) * 4
        d2h = L * w.n_heads * D * 4
    for _ in range(2):
        step()
    if world > 1:
        pg.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    el = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([el], device=torch.device("cuda", local))
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        el = float(t.item())
    return {"value": steps / el, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "api": "ligguf_cuda_attn_decode (host pointers)" if world == 1 else
            (f"ligguf_cuda_attn_decode_gather_async + gather_wait_async (NVLink peer stores), pinned host copies"
             if args.gather == "p2p" else "ligguf_cuda_attn_decode_async + NCCL all-gather, pinned host copies")}


# ------------------------------------------------------------------------------ other configurations
def _time_ms(fn, iters, warm=3):
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def extra_decode_graph(peaks, w):
    """A decode workload that fits L2 poorly or not at all: one token step (a launch per layer)
    captured in a CUDA graph and replayed.  The replays run back to back, so a layer's cache rows may
    still be in L2 from the previous replay only when the whole step's cache fits L2 (the 4K step
    is 1.2 GB, the TinyLlama step 23 MB: that one is reported with an L2 flush between replays)."""
    import torch
    h, s, q, k, v = decode_setup(w, 0, 1, torch.cuda.current_device())
    out = torch.empty(w.n_layers, w.n_heads * w.head_dim, device=q.device)
    step_bytes = w.kv_bytes_per_token()
    flush = None
    if step_bytes < 512 << 20:  # fits (or nearly fits) the 126 MB L2: flush it between replays
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=q.device)

    def step():
        for l in range(w.n_layers):
            h.decode_async(l, w.pos, q[l], k[l], v[l], out[l])
    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    if flush is None:
        ms = _time_ms(g.replay, 50)
    else:  # time each replay alone, after writing a buffer twice the L2 size
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(50)]
        for _ in range(3):
            flush.zero_()
            g.replay()
        for a, b in ev:
            flush.zero_()
            a.record()
            g.replay()
            b.record()
        torch.cuda.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    h.sync()
    del g
    h.close()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    return {"tokens_s": 1e3 / ms, "ms_per_token": ms, "hbm_gbs": gbs, "frac_of_hbm": gbs / peaks["hbm_gbs"],
            "layers": w.n_layers, "ctx": w.pos + 1,
            "note": "CUDA-graph replay of the per-layer launches; GB/s counts algorithmic K+V bytes"
                    + ("; L2 flushed (256 MB write) before each timed replay" if flush is not None else
                       "; inputs larger than L2, replays back to back")}


# FP32 FMA peak of one B200 (the SIMT paths' roofline): 148 SMs x 128 FP32 lanes x 2 FLOP per FMA x
# the 1965 MHz maximum SM clock; nominal (MEASURED_PEAKS.json holds no FP32 figure).
FP32_FMA_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def extra_prefill(peaks, mode):
    import torch
    from ligguf_b200 import AttnConfig, CudaAttention, synth_fill
    from ligguf_b200.workloads import QWEN3_PREFILL as w
    from ligguf_b200.workloads import SYNTH_KNEW, SYNTH_Q, SYNTH_VNEW, stream_id
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = AttnConfig(n_layers=w.n_layers, n_heads=w.n_heads, n_kv_heads=w.n_kv_heads, head_dim=w.head_dim,
                     n_context=w.n_context, rope_dim=w.rope_dim, rope_base=w.rope_base, rms_epsilon=w.eps,
                     qk_norm=w.qk_norm, device=dev.index)
    h = CudaAttention(cfg)
    import numpy as np
    g = np.ones(w.head_dim, dtype=np.float32)
    for l in range(w.n_layers):
        h.set_qk_norm(l, g, g)
    n, D = w.n_tokens, w.head_dim
    q = torch.empty(n, w.n_heads * D, device=dev)
    k = torch.empty(n, w.n_kv_heads * D, device=dev)
    v = torch.empty_like(k)
    out = torch.empty_like(q)
    synth_fill(q, q.numel(), w.seed, stream_id(SYNTH_Q, 0), 0, w.scale)
    synth_fill(k, k.numel(), w.seed, stream_id(SYNTH_KNEW, 0), 0, w.scale)
    synth_fill(v, v.numel(), w.seed, stream_id(SYNTH_VNEW, 0), 0, w.scale)

    def run():
        for l in range(w.n_layers):
            h.prefill_async(l, w.pos0, n, q, k, v, out, mode)
    ms = _time_ms(run, 3 if mode == 0 else 10, warm=1)
    h.sync()
    h.close()
    flops = w.causal_flops_per_layer() * w.n_layers
    tf = flops / (ms * 1e-3) / 1e12
    peak = peaks["bf16_tflops"] if mode == 1 else None
    r = {"ms_36_layers": ms, "tflops": tf, "causal_flops": flops}
    if mode == 0:
        r["frac_of_fp32_fma_peak"] = tf / FP32_FMA_PEAK_TFLOPS
        r["fp32_fma_peak_tflops"] = FP32_FMA_PEAK_TFLOPS
    if peak:
        r["frac_of_bf16_peak"] = tf / peak
    return r


def extra_bert(peaks, mode):
    import torch
    from ligguf_b200 import CudaBertAttention, synth_fill
    from ligguf_b200.workloads import BERT_BASE as w
    from ligguf_b200.workloads import SYNTH_K, SYNTH_Q, SYNTH_V, stream_id
    dev = torch.device("cuda", torch.cuda.current_device())
    E = w.n_heads * w.head_dim
    n = w.batch * w.max_len * E
    q, k, v, out = (torch.empty(n, device=dev) for _ in range(4))
    for t, x in ((SYNTH_Q, q), (SYNTH_K, k), (SYNTH_V, v)):
        synth_fill(x, n, w.seed, stream_id(t, 0), 0, w.scale)
    lens = torch.tensor(w.lens(), dtype=torch.int32, device=dev)
    h = CudaBertAttention(w.n_heads, w.head_dim, w.batch, w.max_len, dev.index)

    def run():
        for _ in range(w.n_layers):
            h.attn_async(w.batch, w.max_len, lens, q, k, v, out, mode)
    ms = _time_ms(run, 5, warm=1)
    h.close()
    flops = w.flops_per_layer() * w.n_layers
    tf = flops / (ms * 1e-3) / 1e12
    r = {"ms_12_layers": ms, "tflops": tf, "flops": flops}
    if mode == 0:
        r["frac_of_fp32_fma_peak"] = tf / FP32_FMA_PEAK_TFLOPS
        r["fp32_fma_peak_tflops"] = FP32_FMA_PEAK_TFLOPS
    if mode == 1:
        r["frac_of_bf16_peak"] = tf / peaks["bf16_tflops"]
    # The layer's roofline is the slower of its arithmetic at peak and its fp32 interface in HBM (the
    # valid rows of q, k and v read, the output written: the reference's types, so no kernel of
    # either path can move fewer bytes).
    io_bytes = 4 * sum(w.lens()) * E * 4
    t_io = io_bytes / (peaks["hbm_gbs"] * 1e3)  # us
    t_math = w.flops_per_layer() / ((FP32_FMA_PEAK_TFLOPS if mode == 0 else peaks["bf16_tflops"]) * 1e6)
    us_layer = ms * 1e3 / w.n_layers
    r["layer_roofline"] = {"bound": "hbm" if t_io > t_math else ("fma" if mode == 0 else "tensor"),
                           "io_bytes": io_bytes, "us_hbm": t_io, "us_math": t_math, "us_measured": us_layer,
                           "frac": max(t_io, t_math) / us_layer}
    return r


def extra_qkv(peaks, types, n_distinct: int = 12, n_tok: int = 1):
    """The Qwen3-8B QKV projection (x [4096] -> q [4096], k [1024], v [1024];
    fast/ligguf_fast_qk.cpp:39-40) with weights of the given GGUF types.  n_tok = 1: one decode token,
    36 launches per step (one per layer) over `n_distinct` synthetic weight sets used in turn (more
    bytes than L2 holds), CUDA-graph replay.  n_tok > 1: the batched prompt form, one call per layer
    for n_tok tokens (the weights stream once per group of up to 8 tokens).  GB/s counts the weight
    bytes of one pass per layer; the batched form also reports the int8 MAC rate."""
    import numpy as np
    import torch
    from ligguf_b200.qmat import QT, QuantMatrix, matmul3_async, matmul3_batch_async, row_bytes, synthetic_rows
    n, dims, L = 4096, (4096, 1024, 1024), 36
    dev = torch.device("cuda", torch.cuda.current_device())
    layers = [[QuantMatrix(QT[t], n, synthetic_rows(QT[t], n, d, seed=97 * i + j), dev.index)
               for j, (t, d) in enumerate(zip(types, dims))] for i in range(n_distinct)]
    nx = L if n_tok == 1 else 1  # the prompt form reuses one [n_tok][n] activation for every layer
    x = torch.from_numpy(np.random.default_rng(1).standard_normal((nx, n_tok, n)).astype(np.float32)).to(dev)
    outs = [torch.empty(nx, n_tok, d, device=dev) for d in dims]

    def step():
        for l in range(L):
            w = layers[l % n_distinct]
            if n_tok == 1:
                matmul3_async(w[0], w[1], w[2], x[l, 0], outs[0][l, 0], outs[1][l, 0], outs[2][l, 0])
            else:
                matmul3_batch_async(w[0], w[1], w[2], x[0], n_tok, outs[0][0], outs[1][0], outs[2][0])
    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    ms = _time_ms(g.replay, 30 if n_tok == 1 else 3)
    del g
    for ws in layers:
        for m in ws:
            m.close()
    wbytes = sum(row_bytes(QT[t], n) * d for t, d in zip(types, dims))
    r = {"types": list(types), "tokens": n_tok, "us_per_layer": ms * 1e3 / L, "weight_bytes_per_layer": wbytes}
    if n_tok == 1:
        gbs = wbytes * L / (ms * 1e-3) / 1e9
        r.update(hbm_gbs=gbs, frac_of_hbm=gbs / peaks["hbm_gbs"])
    else:
        r.update(tokens_s=n_tok * L / (ms * 1e-3) / L, int8_tmacs=n_tok * n * sum(dims) * L / (ms * 1e-3) / 1e12)
    r["note"] = (f"36 per-layer launches over {n_distinct} distinct synthetic weight sets "
                 f"({n_distinct * wbytes / 1e6:.0f} MB, more than L2), CUDA-graph replay; x quantized on the device "
                 f"as the reference does")
    return r


def run_extras(peaks):
    extra = {}
    from ligguf_b200.workloads import QWEN3_DECODE_4K, TINYLLAMA_DECODE
    jobs = [("tinyllama_decode_512", lambda: extra_decode_graph(peaks, TINYLLAMA_DECODE)),
            ("qwen3_8b_decode_4k", lambda: extra_decode_graph(peaks, QWEN3_DECODE_4K)),
            ("qwen3_8b_prefill_2048_simt_fp32", lambda: extra_prefill(peaks, 0)),
            ("qwen3_8b_prefill_2048_tc_bf16", lambda: extra_prefill(peaks, 1)),
            ("bert_base_attn_simt_fp32", lambda: extra_bert(peaks, 0)),
            ("bert_base_attn_tc_bf16", lambda: extra_bert(peaks, 1)),
            ("qwen3_8b_qkv_q8_0", lambda: extra_qkv(peaks, ("Q8_0", "Q8_0", "Q8_0"))),
            ("qwen3_8b_qkv_q4_k_m", lambda: extra_qkv(peaks, ("Q4_K", "Q4_K", "Q6_K"))),
            ("qwen3_8b_qkv_q4_k_m_prompt_2048", lambda: extra_qkv(peaks, ("Q4_K", "Q4_K", "Q6_K"), n_tok=2048))]
    for name, fn in jobs:
        try:
            extra[name] = fn()
        except Exception as e:  # the headline line must still print
            extra[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return extra


def run_case(case: str, reps: int = 3):
    """Small single-GPU cases for profiling: the kernel of one layer of the named configuration,
    `reps` launches, a few hundred MB on the device."""
    import numpy as np
    import torch
    from ligguf_b200 import AttnConfig, CudaAttention, CudaBertAttention, synth_fill
    from ligguf_b200.workloads import BERT_BASE, QWEN3_DECODE_4K, QWEN3_DECODE_32K, QWEN3_PREFILL
    dev = torch.device("cuda", 0)
    g = np.ones(128, dtype=np.float32)
    if case == "decode-layer":  # qwen3_8b_decode_32k shapes, 2 layers of cache (537 MB), layer 0
        w = QWEN3_DECODE_32K
        h = CudaAttention(AttnConfig(n_layers=2, n_heads=w.n_heads, n_kv_heads=w.n_kv_heads, head_dim=w.head_dim,
                                     n_context=w.n_context, rope_dim=w.rope_dim, rope_base=w.rope_base,
                                     rms_epsilon=w.eps, qk_norm=True))
        h.set_qk_norm(0, g, g)
        h.kv_synth(0, 1, 0, w.pos, w.seed, w.scale)
        q, k, v = torch.empty(w.q_dim, device=dev), torch.empty(w.kv_dim, device=dev), torch.empty(w.kv_dim, device=dev)
        out = torch.empty(w.q_dim, device=dev)
        for t, x in ((3, q), (4, k), (5, v)):
            synth_fill(x, x.numel(), w.seed, t << 32, 0, w.scale)
        for _ in range(reps):
            h.decode_async(0, w.pos, q, k, v, out)
    elif case == "decode-4k-layer":
        # qwen3_8b_decode_4k shapes, 8 layers of cache (268 MB, more than L2), two passes over the
        # layers: a launch of the second pass reads a layer that 7 others have since evicted.
        w = QWEN3_DECODE_4K
        L = 8
        h = CudaAttention(AttnConfig(n_layers=L, n_heads=w.n_heads, n_kv_heads=w.n_kv_heads, head_dim=w.head_dim,
                                     n_context=w.n_context, rope_dim=w.rope_dim, rope_base=w.rope_base,
                                     rms_epsilon=w.eps, qk_norm=True))
        for l in range(L):
            h.set_qk_norm(l, g, g)
        h.kv_synth(0, L, 0, w.pos, w.seed, w.scale)
        q, k, v = torch.empty(w.q_dim, device=dev), torch.empty(w.kv_dim, device=dev), torch.empty(w.kv_dim, device=dev)
        out = torch.empty(w.q_dim, device=dev)
        for t, x in ((3, q), (4, k), (5, v)):
            synth_fill(x, x.numel(), w.seed, t << 32, 0, w.scale)
        for _ in range(2):
            for l in range(L):
                h.decode_async(l, w.pos, q, k, v, out)
    elif case == "qkv-layer":
        # the Qwen3-8B Q8_0 QKV projection of one decode token over 12 distinct weight sets (321 MB,
        # more than L2), two passes: a launch of the second pass reads weights that 11 others have
        # since evicted
        from ligguf_b200.qmat import QT, QuantMatrix, matmul3_async, synthetic_rows
        n, dims = 4096, (4096, 1024, 1024)
        mats = [[QuantMatrix(QT["Q8_0"], n, synthetic_rows(QT["Q8_0"], n, d, seed=97 * i + j), 0)
                 for j, d in enumerate(dims)] for i in range(12)]
        x = torch.randn(n, device=dev)
        outs = [torch.empty(d, device=dev) for d in dims]
        for _ in range(2):
            for m in mats:
                matmul3_async(m[0], m[1], m[2], x, *outs)
        torch.cuda.synchronize()
        for m in mats:
            for w_ in m:
                w_.close()
        print(f"case {case}: ok")
        return 0
    elif case == "prefill-layer":  # qwen3_8b_prefill_2048, one layer, tensor-core path
        w = QWEN3_PREFILL
        h = CudaAttention(AttnConfig(n_layers=1, n_heads=w.n_heads, n_kv_heads=w.n_kv_heads, head_dim=w.head_dim,
                                     n_context=w.n_context, rope_dim=w.rope_dim, rope_base=w.rope_base,
                                     rms_epsilon=w.eps, qk_norm=True))
        h.set_qk_norm(0, g, g)
        n = w.n_tokens
        q = torch.empty(n, w.n_heads * w.head_dim, device=dev)
        k = torch.empty(n, w.n_kv_heads * w.head_dim, device=dev)
        v, out = torch.empty_like(k), torch.empty_like(q)
        for t, x in ((3, q), (4, k), (5, v)):
            synth_fill(x, x.numel(), w.seed, t << 32, 0, w.scale)
        for _ in range(reps):
            h.prefill_async(0, 0, n, q, k, v, out, 1)
    else:  # bert_base_attn, one layer, tensor-core path
        w = BERT_BASE
        n = w.batch * w.max_len * w.n_heads * w.head_dim
        q, k, v, out = (torch.empty(n, device=dev) for _ in range(4))
        for t, x in ((3, q), (1, k), (2, v)):
            synth_fill(x, n, w.seed, t << 32, 0, w.scale)
        lens = torch.tensor(w.lens(), dtype=torch.int32, device=dev)
        h = CudaBertAttention(w.n_heads, w.head_dim, w.batch, w.max_len, 0)
        for _ in range(reps):
            h.attn_async(w.batch, w.max_len, lens, q, k, v, out, 1)
    torch.cuda.synchronize()
    h.close()
    print(f"case {case}: ok")
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.case:
        return run_case(args.case)
    import torch
    from ligguf_b200 import load
    from ligguf_b200.workloads import DECODE_WORKLOADS
    load()
    rank, world, local, pg = setup_dist(args)
    peaks = load_peaks()
    w = DECODE_WORKLOADS[WORKLOAD]
    res = bench_decode(args, w, rank, world, local, pg, peaks)
    extra = {}
    cb = None
    if world == 1 and rank == 0:
        if not args.no_extra:
            extra = run_extras(peaks)
        if not args.no_cpu:
            cb = cpu_baseline(w)
    if rank == 0:
        line = {
            "metric": METRIC, "value": res["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded generator, ~N(0,1)); random-init QK-norm weights",
            "config": bench_config(w, world, args.gather),
            "hbm_gbs": res["hbm_gbs_step"],
            "roofline": res["roofline"], "clocks": res["clocks"], "e2e": res["e2e"],
            "gpu_launches": res["gpu_launches"], "parity": res["parity"],
            "timing": ("CUDA events around K replays of a CUDA graph of one step (36 decode launches"
                       + (", 36 gather waits" if world > 1 else "") + "), max over ranks"),
        }
        if res.get("other_gather"):
            line["other_gather"] = res["other_gather"]
        if res.get("sara_layer"):
            line["sara_layer"] = res["sara_layer"]
        if cb is not None:
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        if extra:
            line["extra"] = extra
        print(json.dumps(line), flush=True)
    if world > 1:
        pg.barrier()
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
