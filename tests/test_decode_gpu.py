"""Decode attention on the GPU (through the C ABI) against the CPU checkers.

Tolerance (from the north star): max |gpu - ref| <= 1e-4 * max |ref| for the fp32 arithmetic paths.
The cache is filled on the device by the library's generator and on the host by the restatement;
the two are bit-identical, which test_kv_synth_matches_host checks first.
"""
import json
import os

import numpy as np
import pytest

import cases
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL = 1e-4
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def make_handle(c, n_layers=None, layer=None, kv_head0=None, kv_headn=None):
    from ligguf_b200 import AttnConfig, CudaAttention
    layer = c["layer"] if layer is None else layer
    n_layers = (layer + 1) if n_layers is None else n_layers
    cfg = AttnConfig(n_layers=n_layers, n_heads=c["H"], n_kv_heads=c["Hk"], head_dim=c["D"], n_context=c["n_ctx"],
                     rope_dim=c["rope_dim"], rope_base=c["theta"], rms_epsilon=c["eps"], qk_norm=bool(c["qk_norm"]),
                     kv_type=c["kv_type"], scale_mode=c["scale_mode"],
                     kv_head0=c["kv_head0"] if kv_head0 is None else kv_head0,
                     kv_headn=(c["kv_headn"] if c["kv_headn"] != c["Hk"] else 0) if kv_headn is None else kv_headn)
    h = CudaAttention(cfg)
    if c["qk_norm"]:
        for l in range(n_layers):
            h.set_qk_norm(l, c["qg"], c["kg"])
    return h


def gpu_decode(c, h=None):
    h = h or make_handle(c)
    if c["qk_norm"]:
        h.set_qk_norm(c["layer"], c["qg"], c["kg"])
    if c["pos"] > 0:
        h.kv_synth(c["layer"], 1, 0, c["pos"], c["seed"], c["scale"])
    out = h.decode(c["layer"], c["pos"], c["q"], c["k"], c["v"])
    k, v = h.kv_download(c["layer"], c["pos"], 1)
    return out, k[0], v[0], h


def test_kv_synth_matches_host(gpu):
    for kv_type in (0, 1, 2):
        c = cases.decode_case(H=8, Hk=2, D=128, n_ctx=80, kv_type=kv_type, pos=77, seed=99, layer=2, scale=0.7)
        h = make_handle(c)
        h.kv_synth(2, 1, 0, 77, 99, 0.7)
        k, v = h.kv_download(2, 0, 77)
        assert np.array_equal(k, c["kc"][:77]) and np.array_equal(v, c["vc"][:77]), kv_type
        h.close()


@pytest.mark.parametrize("key", ["decode_f32_tinyllama_like", "decode_f16_fast_qwen3", "decode_f32_div_gqa4",
                                 "decode_f16_rope_partial"])
def test_decode_vs_reference_golden(gpu, key):
    spec = dict(json.load(open(os.path.join(GOLDEN, "golden.json")))[key])
    pos_list = spec.pop("pos_list")
    gold = np.load(os.path.join(GOLDEN, key + ".npz"))
    for pos in pos_list:
        c = cases.decode_case(pos=pos, **spec)
        out, krow, vrow, h = gpu_decode(c)
        assert cases.rel_err(out, gold[f"out_{pos}"]) <= TOL, (key, pos)
        assert np.array_equal(vrow, gold[f"vrow_{pos}"]), (key, pos)
        kt = spec.get("kv_type", 0)
        ka, kb = orc.to_f32(krow, kt), orc.to_f32(gold[f"krow_{pos}"], kt)
        assert np.abs(ka - kb).max() <= (2.0 ** -10 if kt == 1 else 4e-6) * np.abs(kb).max(), (key, pos)
        h.close()


SHAPES = [(32, 4, 64), (32, 8, 128), (8, 8, 64), (16, 8, 128), (16, 2, 128)]


@pytest.mark.parametrize("kv_type", [0, 1, 2])
@pytest.mark.parametrize("shape", SHAPES)
def test_decode_sweep_vs_port(gpu, kv_type, shape):
    H, Hk, D = shape
    port = orc.Checker("port")
    h = None
    for pos in (0, 1, 31, 32, 33, 127, 511, 1000):
        c = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=1024, theta=1e6, qk_norm=int(D == 128), kv_type=kv_type,
                              pos=pos, seed=1000 + pos, scale=1.0 if D == 128 else 0.125, layer=1)
        h = h or make_handle(c, n_layers=2)
        out, krow, vrow, _ = gpu_decode(c, h)
        ref, kref, vref = cases.run_decode(port, c)
        assert cases.rel_err(out, ref) <= TOL, (shape, kv_type, pos)
        assert np.array_equal(vrow, vref), (shape, kv_type, pos)
    h.close()


def test_decode_scale_div_and_rope_partial(gpu):
    port = orc.Checker("port")
    c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=700, rope_dim=96, theta=5e5, qk_norm=1, scale_mode=1, pos=650,
                          seed=5, scale=1.0)
    out, _, _, h = gpu_decode(c)
    ref, _, _ = cases.run_decode(port, c)
    assert cases.rel_err(out, ref) <= TOL
    h.close()


@pytest.mark.parametrize("name,pos,layer", [("qwen3_8b_decode_4k", 4096, 35), ("qwen3_8b_decode_32k", 32768, 7),
                                            ("tinyllama_decode_512", 512, 21)])
def test_decode_full_size_layer(gpu, name, pos, layer):
    """Full BASELINE configuration sizes (one layer each) against the port."""
    from ligguf_b200.workloads import DECODE_WORKLOADS
    w = DECODE_WORKLOADS[name]
    c = cases.decode_case(H=w.n_heads, Hk=w.n_kv_heads, D=w.head_dim, n_ctx=w.n_context, theta=w.rope_base,
                          qk_norm=int(w.qk_norm), eps=w.eps, pos=pos, seed=w.seed, scale=w.scale, layer=layer)
    out, _, _, h = gpu_decode(c)
    ref, _, _ = cases.run_decode(orc.Checker("port"), c)
    assert cases.rel_err(out, ref) <= TOL
    h.close()


def test_decode_repeat_and_layers_independent(gpu):
    """Repeated calls agree to fp32 rounding (tiles are handed out dynamically, so the merge order of
    the split partials - not the set of terms - can change between calls), and layers are separate."""
    c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=5000, theta=1e6, qk_norm=1, pos=4500, seed=8, layer=2)
    h = make_handle(c, n_layers=4)
    h.kv_synth(0, 4, 0, 4500, c["seed"], 1.0)
    a = h.decode(2, 4500, c["q"], c["k"], c["v"])
    for _ in range(5):
        b = h.decode(2, 4500, c["q"], c["k"], c["v"])
        assert cases.rel_err(b, a) <= 1e-6
    other = h.decode(1, 4500, c["q"], c["k"], c["v"])  # different cache contents -> different result
    assert not np.array_equal(a, other)
    c1 = cases.decode_case(H=32, Hk=8, D=128, n_ctx=5000, theta=1e6, qk_norm=1, pos=4500, seed=8, layer=1)
    c1["q"], c1["k"], c1["v"] = c["q"], c["k"], c["v"]
    c1["qg"], c1["kg"] = c["qg"], c["kg"]  # make_handle gave every layer layer 2's norm weights
    ref1, _, _ = cases.run_decode(orc.Checker("port"), c1)
    assert cases.rel_err(other, ref1) <= TOL
    h.close()


def test_decode_async_device_tensors(gpu):
    import torch
    from ligguf_b200 import synth_fill
    from ligguf_b200.workloads import SYNTH_KNEW, SYNTH_Q, SYNTH_VNEW, stream_id
    c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=2100, theta=1e6, qk_norm=1, pos=2049, seed=21, layer=0)
    h = make_handle(c)
    h.kv_synth(0, 1, 0, 2049, 21, 1.0)
    dev = torch.device("cuda", 0)
    q = torch.empty(32 * 128, device=dev)
    k = torch.empty(8 * 128, device=dev)
    v = torch.empty(8 * 128, device=dev)
    out = torch.empty(32 * 128, device=dev)
    synth_fill(q, q.numel(), 21, stream_id(SYNTH_Q, 0), 0, 1.0)
    synth_fill(k, k.numel(), 21, stream_id(SYNTH_KNEW, 0), 0, 1.0)
    synth_fill(v, v.numel(), 21, stream_id(SYNTH_VNEW, 0), 0, 1.0)
    assert np.array_equal(q.cpu().numpy(), c["q"])
    h.decode_async(0, 2049, q, k, v, out)
    torch.cuda.synchronize()
    h.sync()
    ref, _, _ = cases.run_decode(orc.Checker("port"), c)
    assert cases.rel_err(out.cpu().numpy(), ref) <= TOL
    h.close()


def test_decode_host_pinned_buffers(gpu):
    """The host-pointer call with pinned host buffers (the output is then written in place over the
    host link) and with pageable ones (a staging copy)."""
    import torch
    c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=2100, theta=1e6, qk_norm=1, pos=2000, seed=23, layer=0)
    h = make_handle(c)
    h.kv_synth(0, 1, 0, 2000, 23, 1.0)
    ref, _, _ = cases.run_decode(orc.Checker("port"), c)
    q, k, v = (torch.from_numpy(c[x].copy()).pin_memory() for x in ("q", "k", "v"))
    out = torch.full((32 * 128,), float("nan")).pin_memory()
    rc = h.lib.ligguf_cuda_attn_decode(h.handle, 0, 2000, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr())
    assert rc == 0, h.lib.ligguf_cuda_attn_last_error()
    assert cases.rel_err(out.numpy(), ref) <= TOL
    # pageable inputs and output, then pinned inputs with a pageable output
    h.kv_synth(0, 1, 0, 2000, 23, 1.0)
    qp, kp, vp = (np.ascontiguousarray(c[x]) for x in ("q", "k", "v"))
    outp = np.full(32 * 128, np.nan, dtype=np.float32)
    rc = h.lib.ligguf_cuda_attn_decode(h.handle, 0, 2000, qp.ctypes.data, kp.ctypes.data, vp.ctypes.data,
                                       outp.ctypes.data)
    assert rc == 0, h.lib.ligguf_cuda_attn_last_error()
    assert cases.rel_err(outp, ref) <= TOL
    h.kv_synth(0, 1, 0, 2000, 23, 1.0)
    outp[:] = np.nan
    rc = h.lib.ligguf_cuda_attn_decode(h.handle, 0, 2000, q.data_ptr(), k.data_ptr(), v.data_ptr(), outp.ctypes.data)
    assert rc == 0, h.lib.ligguf_cuda_attn_last_error()
    assert cases.rel_err(outp, ref) <= TOL
    h.close()


@pytest.mark.parametrize("H,Hk,D,kv_type", [
    (32, 8, 128, 0),  # Qwen3-8B heads, fp32 cache
    (64, 8, 128, 1),  # nrep 8, fp16: the prologue's second round of jobs reads q, k, v again
    (64, 8, 64, 2),   # nrep 8, head_dim 64, bf16
])
def test_decode_host_call_and_device_call_alternate(gpu, H, Hk, D, kv_type):
    """The host-pointer call (one staging copy of q, k, v) alternates with the device-pointer call on
    the same handle, at positions 0, 1 and 700: every output equals the reference's."""
    import torch
    port = orc.Checker("port")
    for pos in (0, 1, 700):
        c = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=768, theta=1e6, qk_norm=1, kv_type=kv_type, pos=pos,
                              seed=80 + pos, scale=1.0 if D == 128 else 0.125, layer=0)
        h = make_handle(c)
        out, krow, vrow, _ = gpu_decode(c, h)
        ref, kref, vref = cases.run_decode(port, c)
        assert cases.rel_err(out, ref) <= TOL, pos
        assert np.array_equal(vrow, vref), pos
        dev = torch.device("cuda", 0)
        qd, kd, vd = (torch.from_numpy(np.ascontiguousarray(c[x])).to(dev) for x in ("q", "k", "v"))
        od = torch.empty(H * D, device=dev)
        h.decode_async(0, pos, qd, kd, vd, od)
        torch.cuda.synchronize()
        h.sync()
        assert cases.rel_err(od.cpu().numpy(), ref) <= TOL, pos
        assert cases.rel_err(h.decode(0, pos, c["q"], c["k"], c["v"]), ref) <= TOL, pos
        h.close()


def test_back_to_back_steps_read_the_rows_they_append(gpu):
    """Decode steps launched back to back on one stream with no host synchronisation, alternating two
    layers: every step reads the row its layer's previous step appended.  (A decode may start loading
    cache rows while the previous kernel finishes, but only rows no kernel still in flight can write.)"""
    import torch
    P0, steps, H, Hk, D = 1000, 6, 32, 8, 128
    cs = [cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=1100, theta=1e6, qk_norm=1, pos=P0, seed=33, layer=l)
          for l in (0, 1)]
    h = make_handle(cs[0], n_layers=2)  # both layers get layer 0's norm weights
    h.kv_synth(0, 2, 0, P0, 33, 1.0)
    rng = np.random.default_rng(5)
    ins = [[rng.standard_normal(n).astype(np.float32) for n in (H * D, Hk * D, Hk * D)] for _ in range(2 * steps)]
    dev = torch.device("cuda", 0)
    dins = [[torch.from_numpy(x).to(dev) for x in xs] for xs in ins]
    outs = [torch.empty(H * D, device=dev) for _ in range(2 * steps)]
    torch.cuda.synchronize()
    h.sync()
    for i in range(steps):
        for l in (0, 1):
            q, k, v = dins[2 * i + l]
            h.decode_async(l, P0 + i, q, k, v, outs[2 * i + l])
    torch.cuda.synchronize()
    port = orc.Checker("port")
    cfg = orc.Checker.cfg(H, Hk, D, 1100, D, cs[0]["eps"], 1, 0, 0)
    caches = [(c["kc"].copy(), c["vc"].copy()) for c in cs]
    for i in range(steps):
        for l in (0, 1):
            kc, vc = caches[l]
            q, k, v = ins[2 * i + l]
            ref = port.decode_layer(cfg, kc, vc, cs[0]["freq"], cs[0]["qg"], cs[0]["kg"], P0 + i, q, k, v)
            assert cases.rel_err(outs[2 * i + l].cpu().numpy(), ref) <= TOL, (i, l)
    h.close()


@pytest.mark.parametrize("kv_head0", [0, 5])
def test_decode_one_kv_head_two_level_merge(gpu, kv_head0):
    """A one-KV-head shard at 4100 positions splits each head over more CTAs than two ring loads of
    partials: the merge takes two levels (groups of partials, then the group results)."""
    port = orc.Checker("port")
    c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=4200, theta=1e6, qk_norm=1, pos=4100, seed=91, layer=0,
                          kv_head0=kv_head0, kv_headn=1)
    h = make_handle(c, kv_head0=kv_head0, kv_headn=1)
    out, _, _, _ = gpu_decode(c, h)
    ref, _, _ = cases.run_decode(port, c)
    assert cases.rel_err(out, ref) <= TOL
    h.close()


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_sharded_decode_matches_unsharded(gpu, nranks):
    """SARA split by KV head (cpp/ligguf_distrib.cpp:665-679): the shards' outputs, concatenated in
    rank order, equal the unsharded result (one GPU hosts every shard here)."""
    from ligguf_b200 import shard_of
    port = orc.Checker("port")
    full = cases.decode_case(H=32, Hk=8, D=128, n_ctx=3000, theta=1e6, qk_norm=1, pos=2900, seed=77, layer=0)
    ref, _, _ = cases.run_decode(port, full)
    parts = []
    for r in range(nranks):
        s = shard_of(8, 32, r, nranks)
        c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=3000, theta=1e6, qk_norm=1, pos=2900, seed=77, layer=0,
                              kv_head0=s["kv_head0"], kv_headn=s["kv_headn"])
        h = make_handle(c, kv_head0=s["kv_head0"], kv_headn=s["kv_headn"])
        out, _, _, _ = gpu_decode(c, h)
        parts.append(out)
        h.close()
    assert cases.rel_err(np.concatenate(parts), ref) <= TOL


def test_kv_roundtrip_fp16_state_layout(gpu):
    """kv_download/upload move the fast/ligguf_fast_qk.cpp:236-247 per-layer fp16 rows byte for byte."""
    c = cases.decode_case(H=8, Hk=2, D=64, n_ctx=64, kv_type=1, pos=40, seed=3)
    h = make_handle(c, n_layers=3)
    rows_k = orc.from_f32(orc.synth_f32(40 * 128, 1, 1, 0, 1.0), 1).reshape(40, 128)
    rows_v = orc.from_f32(orc.synth_f32(40 * 128, 1, 2, 0, 1.0), 1).reshape(40, 128)
    h.kv_upload(2, 0, rows_k, rows_v)
    k, v = h.kv_download(2, 0, 40)
    assert np.array_equal(k, rows_k) and np.array_equal(v, rows_v)
    k0, _ = h.kv_download(1, 0, 40)
    assert not np.any(k0)  # other layers untouched (zero-initialised like kc.resize(...,0))
    h.close()


def test_gather_wait_gives_up_and_reports(gpu):
    """A bounded in-kernel wait that runs out: a shard holding half the KV heads opens a one-rank
    gather, so the other half's words are never stored.  The wait kernel gives up after its limit,
    the host reads a timeout status, and the handle stays usable."""
    import torch
    from ligguf_b200 import LigGufAttnError
    c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=300, theta=1e6, qk_norm=1, pos=200, seed=4, layer=0,
                          kv_head0=0, kv_headn=4)
    h = make_handle(c, kv_head0=0, kv_headn=4)
    h.kv_synth(0, 1, 0, 200, 4, 1.0)
    h.gather_open(0, [h.gather_ipc_handle()])
    dev = torch.device("cuda", 0)
    q, k, v = (torch.from_numpy(np.ascontiguousarray(c[x])).to(dev) for x in ("q", "k", "v"))
    full = torch.empty(32 * 128, device=dev)
    h.decode_gather_async(0, 200, q, k, v)
    h.gather_wait_async(0, full)
    torch.cuda.synchronize()  # returns once the wait has given up (about 2 s)
    with pytest.raises(LigGufAttnError) as e:
        h.sync()
    assert e.value.status == -4  # LIGGUF_ATTN_ETIMEDOUT
    ref, _, _ = cases.run_decode(orc.Checker("port"), c)
    out, _, _, _ = gpu_decode(c, h)  # still usable
    assert cases.rel_err(out, ref) <= TOL
    h.close()


def test_errors_are_reported_not_fatal(gpu):
    from ligguf_b200 import LigGufAttnError
    c = cases.decode_case(H=8, Hk=2, D=64, n_ctx=16, qk_norm=1, pos=3)
    from ligguf_b200 import AttnConfig, CudaAttention
    h = CudaAttention(AttnConfig(n_layers=1, n_heads=8, n_kv_heads=2, head_dim=64, n_context=16, rope_dim=64,
                                 qk_norm=True))
    with pytest.raises(LigGufAttnError) as e:  # QK-norm weights not set
        h.decode(0, 3, c["q"], c["k"], c["v"])
    assert e.value.status == -6
    h.set_qk_norm(0, c["qg"], c["kg"])
    with pytest.raises(LigGufAttnError) as e:
        h.decode(0, 16, c["q"], c["k"], c["v"])  # pos == n_context
    assert e.value.status == -1
    with pytest.raises(LigGufAttnError):
        h.decode(1, 3, c["q"], c["k"], c["v"])  # layer out of range
    h.decode(0, 3, c["q"], c["k"], c["v"])  # still usable
    h.close()


@pytest.mark.parametrize("H,Hk,D,pos,kv_headn,scale", [
    (32, 4, 64, 512, 0, 0.125),      # TinyLlama-shaped: one tile per CTA
    (32, 8, 128, 4096, 0, 1.0),      # 4K: static chunks of a few tiles
    (32, 8, 128, 32768, 1, 1.0),     # one KV head at 32K (the 8-GPU shard): two-level merge
    (16, 4, 128, 2000, 0, 3.0),      # peaked softmax: one split's maximum dominates the merge
])
def test_decode_short_streams(gpu, H, Hk, D, pos, kv_headn, scale):
    """Few tiles per CTA: static equal chunks (no grabs), every chunk requested before the previous
    kernel completes, then the merge of the splits' partials."""
    port = orc.Checker("port")
    c = cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=pos + 64, theta=1e6, qk_norm=int(D == 128), pos=pos, seed=pos + H,
                          scale=scale, layer=0, kv_head0=0, kv_headn=kv_headn)
    h = make_handle(c, kv_head0=0, kv_headn=kv_headn)
    for _ in range(2):  # twice: the tickets and counters must be back at zero after each call
        out, _, _, _ = gpu_decode(c, h)
        ref, _, _ = cases.run_decode(port, c)
        assert cases.rel_err(out, ref) <= TOL
    h.close()


def test_self_gather_epochs_advance_on_device_and_replay(gpu):
    """A one-rank gather (the whole model on one GPU, the rank storing into its own buffer): calls
    issued directly, then the same calls captured in a CUDA graph and replayed several times.  The
    gather epoch and slot are decided on the device, so every replay tags its words with a new epoch
    and the waits never take a stale word: each output equals the reference's."""
    import torch
    port = orc.Checker("port")
    H, Hk, D, L, pos = 16, 4, 128, 3, 700
    cs = [cases.decode_case(H=H, Hk=Hk, D=D, n_ctx=768, theta=1e6, qk_norm=1, pos=pos, seed=60 + l, layer=l)
          for l in range(L)]
    h = make_handle(cs[0], n_layers=L, layer=0)
    for l, c in enumerate(cs):
        h.set_qk_norm(l, c["qg"], c["kg"])
        h.kv_synth(l, 1, 0, pos, c["seed"], c["scale"])
    h.gather_open(0, [h.gather_ipc_handle()])
    dev = torch.device("cuda", 0)
    ins = [tuple(torch.from_numpy(c[x]).to(dev) for x in ("q", "k", "v")) for c in cs]
    outs = torch.full((L, H * D), float("nan"), device=dev)
    refs = [cases.run_decode(port, c)[0] for c in cs]

    def step():
        for l in range(L):
            h.decode_gather_async(l, pos, *ins[l])
            h.gather_wait_async(l, outs[l])

    def check():
        torch.cuda.synchronize()
        h.sync()
        for l in range(L):
            assert cases.rel_err(outs[l].cpu().numpy(), refs[l]) <= TOL, l
        outs.fill_(float("nan"))

    for _ in range(3):
        step()
        check()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(4):
        g.replay()
        check()
    step()  # direct calls after the replays continue the device's epoch sequence
    check()
    del g
    h.close()


@pytest.mark.parametrize("H,Hk,kv_type", [
    (4, 1, 0),   # one KV head at 32K (the 8-GPU shard's shape): 256 static splits in 6 merge groups
    (4, 1, 1),   # the same in fp16: 256 splits of 2 tiles, 6 groups
    (16, 4, 0),  # four KV heads: 74 splits per head with grabs, in 2 groups
])
def test_self_gather_merges_group_results(gpu, H, Hk, kv_type):
    """A gathered decode with several first-level merge groups per KV head stores each group's
    (max, sum, o) and the gather wait merges them, in place of a second merge level on the shard's
    GPU.  With grabs, the head's last group merger frees the grab counter, so repeated calls (direct,
    then from a CUDA graph) must each see zeroed counters.  A one-rank gather of the whole model
    exercises the same words as a multi-GPU one; every output equals the reference's."""
    import torch
    port = orc.Checker("port")
    pos = 32768
    c = cases.decode_case(H=H, Hk=Hk, D=128, n_ctx=pos + 64, kv_type=kv_type, theta=1e6, qk_norm=1, pos=pos,
                          seed=70 + H + kv_type, layer=0)
    h = make_handle(c)
    h.kv_synth(0, 1, 0, pos, c["seed"], c["scale"])
    h.gather_open(0, [h.gather_ipc_handle()])
    dev = torch.device("cuda", 0)
    q, k, v = (torch.from_numpy(np.ascontiguousarray(c[x])).to(dev) for x in ("q", "k", "v"))
    out = torch.full((H * 128,), float("nan"), device=dev)
    ref, _, _ = cases.run_decode(port, c)

    def step():
        h.decode_gather_async(0, pos, q, k, v)
        h.gather_wait_async(0, out)

    def check():
        torch.cuda.synchronize()
        h.sync()
        assert cases.rel_err(out.cpu().numpy(), ref) <= TOL
        out.fill_(float("nan"))

    for _ in range(3):
        step()
        check()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(3):
        g.replay()
        check()
    del g
    h.close()
