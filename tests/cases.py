"""Seeded test cases: host inputs from the generator restatement (oracle/attn_oracle.c), identical to
what the CUDA library's generator produces on the device.  Test infrastructure only."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import oracle as orc  # noqa: E402

SYNTH_K, SYNTH_V, SYNTH_Q, SYNTH_KNEW, SYNTH_VNEW, SYNTH_QGAMMA, SYNTH_KGAMMA = 1, 2, 3, 4, 5, 6, 7


def sid(tensor, layer):
    return (tensor << 32) | (layer & 0xFFFFFFFF)


def decode_case(H=8, Hk=2, D=64, n_ctx=64, rope_dim=None, theta=1e4, qk_norm=0, eps=1e-6, kv_type=0,
                scale_mode=0, pos=10, scale=1.0, seed=1234, layer=0, kv_head0=0, kv_headn=0):
    """Inputs of one decode step of one layer (optionally one SARA shard of it)."""
    rope_dim = D if rope_dim is None else rope_dim
    kvn = kv_headn or Hk
    nrep = H // Hk
    kv_full, kv_dim = Hk * D, kvn * D
    c = dict(H=H, Hk=Hk, D=D, n_ctx=n_ctx, rope_dim=rope_dim, theta=theta, qk_norm=qk_norm, eps=eps,
             kv_type=kv_type, scale_mode=scale_mode, pos=pos, scale=scale, seed=seed, layer=layer,
             kv_head0=kv_head0, kv_headn=kvn, q_headn=kvn * nrep)
    dt = orc.kv_dtype(kv_type)
    kc = np.zeros((n_ctx, kv_dim), dtype=dt)
    vc = np.zeros((n_ctx, kv_dim), dtype=dt)
    if pos > 0:
        orc.kv_synth(kc, kv_type, kv_dim, kv_full, kv_head0 * D, layer, SYNTH_K, 0, pos, seed, scale)
        orc.kv_synth(vc, kv_type, kv_dim, kv_full, kv_head0 * D, layer, SYNTH_V, 0, pos, seed, scale)
    c["kc"], c["vc"] = kc, vc
    c["q"] = orc.synth_f32(kvn * nrep * D, seed, sid(SYNTH_Q, layer), kv_head0 * nrep * D, scale)
    c["k"] = orc.synth_f32(kv_dim, seed, sid(SYNTH_KNEW, layer), kv_head0 * D, scale)
    c["v"] = orc.synth_f32(kv_dim, seed, sid(SYNTH_VNEW, layer), kv_head0 * D, scale)
    c["qg"] = orc.synth_f32(D, seed, sid(SYNTH_QGAMMA, layer), 0, 0.02, 1.0)
    c["kg"] = orc.synth_f32(D, seed, sid(SYNTH_KGAMMA, layer), 0, 0.02, 1.0)
    c["freq"] = orc.rope_table(rope_dim, theta)
    return c


def run_decode(checker, c):
    """Runs the checker on copies of the cache; returns (out, k_row, v_row) (the written cache row)."""
    cfg = orc.Checker.cfg(c["q_headn"], c["kv_headn"], c["D"], c["n_ctx"], c["rope_dim"], c["eps"],
                          c["qk_norm"], c["kv_type"], c["scale_mode"])
    kc, vc = c["kc"].copy(), c["vc"].copy()
    out = checker.decode_layer(cfg, kc, vc, c["freq"], c["qg"], c["kg"], c["pos"], c["q"], c["k"], c["v"])
    return out, kc[c["pos"]].copy(), vc[c["pos"]].copy()


def prefill_case(H=4, Hk=2, D=64, n_ctx=64, rope_dim=None, theta=1e4, qk_norm=0, eps=1e-6, kv_type=0,
                 scale_mode=0, pos0=0, n=8, scale=1.0, seed=4321, layer=0):
    rope_dim = D if rope_dim is None else rope_dim
    kv_dim = Hk * D
    c = dict(H=H, Hk=Hk, D=D, n_ctx=n_ctx, rope_dim=rope_dim, theta=theta, qk_norm=qk_norm, eps=eps,
             kv_type=kv_type, scale_mode=scale_mode, pos0=pos0, n=n, scale=scale, seed=seed, layer=layer)
    dt = orc.kv_dtype(kv_type)
    kc = np.zeros((n_ctx, kv_dim), dtype=dt)
    vc = np.zeros((n_ctx, kv_dim), dtype=dt)
    if pos0 > 0:
        orc.kv_synth(kc, kv_type, kv_dim, kv_dim, 0, layer, SYNTH_K, 0, pos0, seed, scale)
        orc.kv_synth(vc, kv_type, kv_dim, kv_dim, 0, layer, SYNTH_V, 0, pos0, seed, scale)
    c["kc"], c["vc"] = kc, vc
    c["q"] = orc.synth_f32(n * H * D, seed, sid(SYNTH_Q, layer), pos0 * H * D, scale).reshape(n, H * D)
    c["k"] = orc.synth_f32(n * kv_dim, seed, sid(SYNTH_KNEW, layer), pos0 * kv_dim, scale).reshape(n, kv_dim)
    c["v"] = orc.synth_f32(n * kv_dim, seed, sid(SYNTH_VNEW, layer), pos0 * kv_dim, scale).reshape(n, kv_dim)
    c["qg"] = orc.synth_f32(D, seed, sid(SYNTH_QGAMMA, layer), 0, 0.02, 1.0)
    c["kg"] = orc.synth_f32(D, seed, sid(SYNTH_KGAMMA, layer), 0, 0.02, 1.0)
    c["freq"] = orc.rope_table(rope_dim, theta)
    return c


def run_prefill(checker, c):
    cfg = orc.Checker.cfg(c["H"], c["Hk"], c["D"], c["n_ctx"], c["rope_dim"], c["eps"], c["qk_norm"],
                          c["kv_type"], c["scale_mode"])
    kc, vc = c["kc"].copy(), c["vc"].copy()
    out = checker.prefill_layer(cfg, kc, vc, c["freq"], c["qg"], c["kg"], c["pos0"], c["n"], c["q"], c["k"], c["v"])
    return out, kc, vc


def bert_case(H=4, D=64, lens=(1, 7, 20), max_len=20, scale=0.125, seed=777, layer=0):
    lens = np.asarray(lens, dtype=np.int32)
    B, E = lens.size, H * D
    n = B * max_len * E
    c = dict(H=H, D=D, lens=lens, max_len=max_len, scale=scale, seed=seed, layer=layer)
    c["q"] = orc.synth_f32(n, seed, sid(SYNTH_Q, layer), 0, scale).reshape(B, max_len, E)
    c["k"] = orc.synth_f32(n, seed, sid(SYNTH_K, layer), 0, scale).reshape(B, max_len, E)
    c["v"] = orc.synth_f32(n, seed, sid(SYNTH_V, layer), 0, scale).reshape(B, max_len, E)
    return c


def run_bert(checker, c):
    return checker.bert_attn(c["H"], c["D"], c["lens"], c["max_len"], c["q"], c["k"], c["v"])


def rel_err(got, ref):
    """max |got - ref| / max |ref| (the tolerance measure: error relative to the output scale)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / scale)


# ------------------------------------------------------------------ golden case lists
GOLDEN_DECODE = [
    dict(name="f32_tinyllama_like", H=8, Hk=2, D=64, n_ctx=64, theta=1e4, pos_list=(0, 1, 31, 33, 63), scale=0.125),
    dict(name="f16_fast_qwen3", H=8, Hk=2, D=128, n_ctx=64, theta=1e6, qk_norm=1, kv_type=1,
         pos_list=(0, 5, 47), scale=1.0),
    dict(name="f32_div_gqa4", H=16, Hk=4, D=128, n_ctx=160, theta=1e6, qk_norm=1, scale_mode=1,
         pos_list=(2, 129), scale=1.0),
    dict(name="f16_rope_partial", H=4, Hk=4, D=64, n_ctx=48, rope_dim=32, theta=1e4, kv_type=1,
         pos_list=(17,), scale=0.5),
]
GOLDEN_PREFILL = [
    dict(name="f32_p0", H=4, Hk=2, D=64, n_ctx=64, theta=1e4, pos0=0, n=12, scale=0.5),
    dict(name="f32_qwen3_p5", H=8, Hk=2, D=128, n_ctx=64, theta=1e6, qk_norm=1, pos0=5, n=9, scale=1.0),
]
GOLDEN_BERT = [
    dict(name="bert_small", H=4, D=64, lens=(1, 7, 20), max_len=20, scale=0.125),
    dict(name="bert_empty_and_full", H=2, D=64, lens=(0, 16, 5), max_len=16, scale=0.125),
]
