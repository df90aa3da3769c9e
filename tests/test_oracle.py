"""Pins the C restatement (oracle/attn_oracle.c) to the reference's own compiled arithmetic.

Two anchors: the golden fixtures under tests/golden (made by tests/golden/make_golden.py from the
reference's fast/lil_math.cpp built from source), and - where oracle/_ref was built - a direct run
of the reference-compiled harness on fresh cases.  Runs on the CPU only.
"""
import json
import os

import numpy as np
import pytest

import cases
from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
META = json.load(open(os.path.join(GOLDEN, "golden.json")))
# The port sums in plain loop order; the reference's AVX2 dot (fast/arch_avx2.h:83-109) accumulates in
# 8 lanes, built -Ofast.  Differences are rounding-order only.
PORT_TOL = 2e-6


def test_synth_numpy_matches_c():
    for seed, stream, idx0, scale, add in [(1, 2, 0, 1.0, 0.0), (77, (3 << 32) | 5, 123456789, 0.125, 0.0),
                                           (5, 6, 0, 0.02, 1.0)]:
        a = orc.synth_f32(5000, seed, stream, idx0, scale, add)
        b = orc.synth_numpy(5000, seed, stream, idx0, scale, add)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_synth_distribution():
    x = orc.synth_f32(200000, 3, 1, 0, 1.0)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1.0) < 0.01
    assert np.abs(x).max() < 3.5


def test_fp16_conversion_bit_exact_vs_reference():
    """Bit-exact over everything that rounds to a finite half or to +-inf at the boundary.

    Above 65520 the reference's own build diverges from its source: fp32_to_fp16
    (fast/lil_math.cpp:57-76) scales by 2^112 then 2^-110 to saturate, and -Ofast (fast/Makefile:7)
    folds the two multiplies, so e.g. 1e9 becomes 0x3373 and 70000 a NaN pattern.  This library
    (and the port) round such values to +-inf as IEEE and the source intend."""
    d = np.load(os.path.join(GOLDEN, "fp16_convert.npz"))
    x = d["x"]
    mine = np.array([orc.port_lib().lo_f32_to_f16(float(v)) for v in x], dtype=np.uint16)
    in_range = np.abs(x) <= 65520.0
    assert in_range.sum() >= x.size - 4
    assert np.array_equal(mine[in_range], d["h"][in_range])


def test_fp16_roundtrip_all_finite_halves():
    h = np.arange(0, 0x7C00, dtype=np.uint16)
    f = orc.to_f32(h, orc.KV_F16)
    back = orc.from_f32(f, orc.KV_F16)
    assert np.array_equal(back, h)


@pytest.mark.parametrize("key", [k for k in META if k.startswith("decode_")])
def test_port_decode_vs_golden(key):
    spec = dict(META[key])
    pos_list = spec.pop("pos_list")
    gold = np.load(os.path.join(GOLDEN, key + ".npz"))
    port = orc.Checker("port")
    for pos in pos_list:
        c = cases.decode_case(pos=pos, **spec)
        out, krow, vrow = cases.run_decode(port, c)
        assert cases.rel_err(out, gold[f"out_{pos}"]) <= PORT_TOL, (key, pos)
        # v is stored unmodified: its row is byte work (a copy, or the fp16 conversion) - exact.
        assert np.array_equal(vrow, gold[f"vrow_{pos}"]), (key, pos, "v row")
        # k is stored after norm and RoPE (float arithmetic): within one ulp of the cache type.
        kt = spec.get("kv_type", 0)
        ulp = 2.0 ** -10 if kt == 1 else 2e-6
        ka, kb = orc.to_f32(krow, kt), orc.to_f32(gold[f"krow_{pos}"], kt)
        assert np.abs(ka - kb).max() <= ulp * np.abs(kb).max(), (key, pos, "k row")


@pytest.mark.parametrize("key", [k for k in META if k.startswith("prefill_")])
def test_port_prefill_vs_golden(key):
    spec = dict(META[key])
    gold = np.load(os.path.join(GOLDEN, key + ".npz"))
    out, _, _ = cases.run_prefill(orc.Checker("port"), cases.prefill_case(**spec))
    assert cases.rel_err(out, gold["out"]) <= PORT_TOL


@pytest.mark.parametrize("key", [k for k in META if k.startswith("bert_")])
def test_port_bert_vs_golden(key):
    spec = dict(META[key])
    gold = np.load(os.path.join(GOLDEN, key + ".npz"))
    out = cases.run_bert(orc.Checker("port"), cases.bert_case(**spec))
    assert cases.rel_err(out, gold["out"]) <= PORT_TOL
    lens = spec["lens"]
    for b, n in enumerate(lens):  # padded rows are zero
        assert not np.any(out[b, n:])


def test_prefill_equals_repeated_decode():
    """fast/ligguf_fast_qk.cpp:340-356: a prompt is fed one inference() per token."""
    c = cases.prefill_case(H=4, Hk=2, D=64, n_ctx=32, pos0=3, n=6, scale=0.5, qk_norm=1)
    port = orc.Checker("port")
    out, kc, vc = cases.run_prefill(port, c)
    kc2, vc2 = c["kc"].copy(), c["vc"].copy()
    cfg = orc.Checker.cfg(4, 2, 64, 32, 64, 1e-6, 1, 0, 0)
    for i in range(6):
        o = port.decode_layer(cfg, kc2, vc2, c["freq"], c["qg"], c["kg"], 3 + i, c["q"][i], c["k"][i], c["v"][i])
        assert np.array_equal(o, out[i])
    assert np.array_equal(kc, kc2) and np.array_equal(vc, vc2)


ref_missing = orc.ref_lib() is None


@pytest.mark.skipif(ref_missing, reason="reference build oracle/_ref not present")
@pytest.mark.parametrize("kv_type", [0, 1])
@pytest.mark.parametrize("pos", [0, 7, 200])
def test_port_vs_reference_fresh(kv_type, pos):
    c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=256, theta=1e6, qk_norm=1, kv_type=kv_type, pos=pos,
                          seed=31 + pos, layer=3)
    a, ka, va = cases.run_decode(orc.Checker("port"), c)
    b, kb, vb = cases.run_decode(orc.Checker("ref"), c)
    assert cases.rel_err(a, b) <= PORT_TOL
    assert np.array_equal(va, vb)
    ka, kb = orc.to_f32(ka, kv_type), orc.to_f32(kb, kv_type)
    assert np.abs(ka - kb).max() <= (2.0 ** -10 if kv_type else 2e-6) * np.abs(kb).max()


@pytest.mark.skipif(ref_missing, reason="reference build oracle/_ref not present")
def test_rope_and_norm_vs_reference():
    port, ref = orc.port_lib(), orc.ref_lib()
    x = orc.synth_f32(4 * 128, 5, 9, 0, 1.0)
    w = orc.synth_f32(128, 5, 10, 0, 0.02, 1.0)
    freq = orc.rope_table(128, 1e6)
    a, b = x.copy(), x.copy()
    for h in range(4):
        port.lo_rmsnorm_inplace(a[h * 128:].ctypes.data, w.ctypes.data, 128, 1e-6)
        ref.rf_rmsnorm_inplace(b[h * 128:].ctypes.data, w.ctypes.data, 128, 1e-6)
    assert np.abs(a - b).max() <= 1e-6 * np.abs(b).max()
    for pos in (0, 1, 4096, 32768):
        a2, b2 = a.copy(), a.copy()
        port.lo_rope(a2.ctypes.data, 4, 128, 128, pos, freq.ctypes.data)
        ref.rf_rope(b2.ctypes.data, 4, 128, 128, pos, freq.ctypes.data)
        assert np.abs(a2 - b2).max() <= 2e-6 * np.abs(b2).max(), pos


def test_split_even_matches_sara():
    from ligguf_b200.attn import split_even
    for total in (1, 4, 7, 8, 36):
        for parts in range(1, total + 1):
            offs = []
            for i in range(parts):
                assert split_even(total, i, parts) == orc.split_even(total, i, parts)
                offs.append(split_even(total, i, parts))
            assert offs[0][0] == 0 and sum(c for _, c in offs) == total
            for (o0, c0), (o1, _) in zip(offs, offs[1:]):
                assert o0 + c0 == o1
