"""Generates tests/golden/*.npz from the REFERENCE's own compiled code.

The reference ships no tests, fixtures or golden vectors, so these are made here: the inputs come
from the seeded generator (re-created by the tests from the seed, not stored), the outputs from
oracle/_ref/libligguf_ref.so - the reference's fast/lil_math.cpp built from its source tree by
oracle/Makefile and driven through the loop of fast/ligguf_fast_qk.cpp:42-105 (decode, prefill as
repeated decode) or fast/vdb.cpp:189-212 (BERT) by oracle/ref_harness.cpp.

    make -C oracle && python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import cases  # noqa: E402
from oracle import oracle as orc  # noqa: E402


def main():
    orc.build()
    ref = orc.Checker("ref")
    meta = {}
    for spec in cases.GOLDEN_DECODE:
        spec = dict(spec)
        name, pos_list = spec.pop("name"), spec.pop("pos_list")
        arrays = {}
        for pos in pos_list:
            c = cases.decode_case(pos=pos, **spec)
            out, krow, vrow = cases.run_decode(ref, c)
            arrays[f"out_{pos}"] = out
            arrays[f"krow_{pos}"] = krow
            arrays[f"vrow_{pos}"] = vrow
        np.savez_compressed(os.path.join(HERE, f"decode_{name}.npz"), **arrays)
        meta[f"decode_{name}"] = dict(spec, pos_list=list(pos_list))
    for spec in cases.GOLDEN_PREFILL:
        spec = dict(spec)
        name = spec.pop("name")
        c = cases.prefill_case(**spec)
        out, kc, vc = cases.run_prefill(ref, c)
        np.savez_compressed(os.path.join(HERE, f"prefill_{name}.npz"), out=out)
        meta[f"prefill_{name}"] = spec
    for spec in cases.GOLDEN_BERT:
        spec = dict(spec)
        name = spec.pop("name")
        c = cases.bert_case(**spec)
        out = cases.run_bert(ref, c)
        np.savez_compressed(os.path.join(HERE, f"bert_{name}.npz"), out=out)
        meta[f"bert_{name}"] = dict(spec, lens=list(spec["lens"]))
    # fp32 -> fp16 conversion of the reference (f32_to_f16_row, fast/lil_math.cpp:57-86) on edge values
    edge = np.concatenate([
        np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, np.inf, -np.inf,
                  2.0 ** -14, 2.0 ** -24, 2.0 ** -25, 2.0 ** -25 * 1.0001, 2.0 ** -26, 5.96e-8, 6.1e-5,
                  1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, 0.1, 1.0 / 3.0], dtype=np.float32),
        orc.synth_f32(4096, 99, 1, 0, 3.0),
        orc.synth_f32(4096, 98, 1, 0, 1e-5),
    ]).astype(np.float32)
    h = np.zeros(edge.size, dtype=np.uint16)
    orc.ref_lib().rf_f32_to_f16_row(edge.ctypes.data, h.ctypes.data, edge.size)
    np.savez_compressed(os.path.join(HERE, "fp16_convert.npz"), x=edge, h=h)
    meta["fp16_convert"] = {"n": int(edge.size)}
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print(f"wrote {len(meta)} fixtures to {HERE}")


if __name__ == "__main__":
    main()
