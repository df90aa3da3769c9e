"""The tensor-core softmax's polynomial 2^x (exp2_poly2 in ligguf_b200/csrc/flash_tc.cuh), emulated
step by step in float32 with the coefficients read from the kernel source (CPU only).

The kernel takes a quarter of the exponentials of P this way instead of ex2.approx.  P is rounded to
bf16 (relative step 2^-8), so the stated bound of the cubic, 1.03e-4 relative, is what matters; the
end-to-end tolerance is covered by the bf16 parity tests on the GPU."""
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "ligguf_b200", "csrc", "flash_tc.cuh")


def _body():
    text = open(SRC).read()
    start = text.index("__device__ __forceinline__ float2 exp2_poly2(float2 x) {")
    return text[start:text.index("\n}\n", start)]


def _coefficients():
    """c3, c2 (first ffma2), c1 (second), 1 (third): the Horner steps in source order."""
    body = _body()
    consts = [float(v) for v in re.findall(r"make_float2\(([-0-9.e]+)f, \1f\)", body)]
    # clamp bound and the 1.5 * 2^23 shifter appear first; then f = n * -1 + x; then the Horner terms
    horner = consts[consts.index(-1.0) + 1:]
    assert len(horner) == 4, horner
    return [np.float32(v) for v in horner]


def _exp2_poly(x):
    c3, c2, c1, c0 = _coefficients()
    f32 = np.float32
    x = np.maximum(x.astype(np.float32), f32(-127.0))
    t = (x + f32(12582912.0)).astype(np.float32)
    n = (t + f32(-12582912.0)).astype(np.float32)
    f = (n * f32(-1.0) + x).astype(np.float32)
    p = (f * c3 + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    bits = (p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_coefficients_pin_p0_to_one():
    assert _coefficients()[3] == np.float32(1.0)


def test_relative_error_within_stated_bound():
    x = np.linspace(-125.0, 8.5, 1_000_001).astype(np.float32)
    y = _exp2_poly(x).astype(np.float64)
    rel = np.abs(y / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() <= 1.04e-4, rel.max()


def test_special_inputs():
    x = np.array([-np.inf, -1000.0, -127.0, 0.0, 1.0, -1.0, 8.0], np.float32)
    y = _exp2_poly(x)
    assert y[0] == 0.0 and y[1] == 0.0 and y[2] == 0.0
    assert y[3] == 1.0 and y[6] == 256.0
    assert abs(y[4] / 2.0 - 1.0) < 1.04e-4 and abs(y[5] / 0.5 - 1.0) < 1.04e-4


def test_tiny_inputs_stay_below_normal_range():
    x = np.linspace(-127.0, -125.0, 10001).astype(np.float32)
    y = _exp2_poly(x).astype(np.float64)
    assert np.all(y >= 0.0) and np.all(y <= 2.0 ** -125 * 1.001)
