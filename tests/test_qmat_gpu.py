"""The QKV projection on the GPU (ligguf_cuda_matmul3*, ligguf_cuda_quantize_*) against the
reference's own code compiled here (oracle/_ref: matmul3 / matmul / quantize_q8_K / quantize_q8_0 of
fast/lil_math.cpp, AVX2).  The quantized activation is integer work: bit-exact.  Outputs: fp32 path,
max |gpu - ref| <= 1e-4 * max |ref| (only the order of the fp32 sum over blocks differs)."""
import numpy as np
import pytest

from oracle import oracle as orc
from ligguf_b200.qmat import (QT, QuantMatrix, matmul3, matmul3_async, matmul3_batch, matmul3_batch_async,
                              synthetic_rows)

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _x(n, seed, mag=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * mag).astype(np.float32)
    x[:40] = 0.0
    x[300:305] = -3.0
    return x


def _rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("mag", [1e-3, 1.0, 40.0])
def test_quantizers_bit_exact(gpu, mag):
    import torch
    from ligguf_b200 import _lib
    lib = _lib.load()
    x = _x(4096 * 64, 11, mag)
    x[1024:1280] = 0.0
    dx = torch.from_numpy(x).cuda()
    k = torch.zeros(x.size // 256 * 292, dtype=torch.uint8, device="cuda")
    z = torch.zeros(x.size // 32 * 34, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.ligguf_cuda_quantize_q8_K_async(dx.data_ptr(), x.size, k.data_ptr(), s) == 0
    assert lib.ligguf_cuda_quantize_q8_0_async(dx.data_ptr(), x.size, z.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert np.array_equal(k.cpu().numpy(), orc.quantize_q8_K(x, "ref"))
    assert np.array_equal(z.cpu().numpy(), orc.quantize_q8_0(x, "ref"))


@pytest.mark.parametrize("name", list(QT))
@pytest.mark.parametrize("n,d", [(4096, 520), (1024, 33)])
def test_matmul_each_type(gpu, name, n, d):
    t = QT[name]
    w = synthetic_rows(t, n, d, seed=t * 7 + n)
    x = _x(n, n + t)
    m = QuantMatrix(t, n, w)
    (got,) = matmul3(m, None, None, x)
    m.close()
    ref = orc.matmul(t, w, n, x, "ref")
    assert _rel(got, ref) <= TOL, name


@pytest.mark.parametrize("types", [("Q8_0", "Q8_0", "Q8_0"), ("Q4_K", "Q4_K", "Q6_K"), ("Q5_K", "Q1_0", "F16")])
def test_matmul3_qwen3_8b_shapes(gpu, types):
    """The Qwen3-8B QKV step: x [4096] -> q [4096], k [1024], v [1024], one launch for all three
    matrices (mixed types as a Q4_K_M file has them), device pointers, against the engine's
    quantize_q8_K + matmul3."""
    import torch
    n, dims = 4096, (4096, 1024, 1024)
    ws = [(QT[nm], synthetic_rows(QT[nm], n, d, seed=i + 31)) for i, (nm, d) in enumerate(zip(types, dims))]
    x = _x(n, 3)
    mats = [QuantMatrix(t, n, w) for t, w in ws]
    dx = torch.from_numpy(x).cuda()
    outs = [torch.full((d,), float("nan"), device="cuda") for d in dims]
    matmul3_async(*mats, dx, *outs)
    torch.cuda.synchronize()
    refs = orc.matmul3(ws, n, x)
    for o, r in zip(outs, refs):
        assert _rel(o.cpu().numpy(), r) <= TOL, types
    for m in mats:
        m.close()


@pytest.mark.parametrize("name", ["F32", "F16", "Q8_0", "Q1_0"])
@pytest.mark.parametrize("n,d", [(96, 7), (864, 131), (16384, 40)])
def test_matmul_ragged_widths(gpu, name, n, d):
    """Widths that are a multiple of the 32-element block but not of 256 or 1024 (the tail of the
    Q8_0 quantizer's lane-per-block pass and of the fp32 copy), row counts that leave a partial
    tile, and the widest input the kernel takes (16384; for F32, whose row must fit a 32 KB stream
    stage, 8192), one token and a batch of 5."""
    if name == "F32" and n > 8192:
        n = 8192
    t = QT[name]
    w = synthetic_rows(t, n, d, seed=t * 13 + n)
    m = QuantMatrix(t, n, w)
    xs = np.stack([_x(n, n + t + i, mag=0.5 + i) for i in range(5)])
    (one,) = matmul3(m, None, None, xs[0])
    (batch,) = matmul3_batch(m, None, None, xs)
    m.close()
    for i in range(5):
        ref = orc.matmul(t, w, n, xs[i], "ref")
        assert _rel(batch[i], ref) <= TOL, (name, i)
    assert np.array_equal(one, batch[0])


@pytest.mark.parametrize("n_tok", [1, 3, 8, 21])
@pytest.mark.parametrize("types", [("Q4_K", "Q4_K", "Q6_K"), ("Q8_0", "Q8_0", "Q8_0"), ("F16", "Q2_K", "Q1_G")])
def test_matmul3_batch_equals_token_loop(gpu, n_tok, types):
    """Batched prompt projections: n_tok tokens in groups of up to 8 per weight pass, each token's
    outputs equal to the reference's matmul3 on that token (the feed_text loop,
    fast/ligguf_fast_qk.cpp:340-356)."""
    import torch
    n, dims = 2048, (2048, 512, 256)
    ws = [(QT[nm], synthetic_rows(QT[nm], n, d, seed=i + 7 * n_tok)) for i, (nm, d) in enumerate(zip(types, dims))]
    mats = [QuantMatrix(t, n, w) for t, w in ws]
    x = np.stack([_x(n, 100 + i, mag=0.5 + i) for i in range(n_tok)])
    dx = torch.from_numpy(x).cuda()
    outs = [torch.full((n_tok, d), float("nan"), device="cuda") for d in dims]
    matmul3_batch_async(*mats, dx, n_tok, *outs)
    torch.cuda.synchronize()
    host = matmul3_batch(*mats, x)  # the host-pointer form too
    for i in range(n_tok):
        refs = orc.matmul3(ws, n, x[i])
        for j in range(3):
            assert _rel(outs[j][i].cpu().numpy(), refs[j]) <= TOL, (types, i, j)
            assert np.array_equal(host[j][i], outs[j][i].cpu().numpy())
    for m in mats:
        m.close()


@pytest.mark.parametrize("types", [("Q8_0", "Q8_0", "Q8_0"), ("Q4_K", "Q4_K", "Q6_K"), ("F32", "Q1_0", "Q3_K")])
def test_one_token_and_batch_quantize_alike(gpu, types):
    """A token alone (quantized inside the projection kernel, a lane per Q8_0 block) and the same
    token inside a batch (quantized once per call by the activation kernel, a warp per block) give
    bit-identical outputs: both are the reference's quantizer, and the dots run in the same order."""
    import torch
    n, dims = 4096, (1024, 512, 256)
    ws = [(QT[nm], synthetic_rows(QT[nm], n, d, seed=31 + i)) for i, (nm, d) in enumerate(zip(types, dims))]
    mats = [QuantMatrix(t, n, w) for t, w in ws]
    xs = np.stack([_x(n, 200 + i, mag=[1e-3, 1.0, 40.0][i]) for i in range(3)])
    batch = matmul3_batch(*mats, xs)
    for i in range(3):
        one = matmul3(*mats, xs[i])
        for j in range(3):
            assert np.array_equal(one[j], batch[j][i]), (types, i, j)
    for m in mats:
        m.close()


def test_matmul3_shapes_and_errors(gpu):
    from ligguf_b200 import _lib
    from ligguf_b200._lib import LigGufAttnError
    t = QT["Q4_K"]
    a = QuantMatrix(t, 2048, synthetic_rows(t, 2048, 7, 1))     # fewer rows than one tile
    b = QuantMatrix(t, 4096, synthetic_rows(t, 4096, 16, 2))
    x = _x(2048, 5)
    (got,) = matmul3(a, None, None, x)
    assert _rel(got, orc.matmul(t, synthetic_rows(t, 2048, 7, 1), 2048, x, "ref")) <= TOL
    with pytest.raises(LigGufAttnError) as e:  # different input widths in one call
        matmul3(a, b, None, x)
    assert e.value.status == _lib.EINVAL
    import torch
    dx = torch.zeros(2048 + 4, device="cuda")
    out = torch.empty(7, device="cuda")
    with pytest.raises(LigGufAttnError) as e:  # x not on a 16-byte boundary (read in 16-byte vectors)
        matmul3_async(a, None, None, dx.data_ptr() + 4, out)
    assert e.value.status == _lib.EINVAL
    a.close()
    b.close()
