"""The port's restatement of the QKV projection arithmetic (oracle/qmat_oracle.c) against the
reference's own code compiled here (oracle/_ref: fast/lil_math.cpp with the reference's flags).
CPU only.  The activation quantizers are integer work: bit-exact.  The row dots sum fp32 block
terms in another order than the AVX2 loops: within 1e-5 of the output scale."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from ligguf_b200.qmat import BLOCK, QT, row_bytes, synthetic_rows

HAVE_REF = orc.ref_lib() is not None


def _x(n, seed, mag=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * mag).astype(np.float32)
    x[:16] = 0.0           # a zero run
    x[300:310] = 2.5       # ties of the largest magnitude inside a 256-block
    x[310] = -2.5
    return x


@pytest.mark.skipif(not HAVE_REF, reason="reference build absent")
@pytest.mark.parametrize("mag", [1e-3, 1.0, 40.0, 1000.0])
def test_quantizers_bit_exact_with_reference(mag):
    """Over 2M values: includes elements that land exactly on a .5 of x*127/amax, where computing
    1/d instead of 127/amax (as the source reads) would round the other way."""
    x = _x(4096 * 512, 5, mag)
    x[512:768] = 0.0       # an all-zero Q8_K block
    assert np.array_equal(orc.quantize_q8_K(x, "port"), orc.quantize_q8_K(x, "ref"))
    assert np.array_equal(orc.quantize_q8_0(x, "port"), orc.quantize_q8_0(x, "ref"))


@pytest.mark.skipif(not HAVE_REF, reason="reference build absent")
@pytest.mark.parametrize("name", list(QT))
def test_port_matmul_matches_reference(name):
    t = QT[name]
    n, d = 1024, 96
    w = synthetic_rows(t, n, d, seed=100 + t)
    x = _x(n, 7)
    port = orc.matmul(t, w, n, x, "port")
    ref = orc.matmul(t, w, n, x, "ref")
    assert np.isfinite(ref).all()
    assert np.abs(port - ref).max() <= 1e-5 * np.abs(ref).max(), name


def test_row_bytes_match_the_library():
    from ligguf_b200 import _lib
    lib = _lib.load()
    for t, (bb, be) in BLOCK.items():
        for n in (256, 4096):
            assert lib.ligguf_cuda_qmat_row_bytes(t, n) == row_bytes(t, n) == n // be * bb
    assert lib.ligguf_cuda_qmat_row_bytes(12, 100) == 0 and lib.ligguf_cuda_qmat_row_bytes(99, 256) == 0


def test_qmat_argument_checks_without_gpu():
    from ligguf_b200 import _lib
    lib = _lib.load()
    out = ctypes.c_void_p()
    row = (ctypes.c_uint8 * 64)()
    assert lib.ligguf_cuda_qmat_init(99, 256, 1, row, 0, 0, ctypes.byref(out)) == _lib.EUNSUPPORTED
    assert lib.ligguf_cuda_qmat_init(12, 100, 1, row, 0, 0, ctypes.byref(out)) == _lib.EINVAL
    assert lib.ligguf_cuda_qmat_init(8, 32768, 1, row, 0, 0, ctypes.byref(out)) == _lib.EUNSUPPORTED
    assert lib.ligguf_cuda_matmul3_async(None, None, None, None, None, None, None, None) == _lib.EINVAL
    assert lib.ligguf_cuda_matmul3_batch_async(None, None, None, None, 4, None, None, None, None) == _lib.EINVAL
    assert lib.ligguf_cuda_quantize_q8_K_async(None, 256, None, None) == _lib.EINVAL
    assert lib.ligguf_cuda_qmat_free(None) == _lib.OK


def test_column_slice_and_reduce_argument_checks_without_gpu():
    from ligguf_b200 import _lib
    lib = _lib.load()
    out = ctypes.c_void_p()
    row = (ctypes.c_uint8 * 64)()
    # columns must be whole blocks of the type (32 for Q8_0)
    assert lib.ligguf_cuda_qmat_init_cols(8, 256, 1, row, 16, 64, 0, 0, ctypes.byref(out)) == _lib.EINVAL
    assert lib.ligguf_cuda_qmat_init_cols(8, 256, 1, row, 224, 64, 0, 0, ctypes.byref(out)) == _lib.EINVAL
    assert lib.ligguf_cuda_reduce_init(0, 2, 0, 0, ctypes.byref(out)) == _lib.EINVAL
    assert lib.ligguf_cuda_reduce_init(16, 2, 2, 0, ctypes.byref(out)) == _lib.EINVAL
    assert lib.ligguf_cuda_matmul_reduce_async(None, None, None, None) == _lib.EINVAL
    assert lib.ligguf_cuda_reduce_free(None) == _lib.OK
