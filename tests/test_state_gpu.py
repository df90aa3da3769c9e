"""The engine's state file (`model_file`, fast/common.h:26-31; save_model_state / load_model_state,
fast/ligguf_fast_qk.cpp:216-302) written from and read into the HBM-resident fp16 cache.

A model decodes a prompt, its state is saved, a fresh handle loads it and both continue: the next
tokens must agree bit for bit (same cache bytes, same kernel).  The file is checked byte for byte
against a restatement of save_model_state over the cache rows kv_download returns, and files that
fail the reference's checks are refused without touching the cache."""
import os
import struct

import numpy as np
import pytest

import cases
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
H, HK, D, NCTX, L = 8, 2, 128, 256, 2
N_LOGITS = 1000


def _handle(kv_type=1):
    from ligguf_b200 import AttnConfig, CudaAttention
    return CudaAttention(AttnConfig(n_layers=L, n_heads=H, n_kv_heads=HK, head_dim=D, n_context=NCTX, rope_dim=D,
                                    rope_base=1e6, rms_epsilon=1e-6, qk_norm=True, kv_type=kv_type))


def _step(h, pos):
    outs = []
    for layer in range(L):
        c = cases.decode_case(H=H, Hk=HK, D=D, n_ctx=NCTX, theta=1e6, qk_norm=1, kv_type=1, pos=pos,
                              seed=500 + layer, layer=layer)
        h.set_qk_norm(layer, c["qg"], c["kg"])
        outs.append(h.decode(layer, pos, c["q"], c["k"], c["v"]))
    return np.concatenate(outs)


def _reference_file_bytes(h, pos, logits):
    """save_model_state's bytes (fast/ligguf_fast_qk.cpp:274-298) from the downloaded cache rows."""
    kv_dim = HK * D
    hdr = struct.pack("<iiQQ", pos, NCTX, L * pos * kv_dim, logits.size)
    rows = [h.kv_download(layer, 0, pos) for layer in range(L)]
    body = b"".join(k.tobytes() for k, _ in rows) + b"".join(v.tobytes() for _, v in rows)
    return hdr + body + logits.astype(np.float32).tobytes()


def test_state_round_trip_continues_identically(gpu, tmp_path):
    P = 70
    a = _handle()
    for pos in range(P):
        _step(a, pos)
    logits = np.random.default_rng(7).standard_normal(N_LOGITS).astype(np.float32)
    path = str(tmp_path / "state.bin")
    a.state_save(path, P, logits)
    assert open(path, "rb").read() == _reference_file_bytes(a, P, logits)
    b = _handle()
    pos, n_ctx, lg = b.state_load(path, N_LOGITS)
    assert (pos, n_ctx) == (P, NCTX) and np.array_equal(lg, logits)
    for layer in range(L):
        ka, va = a.kv_download(layer, 0, P)
        kb, vb = b.kv_download(layer, 0, P)
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    for pos in (P, P + 1):  # both continue the same sequence
        assert np.array_equal(_step(a, pos), _step(b, pos))
    # and the continuation is still the reference's attention
    c = cases.decode_case(H=H, Hk=HK, D=D, n_ctx=NCTX, theta=1e6, qk_norm=1, kv_type=1, pos=P + 2, seed=500, layer=0)
    b.set_qk_norm(0, c["qg"], c["kg"])
    kc, vc = b.kv_download(0, 0, P + 2)
    c["kc"][:P + 2], c["vc"][:P + 2] = kc, vc
    ref, _, _ = cases.run_decode(orc.Checker("port"), c)
    assert cases.rel_err(b.decode(0, P + 2, c["q"], c["k"], c["v"]), ref) <= 1e-4
    a.close()
    b.close()


def test_state_files_that_fail_the_checks_change_nothing(gpu, tmp_path):
    from ligguf_b200 import _lib
    from ligguf_b200._lib import LigGufAttnError
    a = _handle()
    for pos in range(5):
        _step(a, pos)
    logits = np.ones(N_LOGITS, dtype=np.float32)
    good = str(tmp_path / "good.bin")
    a.state_save(good, 5, logits)
    blob = open(good, "rb").read()
    b = _handle()
    for pos in range(3):
        _step(b, pos)
    before = [b.kv_download(layer, 0, 5) for layer in range(L)]
    bad_files = {
        "short": blob[:-4],                                                    # truncated logits
        "zero_pos": struct.pack("<iiQQ", 0, NCTX, 0, N_LOGITS) + blob[24:],    # empty state
        "kv_size": struct.pack("<iiQQ", 5, NCTX, 7, N_LOGITS) + blob[24:],     # wrong cache size
    }
    for name, data in bad_files.items():
        p = str(tmp_path / f"{name}.bin")
        open(p, "wb").write(data)
        with pytest.raises(LigGufAttnError) as e:
            b.state_load(p, N_LOGITS)
        assert e.value.status == _lib.EINVAL, name
    with pytest.raises(LigGufAttnError):
        b.state_load(good, N_LOGITS + 1)  # logits size differs
    after = [b.kv_download(layer, 0, 5) for layer in range(L)]
    for (k0, v0), (k1, v1) in zip(before, after):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
    f32 = _handle(kv_type=0)
    with pytest.raises(LigGufAttnError) as e:
        f32.state_save(str(tmp_path / "f32.bin"), 1, logits)
    assert e.value.status == _lib.EUNSUPPORTED
    for h in (a, b, f32):
        h.close()
    assert not os.path.exists(str(tmp_path / "f32.bin"))
