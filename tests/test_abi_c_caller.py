"""A plain C99 translation unit (tests/abi_caller.c) includes include/ligguf_cuda_attn.h and links
libligguf_cuda_attn.so, as an engine binding does: it compiles warning-free, its argument checks pass
without a GPU, and (GPU) one decode step through the host-pointer call matches the C restatement of
the reference within 1e-4 of the output scale."""
import os
import subprocess

import numpy as np
import pytest

import cases
from oracle import oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def caller(tmp_path_factory):
    from ligguf_b200 import build
    libdir = os.path.dirname(build.build())
    exe = str(tmp_path_factory.mktemp("caller") / "abi_caller")
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"), "-o",
                        exe, os.path.join(ROOT, "tests", "abi_caller.c"), "-L", libdir, "-lligguf_cuda_attn",
                        f"-Wl,-rpath,{libdir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c_caller_argument_checks(caller):
    r = subprocess.run([caller], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stderr


@pytest.mark.gpu
def test_c_caller_decode_matches_reference(gpu, caller, tmp_path):
    c = cases.decode_case(H=32, Hk=8, D=128, n_ctx=320, theta=1e6, qk_norm=1, pos=300, seed=11, layer=0)
    blob = np.concatenate([c["q"], c["k"], c["v"], c["qg"], c["kg"]]).astype(np.float32)
    inp, out = tmp_path / "in.bin", tmp_path / "out.bin"
    blob.tofile(inp)
    r = subprocess.run([caller, "decode", str(inp), str(out)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(out, dtype=np.float32)
    ref, _, _ = cases.run_decode(orc.Checker("port"), c)
    assert cases.rel_err(got, ref) <= 1e-4
