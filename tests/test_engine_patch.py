"""The FAST engine patch (integration/fast_cuda_attn.patch): it only inserts lines, it applies to the
reference's fast/ tree, the patched engine compiles and links against include/ligguf_cuda_attn.h and
libligguf_cuda_attn.so (and starts: the dynamic loader resolves the library), and with CUDA_ATTN unset
the patched sources preprocess to exactly the reference's.  CPU only (no model is needed); the tree is
the checkout named `reference` beside this repository, or LIGGUF_REFERENCE_TREE, else skipped."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PATCH = os.path.join(ROOT, "integration", "fast_cuda_attn.patch")
REF = os.environ.get("LIGGUF_REFERENCE_TREE", os.path.join(os.path.dirname(ROOT), "reference"))
HAVE_REF = os.path.exists(os.path.join(REF, "fast", "ligguf_fast_qk.cpp"))
# the reference's flags (fast/Makefile:7-8), -march portable as in oracle/Makefile
CXXFLAGS = ["-Wall", "-Ofast", "-fopenmp", "-march=x86-64-v3", "-mavx2", "-mfma"]
SOURCES = ["ligguf_fast_qk", "lil_gguf", "lil_math", "tokenize", "common", "vdb"]  # no SDL here


def test_patch_only_inserts_lines():
    body = [l for l in open(PATCH).read().splitlines() if not l.startswith(("---", "+++"))]
    assert not [l for l in body if l.startswith("-")]
    assert any(l.startswith("+") for l in body)


@pytest.fixture(scope="module")
def patched(tmp_path_factory):
    if not HAVE_REF:
        pytest.skip("reference tree not present")
    d = tmp_path_factory.mktemp("engine")
    shutil.copytree(os.path.join(REF, "fast"), d / "fast")
    r = subprocess.run(["patch", "-p1", "-s", "--no-backup-if-mismatch", "-i", PATCH], cwd=d, capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return d / "fast"


def test_patched_engine_compiles_links_and_starts(patched):
    from ligguf_b200 import build
    lib = build.build()
    libdir = os.path.dirname(lib)
    procs = [subprocess.Popen(["g++", *CXXFLAGS, "-DLIGGUF_CUDA_ATTN=1", "-I", os.path.join(ROOT, "include"), "-c",
                               "-o", f"{s}.o", f"{s}.cpp"], cwd=patched, stderr=subprocess.PIPE, text=True)
             for s in SOURCES + ["cuda_attn"]]
    for p in procs:
        _, err = p.communicate(timeout=300)
        assert p.returncode == 0, err
    objs = [f"{s}.o" for s in SOURCES + ["cuda_attn"]]
    r = subprocess.run(["g++", "-fopenmp", "-o", "engine", *objs, "-L", libdir, "-lligguf_cuda_attn",
                        f"-Wl,-rpath,{libdir}"], cwd=patched, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    undef = subprocess.run(["nm", "-u", "engine"], cwd=patched, capture_output=True, text=True).stdout
    for sym in ("ligguf_cuda_attn_init", "ligguf_cuda_attn_set_qk_norm", "ligguf_cuda_attn_decode",
                "ligguf_cuda_attn_state_save", "ligguf_cuda_attn_state_load", "ligguf_cuda_attn_free"):
        assert sym in undef, sym
    # no model: the engine stops at its model check, after the loader has resolved the library
    r = subprocess.run(["./engine"], cwd=patched, capture_output=True, text=True, timeout=60)
    assert "error while loading shared libraries" not in r.stderr and r.returncode != 127, r.stderr


def test_without_the_flag_the_engine_is_unchanged(patched):
    for s in SOURCES:
        pre = []
        for d in (os.path.join(REF, "fast"), str(patched)):
            r = subprocess.run(["g++", *CXXFLAGS, "-E", "-P", f"{s}.cpp"], cwd=d, capture_output=True, text=True)
            assert r.returncode == 0, r.stderr
            pre.append(r.stdout)
        assert pre[0] == pre[1], s
