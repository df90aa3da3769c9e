"""The C ABI library: built, loadable, exports every entry point include/ligguf_cuda_attn.h declares.
No compute calls (CPU only)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ligguf_cuda_attn.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ligguf_cuda_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from ligguf_b200 import build, _lib
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = _declared()
    assert "ligguf_cuda_attn_decode" in names and "ligguf_cuda_attn_init" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from ligguf_b200 import _lib
    assert sorted(_lib.exported_names()) == _declared()


def test_strerror_and_invalid_args_without_gpu(lib):
    from ligguf_b200 import _lib
    assert lib.ligguf_cuda_attn_strerror(_lib.EINVAL) == b"invalid argument"
    assert lib.ligguf_cuda_attn_strerror(12345) == b"unknown status"
    # argument checks that return before touching the device
    assert lib.ligguf_cuda_attn_init(None, None) == _lib.EINVAL
    out = ctypes.c_void_p()
    bad = _lib.AttnCfg()
    bad.n_layers, bad.n_heads, bad.n_kv_heads, bad.head_dim, bad.n_context = 1, 6, 4, 64, 16
    assert lib.ligguf_cuda_attn_init(ctypes.byref(bad), ctypes.byref(out)) == _lib.EINVAL
    assert b"multiple" in lib.ligguf_cuda_attn_last_error()
    bad.n_heads, bad.head_dim = 8, 96
    assert lib.ligguf_cuda_attn_init(ctypes.byref(bad), ctypes.byref(out)) == _lib.EUNSUPPORTED
    assert lib.ligguf_cuda_attn_decode(None, 0, 0, None, None, None, None) == _lib.EINVAL
    assert lib.ligguf_cuda_attn_free(None) == _lib.OK


def test_cfg_struct_layout_matches_header():
    from ligguf_b200 import _lib
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct ligguf_attn_cfg \{(.*?)\} ligguf_attn_cfg;", text, re.S).group(1)
    fields = re.findall(r"\b(\w+);", body)
    assert fields == [f for f, _ in _lib.AttnCfg._fields_]


def test_no_cpu_fallback_in_package():
    """The product package never loads the CPU checkers."""
    pkg = os.path.join(ROOT, "ligguf_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                src = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in src.replace("oracle/attn_oracle.c", ""), f
