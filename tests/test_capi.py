"""CPU checks of the C ABI: the library loads, exports every function that
include/scope_b200.h declares, and the ctypes binding covers all of them.
No compute call is made (there is no GPU here)."""
import ctypes
import os
import re
import subprocess

import pytest

from scope_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "scope_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ws_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def built_lib():
    if not os.path.exists(_lib.LIB_PATH):
        from scope_b200.compile_lib import build
        build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_entry_points():
    fns = declared_functions()
    assert "ws_gqa_decode" in fns and "ws_lse_merge" in fns
    assert len(fns) >= 8


def test_every_declared_symbol_is_exported(built_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (ws_[a-z0-9_]+)", out))
    for fn in declared_functions():
        assert fn in exported, fn
        assert getattr(built_lib, fn) is not None


def test_binding_covers_header():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_library_has_no_torch_dependency():
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "libtorch" not in out and "libc10" not in out


def test_cpu_tensors_are_rejected():
    import torch
    import scope_b200
    ext = scope_b200.build()
    q = torch.zeros(1, 8, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 16, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ext.fused_cpu_attn(q, k, k, 0.1)
    with pytest.raises(RuntimeError):
        ext.fused_cpu_attn(q.float(), k, k, 0.1)


def test_error_string_and_version(built_lib):
    built_lib.ws_version.restype = ctypes.c_int
    assert built_lib.ws_version() >= 100
    built_lib.ws_last_error.restype = ctypes.c_char_p
    assert isinstance(built_lib.ws_last_error(), bytes)
