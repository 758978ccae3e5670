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


def test_exchange_sizes_and_argument_checks():
    """Host-only parts of the NVLink exchange entries: buffer sizes, and the
    argument checks that return before any CUDA call."""
    L = _lib.lib()
    # gather form: 1 KB control block + one slot per rank of rows*dim + rows floats, rounded to 64 floats
    slot = -(-(1024 * 128 + 1024) // 64) * 64
    assert L.ws_peer_exchange_bytes(8, 1024, 128) == 1024 + 8 * slot * 4
    assert L.ws_peer_slot_offset(8, 1024, 128, 3) == 1024 + 3 * slot * 4
    assert L.ws_peer_exchange_bytes(0, 1024, 128) == 0 and L.ws_peer_exchange_bytes(65, 16, 128) == 0
    # scatter-merge form: 2 KB control block, one slot per rank of the largest share, then the gather area
    for world, rows, dim in ((8, 2048, 128), (2, 35, 128), (3, 1024, 512), (32, 1, 4)):
        share = -(-rows // world)
        sf = -(-(share * dim + share) // 64) * 64
        area = -(-(rows * dim + rows) // 64) * 64
        assert L.ws_peer_rs_bytes(world, rows, dim) == 2048 + world * sf * 4 + area * 4
    assert L.ws_peer_rs_bytes(33, 64, 128) == 0          # world > 32
    assert L.ws_peer_rs_bytes(2, 64, 6) == 0             # dim % 4 != 0
    # rejected before any launch: a rank 0 push, null pointers, an output dtype that is not bf16 / fp32
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    assert L.ws_peer_push(p, p, 2, 16, 128, 0, p, None) == 1
    assert L.ws_peer_rs_scatter(None, p, 2, 16, 128, 0, p, None) == 1
    assert L.ws_peer_rs_merge(p, p, 2, 16, 128, 0, p, None, 0, None, None) == 1   # rank 0 without out
    assert L.ws_peer_rs_merge(p, p, 2, 16, 128, 1, p, None, 7, None, None) == 1   # bad out dtype
    assert b"peer" in L.ws_last_error()
