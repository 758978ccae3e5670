"""scope_b200 -- B200-native (sm_100a) decode attention for physically
partitioned KV caches.

Reference-compatible loaders (the reference binds its CPU kernels through
``kernel/build.py:build``, ``kernel/build_tile.py:build`` and
``kernel/cpu_attn_ds4_ext/build.py:build_csa_attn``):

    ext = scope_b200.build()            # fused_cpu_attn, fused_cpu_attn_mla, ...
    csa = scope_b200.build_csa_attn()   # fused_csa_attn, indexer_attn_cpu, ...

Both return modules with the reference's attribute names and signatures that
run on CUDA tensors through libscope_b200.so.  There is no CPU fallback.
"""
from __future__ import annotations

import os

from . import cpu_attn as _cpu_attn
from ._lib import LIB_PATH, ScopeError, lib
from .ops import Share, gqa_decode_shares, lse_merge

__all__ = ["build", "build_tile", "build_csa_attn", "lib", "ScopeError", "Share", "gqa_decode_shares", "lse_merge",
           "status_take"]


def _ensure_library(verbose: bool = False) -> None:
    if not os.path.exists(LIB_PATH):
        from .compile_lib import build as _build_lib
        _build_lib(verbose=verbose)


def build(verbose: bool = False):
    """Mirror of the reference's ``kernel/build.py:build``: returns the module
    exposing fused_cpu_attn, fused_cpu_attn_mla, fused_cpu_attn_fp32,
    fused_cpu_attn_mla_compressed, set_num_threads, get_num_threads."""
    _ensure_library(verbose)
    lib()
    return _cpu_attn


def build_tile(verbose: bool = False):
    """Mirror of ``kernel/build_tile.py:build`` (the MLA_TILE variant).  The
    token tile of the GPU kernel is fixed by its pipeline, so this returns the
    same module as build()."""
    return build(verbose)


def build_csa_attn():
    """Mirror of ``kernel/cpu_attn_ds4_ext/build.py:build_csa_attn``."""
    _ensure_library(False)
    lib()
    from . import csa_attn as _csa_attn
    return _csa_attn


def status_take(device=None) -> int:
    """Read and clear the device status word of ``device`` (synchronises its
    current stream): 0 when no kernel reported a problem since the last call,
    else WS_ERR_DEVICE (5): a bounded wait gave up, or a CSA id outside the
    KV buffer was skipped.  On WS_ERR_DEVICE the device's pooled workspaces
    are dropped, so the next launch runs on a freshly zeroed one (a launch
    that gave up may have left a merge counter set)."""
    import torch
    from ._lib import workspaces
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        rc = int(lib().ws_status_take(torch.cuda.current_stream(dev).cuda_stream))
    if rc != 0:
        workspaces.drop_device(dev.index if dev.index is not None else torch.cuda.current_device())
    return rc
