"""ws_gqa_decode_noalloc: the GQA decode for callers that cannot allocate.

Some callers can give the library their inputs and outputs but no further
device memory: a serving process whose memory manager already holds the GPU's
free HBM for its KV-cache pool (a cudaMalloc would fail there, and it would
also synchronise the device in the middle of a decode loop), or a plugin host
that passes only tensors across its boundary.  For them the entry point keeps
the kernel's scratch in a built-in per-device array instead of a workspace.

These tests call it through the C ABI and compare it with ws_gqa_decode (the
workspace entry point) on two calls in a row -- the second call runs on
scratch that still holds the first call's contents -- within the tolerances
the other GPU tests use.  The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from scope_b200 import _lib

pytestmark = pytest.mark.gpu

TOL_OUT = 2e-2
TOL_LSE = 1e-3


def _inputs(B_kv, G, D, L, seed):
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    q = torch.randn(B_kv, G, D, device="cuda:0", generator=g).bfloat16()
    k = torch.randn(B_kv, L, D, device="cuda:0", generator=g).bfloat16()
    v = torch.randn(B_kv, L, D, device="cuda:0", generator=g).bfloat16()
    return q, k, v


def _with_workspace(q, k, v, scale):
    L_ = _lib.lib()
    B_kv, G, D = q.shape
    L = k.shape[1]
    out = torch.empty(B_kv, G, D, dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(B_kv, G, dtype=torch.float32, device=q.device)
    ws = torch.zeros(L_.ws_gqa_decode_workspace_size(B_kv, G, D, L), dtype=torch.uint8, device=q.device)
    rc = L_.ws_gqa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), v.stride(0),
                          v.stride(1), B_kv, G, D, D, L, scale, _lib.WS_DTYPE_BF16, _lib.WS_OUT_NORM_BF16,
                          out.data_ptr(), None, None, lse.data_ptr(), ws.data_ptr(), ws.numel(),
                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L_.ws_last_error()
    return out, lse


def _without_workspace(q, k, v, scale):
    L_ = _lib.lib()
    B_kv, G, D = q.shape
    L = k.shape[1]
    out = torch.empty(B_kv, G, D, dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(B_kv, G, dtype=torch.float32, device=q.device)
    rc = L_.ws_gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), v.stride(0),
                                  v.stride(1), B_kv, G, D, D, L, scale, _lib.WS_OUT_NORM_BF16,
                                  out.data_ptr(), None, None, lse.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L_.ws_last_error()
    return out, lse


@pytest.mark.parametrize("B_kv,G,D,L", [(4, 8, 128, 4096), (64, 8, 128, 20000)])
def test_noalloc_matches_workspace_entry_two_calls(B_kv, G, D, L):
    scale = D ** -0.5
    first = _inputs(B_kv, G, D, L, seed=1)
    second = _inputs(B_kv, G, D, L, seed=2)
    for q, k, v in (first, second):
        ref_out, ref_lse = _with_workspace(q, k, v, scale)
        out, lse = _without_workspace(q, k, v, scale)
        torch.cuda.synchronize()
        assert (out.float() - ref_out.float()).abs().max().item() < TOL_OUT
        assert (lse - ref_lse).abs().max().item() < TOL_LSE
    assert _lib.lib().ws_status_take(torch.cuda.current_stream().cuda_stream) == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    L_ = _lib.lib()
    cap = L_.ws_gqa_decode_noalloc_max_scratch()
    B_kv, G, D, L = 4096, 8, 128, 64
    assert L_.ws_gqa_decode_workspace_size(B_kv, G, D, L) > cap
    dummy = torch.empty(16, dtype=torch.bfloat16, device="cuda:0")
    p = dummy.data_ptr()
    rc = L_.ws_gqa_decode_noalloc(p, p, p, L * D, D, L * D, D, B_kv, G, D, D, L, 0.1, _lib.WS_OUT_NORM_BF16,
                                  p, None, None, None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.WS_ERR_WORKSPACE
    assert b"scratch" in L_.ws_last_error()
