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


def _inputs(B_kv, G, Dk, Dv, L, seed):
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    q = torch.randn(B_kv, G, Dk, device="cuda:0", generator=g).bfloat16()
    k = torch.randn(B_kv, L, Dk, device="cuda:0", generator=g).bfloat16()
    v = torch.randn(B_kv, L, Dv, device="cuda:0", generator=g).bfloat16()
    return q, k, v


def _outputs(q, Dv, mode):
    B_kv, G, _ = q.shape
    odt = torch.bfloat16 if mode == _lib.WS_OUT_NORM_BF16 else torch.float32
    out = torch.empty(B_kv, G, Dv, dtype=odt, device=q.device)
    lse = torch.empty(B_kv, G, dtype=torch.float32, device=q.device)
    mx = sm = None
    if mode == _lib.WS_OUT_UNNORM_F32:   # the fused_cpu_attn_mla outputs: un-normalised o, max and sum
        mx = torch.empty(B_kv, G, dtype=torch.float32, device=q.device)
        sm = torch.empty(B_kv, G, dtype=torch.float32, device=q.device)
    return out, mx, sm, lse


def _ptr(t):
    return None if t is None else t.data_ptr()


def _with_workspace(q, k, v, scale, mode):
    L_ = _lib.lib()
    B_kv, G, Dk = q.shape
    L, Dv = k.shape[1], v.shape[2]
    out, mx, sm, lse = _outputs(q, Dv, mode)
    ws = torch.zeros(L_.ws_gqa_decode_workspace_size(B_kv, G, Dv, L), dtype=torch.uint8, device=q.device)
    rc = L_.ws_gqa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), v.stride(0),
                          v.stride(1), B_kv, G, Dk, Dv, L, scale, _lib.WS_DTYPE_BF16, mode,
                          out.data_ptr(), _ptr(mx), _ptr(sm), lse.data_ptr(), ws.data_ptr(), ws.numel(),
                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L_.ws_last_error()
    return out, mx, sm, lse


def _without_workspace(q, k, v, scale, mode):
    L_ = _lib.lib()
    B_kv, G, Dk = q.shape
    L, Dv = k.shape[1], v.shape[2]
    out, mx, sm, lse = _outputs(q, Dv, mode)
    rc = L_.ws_gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), v.stride(0),
                                  v.stride(1), B_kv, G, Dk, Dv, L, scale, mode,
                                  out.data_ptr(), _ptr(mx), _ptr(sm), lse.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L_.ws_last_error()
    return out, mx, sm, lse


CASES = [
    # (B_kv, G, Dk, Dv, L, out_mode): a short row (in-launch ticket merge), long rows (deferred merge),
    # 16 heads per kv row (two MMA column tiles) with the 192/128 MLA head dims, the un-normalised
    # fused_cpu_attn_mla outputs with max and sum, and an empty cache
    (4, 8, 128, 128, 4096, _lib.WS_OUT_NORM_BF16),
    (64, 8, 128, 128, 20000, _lib.WS_OUT_NORM_BF16),
    (8, 16, 192, 128, 3000, _lib.WS_OUT_NORM_F32),
    (16, 8, 128, 128, 5000, _lib.WS_OUT_UNNORM_F32),
    (4, 8, 128, 128, 0, _lib.WS_OUT_NORM_BF16),
]


@pytest.mark.parametrize("B_kv,G,Dk,Dv,L,mode", CASES)
def test_noalloc_matches_workspace_entry_two_calls(B_kv, G, Dk, Dv, L, mode):
    scale = Dk ** -0.5
    first = _inputs(B_kv, G, Dk, Dv, L, seed=1)
    second = _inputs(B_kv, G, Dk, Dv, L, seed=2)
    for q, k, v in (first, second):
        ref = _with_workspace(q, k, v, scale, mode)
        got = _without_workspace(q, k, v, scale, mode)
        torch.cuda.synchronize()
        r_out, r_mx, r_sm, r_lse = ref
        out, mx, sm, lse = got
        if mode == _lib.WS_OUT_UNNORM_F32:   # compare the normalised rows and the max / log-sum
            assert (mx - r_mx).abs().max().item() < TOL_LSE
            assert (sm.log() - r_sm.log()).abs().max().item() < TOL_LSE
            out, r_out = out / sm[..., None], r_out / r_sm[..., None]
        if L == 0:
            assert torch.isneginf(lse).all() and torch.isneginf(r_lse).all()
            assert (out.float() == 0).all() and (r_out.float() == 0).all()
            continue
        assert (out.float() - r_out.float()).abs().max().item() < TOL_OUT
        assert (lse - r_lse).abs().max().item() < TOL_LSE
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
