"""Entry points beyond the reference's extension surface: the ragged
multi-share decode with fused LSE merge, and the standalone LSE merge.

These replace the runtime-side pieces around the reference kernels: the
per-share ``fused_cpu_attn`` calls and the Python log-sum-exp merges of
``system/mixoffload.py:1263-1268, :1333-1334, :1456-1464`` and
``system/qwenoffload.py:1606-1617``.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _lib
from ._lib import KvShare, check, lib, ptr, on_device, stream_ptr, workspaces


class Share:
    """One physical KV share of a ragged batch, in one of two layouts.

    packed -- ``Share(k, v, cu_seqlens=cu)``: k, v [n_tok, Hkv, D] bf16 (any
        strides on the first two dims, e.g. a token-major buffer or the
        transpose of a head-major [Hkv, n_tok, D] one); cu int32 [B+1]:
        sequence b owns tokens [cu[b], cu[b+1]).
    padded -- ``Share(k, v, seqlens=lens)``: k, v [B*Hkv, cap, D] bf16, one
        capacity-sized row per (sequence, kv-head) like the reference's
        InplaceKVCache (system/qwenoffload.py:59-141); lens int32 [B]: tokens
        [0, lens[b]) of rows b*Hkv .. b*Hkv+Hkv-1 are valid.
    Length arrays live on the same device as k and v.
    """

    __slots__ = ("k", "v", "cu_seqlens", "seqlens")

    def __init__(self, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor | None = None,
                 seqlens: torch.Tensor | None = None):
        if (cu_seqlens is None) == (seqlens is None):
            raise ValueError("Share: give exactly one of cu_seqlens (packed) or seqlens (padded)")
        self.k, self.v, self.cu_seqlens, self.seqlens = k, v, cu_seqlens, seqlens

    @property
    def padded(self) -> bool:
        return self.seqlens is not None


def gqa_decode_shares(q: torch.Tensor, shares: Sequence[Share], scale: float,
                      out: torch.Tensor | None = None, lse: torch.Tensor | None = None):
    """Ragged-batch GQA decode over up to 4 KV shares per sequence, merged by
    log-sum-exp in the same launch.

    q [B, H, Dk] bf16 contiguous with H = Hkv * G (head h = kvh * G + g).
    Returns (out bf16 [B, H, Dv] normalised, lse fp32 [B, H]).
    """
    if not q.is_cuda or q.dtype != torch.bfloat16 or q.dim() != 3 or not q.is_contiguous():
        raise RuntimeError("gqa_decode_shares: q must be a contiguous bf16 CUDA tensor [B, H, Dk]")
    if not 1 <= len(shares) <= 4:
        raise RuntimeError("gqa_decode_shares: 1 to 4 shares")
    B, H, Dk = q.shape
    s0 = shares[0]
    Hkv = s0.k.shape[0] // B if s0.padded else s0.k.shape[1]
    Dv = s0.v.shape[2]
    if Hkv < 1 or H % Hkv:
        raise RuntimeError("gqa_decode_shares: query heads must be a multiple of KV heads")
    G = H // Hkv
    dev = q.device
    arr = (KvShare * len(shares))()
    for i, s in enumerate(shares):
        lens = s.seqlens if s.padded else s.cu_seqlens
        for t in (s.k, s.v, lens):
            if not t.is_cuda or t.device != dev:
                raise RuntimeError("gqa_decode_shares: all tensors must be on q's device")
        if s.k.dtype != torch.bfloat16 or s.v.dtype != torch.bfloat16:
            raise RuntimeError("gqa_decode_shares: k/v must be bf16")
        if s.k.dim() != 3 or s.v.dim() != 3 or s.k.shape[2] != Dk or s.v.shape[2] != Dv:
            raise RuntimeError("gqa_decode_shares: k/v must be 3-D with head dims Dk / Dv")
        if s.k.shape[:2] != s.v.shape[:2]:
            raise RuntimeError("gqa_decode_shares: k/v shape mismatch")
        if s.k.stride(2) != 1 or s.v.stride(2) != 1:
            raise RuntimeError("gqa_decode_shares: unit stride on the head dim required")
        if lens.dtype != torch.int32:
            raise RuntimeError("gqa_decode_shares: length arrays must be int32")
        if s.padded:
            if s.k.shape[0] != B * Hkv or lens.numel() != B:
                raise RuntimeError("gqa_decode_shares: padded share must be [B*Hkv, cap, D] with seqlens [B]")
            arr[i] = KvShare(ptr(s.k), ptr(s.v), None, ptr(lens), s.k.shape[1],
                             s.k.stride(1), s.k.stride(0), s.v.stride(1), s.v.stride(0))
        else:
            if s.k.shape[1] != Hkv or lens.numel() != B + 1:
                raise RuntimeError("gqa_decode_shares: packed share must be [n_tok, Hkv, D] with cu_seqlens [B+1]")
            arr[i] = KvShare(ptr(s.k), ptr(s.v), ptr(lens), None, s.k.shape[0],
                             s.k.stride(0), s.k.stride(1), s.v.stride(0), s.v.stride(1))
    if out is None:
        out = torch.empty(B, H, Dv, dtype=torch.bfloat16, device=dev)
    if lse is None:
        lse = torch.empty(B, H, dtype=torch.float32, device=dev)
    L_ = lib()
    with on_device(dev):
        nbytes = L_.ws_gqa_decode_shares_workspace_size(B, Hkv, G, Dv, len(shares))
        ws = workspaces.get(nbytes, dev)
        rc = L_.ws_gqa_decode_shares(ptr(q), B, Hkv, G, Dk, Dv, float(scale), arr, len(shares),
                                     ptr(out), ptr(lse), ptr(ws), ws.numel(), stream_ptr(dev))
    check(rc, "ws_gqa_decode_shares")
    return out, lse


def lse_merge(o_parts: torch.Tensor, lse_parts: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
              out: torch.Tensor | None = None, out_lse: torch.Tensor | None = None):
    """Merge P normalised partials: o_parts [P, R, D] fp32, lse_parts [P, R] fp32.

    Returns (out [R, D] in out_dtype, lse [R] fp32).  Leading dims after P may
    be any shape; they are flattened into R.
    """
    if not (o_parts.is_cuda and lse_parts.is_cuda):
        raise RuntimeError("lse_merge: CUDA tensors required (there is no CPU path)")
    if o_parts.dtype != torch.float32 or lse_parts.dtype != torch.float32:
        raise RuntimeError("lse_merge: fp32 partials required")
    P = o_parts.shape[0]
    D = o_parts.shape[-1]
    lead = o_parts.shape[1:-1]
    o_c = o_parts.contiguous().view(P, -1, D)
    l_c = lse_parts.contiguous().view(P, -1)
    R = o_c.shape[1]
    if l_c.shape[1] != R:
        raise RuntimeError("lse_merge: lse_parts must match o_parts' leading dims")
    dev = o_parts.device
    if out is None:
        out = torch.empty(*lead, D, dtype=out_dtype, device=dev)
    if out_lse is None:
        out_lse = torch.empty(*lead, dtype=torch.float32, device=dev)
    code = _lib.WS_DTYPE_BF16 if out.dtype == torch.bfloat16 else _lib.WS_DTYPE_F32
    with on_device(dev):
        rc = lib().ws_lse_merge(ptr(o_c), ptr(l_c), P, R, D, ptr(out), code, ptr(out_lse), stream_ptr(dev))
    check(rc, "ws_lse_merge")
    return out, out_lse
