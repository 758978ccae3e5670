"""Drop-in for the reference's `cpu_attn_ext` / `cpu_attn_tile_ext` modules.

The reference builds these with ``kernel/build.py:8-26`` /
``kernel/build_tile.py`` and binds them at ``kernel/cpu_attn.cpp:1024-1054``.
Same attribute names, positional/keyword signatures, output dtypes and
normalisation; the tensors are CUDA tensors instead of CPU tensors and every
call runs the sm_100a kernels of libscope_b200.so on the current stream.
There is no CPU fallback: a CPU tensor raises RuntimeError.

    ext = scope_b200.build()
    out, mx, sm = ext.fused_cpu_attn(q, k, v, scale)
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import check, lib, ptr, on_device, stream_ptr, workspaces

_num_threads = [0]


def _require_cuda(name: str, *ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name}: expected tensors")
        if not t.is_cuda:
            raise RuntimeError(f"{name}: scope_b200 ops take CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{name}: all tensors must be on the same device")
    return dev


def _gqa_common(name, q, k, v):
    dev = _require_cuda(name, q, k, v)
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise RuntimeError(f"{name}: q, k, v must be 3-D ([B_kv, G, D], [B_kv, L, D], [B_kv, L, Dv])")
    if not q.is_contiguous():
        raise RuntimeError("q must be contiguous")
    if k.stride(2) != 1 or v.stride(2) != 1:
        raise RuntimeError(f"{name}: k and v must have unit stride on the head dim")
    B, G, Dk = q.shape
    if k.shape[0] != B or v.shape[0] != B or k.shape[2] != Dk or k.shape[1] != v.shape[1]:
        raise RuntimeError(f"{name}: shape mismatch between q, k, v")
    return dev, B, G, Dk, k.shape[1], v.shape[2]


def _run_gqa(q, k, v, scale, dtype_code, out_mode, out, mx, sm, lse):
    dev = q.device
    B, G, Dk = q.shape
    L, Dv = k.shape[1], v.shape[2]
    L_ = lib()
    with on_device(dev):
        nbytes = L_.ws_gqa_decode_workspace_size(B, G, Dv, L)
        ws = workspaces.get(nbytes, dev)
        rc = L_.ws_gqa_decode(ptr(q), ptr(k), ptr(v), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
                              B, G, Dk, Dv, L, float(scale), dtype_code, out_mode,
                              ptr(out), ptr(mx), ptr(sm), ptr(lse), ptr(ws), ws.numel(), stream_ptr(dev))
    check(rc, "ws_gqa_decode")


def fused_cpu_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float):
    """GQA decode (kernel/cpu_attn.cpp:572-636).

    q [B_kv, G, D] contiguous, k/v [B_kv, L, D] with any strides on dims 0-1;
    fp32 or bf16 (all three alike); D % 16 == 0.
    Returns (out [B_kv, G, D] normalised, max [B_kv, G, 1], sum [B_kv, G, 1]),
    all bf16 for bf16 inputs and fp32 for fp32 inputs, like the reference.
    """
    if q.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("q must be float32 or bfloat16")
    if k.dtype != q.dtype:
        raise RuntimeError("k dtype must match q")
    if v.dtype != q.dtype:
        raise RuntimeError("v dtype must match q")
    dev, B, G, D, L, Dv = _gqa_common("fused_cpu_attn", q, k, v)
    if D % 16 != 0:
        raise RuntimeError("head_dim must be multiple of 16 for AVX512")
    if Dv != D:
        raise RuntimeError("fused_cpu_attn: k and v head dims must match (use fused_cpu_attn_mla)")
    if q.dtype == torch.bfloat16:
        out = torch.empty(B, G, D, dtype=torch.bfloat16, device=dev)
        mx = torch.empty(B, G, 1, dtype=torch.bfloat16, device=dev)
        sm = torch.empty(B, G, 1, dtype=torch.bfloat16, device=dev)
        _run_gqa(q, k, v, scale, _lib.WS_DTYPE_BF16, _lib.WS_OUT_NORM_BF16, out, mx, sm, None)
    else:
        out = torch.empty(B, G, D, dtype=torch.float32, device=dev)
        mx = torch.empty(B, G, 1, dtype=torch.float32, device=dev)
        sm = torch.empty(B, G, 1, dtype=torch.float32, device=dev)
        _run_gqa(q, k, v, scale, _lib.WS_DTYPE_F32, _lib.WS_OUT_NORM_F32, out, mx, sm, None)
    return out, mx, sm


def fused_cpu_attn_mla(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float):
    """Decode with k_head_dim != v_head_dim allowed (kernel/cpu_attn.cpp:638-672).

    bf16 only.  Returns fp32 (o NOT normalised [B_kv, G, Dv], max [B_kv, G, 1],
    sum [B_kv, G, 1]) like the reference; o / sum is the attention output and
    max + log(sum) its log-sum-exp.
    """
    if q.dtype != torch.bfloat16:
        raise RuntimeError("fused_cpu_attn_mla requires bf16 inputs")
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise RuntimeError("fused_cpu_attn_mla requires bf16 inputs")
    dev, B, G, Dk, L, Dv = _gqa_common("fused_cpu_attn_mla", q, k, v)
    out = torch.empty(B, G, Dv, dtype=torch.float32, device=dev)
    mx = torch.empty(B, G, 1, dtype=torch.float32, device=dev)
    sm = torch.empty(B, G, 1, dtype=torch.float32, device=dev)
    _run_gqa(q, k, v, scale, _lib.WS_DTYPE_BF16, _lib.WS_OUT_UNNORM_F32, out, mx, sm, None)
    return out, mx, sm


def fused_cpu_attn_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float):
    """fp32 decode (kernel/cpu_attn.cpp:817-848): (out normalised, max, sum), all fp32."""
    for t in (q, k, v):
        if t.dtype != torch.float32:
            raise RuntimeError("fused_cpu_attn_fp32 requires float32 inputs")
    dev, B, G, D, L, Dv = _gqa_common("fused_cpu_attn_fp32", q, k, v)
    out = torch.empty(B, G, D, dtype=torch.float32, device=dev)
    mx = torch.empty(B, G, 1, dtype=torch.float32, device=dev)
    sm = torch.empty(B, G, 1, dtype=torch.float32, device=dev)
    _run_gqa(q, k, v, scale, _lib.WS_DTYPE_F32, _lib.WS_OUT_NORM_F32, out, mx, sm, None)
    return out, mx, sm


def _run_mla(q_proj, q_pe, c_kv, k_pe, scale, out_mode, out, mx, sm, lse):
    """One ws_mla_decode_strided launch.  c_kv / k_pe may be views of a larger
    cache (unit stride on the feature dim, tokens contiguous, any batch
    stride).  A head count that is not a multiple of 16 runs on zero-padded
    query rows; the padded rows' outputs are dropped."""
    dev = _require_cuda("fused_cpu_attn_mla_compressed", q_proj, q_pe, c_kv, k_pe)
    for t in (q_proj, q_pe, c_kv, k_pe):
        if t.dtype != torch.bfloat16:
            raise RuntimeError("fused_cpu_attn_mla_compressed requires bf16 inputs")
    if not q_proj.is_contiguous() or not q_pe.is_contiguous():
        raise RuntimeError("q_proj and q_pe must be contiguous")
    if c_kv.dim() != 3 or k_pe.dim() != 3:
        raise RuntimeError("expected c_kv [B, S, 512] and k_pe [B, S, 64]")
    B, S, CLR = c_kv.shape
    if B == 0 or q_proj.shape[0] % B:
        raise RuntimeError("q_proj rows must be a multiple of the batch")
    nH = q_proj.shape[0] // B
    if not (q_proj.shape[1] == 512 and q_pe.shape[1] == 64 and CLR == 512 and k_pe.shape[2] == 64):
        raise RuntimeError("expected q_proj [B*nH, 512], q_pe [B*nH, 64], c_kv [B, S, 512], k_pe [B, S, 64]")
    if q_pe.shape[0] != B * nH or k_pe.shape[0] != B or k_pe.shape[1] != S:
        raise RuntimeError("shape mismatch between q_proj, q_pe, c_kv, k_pe")
    for t, w in ((c_kv, 512), (k_pe, 64)):
        rows_ok = t.stride(2) == 1 and (S <= 1 or t.stride(1) == w)
        if not rows_ok or (B > 1 and (t.stride(0) % 8 or t.stride(0) < S * w)):
            raise RuntimeError("c_kv and k_pe must be contiguous per sequence (batch stride a multiple of 8)")
    c_bs = c_kv.stride(0) if B > 1 else S * 512
    pe_bs = k_pe.stride(0) if B > 1 else S * 64
    nHp = -(-nH // 16) * 16
    if nHp != nH:   # zero query rows up to a multiple of 16 heads; outputs go through padded buffers
        qp = torch.zeros(B, nHp, 512, dtype=q_proj.dtype, device=dev)
        qp[:, :nH] = q_proj.view(B, nH, 512)
        qe = torch.zeros(B, nHp, 64, dtype=q_pe.dtype, device=dev)
        qe[:, :nH] = q_pe.view(B, nH, 64)

        def wide(t, tail):
            return None if t is None else torch.empty(B, nHp, *tail, dtype=t.dtype, device=dev)
        wo, wm, ws_, wl = wide(out, (512,)), wide(mx, ()), wide(sm, ()), wide(lse, ())
        _run_mla(qp.view(B * nHp, 512), qe.view(B * nHp, 64), c_kv, k_pe, scale, out_mode,
                 wo.view(B * nHp, 512), None if wm is None else wm.view(-1), None if ws_ is None else ws_.view(-1),
                 None if wl is None else wl.view(-1))
        out.view(B, nH, 512).copy_(wo[:, :nH])
        for dst, src in ((mx, wm), (sm, ws_), (lse, wl)):
            if dst is not None:
                dst.view(B, nH).copy_(src[:, :nH])
        return
    L_ = lib()
    with on_device(dev):
        ws = workspaces.get(L_.ws_mla_decode_workspace_size(B, nH, S), dev)
        rc = L_.ws_mla_decode_strided(ptr(q_proj), ptr(q_pe), ptr(c_kv), c_bs, ptr(k_pe), pe_bs, B, nH, S,
                                      float(scale), out_mode, ptr(out), ptr(mx), ptr(sm), ptr(lse), ptr(ws),
                                      ws.numel(), stream_ptr(dev))
    check(rc, "ws_mla_decode")


def fused_cpu_attn_mla_compressed(q_proj: torch.Tensor, q_pe: torch.Tensor, c_kv: torch.Tensor,
                                  k_pe: torch.Tensor, scale: float):
    """Absorbed MLA decode (kernel/cpu_attn.cpp:852-1022).

    q_proj [B*nH, 512], q_pe [B*nH, 64], c_kv [B, S, 512], k_pe [B, S, 64], bf16.
    Returns fp32 (o NOT normalised [B*nH, 512], max [B*nH], sum [B*nH]) like the
    reference; o / sum[:, None] is the attention output over the latent.
    """
    B, S, _ = c_kv.shape
    R = q_proj.shape[0]
    dev = c_kv.device
    out = torch.empty(R, 512, dtype=torch.float32, device=dev)
    mx = torch.empty(R, dtype=torch.float32, device=dev)
    sm = torch.empty(R, dtype=torch.float32, device=dev)
    _run_mla(q_proj, q_pe, c_kv, k_pe, scale, _lib.WS_OUT_UNNORM_F32, out, mx, sm, None)
    return out, mx, sm


def mla_decode(q_proj: torch.Tensor, q_pe: torch.Tensor, c_kv: torch.Tensor, k_pe: torch.Tensor, scale: float,
               out_dtype=torch.bfloat16, out: torch.Tensor | None = None, lse: torch.Tensor | None = None):
    """Absorbed MLA decode returning (out [B*nH, 512] normalised in out_dtype
    (bf16, or fp32: the partial a sharded cache exchanges), lse fp32 [B*nH]).
    ``out`` / ``lse`` may be given (contiguous, of those shapes) to be written
    in place."""
    R = q_proj.shape[0]
    dev = c_kv.device
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError("mla_decode: out_dtype must be bf16 or fp32")
    out = torch.empty(R, 512, dtype=out_dtype, device=dev) if out is None else out
    lse = torch.empty(R, dtype=torch.float32, device=dev) if lse is None else lse
    if out.dtype != out_dtype or out.numel() != R * 512 or not out.is_contiguous() or lse.numel() != R \
            or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise RuntimeError("mla_decode: out / lse must be contiguous [B*nH, 512] out_dtype and [B*nH] fp32")
    mode = _lib.WS_OUT_NORM_BF16 if out_dtype == torch.bfloat16 else _lib.WS_OUT_NORM_F32
    _run_mla(q_proj, q_pe, c_kv, k_pe, scale, mode, out, None, None, lse)
    return out, lse


def mla_decode_absorbed(q_nope: torch.Tensor, q_pe: torch.Tensor, c_kv: torch.Tensor, k_pe: torch.Tensor,
                        kv_b_proj_weight: torch.Tensor, scale: float, return_lse: bool = False):
    """The decode branch of the reference's absorbed MLA forward with the projections
    either side of the attention (system/deepseek.py:257-265 absorb, :355-404 attention
    and merge, :405-407 up-projection), on the GPU:

        q_proj = q_nope . W_UK ;  o = attention over (c_kv, k_pe) ;  out = bf16(o) . W_UV^T

    q_nope [B, nH, nop] (or [B, nH, 1, nop]), q_pe [B, nH, 64] (or [B*nH, 64] / [B, nH, 1, 64]),
    c_kv [B, S, 512], k_pe [B, S, 64], kv_b_proj_weight [nH * (nop + vhd), 512], all bf16.
    Returns out [B, nH, vhd] bf16 (and lse [B, nH] fp32 with return_lse)."""
    dev = _require_cuda("mla_decode_absorbed", q_nope, q_pe, c_kv, k_pe, kv_b_proj_weight)
    for t in (q_nope, q_pe, c_kv, k_pe, kv_b_proj_weight):
        if t.dtype != torch.bfloat16:
            raise RuntimeError("mla_decode_absorbed requires bf16 inputs")
    B, S, CLR = c_kv.shape
    if CLR != 512 or k_pe.shape != (B, S, 64):
        raise RuntimeError("expected c_kv [B, S, 512] and k_pe [B, S, 64]")
    nH = q_nope.shape[1]
    nop = q_nope.shape[-1]
    qn = q_nope.reshape(B, nH, nop).contiguous()
    qpe = q_pe.reshape(B * nH, 64).contiguous()
    w = kv_b_proj_weight if kv_b_proj_weight.is_contiguous() else kv_b_proj_weight.contiguous()
    w = w.reshape(nH, -1, 512)
    vhd = w.shape[1] - nop
    if vhd < 1:
        raise RuntimeError("kv_b_proj_weight must hold nH x (nop + vhd) rows of 512")
    hs = (nop + vhd) * 512   # W_UK and W_UV are read in place: head blocks at this stride
    # the latent may be a view of a [B, cap, *] cache: read in place through its batch stride when the
    # tokens of each sequence are contiguous, else copied
    def seq_contiguous(t, w):
        return t.stride(2) == 1 and (S <= 1 or t.stride(1) == w) and (B <= 1 or (t.stride(0) % 8 == 0
                                                                                   and t.stride(0) >= S * w))
    if not seq_contiguous(c_kv, 512):
        c_kv = c_kv.contiguous()
    if not seq_contiguous(k_pe, 64):
        k_pe = k_pe.contiguous()
    c_bs = c_kv.stride(0) if B > 1 else S * 512
    pe_bs = k_pe.stride(0) if B > 1 else S * 64
    out = torch.empty(B, nH, vhd, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, nH, dtype=torch.float32, device=dev) if return_lse else None
    L_ = lib()
    with on_device(dev):
        ws = workspaces.get(L_.ws_mla_decode_absorbed_workspace_size(B, nH, S), dev)
        rc = L_.ws_mla_decode_absorbed_strided(ptr(qn), w.data_ptr(), hs, ptr(qpe), ptr(c_kv), c_bs, ptr(k_pe), pe_bs,
                                               w.data_ptr() + nop * 512 * 2, hs, B, nH, S, nop, vhd, float(scale),
                                               ptr(out), ptr(lse), ptr(ws), ws.numel(), stream_ptr(dev))
    check(rc, "ws_mla_decode_absorbed")
    return (out, lse) if return_lse else out


def gqa_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, out_dtype=torch.bfloat16,
               out: torch.Tensor | None = None, lse: torch.Tensor | None = None):
    """GQA decode returning (out [B_kv, G, Dv] normalised in out_dtype (bf16 or fp32),
    lse fp32 [B_kv, G]).

    The fp32 log-sum-exp (max + log sum) is what the LSE merges consume; the
    reference's bf16 fused_cpu_attn rounds max and sum to bf16 (~1e-2 LSE error).
    An fp32 out is the partial a sharded cache exchanges.  ``out`` / ``lse``
    may be given (contiguous, of those shapes) to be written in place.
    """
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise RuntimeError("gqa_decode requires bf16 inputs")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError("gqa_decode: out_dtype must be bf16 or fp32")
    dev, B, G, Dk, L, Dv = _gqa_common("gqa_decode", q, k, v)
    out = torch.empty(B, G, Dv, dtype=out_dtype, device=dev) if out is None else out
    lse = torch.empty(B, G, dtype=torch.float32, device=dev) if lse is None else lse
    if out.dtype != out_dtype or out.numel() != B * G * Dv or not out.is_contiguous() or lse.numel() != B * G \
            or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise RuntimeError("gqa_decode: out / lse must be contiguous [B_kv, G, Dv] out_dtype and [B_kv, G] fp32")
    mode = _lib.WS_OUT_NORM_BF16 if out_dtype == torch.bfloat16 else _lib.WS_OUT_NORM_F32
    _run_gqa(q, k, v, scale, _lib.WS_DTYPE_BF16, mode, out, None, None, lse)
    return out, lse


def set_num_threads(n: int) -> None:
    """Kept for API compatibility (kernel/cpu_attn.cpp:1046-1050).  The GPU
    kernels size their grids from the SM count; the value is only remembered."""
    _num_threads[0] = int(n)


def get_num_threads() -> int:
    """Last value given to set_num_threads, else the device's SM count."""
    if _num_threads[0] > 0:
        return _num_threads[0]
    if torch.cuda.is_available():
        return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return 1


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
