"""Drop-in for the reference's `csa_attn_kernel` module
(kernel/cpu_attn_ds4_ext/csa_attn.cpp:1885-1977), on CUDA tensors.

Same attribute names and positional/keyword signatures (``n_threads=0`` kept
and ignored), same output dtypes (fp32 normalised ``o``, fp32 ``lse``), same
in-place behaviour for the ``_bsq*`` / ``_inplace`` / ``indexer_attn_cpu``
variants.  Every attention entry runs the one tcgen05 CSA kernel of
libscope_b200.so (``ws_csa_decode``): bf16 or int8+scale entries, gathered by
top-k ids or over a dense range; its workspace comes from the per-stream pool.
There is no CPU path: CPU tensors raise.

Arithmetic:
  * an fp32 query is held as two bf16 parts (hi + lo) inside the kernel, so
    the scores keep ~16 mantissa bits of it (fp32 accumulation); a bf16 query
    is used as it is;
  * the int8 operators (``_bsq_int8``, ``_int8_preq``, ``_int8_full``) compute
    the reference's own integer score: the query quantised to u8 codes
    (bit-exact with the reference's quantiser), the exact integer dot with the
    s8 entry codes less ``128 * kv_sums``, times the query scale, the entry
    scale and the softmax scale (``ws_csa_decode_qcodes``);
  * ``fused_csa_attn_int8_exact`` is the one addition: int8 entries attended
    with an unquantised query (``value = int8 * scale`` in both products), the
    arithmetic the cfg5 sparse decode uses.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, on_device, stream_ptr, workspaces
from .cpu_attn import _require_cuda, get_num_threads, set_num_threads  # noqa: F401

HD = 512

_IDX_MODES = {"all": _lib.WS_CSA_IDX_ALL, "sorted_shard": _lib.WS_CSA_IDX_SORTED_SHARD,
              "shard": _lib.WS_CSA_IDX_SHARD}


_EMPTY_IDS: dict = {}


def _nonempty_ids(dev):
    t = _EMPTY_IDS.get(dev)
    if t is None:
        t = _EMPTY_IDS[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
    return t


def _launch(q, kv, scale, out, lse, *, idx=None, kv_scales=None, kv_range=None, shard_lo=0, idx_mode="all"):
    """q [bs, nq..., hd] (fp32 or bf16), kv [bs, nc, hd] (bf16 or int8), out like q's rows."""
    dev = _require_cuda("csa", q, kv, out, lse, *(t for t in (idx, kv_scales) if t is not None))
    bs, hd = q.shape[0], q.shape[-1]
    nq = q.numel() // max(1, bs * hd) if bs else 0
    nc = kv.shape[1]
    if hd > HD or hd % 16 or hd == 0:
        raise RuntimeError(f"csa: head_dim must be a multiple of 16 and at most {HD} (got {hd})")
    if kv.dim() != 3 or kv.shape[0] != bs or kv.shape[2] != hd:
        raise RuntimeError("kv shape mismatch")
    for name, t in (("q", q), ("kv", kv), ("o_out", out), ("lse_out", lse)):
        if not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous")
    if out.numel() != bs * nq * hd or lse.numel() != bs * nq:
        raise RuntimeError("o_out / lse_out shape mismatch")
    if hd < HD:
        # the kernel's latent is 512 wide: narrower heads run on zero-padded copies (zero dims add
        # nothing to a score or to an output row); the result's first hd dims are copied back
        if bs == 0 or nq == 0:
            return
        wide = torch.empty(bs, nq, HD, dtype=out.dtype, device=dev)
        _launch(_pad_dims(q.reshape(bs, nq, hd), HD), _pad_dims(kv, HD), scale, wide, lse, idx=idx,
                kv_scales=kv_scales, kv_range=kv_range, shard_lo=shard_lo, idx_mode=idx_mode)
        out.view(bs, nq, hd).copy_(wide[..., :hd])
        return
    if lse.dtype != torch.float32:
        raise RuntimeError("lse_out must be float32")
    q_code = {torch.float32: _lib.WS_DTYPE_F32, torch.bfloat16: _lib.WS_DTYPE_BF16}.get(q.dtype)
    kv_code = {torch.bfloat16: _lib.WS_DTYPE_BF16, torch.int8: _lib.WS_DTYPE_I8}.get(kv.dtype)
    out_code = {torch.float32: _lib.WS_DTYPE_F32, torch.bfloat16: _lib.WS_DTYPE_BF16}.get(out.dtype)
    if q_code is None or kv_code is None or out_code is None:
        raise RuntimeError("q must be fp32/bf16, kv bf16/int8, o_out fp32/bf16")
    if kv_code == _lib.WS_DTYPE_I8:
        if kv_scales is None or kv_scales.dtype != torch.float32 or kv_scales.shape != (bs, nc) \
                or not kv_scales.is_contiguous():
            raise RuntimeError("int8 kv needs contiguous float32 kv_scales [bs, nc]")
    k = 0
    if idx is not None:
        if idx.dtype != torch.int32 or idx.dim() != 2 or idx.shape[0] != bs or not idx.is_contiguous():
            raise RuntimeError("topk_idxs must be contiguous int32 [bs, k]")
        k = idx.shape[1]
        if k == 0:   # an empty id list still selects the gather form (a null pointer means dense)
            idx = _nonempty_ids(dev)
    kv_s, kv_e = kv_range if kv_range is not None else (shard_lo, shard_lo + nc)
    if bs == 0 or nq == 0:
        return
    with on_device(dev):
        L_ = lib()
        ws = workspaces.get(L_.ws_csa_decode_workspace_size(bs, nq, q_code), dev)
        rc = L_.ws_csa_decode(ptr(q), q_code, bs, nq, hd, ptr(kv), kv_code, ptr(kv_scales), nc, int(shard_lo),
                              ptr(idx), k, _IDX_MODES[idx_mode], int(kv_s), int(kv_e), float(scale),
                              ptr(out), out_code, ptr(lse), ptr(ws), ws.numel(), stream_ptr(dev))
    check(rc, "ws_csa_decode")


def _new_outputs(q):
    bs, nh, sq, hd = q.shape
    o = torch.empty((bs, nh, sq, hd), dtype=torch.float32, device=q.device)
    lse = torch.empty((bs, nh, sq), dtype=torch.float32, device=q.device)
    return o, lse


def _check_dense(q, kv, q_dtype=None):
    _require_cuda("fused_csa_attn", q, kv)
    if q.dim() != 4:
        raise RuntimeError("q must be 4D")
    if kv.dim() != 3:
        raise RuntimeError("kv must be 3D")
    if q_dtype is not None and q.dtype != q_dtype:
        raise RuntimeError(f"q must be {'fp32' if q_dtype == torch.float32 else 'bf16'}")
    if kv.dtype != torch.bfloat16:
        raise RuntimeError("kv must be bf16")
    if not q.is_contiguous() or not kv.is_contiguous():
        raise RuntimeError("must be contiguous")
    if kv.shape[0] != q.shape[0]:
        raise RuntimeError("kv batch mismatch")
    if kv.shape[2] != q.shape[3]:
        raise RuntimeError("kv head_dim mismatch")
    if q.shape[3] % 16:
        raise RuntimeError("head_dim must be multiple of 16")


# ---------------------------------------------------------------- dense family
def fused_csa_attn(q: torch.Tensor, kv: torch.Tensor, scale: float):
    """Dense CSA (csa_attn.cpp:200-281): q fp32 [bs, nH, sq, hd], kv bf16 [bs, nc, hd]
    -> (o fp32 [bs, nH, sq, hd] normalised, lse fp32 [bs, nH, sq])."""
    _check_dense(q, kv, torch.float32)
    o, lse = _new_outputs(q)
    _launch(q, kv, scale, o, lse)
    return o, lse


def fused_csa_attn_pool(q: torch.Tensor, kv: torch.Tensor, scale: float, n_threads: int = 0):
    """Thread-pool form of fused_csa_attn (csa_attn.cpp:283-377); same result."""
    return fused_csa_attn(q, kv, scale)


def fused_csa_attn_pool_bf16(q: torch.Tensor, kv: torch.Tensor, scale: float, n_threads: int = 0):
    """bf16-query form (csa_attn.cpp:379-474); outputs fp32."""
    _check_dense(q, kv, torch.bfloat16)
    o, lse = _new_outputs(q)
    _launch(q, kv, scale, o, lse)
    return o, lse


def fused_csa_attn_range(q: torch.Tensor, kv: torch.Tensor, scale: float, kv_s: int, kv_e: int):
    """Dense CSA over kv[:, kv_s:kv_e] (csa_attn.cpp:1587-1656)."""
    _require_cuda("fused_csa_attn_range", q, kv)
    if not q.is_contiguous() or not kv.is_contiguous():
        raise RuntimeError("must be contiguous")
    if not (kv_s >= 0 and kv_e <= kv.shape[1] and kv_s < kv_e):
        raise RuntimeError("invalid kv range")
    if q.dtype != torch.float32:
        raise RuntimeError("q must be fp32")
    o = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=q.device)
    _launch(q, kv, scale, o, lse, kv_range=(kv_s, kv_e))
    return o, lse


def _inplace(q, kv, scale, o_out, lse_out, q_dtype=None):
    _require_cuda("fused_csa_attn", q, kv, o_out, lse_out)
    if not q.is_contiguous() or not kv.is_contiguous():
        raise RuntimeError("q/kv must be contiguous")
    if not o_out.is_contiguous() or not lse_out.is_contiguous():
        raise RuntimeError("o/lse must be contiguous")
    if q_dtype is not None and q.dtype != q_dtype:
        raise RuntimeError("q must be bf16" if q_dtype == torch.bfloat16 else "q must be fp32")
    if kv.dtype != torch.bfloat16:
        raise RuntimeError("kv must be bf16")
    if q.shape[-1] % 16:
        raise RuntimeError("head_dim must be multiple of 16")
    _launch(q, kv, scale, o_out, lse_out)


def fused_csa_attn_bsq(q, kv, scale, o_out, lse_out, n_threads: int = 0) -> None:
    """In-place dense CSA, fp32 q (csa_attn.cpp:476-578)."""
    _inplace(q, kv, scale, o_out, lse_out, torch.float32)


def fused_csa_attn_bsq_bf16(q, kv, scale, o_out, lse_out, n_threads: int = 0) -> None:
    """In-place dense CSA, bf16 q (csa_attn.cpp:580-764)."""
    _inplace(q, kv, scale, o_out, lse_out, torch.bfloat16)


def fused_csa_attn_2pass_bf16(q, kv, scale, o_out, lse_out, n_threads: int = 0) -> None:
    """Two-pass form (csa_attn.cpp:1050-1173); same result as the one-pass kernel."""
    _inplace(q, kv, scale, o_out, lse_out, torch.bfloat16)


def fused_csa_attn_fast_bf16(q, kv, scale, o_out, lse_out, n_threads: int = 0) -> None:
    """Blocked form (csa_attn.cpp:885-1048); same result."""
    _inplace(q, kv, scale, o_out, lse_out, torch.bfloat16)


def fused_csa_attn_inplace(q, kv, scale, o_out, lse_out, n_threads: int = 0) -> None:
    """In-place dense CSA, caller-allocated outputs (csa_attn.cpp:1485-1585)."""
    _inplace(q, kv, scale, o_out, lse_out)


def _check_int8_family(hd):
    if hd % 64 or hd > 512:
        raise RuntimeError("head_dim must be multiple of 64 and <=512")


def _pad_dims(t, hd):
    """t [..., d] -> [..., hd] with zeros beyond d (a copy; only when d < hd)."""
    d = t.shape[-1]
    if d == hd:
        return t.contiguous()
    out = torch.zeros(*t.shape[:-1], hd, dtype=t.dtype, device=t.device)
    out[..., :d] = t
    return out


def _launch_qcodes(q_u8, q_scales, kv_i8, kv_scales, kv_sums, kv_vals, scale, o_out, lse_out):
    """The integer-score CSA kernel over every entry of each sequence.

    q_u8 [bs, nH, sq, hd] codes, q_scales [bs, nH, sq]; kv_i8 [bs, nc, hd],
    kv_scales / kv_sums [bs, nc]; kv_vals None (values int8 * scale) or bf16
    [bs, nc, hd].  hd < 512 (a multiple of 64) runs on zero-padded copies:
    zero codes add nothing to the dot, zero values nothing to the output.
    """
    bs, hd = q_u8.shape[0], q_u8.shape[-1]
    nc = kv_i8.shape[1]
    nq = q_u8.numel() // max(1, bs * hd) if bs else 0
    if bs == 0 or nq == 0:
        return
    dev = q_u8.device
    if o_out.numel() != bs * nq * hd or lse_out.numel() != bs * nq:
        raise RuntimeError("o_out / lse_out shape mismatch")
    if lse_out.dtype != torch.float32 or o_out.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("o_out must be fp32 or bf16 and lse_out fp32")
    if kv_i8.dim() != 3 or kv_i8.shape[0] != bs or kv_i8.shape[2] != hd:
        raise RuntimeError("kv shape mismatch")
    if tuple(kv_scales.shape) != (bs, nc) or tuple(kv_sums.shape) != (bs, nc):
        raise RuntimeError("kv_scales / kv_sums must be [bs, nc]")
    if kv_scales.dtype != torch.float32 or kv_sums.dtype != torch.int32:
        raise RuntimeError("kv_scales must be float32 and kv_sums int32")
    qp = _pad_dims(q_u8.reshape(bs, nq, hd), HD)
    kp = _pad_dims(kv_i8, HD)
    vp = None if kv_vals is None else _pad_dims(kv_vals, HD)
    out = o_out if hd == HD else torch.empty(bs, nq, HD, dtype=o_out.dtype, device=dev)
    with on_device(dev):
        L_ = lib()
        ws = workspaces.get(L_.ws_csa_decode_workspace_size(bs, nq, _lib.WS_DTYPE_BF16), dev)
        rc = L_.ws_csa_decode_qcodes(ptr(qp), ptr(q_scales.contiguous()), bs, nq, HD, ptr(kp),
                                     ptr(kv_scales.contiguous()), ptr(kv_sums.contiguous()), ptr(vp), nc, 0, None, 0,
                                     _lib.WS_CSA_IDX_ALL, 0, nc, float(scale), ptr(out),
                                     _lib.WS_DTYPE_F32 if out.dtype == torch.float32 else _lib.WS_DTYPE_BF16,
                                     ptr(lse_out), ptr(ws), ws.numel(), stream_ptr(dev))
    check(rc, "ws_csa_decode_qcodes")
    if out is not o_out:
        o_out.view(bs, nq, hd).copy_(out[..., :hd])


def fused_csa_attn_bsq_int8(q, kv, scale, o_out, lse_out, n_threads: int = 0) -> None:
    """csa_attn.cpp:766-883: q fp32 [bs, nH, sq, hd] and kv bf16 [bs, nc, hd]
    are both quantised inside the call (q to u8 per row, kv to s8 per entry,
    each bit-exact with the reference's quantisers), the score is the integer
    dot and the values are ``int8 * scale``; writes o_out / lse_out."""
    _require_cuda("fused_csa_attn_bsq_int8", q, kv, o_out, lse_out)
    if not q.is_contiguous() or not kv.is_contiguous():
        raise RuntimeError("q/kv must be contiguous")
    if not o_out.is_contiguous() or not lse_out.is_contiguous():
        raise RuntimeError("o/lse must be contiguous")
    _check_int8_family(q.shape[-1])
    if q.dtype != torch.float32:
        raise RuntimeError("q must be fp32")
    if kv.dtype != torch.bfloat16:
        raise RuntimeError("kv must be bf16")
    kv_i8, kv_scales, kv_sums = kv_quantize_bf16_to_int8(kv)
    q_u8, q_scales = q_quantize_fp32_to_u8(q)
    _launch_qcodes(q_u8, q_scales, kv_i8, kv_scales, kv_sums, None, scale, o_out, lse_out)


# ------------------------------------------------------------- int8 storage
def kv_quantize_bf16_to_int8(kv: torch.Tensor, n_threads: int = 0):
    """bf16 [bs, nc, hd] -> (int8 [bs, nc, hd], scales fp32 [bs, nc], sums int32 [bs, nc]),
    bit-exact with csa_attn.cpp:1203-1233."""
    _require_cuda("kv_quantize_bf16_to_int8", kv)
    if kv.dtype != torch.bfloat16 or kv.dim() != 3 or not kv.is_contiguous():
        raise RuntimeError("kv must be contiguous bf16 [bs, nc, hd]")
    bs, nc, hd = kv.shape
    out = torch.empty((bs, nc, hd), dtype=torch.int8, device=kv.device)
    scales = torch.empty((bs, nc), dtype=torch.float32, device=kv.device)
    sums = torch.empty((bs, nc), dtype=torch.int32, device=kv.device)
    with on_device(kv.device):
        rc = lib().ws_csa_kv_quantize_s8(ptr(kv), bs * nc, hd, ptr(out), ptr(scales), ptr(sums),
                                         stream_ptr(kv.device))
    check(rc, "ws_csa_kv_quantize_s8")
    return out, scales, sums


def q_quantize_fp32_to_u8(q: torch.Tensor, n_threads: int = 0):
    """fp32 [bs, nh, sq, hd] -> (uint8 [bs, nh, sq, hd], scales fp32 [bs, nh, sq]),
    bit-exact with csa_attn.cpp:1175-1201."""
    _require_cuda("q_quantize_fp32_to_u8", q)
    if q.dtype != torch.float32 or not q.is_contiguous():
        raise RuntimeError("q must be contiguous fp32")
    hd = q.shape[-1]
    rows = q.numel() // hd if hd else 0
    out = torch.empty(q.shape, dtype=torch.uint8, device=q.device)
    scales = torch.empty(q.shape[:-1], dtype=torch.float32, device=q.device)
    with on_device(q.device):
        rc = lib().ws_csa_q_quantize_u8(ptr(q), rows, hd, ptr(out), ptr(scales), stream_ptr(q.device))
    check(rc, "ws_csa_q_quantize_u8")
    return out, scales


def fused_csa_attn_bsq_int8_preq(q, kv_i8, kv_scales, kv_sums, scale, o_out, lse_out, n_threads: int = 0) -> None:
    """csa_attn.cpp:1235-1357: pre-quantised entries (int8 codes, scales,
    code sums), the fp32 query quantised to u8 inside the call; score
    ``((sum u8*s8) - 128*kv_sums) * q_scale * k_scale * scale``, values
    ``int8 * k_scale``; writes o_out / lse_out."""
    _require_cuda("fused_csa_attn_bsq_int8_preq", q, kv_i8, kv_scales, kv_sums, o_out, lse_out)
    if not (q.is_contiguous() and kv_i8.is_contiguous() and kv_scales.is_contiguous() and kv_sums.is_contiguous()
            and o_out.is_contiguous() and lse_out.is_contiguous()):
        raise RuntimeError("tensors must be contiguous")
    _check_int8_family(q.shape[-1])
    if q.dtype != torch.float32 or kv_i8.dtype != torch.int8:
        raise RuntimeError("q must be fp32 and kv_i8 int8")
    q_u8, q_scales = q_quantize_fp32_to_u8(q)
    _launch_qcodes(q_u8, q_scales, kv_i8, kv_scales, kv_sums, None, scale, o_out, lse_out)


def fused_csa_attn_bsq_int8_full(q_u8, q_scales, kv_i8, kv_scales, kv_sums, kv_bf16, scale, o_out, lse_out,
                                 n_threads: int = 0) -> None:
    """csa_attn.cpp:1359-1483: a pre-quantised u8 query (codes + scales)
    scored against the int8 entry codes as in ``_preq``, the weighted sum
    taken over the bf16 entries ``kv_bf16``; writes o_out / lse_out."""
    _require_cuda("fused_csa_attn_bsq_int8_full", q_u8, q_scales, kv_i8, kv_scales, kv_sums, kv_bf16, o_out,
                  lse_out)
    if not (q_u8.is_contiguous() and kv_i8.is_contiguous() and kv_bf16.is_contiguous() and q_scales.is_contiguous()
            and kv_scales.is_contiguous() and kv_sums.is_contiguous() and o_out.is_contiguous()
            and lse_out.is_contiguous()):
        raise RuntimeError("tensors must be contiguous")
    _check_int8_family(q_u8.shape[-1])
    if q_u8.dtype != torch.uint8 or kv_i8.dtype != torch.int8 or kv_bf16.dtype != torch.bfloat16:
        raise RuntimeError("q_u8 must be uint8, kv_i8 int8 and kv_bf16 bf16")
    if kv_bf16.shape != kv_i8.shape:
        raise RuntimeError("kv_bf16 shape mismatch")
    _launch_qcodes(q_u8, q_scales, kv_i8, kv_scales, kv_sums, kv_bf16, scale, o_out, lse_out)


def fused_csa_attn_int8_exact(q, kv_i8, kv_scales, scale, o_out, lse_out) -> None:
    """Addition (no reference counterpart): dense CSA over int8 entries with
    one fp32 scale each, the query unquantised (fp32 or bf16); the score and
    the weighted sum both use ``int8 * scale`` exactly."""
    _require_cuda("fused_csa_attn_int8_exact", q, kv_i8, kv_scales, o_out, lse_out)
    if not (q.is_contiguous() and kv_i8.is_contiguous() and kv_scales.is_contiguous() and o_out.is_contiguous()
            and lse_out.is_contiguous()):
        raise RuntimeError("tensors must be contiguous")
    _launch(q, kv_i8, scale, o_out, lse_out, kv_scales=kv_scales)


# ------------------------------------------------------------------ gather
def indexer_attn_cpu(q, kv_compress, topk_idxs, scale, o_out, lse_out, n_threads: int = 0) -> None:
    """Top-k gather + attention (csa_attn.cpp:1819-1883): q fp32 [bs, nH, hd],
    kv_compress bf16 [bs, nc, hd], topk_idxs int32 [bs, k]; writes o_out fp32
    [bs, nH, hd] and lse_out fp32 [bs, nH].  Ids outside [0, nc) are skipped
    and reported by ``scope_b200.status_take()`` (the reference reads out of
    bounds there)."""
    _require_cuda("indexer_attn_cpu", q, kv_compress, topk_idxs, o_out, lse_out)
    if not q.is_contiguous() or not kv_compress.is_contiguous():
        raise RuntimeError("must be contiguous")
    _launch(q, kv_compress, scale, o_out, lse_out, idx=topk_idxs)


def csa_sparse_decode(q, kv, topk_idxs, scale, kv_scales=None, *, shard_lo: int = 0, idx_mode: str = "all",
                      out_dtype=torch.bfloat16):
    """CSA sparse decode over bf16 or int8+scale entries (the cfg5 hot path).

    q [bs, nH, hd] (fp32 or bf16); kv [bs, nc, hd] holding entry ids
    [shard_lo, shard_lo + nc); topk_idxs int32 [bs, k] global ids.
    ``idx_mode``: "all" (every id must be in this buffer), "sorted_shard"
    (ids ascending, only this shard's count) or "shard" (any order).
    Returns (out [bs, nH, hd] normalised in ``out_dtype``, lse fp32 [bs, nH]);
    a row with no entry in the shard gives out 0 and lse -inf.
    """
    out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=q.device)
    if idx_mode not in _IDX_MODES:
        raise ValueError(f"idx_mode must be one of {sorted(_IDX_MODES)}")
    _launch(q, kv, scale, out, lse, idx=topk_idxs, kv_scales=kv_scales, shard_lo=shard_lo, idx_mode=idx_mode)
    return out, lse


# ------------------------------------------------------------ indexer top-k
def indexer_topk(q_idx, kv_idx, weights, k: int, order: str = "score", return_scores: bool = False):
    """Indexer top-k (csa_attn.cpp:1658-1817) on the device.

    q_idx [bs, nH, hd] and kv_idx [bs, nc, hd] fp32 or bf16 (alike), weights
    [bs, nH] fp32; score = sum_h w_h * relu(q_h . kv_j) in fp32.  Returns ids
    int32 [bs, min(k, nc)] in descending score order (ties: lower id first) or,
    with ``order="id"``, ascending (the layout the sharded CSA decode wants);
    with ``return_scores`` also the scores fp32 [bs, nc].
    """
    _require_cuda("indexer_topk", q_idx, kv_idx, weights)
    if q_idx.dim() != 3 or kv_idx.dim() != 3:
        raise RuntimeError("q_idx/kv_idx must be 3D")
    if q_idx.dtype != kv_idx.dtype or q_idx.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("q_idx and kv_idx must both be fp32 or both bf16")
    if not (q_idx.is_contiguous() and kv_idx.is_contiguous() and weights.is_contiguous()):
        raise RuntimeError("must be contiguous")
    bs, nH, hd = q_idx.shape
    nc = kv_idx.shape[1]
    if kv_idx.shape[0] != bs or kv_idx.shape[2] != hd or tuple(weights.shape) != (bs, nH):
        raise RuntimeError("shape mismatch")
    if weights.dtype != torch.float32:
        raise RuntimeError("weights must be fp32")
    if hd % 16:
        raise RuntimeError("hd must be multiple of 16")
    if order not in ("score", "id"):
        raise ValueError("order must be 'score' or 'id'")
    k = min(int(k), nc)
    dev = q_idx.device
    ids = torch.empty(bs, k, dtype=torch.int32, device=dev)
    scores = torch.empty(bs, nc, dtype=torch.float32, device=dev) if return_scores else None
    code = _lib.WS_DTYPE_F32 if q_idx.dtype == torch.float32 else _lib.WS_DTYPE_BF16
    with on_device(dev):
        L_ = lib()
        ws = workspaces.get(L_.ws_indexer_topk_workspace_size(bs, nc), dev)
        rc = L_.ws_indexer_topk(ptr(q_idx), ptr(kv_idx), code, ptr(weights), bs, nH, hd, nc, k,
                                _lib.WS_TOPK_BY_ID if order == "id" else _lib.WS_TOPK_BY_SCORE,
                                ptr(ids), ptr(scores), ptr(ws), ws.numel(), stream_ptr(dev))
    check(rc, "ws_indexer_topk")
    return (ids, scores) if return_scores else ids


def indexer_topk_cpu(q_idx, kv_idx, weights, k: int, n_threads: int = 0):
    """Drop-in for indexer_topk_cpu (csa_attn.cpp:1658-1736): fp32 inputs,
    ids int32 [bs, min(k, nc)] by descending score."""
    if q_idx.dtype != torch.float32 or kv_idx.dtype != torch.float32:
        raise RuntimeError("must be fp32")
    return indexer_topk(q_idx, kv_idx, weights, k)


def indexer_topk_cpu_par(q_idx, kv_idx, weights, k: int, n_threads: int = 0):
    """Drop-in for indexer_topk_cpu_par (csa_attn.cpp:1738-1817); same result."""
    return indexer_topk(q_idx, kv_idx, weights, k)
