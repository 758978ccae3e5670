"""TEST INFRASTRUCTURE ONLY -- the CPU checker for the CUDA decode-attention path.

Two things live here:

* ``liboracle.so`` (``ws_oracle.c``): a plain-C restatement of the reference
  operators, float64 accumulation, called through ctypes on numpy arrays.
* ``_ref/``: the reference's own AVX-512 torch extensions compiled from their
  sources (``make ref``); loaded with :func:`load_ref` when present.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU
baseline and ``--impl reference`` arm) may import this package.  The shipped
``scope_b200`` package never does.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_lib = None

_D = ctypes.POINTER(ctypes.c_double)
_F = ctypes.POINTER(ctypes.c_float)
_I = ctypes.POINTER(ctypes.c_int32)
_V = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int


def build(verbose: bool = False) -> None:
    """Compile liboracle.so (make in this directory)."""
    out = subprocess.run(["make", "-C", HERE, "liboracle.so"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if verbose:
        print(out.stdout)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_gqa_decode.argtypes = [_V, _V, _V, _int, _i64, _i64, _i64, _i64,
                                     _int, _int, _int, _int, _int, ctypes.c_double, _D, _D, _D]
        L.orc_gqa_decode.restype = None
        L.orc_mla_compressed.argtypes = [_V, _V, _V, _V, _int, _int, _int, _int, _int,
                                         ctypes.c_double, _D, _D, _D]
        L.orc_mla_compressed.restype = None
        L.orc_csa_attend.argtypes = [_V, _int, _V, _int, _F, _I, _int, _int, _int,
                                     _int, _int, _int, _int, ctypes.c_double, _D, _D]
        L.orc_csa_attend.restype = ctypes.c_int64
        L.orc_kv_quantize_s8.argtypes = [_V, _i64, _int, _V, _F, _I]
        L.orc_kv_quantize_s8.restype = None
        L.orc_q_quantize_u8.argtypes = [_F, _i64, _int, _V, _F]
        L.orc_q_quantize_u8.restype = None
        L.orc_csa_int8_preq.argtypes = [_F, _V, _F, _I, _int, _int, _int, _int, ctypes.c_float, _D, _D]
        L.orc_csa_int8_preq.restype = None
        L.orc_csa_int8_codes.argtypes = [_V, _F, _V, _F, _I, _V, _I, _int, _int, _int, _int, _int,
                                         ctypes.c_float, _D, _D]
        L.orc_csa_int8_codes.restype = None
        L.orc_indexer_scores_f32.argtypes = [_F, _F, _F, _int, _int, _int, _i64, _int, _F]
        L.orc_indexer_scores_f32.restype = None
        L.orc_lse_merge.argtypes = [_D, _D, _int, _i64, _int, _D, _D]
        L.orc_lse_merge.restype = None
        L.orc_indexer_topk.argtypes = [_F, _F, _F, _int, _int, _int, _int, _int, _I, _D]
        L.orc_indexer_topk.restype = None
        _lib = L
    return _lib


# ----------------------------------------------------------------- helpers
def _p(a: np.ndarray, ct=None):
    return a.ctypes.data_as(ct) if ct is not None else ctypes.c_void_p(a.ctypes.data)


def bf16_bits(x) -> np.ndarray:
    """bf16 storage as uint16 from a torch bf16 tensor or a uint16 array."""
    if hasattr(x, "view") and hasattr(x, "dtype") and str(getattr(x, "dtype", "")) == "torch.bfloat16":
        import torch
        return x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    a = np.asarray(x)
    assert a.dtype == np.uint16
    return a


def bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bits (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


# --------------------------------------------------------------- operators
def gqa_decode(q, k, v, scale, k_strides=None, v_strides=None, kind="bf16"):
    """GQA/MLA decode (kernel/cpu_attn.cpp:193-672).

    q [B_kv, G, Dk]; k [B_kv, L, Dk], v [B_kv, L, Dv] as uint16 bf16 bits
    (kind="bf16") or float32 (kind="fp32").  ``k_strides``/``v_strides``
    (elements, dims 0 and 1) default to contiguous.  Returns float64
    (o_normalised [B_kv,G,Dv], max [B_kv,G], sum [B_kv,G]).
    """
    kid = 0 if kind == "bf16" else 1
    q = np.ascontiguousarray(q)
    B, G, Dk = q.shape
    L = k.shape[1]
    Dv = v.shape[2]
    if k_strides is None:
        k = np.ascontiguousarray(k)
        k_strides = (L * Dk, Dk)
    if v_strides is None:
        v = np.ascontiguousarray(v)
        v_strides = (L * Dv, Dv)
    o = np.zeros((B, G, Dv), np.float64)
    m = np.zeros((B, G), np.float64)
    s = np.zeros((B, G), np.float64)
    lib().orc_gqa_decode(_p(q), _p(k), _p(v), kid, k_strides[0], k_strides[1], v_strides[0], v_strides[1],
                         B, G, Dk, Dv, L, float(scale), _p(o, _D), _p(m, _D), _p(s, _D))
    return o, m, s


def gqa_decode_strided_buffer(q, kbuf, vbuf, L, k_strides, v_strides, Dv, scale, kind="bf16"):
    """Same as gqa_decode but k/v are flat buffers addressed by explicit strides."""
    kid = 0 if kind == "bf16" else 1
    q = np.ascontiguousarray(q)
    B, G, Dk = q.shape
    o = np.zeros((B, G, Dv), np.float64)
    m = np.zeros((B, G), np.float64)
    s = np.zeros((B, G), np.float64)
    lib().orc_gqa_decode(_p(q), _p(kbuf), _p(vbuf), kid, k_strides[0], k_strides[1], v_strides[0], v_strides[1],
                         B, G, Dk, Dv, L, float(scale), _p(o, _D), _p(m, _D), _p(s, _D))
    return o, m, s


def mla_compressed(q_proj, q_pe, c_kv, k_pe, scale):
    """Absorbed MLA (kernel/cpu_attn.cpp:852-1022); uint16 bf16 inputs.

    Returns float64 (o_unnormalised [B*nH, clr], max [B*nH], sum [B*nH]).
    """
    q_proj, q_pe, c_kv, k_pe = (np.ascontiguousarray(a) for a in (q_proj, q_pe, c_kv, k_pe))
    B, S, clr = c_kv.shape
    qrd = k_pe.shape[2]
    nH = q_proj.shape[0] // B
    o = np.zeros((B * nH, clr), np.float64)
    m = np.zeros((B * nH,), np.float64)
    s = np.zeros((B * nH,), np.float64)
    lib().orc_mla_compressed(_p(q_proj), _p(q_pe), _p(c_kv), _p(k_pe), B, nH, S, clr, qrd,
                             float(scale), _p(o, _D), _p(m, _D), _p(s, _D))
    return o, m, s


def bf16_round(x: np.ndarray) -> np.ndarray:
    """x rounded to bf16 (round-half-even) and returned as float64."""
    return bits_to_f32(f32_to_bf16_bits(np.asarray(x, np.float32))).astype(np.float64)


def mla_absorbed(q_nope, q_pe, c_kv, k_pe, w_uk, w_uv, scale):
    """The absorbed-MLA decode step with its projections (system/deepseek.py:257-265
    q_proj = bmm(q_nope, W_UK) in bf16; :355-404 attention over the cache and merge;
    :405-407 o_n = (o / s).to(bf16), out = bmm(o_n, W_UV^T)).  uint16 bf16 inputs:
    q_nope [B, nH, nop], q_pe [B*nH, 64], c_kv [B, S, 512], k_pe [B, S, 64],
    w_uk [nH, nop, 512], w_uv [nH, vhd, 512].

    Returns float64 (out [B, nH, vhd], lse [B*nH]); the bf16 roundings the reference
    makes (q_proj, o_n) are made here too.
    """
    qn = bits_to_f32(np.ascontiguousarray(q_nope)).astype(np.float64)
    wk = bits_to_f32(np.ascontiguousarray(w_uk)).astype(np.float64)
    wv = bits_to_f32(np.ascontiguousarray(w_uv)).astype(np.float64)
    B, nH, nop = qn.shape
    q_proj = bf16_round(np.einsum("bhk,hkc->bhc", qn, wk)).reshape(B * nH, -1)
    o, m, s = mla_compressed(f32_to_bf16_bits(q_proj.astype(np.float32)), q_pe, c_kv, k_pe, scale)
    with np.errstate(divide="ignore", invalid="ignore"):
        on = np.where(s[:, None] > 0, o / s[:, None], 0.0)
        lse = np.where(s > 0, m + np.log(s), -np.inf)
    on = bf16_round(on).reshape(B, nH, -1)
    out = np.einsum("bhc,hvc->bhv", on, wv)
    return out, lse


def csa_attend(q, kv, scale, idx=None, kv_range=None, kv_scale=None):
    """CSA attention over a shared latent (csa_attn.cpp:200-281, :1587-1656, :1819-1883).

    q [bs, nq, hd] float32 or uint16 (bf16 bits); kv [bs, nc, hd] uint16 bf16
    bits or int8 (then ``kv_scale`` [bs, nc] float32 is required).
    ``idx`` [bs, k] int32 gathers entries; else ``kv_range`` (s, e) or all.
    Returns float64 (o_normalised [bs, nq, hd], lse [bs, nq]).
    """
    q = np.ascontiguousarray(q)
    kv = np.ascontiguousarray(kv)
    bs, nq, hd = q.shape
    nc = kv.shape[1]
    q_kind = 1 if q.dtype == np.float32 else 0
    if kv.dtype == np.int8:
        kv_kind = 2
        assert kv_scale is not None
        kv_scale = np.ascontiguousarray(kv_scale, dtype=np.float32)
    else:
        kv_kind = 0
    o = np.zeros((bs, nq, hd), np.float64)
    lse = np.zeros((bs, nq), np.float64)
    if idx is not None:
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        n_idx = idx.shape[1]
        s, e = 0, 0
    else:
        n_idx = 0
        s, e = kv_range if kv_range is not None else (0, nc)
    bad = lib().orc_csa_attend(_p(q), q_kind, _p(kv), kv_kind,
                               _p(kv_scale, _F) if kv_scale is not None else None,
                               _p(idx, _I) if idx is not None else None, n_idx, s, e,
                               bs, nq, hd, nc, float(scale), _p(o, _D), _p(lse, _D))
    return o, lse, int(bad)


def kv_quantize_s8(kv_bits):
    """bf16 -> int8 per row (csa_attn.cpp:729-764); returns (int8, scales f32, sums i32)."""
    kv_bits = np.ascontiguousarray(kv_bits)
    *lead, hd = kv_bits.shape
    rows = int(np.prod(lead)) if lead else 1
    out = np.zeros(kv_bits.shape, np.int8)
    sc = np.zeros(lead, np.float32)
    sm = np.zeros(lead, np.int32)
    lib().orc_kv_quantize_s8(_p(kv_bits), rows, hd, _p(out), _p(sc, _F), _p(sm, _I))
    return out, sc, sm


def q_quantize_u8(q):
    """fp32 -> u8 per row (csa_attn.cpp:704-727); returns (uint8, scales f32)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    *lead, hd = q.shape
    rows = int(np.prod(lead)) if lead else 1
    out = np.zeros(q.shape, np.uint8)
    sc = np.zeros(lead, np.float32)
    lib().orc_q_quantize_u8(_p(q, _F), rows, hd, _p(out), _p(sc, _F))
    return out, sc


def csa_int8_preq(q, kv_i8, kv_scales, kv_sums, scale):
    """fused_csa_attn_bsq_int8_preq (csa_attn.cpp:1235-1357): q fp32 [bs, nq, hd]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    bs, nq, hd = q.shape
    nc = kv_i8.shape[1]
    o = np.zeros((bs, nq, hd), np.float64)
    lse = np.zeros((bs, nq), np.float64)
    lib().orc_csa_int8_preq(_p(q, _F), _p(np.ascontiguousarray(kv_i8)),
                            _p(np.ascontiguousarray(kv_scales, dtype=np.float32), _F),
                            _p(np.ascontiguousarray(kv_sums, dtype=np.int32), _I),
                            bs, nq, hd, nc, float(scale), _p(o, _D), _p(lse, _D))
    return o, lse


def csa_int8_codes(q_u8, q_scales, kv_i8, kv_scales, kv_sums, scale, kv_bf16=None, idx=None):
    """The reference's integer-score CSA (csa_attn.cpp:1235-1483): q_u8 [bs, nq, hd]
    codes with q_scales [bs, nq]; kv_i8 / kv_scales / kv_sums the entry codes;
    values int8 * scale, or the bf16 entries ``kv_bf16`` (uint16 bits) when
    given (the _full operator); ``idx`` [bs, k] selects entries (else all)."""
    q_u8 = np.ascontiguousarray(q_u8, dtype=np.uint8)
    bs, nq, hd = q_u8.shape
    nc = kv_i8.shape[1]
    o = np.zeros((bs, nq, hd), np.float64)
    lse = np.zeros((bs, nq), np.float64)
    kvb = None if kv_bf16 is None else np.ascontiguousarray(kv_bf16, dtype=np.uint16)
    ids = None if idx is None else np.ascontiguousarray(idx, dtype=np.int32)
    lib().orc_csa_int8_codes(_p(q_u8), _p(np.ascontiguousarray(q_scales, dtype=np.float32), _F),
                             _p(np.ascontiguousarray(kv_i8, dtype=np.int8)),
                             _p(np.ascontiguousarray(kv_scales, dtype=np.float32), _F),
                             _p(np.ascontiguousarray(kv_sums, dtype=np.int32), _I),
                             None if kvb is None else _p(kvb), None if ids is None else _p(ids, _I),
                             0 if ids is None else ids.shape[1], bs, nq, hd, nc, float(scale),
                             _p(o, _D), _p(lse, _D))
    return o, lse


def indexer_scores_f32(q_idx, kv_idx, w, contract=True):
    """Indexer scores in the reference's fp32 order (csa_attn.cpp:1706-1724):
    float32 [bs, nc], bit for bit what indexer_topk_cpu ranks."""
    q_idx = np.ascontiguousarray(q_idx, dtype=np.float32)
    kv_idx = np.ascontiguousarray(kv_idx, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    bs, nH, hd = q_idx.shape
    nc = kv_idx.shape[1]
    out = np.zeros((bs, nc), np.float32)
    lib().orc_indexer_scores_f32(_p(q_idx, _F), _p(kv_idx, _F), _p(w, _F), bs, nH, hd, nc, int(bool(contract)),
                                 _p(out, _F))
    return out


def topk_from_scores(scores, k):
    """ids [bs, min(k, nc)] by descending score, ties by the lower id."""
    scores = np.asarray(scores)
    k = min(int(k), scores.shape[1])
    ids = np.argsort(-scores.astype(np.float64), axis=1, kind="stable")[:, :k]
    return ids.astype(np.int32)


def canonical_topk(ids, scores):
    """Reorder each row of ``ids`` by (descending score, ascending id): the
    reference's partial_sort leaves the order of exactly equal scores
    unspecified, so two correct outputs may differ only inside such runs."""
    ids = np.asarray(ids)
    out = np.empty_like(ids)
    for b in range(ids.shape[0]):
        s = np.asarray(scores[b], dtype=np.float64)[ids[b]]
        out[b] = ids[b][np.lexsort((ids[b], -s))]
    return out


def topk_agreement(ids, ref_ids, scores):
    """Compare two top-k id lists under one score array.  Returns a dict:
    ``set_diff`` ids in one set but not the other (summed over rows),
    ``boundary_ties`` how many entries score exactly the k-th score (a set
    may legitimately differ only among those), ``order_diff`` positions that
    differ after both lists are put in canonical tie order."""
    set_diff = boundary = order_diff = 0
    ci, cr = canonical_topk(ids, scores), canonical_topk(ref_ids, scores)
    for b in range(ids.shape[0]):
        a, r = set(ids[b].tolist()), set(ref_ids[b].tolist())
        set_diff += len(a ^ r)
        kth = np.asarray(scores[b])[ref_ids[b][-1]] if len(ref_ids[b]) else 0.0
        boundary += int((np.asarray(scores[b]) == kth).sum()) if len(ref_ids[b]) else 0
        order_diff += int((ci[b] != cr[b]).sum())
    return {"set_diff": set_diff, "boundary_ties": boundary, "order_diff": order_diff}


def lse_merge(o_parts, lse_parts):
    """LSE merge of P partials (system/qwenoffload.py:1606-1617).

    o_parts [P, R, D] normalised, lse_parts [P, R] -> (o [R, D], lse [R]) float64.
    """
    o_parts = np.ascontiguousarray(o_parts, dtype=np.float64)
    lse_parts = np.ascontiguousarray(lse_parts, dtype=np.float64)
    P, R, D = o_parts.shape
    o = np.zeros((R, D), np.float64)
    lse = np.zeros((R,), np.float64)
    lib().orc_lse_merge(_p(o_parts, _D), _p(lse_parts, _D), P, R, D, _p(o, _D), _p(lse, _D))
    return o, lse


def indexer_topk(q_idx, kv_idx, w, k):
    """Indexer top-k (csa_attn.cpp:1658-1736); returns (ids int32 [bs,k], scores f64 [bs,nc])."""
    q_idx = np.ascontiguousarray(q_idx, dtype=np.float32)
    kv_idx = np.ascontiguousarray(kv_idx, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    bs, nH, hd = q_idx.shape
    nc = kv_idx.shape[1]
    k = min(k, nc)
    out = np.zeros((bs, k), np.int32)
    sc = np.zeros((bs, nc), np.float64)
    lib().orc_indexer_topk(_p(q_idx, _F), _p(kv_idx, _F), _p(w, _F), bs, nH, hd, nc, k, _p(out, _I), _p(sc, _D))
    return out, sc


# ------------------------------------------------------ compiled reference
def ref_available() -> bool:
    """True when oracle/_ref holds the compiled reference and this CPU runs it."""
    if not os.path.isdir(REF_DIR) or not any(f.startswith("cpu_attn_ext") for f in os.listdir(REF_DIR)):
        return False
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        return False
    return all(f in flags for f in ("avx512f", "avx512bw", "avx512_vnni"))


def load_ref(name: str):
    """Import a compiled reference extension from oracle/_ref by module name
    ('cpu_attn_ext', 'cpu_attn_tile_ext', 'csa_attn_kernel')."""
    import torch  # noqa: F401  (the extensions link libtorch)
    for f in os.listdir(REF_DIR):
        if f.startswith(name + "."):
            spec = importlib.util.spec_from_file_location(name, os.path.join(REF_DIR, f))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            sys.modules.setdefault("oracle_ref_" + name, mod)
            return mod
    raise FileNotFoundError(name)
