"""Runtime swap-in: the decode-attention steps of the reference's offload
runtimes, with every KV share resident in HBM.

The reference runs one layer's decode attention as a CPU share (its AVX-512
kernel over host KV), a GPU-resident share and a share streamed over PCIe in
512-token chunks, and merges them by log-sum-exp in torch
(roofline/bench_resident_kv.py:129-148 ``_cpu_attn`` / ``_pairwise_merge``,
:254-352 ``run_bkv_resident`` / ``run_kvlen_resident``; the model runtimes do
the same in system/qwenoffload.py:1217-1545 and system/mixoffload.py:1201-1480).
On a B200 box every share is another HBM buffer (or another GPU's shard,
scope_b200.shard), so the functions here keep the harness's split and layout
and replace its three code paths with the library's kernels:

* ``kvlen_decode``: the token split (rows x [share 0 | share 1 | share 2]):
  one ws_gqa_decode_shares launch over up to four shares, merged in the launch
  (the harness's two pairwise merges);
* ``bkv_decode``: the row split (row groups, each with its whole KV): one
  ws_gqa_decode launch per group, written into slices of one output;
* ``pairwise_merge``: the harness's un-normalised (o, max, sum) merge on the
  device, for callers that keep partials in that form;
* ``MlaDecodeLayer``: the single-token branch of ``_mla_compressed_forward``
  (system/deepseek.py:326-407: absorb, attention over the cache, merge,
  up-projection) over a ShardedKVCacheCompressed, with the new token appended
  first (:250-252) -- one call per decode step, nothing copied to the host;
* ``ds4_window_compressed_decode``: the DeepSeek-V4 decode step's attention
  over the sliding-window cache and the compressed cache
  (system/ds4offload.py:280-342), with the compressed cache resident in HBM
  instead of pinned host memory: two CSA launches and one log-sum-exp merge,
  the attention sink entering that merge as a partial with no value.

Layouts follow the harness: q [B*NH, GROUPS, QHD] bf16 (kv row r = b*NH + h,
query head r*GROUPS + g); a share's k, v [B*NH, len, QHD / VHD] bf16; outputs
[B, NH*GROUPS, 1, VHD] bf16 normalised, as ``run_*_resident`` return them.
"""
from __future__ import annotations

from typing import Sequence

import torch

from .ops import Share, gqa_decode_shares, lse_merge


def _rows_of(q: torch.Tensor) -> tuple[int, int, int]:
    if q.dim() != 3 or q.dtype != torch.bfloat16 or not q.is_cuda or not q.is_contiguous():
        raise RuntimeError("q must be a contiguous bf16 CUDA tensor [B*NH, GROUPS, QHD]")
    return q.shape


def kvlen_decode(q: torch.Tensor, ks: Sequence[torch.Tensor], vs: Sequence[torch.Tensor], scale: float,
                 B: int | None = None, return_lse: bool = False):
    """The token-split decode (run_kvlen_resident, roofline/bench_resident_kv.py:314-352).

    q [B*NH, G, QHD]; ks[i], vs[i] [B*NH, len_i, QHD / VHD] -- the shares of
    every row's tokens in order (the harness's streamed, resident and CPU
    shares; any may be empty), at most four.  Returns out [B, NH*G, 1, VHD]
    bf16 (and lse [B, NH*G] fp32 with ``return_lse``).
    """
    bkv, G, Dk = _rows_of(q)
    if not 1 <= len(ks) <= 4 or len(ks) != len(vs):
        raise RuntimeError("kvlen_decode: 1 to 4 shares, as many k as v")
    B = bkv if B is None else B
    if bkv % B:
        raise RuntimeError("kvlen_decode: rows must be a multiple of the batch")
    dev = q.device
    shares = []
    for k, v in zip(ks, vs):
        if k.shape[0] != bkv or v.shape[0] != bkv or k.shape[1] != v.shape[1]:
            raise RuntimeError("kvlen_decode: every share must hold all rows [B*NH, len, D]")
        if k.shape[1] == 0:
            continue   # an empty share adds nothing to any row
        # each kv row is its own sequence of the padded-share layout (one kv head), of this share's length
        lens = torch.full((bkv,), k.shape[1], dtype=torch.int32, device=dev)
        shares.append(Share(k, v, seqlens=lens))
    Dv = vs[0].shape[2]
    if shares:
        out, lse = gqa_decode_shares(q, shares, scale)        # [bkv, G, VHD], [bkv, G]
    else:
        out = torch.zeros(bkv, G, Dv, dtype=torch.bfloat16, device=dev)
        lse = torch.full((bkv, G), float("-inf"), dtype=torch.float32, device=dev)
    out = out.view(B, (bkv // B) * G, 1, Dv)
    return (out, lse.view(B, -1)) if return_lse else out


def bkv_decode(q: torch.Tensor, groups: Sequence[tuple[torch.Tensor, torch.Tensor]], scale: float,
               B: int | None = None):
    """The row-split decode (run_bkv_resident, roofline/bench_resident_kv.py:254-300).

    groups: consecutive row ranges of q, each (k, v) [rows_i, L_i, QHD / VHD]
    holding those rows' whole KV (the harness's CPU rows, resident rows and
    streamed rows).  Returns out [B, NH*G, 1, VHD] bf16.
    """
    from .cpu_attn import gqa_decode
    bkv, G, Dk = _rows_of(q)
    if sum(k.shape[0] for k, _ in groups) != bkv:
        raise RuntimeError("bkv_decode: the groups' rows must add up to q's rows")
    B = bkv if B is None else B
    Dv = groups[0][1].shape[2]
    out = torch.empty(bkv, G, Dv, dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(bkv, G, dtype=torch.float32, device=q.device)
    r0 = 0
    for k, v in groups:
        n = k.shape[0]
        if n:
            gqa_decode(q[r0:r0 + n], k, v, scale, out=out[r0:r0 + n], lse=lse[r0:r0 + n])
        r0 += n
    return out.view(B, (bkv // B) * G, 1, Dv)


def pairwise_merge(o1, m1, s1, o2, m2, s2):
    """The harness's merge of two un-normalised partials (roofline/bench_resident_kv.py:141-148):
    o_i [R..., D] un-normalised, m_i / s_i [R..., 1] max and sum, all fp32 CUDA
    tensors.  Returns (o, m, s) of the union in the same form, computed by the
    device log-sum-exp merge (ws_lse_merge) on the normalised partials."""
    for t in (o1, m1, s1, o2, m2, s2):
        if not t.is_cuda or t.dtype != torch.float32:
            raise RuntimeError("pairwise_merge: fp32 CUDA tensors")
    ninf = torch.tensor(float("-inf"), device=o1.device)
    parts_o = torch.stack([o1 / s1.clamp(min=1e-30), o2 / s2.clamp(min=1e-30)])
    parts_l = torch.stack([torch.where(s1 > 0, m1 + s1.clamp(min=1e-30).log(), ninf)[..., 0],
                           torch.where(s2 > 0, m2 + s2.clamp(min=1e-30).log(), ninf)[..., 0]])
    o, lse = lse_merge(parts_o, parts_l, torch.float32)
    m = torch.maximum(m1, m2)
    s = torch.where(torch.isinf(lse), torch.zeros_like(lse), torch.exp(lse - m[..., 0]))[..., None]
    return o * s, m, s


class MlaDecodeLayer:
    """The single-token decode branch of the reference's absorbed-MLA layer
    (``_mla_compressed_forward``, system/deepseek.py:326-407) on the device.

    Holds the layer's ``kv_b_proj`` weight [nH * (nop + vhd), kv_lora_rank]
    and a ShardedKVCacheCompressed.  ``step(li, q_nope, q_pe, c_kv, k_pe)``
    appends the new token's latent and rope rows to the cache (:250-252), then
    runs absorb -> attention over the whole cache -> merge -> up-projection
    in one ws_mla_decode_absorbed_strided call that reads the cache buffers in
    place (:257-265, :326-407).  Returns the attention output before o_proj,
    [B, 1, nH * vhd] bf16, the tensor the reference passes to
    ``self_attn.o_proj``.  Single-GPU caches (world 1); a sharded cache would
    exchange the latent partials before the up-projection.
    """

    def __init__(self, cache, kv_b_proj_weight: torch.Tensor, n_heads: int, nope_dim: int, v_dim: int,
                 scale: float):
        if cache.world != 1:
            raise RuntimeError("MlaDecodeLayer: a single-GPU cache (world 1)")
        if kv_b_proj_weight.shape != (n_heads * (nope_dim + v_dim), 512):
            raise RuntimeError("kv_b_proj_weight must be [nH * (nope + v), 512]")
        self.cache, self.w = cache, kv_b_proj_weight.contiguous()
        self.nH, self.nop, self.vhd, self.scale = n_heads, nope_dim, v_dim, scale

    def step(self, li: int, q_nope: torch.Tensor, q_pe: torch.Tensor, c_kv: torch.Tensor, k_pe: torch.Tensor):
        """q_nope [B, nH, 1, nop], q_pe [B, nH, 1, 64] (after rope); c_kv [B, 1, 512]
        (after kv_a_layernorm) and k_pe [B, 1, 64] (after rope) of the new token."""
        from .cpu_attn import mla_decode_absorbed
        self.cache.append(li, c_kv, k_pe)
        c, pe = self.cache.get(li)
        B = q_nope.shape[0]
        out = mla_decode_absorbed(q_nope, q_pe, c, pe, self.w, self.scale)   # [B, nH, vhd]
        return out.reshape(B, 1, self.nH * self.vhd)


def ds4_window_compressed_decode(q: torch.Tensor, kv_window: torch.Tensor, kv_compressed: torch.Tensor,
                                 scale: float, *, window_len: int | None = None, n_compress: int | None = None,
                                 topk_idxs: torch.Tensor | None = None, attn_sink: torch.Tensor | None = None,
                                 return_lse: bool = False):
    """The DeepSeek-V4 decode step's attention over its two caches (system/ds4offload.py:280-342).

    q [bsz, 1, nH, hd] (bf16 or fp32, after rope); kv_window [bsz, win, hd]
    bf16, the sliding-window cache, whose first ``window_len`` entries (all
    by default) are attended; kv_compressed [bsz, nc, hd] bf16, the
    compressed cache, resident here (the reference keeps it in pinned host
    memory and attends to it on the CPU).  K = V = the entry, as in the
    reference (MQA over one latent).

    * ``topk_idxs`` None: the reference's parallel branch (:286-327): every
      window entry and the first ``n_compress`` compressed entries (all by
      default), two partials merged by the pairwise formula.  That branch
      applies no attention sink.
    * ``topk_idxs`` int32 [bsz, k]: the gather branch (:328-342): the window
      entries plus the compressed entries the indexer selected, in one
      softmax.  Ids are compressed-cache positions (the reference's
      ``topk_idxs[..., win:] - win``); ids outside [0, nc) are skipped (the
      reference clamps them to entry 0).
    * ``attn_sink`` [nH] (the gather branch's ``sparse_attn`` sink): a
      per-head logit that joins each head's softmax denominator and carries
      no value.  ``sparse_attn`` is a DeepSeek-V4 kernel that the reference
      imports from the model's own code, not shipped with it; this follows
      that published definition of a sink.

    Returns o [bsz, 1, nH, hd] in q's dtype (and lse fp32 [bsz, nH] with
    ``return_lse``).  Two ws_csa_decode launches and one ws_lse_merge.
    """
    from .csa_attn import _launch
    if q.dim() != 4 or q.shape[1] != 1 or not q.is_cuda:
        raise RuntimeError("q must be a CUDA tensor [bsz, 1, nH, hd] (one decode token)")
    bsz, _, nH, hd = q.shape
    if q.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError("q must be bf16 or fp32")
    for name, t in (("kv_window", kv_window), ("kv_compressed", kv_compressed)):
        if t.dim() != 3 or t.shape[0] < bsz or t.shape[2] != hd or t.dtype != torch.bfloat16 or not t.is_cuda:
            raise RuntimeError(f"{name} must be a bf16 CUDA tensor [>= bsz, entries, hd]")
    kv_w, kv_c = kv_window[:bsz].contiguous(), kv_compressed[:bsz].contiguous()
    win, nc = kv_w.shape[1], kv_c.shape[1]
    wl = win if window_len is None else int(window_len)
    ncomp = nc if n_compress is None else int(n_compress)
    if not 0 <= wl <= win or not 0 <= ncomp <= nc:
        raise RuntimeError("window_len / n_compress out of range")
    dev = q.device
    q3 = q.reshape(bsz, nH, hd).contiguous()
    n_parts = 3 if attn_sink is not None else 2
    parts_o = torch.zeros(n_parts, bsz, nH, hd, dtype=torch.float32, device=dev)
    parts_l = torch.full((n_parts, bsz, nH), float("-inf"), dtype=torch.float32, device=dev)
    if wl > 0:   # the window share: entries [0, window_len)
        _launch(q3, kv_w, scale, parts_o[0], parts_l[0], kv_range=(0, wl))
    if topk_idxs is not None:   # the indexer's compressed entries
        if topk_idxs.dtype != torch.int32 or topk_idxs.dim() != 2 or topk_idxs.shape[0] != bsz:
            raise RuntimeError("topk_idxs must be int32 [bsz, k]")
        _launch(q3, kv_c, scale, parts_o[1], parts_l[1], idx=topk_idxs.contiguous(), shard_lo=0, idx_mode="shard")
    elif ncomp > 0:   # every compressed entry so far
        _launch(q3, kv_c, scale, parts_o[1], parts_l[1], kv_range=(0, ncomp))
    if attn_sink is not None:   # the sink: a partial whose lse is the head's logit and whose value is zero
        if attn_sink.numel() != nH:
            raise RuntimeError("attn_sink must hold one logit per head")
        parts_l[2].copy_(attn_sink.to(device=dev, dtype=torch.float32).view(1, nH).expand(bsz, nH))
    out, lse = lse_merge(parts_o, parts_l, out_dtype=q.dtype)
    out = out.view(bsz, 1, nH, hd)
    return (out, lse) if return_lse else out
