"""Device-resident, sequence-sharded KV caches: the physically partitioned
format the decode kernels read, with append.

Mirrors the reference's caches -- ``InplaceKVCache`` (system/qwenoffload.py:59-141,
GQA: per layer k/v ``[B*Hkv, max_seq, D]``, ``append_4d``, ``get``, ``seq_len``,
``reset``) and ``InplaceKVCacheCompressed`` (system/deepseek.py:144-209,
absorbed MLA: per layer latent ``[B, max_seq, 512]`` and rope ``[B, max_seq, 64]``,
``append``) -- with the buffers in HBM instead of pinned host memory and the
host/GPU share replaced by contiguous token shards across GPUs: rank r of
`world` holds positions [r*cap, (r+1)*cap) with cap = ceil(max_seq / world),
so a decode step's new token lands on one rank only.  Appends run the
``ws_kv_append`` kernel; decodes run ``ws_gqa_decode`` / ``ws_mla_decode`` on
the local shard and (world > 1) merge the shards' partials with one exchange
(scope_b200.shard.PartialExchange).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, on_device, stream_ptr


def shard_capacity(max_seq: int, world: int) -> int:
    return -(-max_seq // world)


def local_slice(t: int, n_new: int, cap: int, rank: int) -> tuple[int, int, int]:
    """Of the new tokens at global positions [t, t + n_new), the ones rank
    `rank` stores: returns (first new-token index, count, local position)."""
    lo, hi = rank * cap, (rank + 1) * cap
    a, b = max(t, lo), min(t + n_new, hi)
    if b <= a:
        return 0, 0, 0
    return a - t, b - a, a - lo


def _append(dst: torch.Tensor, src: torch.Tensor, t0: int) -> None:
    """dst [rows, cap, D] <- src [rows, n, D] at local positions [t0, t0 + n)."""
    code = {torch.bfloat16: _lib.WS_DTYPE_BF16, torch.float32: _lib.WS_DTYPE_F32, torch.int8: _lib.WS_DTYPE_I8}[dst.dtype]
    if src.dtype != dst.dtype or src.device != dst.device:
        raise RuntimeError("append: source must match the cache's dtype and device")
    if src.stride(2) != 1:
        src = src.contiguous()
    rows, n, D = src.shape
    with on_device(dst.device):
        rc = lib().ws_kv_append(ptr(dst), dst.stride(0), dst.stride(1), dst.shape[1], ptr(src), src.stride(0),
                                src.stride(1), rows, n, D, code, t0, stream_ptr(dst.device))
    check(rc, "ws_kv_append")


class ShardedKVCache:
    """GQA cache (InplaceKVCache): per layer k, v [B*Hkv, cap, D] on this rank's GPU."""

    def __init__(self, num_layers, batch_size, num_kv_heads, max_seq, head_dim, dtype=torch.bfloat16,
                 world: int = 1, rank: int = 0, device=None):
        self._nl, self._bs, self._kv_h, self._max_seq, self._hd = num_layers, batch_size, num_kv_heads, max_seq, head_dim
        self._bkv = batch_size * num_kv_heads
        self._dtype = dtype
        self.world, self.rank = world, rank
        self.cap = shard_capacity(max_seq, world)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.key_cache = [None] * num_layers
        self.value_cache = [None] * num_layers
        self._filled = [0] * num_layers

    def _ensure_buffer(self, li):
        if self.key_cache[li] is None:
            shape = (self._bkv, self.cap, self._hd)
            self.key_cache[li] = torch.empty(shape, dtype=self._dtype, device=self.device)
            self.value_cache[li] = torch.empty(shape, dtype=self._dtype, device=self.device)

    def append_4d(self, li, k_4d, v_4d):
        """k_4d, v_4d [B, Hkv, new_seq, D] on this rank's device (every rank is given
        the step's tokens; each stores the positions it owns)."""
        new_seq = k_4d.shape[2]
        if self._filled[li] + new_seq > self._max_seq:
            raise RuntimeError("KV cache full")
        self._ensure_buffer(li)
        t = self._filled[li]
        first, cnt, t0 = local_slice(t, new_seq, self.cap, self.rank)
        if cnt:
            k = k_4d.reshape(self._bkv, new_seq, self._hd)[:, first:first + cnt]
            v = v_4d.reshape(self._bkv, new_seq, self._hd)[:, first:first + cnt]
            _append(self.key_cache[li], k, t0)
            _append(self.value_cache[li], v, t0)
        self._filled[li] = t + new_seq

    def local_len(self, li) -> int:
        return min(max(self._filled[li] - self.rank * self.cap, 0), self.cap)

    def get(self, li):
        """This rank's filled part: k, v [B*Hkv, local_len, D] (views)."""
        self._ensure_buffer(li)
        n = self.local_len(li)
        return self.key_cache[li][:, :n], self.value_cache[li][:, :n]

    def seq_len(self, li) -> int:
        return self._filled[li]

    def reset(self):
        for i in range(self._nl):
            self.key_cache[i] = None
            self.value_cache[i] = None
            self._filled[i] = 0

    def decode(self, li, q, scale, exchange=None):
        """q [B, H, D] -> (out [B, H, D] bf16, lse [B, H] fp32) over all tokens of the
        layer.  With world > 1 pass the rank's PartialExchange(B*H, D, world)."""
        from .cpu_attn import gqa_decode
        k, v = self.get(li)
        B, H, D = q.shape
        qv = q.reshape(self._bkv, H // self._kv_h, D)
        if self.world == 1:
            out, lse = gqa_decode(qv, k, v, scale)
            return out.reshape(B, H, D), lse.reshape(B, H)
        if exchange is None:
            raise RuntimeError("decode: a PartialExchange is required when world > 1")
        # the kernel writes this rank's partial straight into the exchange block
        gqa_decode(qv, k, v, scale, out_dtype=torch.float32, out=exchange.part_o.view(self._bkv, H // self._kv_h, D),
                   lse=exchange.part_l.view(self._bkv, H // self._kv_h))
        out, lse = exchange.step(torch.bfloat16)
        return out.reshape(B, H, D), lse.reshape(B, H)


class ShardedKVCacheCompressed:
    """Absorbed-MLA cache (InplaceKVCacheCompressed): per layer c [B, cap, kv_lora_rank]
    and pe [B, cap, qk_rope_head_dim] on this rank's GPU."""

    def __init__(self, num_layers, batch_size, max_seq, kv_lora_rank, qk_rope_head_dim, dtype=torch.bfloat16,
                 world: int = 1, rank: int = 0, device=None):
        self._nl, self._B, self._ms, self._clr, self._qrd = num_layers, batch_size, max_seq, kv_lora_rank, qk_rope_head_dim
        self._dtype = dtype
        self.world, self.rank = world, rank
        self.cap = shard_capacity(max_seq, world)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.cache_c = [None] * num_layers
        self.cache_pe = [None] * num_layers
        self._filled = [0] * num_layers

    def _ensure(self, li):
        if self.cache_c[li] is None:
            self.cache_c[li] = torch.empty(self._B, self.cap, self._clr, dtype=self._dtype, device=self.device)
            self.cache_pe[li] = torch.empty(self._B, self.cap, self._qrd, dtype=self._dtype, device=self.device)

    def append(self, li, c_kv, k_pe, non_blocking=False):
        """c_kv [B, new_seq, kv_lora_rank], k_pe [B, new_seq, rope] on this rank's device."""
        new_seq = c_kv.shape[1]
        if self._filled[li] + new_seq > self._ms:
            raise RuntimeError("KV cache full")
        self._ensure(li)
        t = self._filled[li]
        first, cnt, t0 = local_slice(t, new_seq, self.cap, self.rank)
        if cnt:
            _append(self.cache_c[li], c_kv[:, first:first + cnt], t0)
            _append(self.cache_pe[li], k_pe[:, first:first + cnt], t0)
        self._filled[li] = t + new_seq

    def local_len(self, li) -> int:
        return min(max(self._filled[li] - self.rank * self.cap, 0), self.cap)

    def get(self, li):
        self._ensure(li)
        n = self.local_len(li)
        return self.cache_c[li][:, :n], self.cache_pe[li][:, :n]

    def seq_len(self, li) -> int:
        return self._filled[li]

    def reset(self):
        for i in range(self._nl):
            self._filled[i] = 0

    def decode(self, li, q_proj, q_pe, scale, exchange=None):
        """Absorbed-MLA decode over all tokens of the layer: q_proj [B*nH, 512],
        q_pe [B*nH, 64] -> (out [B*nH, 512] bf16 normalised, lse [B*nH] fp32).
        With world > 1 pass the rank's PartialExchange(B*nH, 512, world): the
        kernel writes this rank's fp32 partial into its block, then one
        exchange merges the shards (a rank holding no token of the layer
        contributes lse = -inf)."""
        from .cpu_attn import mla_decode
        c, pe = self.get(li)   # views of the [B, cap, *] buffers: the kernel reads them in place by batch stride
        if self.world == 1:
            return mla_decode(q_proj, q_pe, c, pe, scale)
        if exchange is None:
            raise RuntimeError("decode: a PartialExchange is required when world > 1")
        mla_decode(q_proj, q_pe, c, pe, scale, out_dtype=torch.float32, out=exchange.part_o, lse=exchange.part_l)
        return exchange.step(torch.bfloat16)
