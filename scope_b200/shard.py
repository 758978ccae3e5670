"""Sequence-sharded decode across GPUs: the shard plan and the one exchange step.

A physically partitioned KV cache puts a contiguous range of every sequence on
each GPU: GQA tokens [r*L/N, (r+1)*L/N) of every (sequence, kv-head) row, or
CSA compressed entries [r*nc/N, (r+1)*nc/N) of every sequence (a rank attends
to the ids of the global top-k list that fall in its range, rebased to its
local rows).  Each rank produces a normalised partial per query row, o fp32
and lse fp32; a rank whose range holds nothing of a row gives o = 0 and
lse = -inf.  The ranks then exchange the partials with one all_gather and merge
them by log-sum-exp -- the merge the reference's runtimes do on the host
(system/qwenoffload.py:1606-1617, system/mixoffload.py:1456-1464) -- here on
the device with ws_lse_merge_strided, straight from the gathered blocks.
There is no other collective on the path.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """The contiguous range [lo, hi) of n items that rank `rank` of `world` holds."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    return n * rank // world, n * (rank + 1) // world


def local_ids(ids: torch.Tensor, lo: int, hi: int) -> torch.Tensor:
    """The ids of one sequence's top-k list that fall in [lo, hi), rebased to
    local rows (host-side statement of what the CSA kernel selects in its
    ``sorted_shard`` / ``shard`` modes; the order of the list is kept)."""
    sel = ids[(ids >= lo) & (ids < hi)]
    return sel - lo


class PartialExchange:
    """Buffers and the exchange step for R query rows of width D over `world` ranks.

    This rank's kernel writes its partial into part_o [R, D] and part_l [R],
    which are views of one block [o (R*D), lse (R)], so ``gather()`` is a single
    all_gather into [world, R*D + R]; ``merge()`` reduces that in place by
    log-sum-exp (ws_lse_merge_strided by default).
    """

    def __init__(self, rows: int, dim: int, world: int, device, group=None):
        self.world, self.group, self.rows, self.dim = world, group, rows, dim
        self.block = rows * dim + rows
        self.part = torch.empty(self.block, dtype=torch.float32, device=device)
        self.part_o = self.part[:rows * dim].view(rows, dim)
        self.part_l = self.part[rows * dim:]
        self.all = torch.empty(world, self.block, dtype=torch.float32, device=device)
        self.all_o = self.all[:, :rows * dim].view(world, rows, dim)   # strided views of the gathered blocks
        self.all_l = self.all[:, rows * dim:]

    def gather(self) -> None:
        dist.all_gather_into_tensor(self.all.view(-1), self.part, group=self.group)

    def merge(self, out_dtype=torch.bfloat16, out=None, out_lse=None, merge_fn: Callable | None = None):
        if merge_fn is not None:
            return merge_fn(self.all_o.contiguous(), self.all_l.contiguous(), out_dtype, out=out, out_lse=out_lse)
        from . import _lib
        from ._lib import check, lib, ptr, stream_ptr
        dev = self.all.device
        if out is None:
            out = torch.empty(self.rows, self.dim, dtype=out_dtype, device=dev)
        if out_lse is None:
            out_lse = torch.empty(self.rows, dtype=torch.float32, device=dev)
        code = _lib.WS_DTYPE_BF16 if out.dtype == torch.bfloat16 else _lib.WS_DTYPE_F32
        with torch.cuda.device(dev):
            rc = lib().ws_lse_merge_strided(ptr(self.all), self.block, ptr(self.all) + 4 * self.rows * self.dim,
                                            self.block, self.world, self.rows, self.dim, ptr(out), code,
                                            ptr(out_lse), stream_ptr(dev))
        check(rc, "ws_lse_merge_strided")
        return out, out_lse

    def step(self, out_dtype=torch.bfloat16, out=None, out_lse=None, merge_fn: Callable | None = None):
        self.gather()
        return self.merge(out_dtype, out=out, out_lse=out_lse, merge_fn=merge_fn)
