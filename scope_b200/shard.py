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
the device with ws_lse_merge.  There is no other collective on the path.
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

    part_o [R, D] / part_l [R] are where this rank's kernel writes its partial;
    ``gather()`` all-gathers them into all_o [world, R, D] / all_l [world, R];
    ``merge()`` reduces those by log-sum-exp (ws_lse_merge by default).
    """

    def __init__(self, rows: int, dim: int, world: int, device, group=None):
        self.world, self.group = world, group
        self.part_o = torch.empty(rows, dim, dtype=torch.float32, device=device)
        self.part_l = torch.empty(rows, dtype=torch.float32, device=device)
        self.all_o = torch.empty(world, rows, dim, dtype=torch.float32, device=device)
        self.all_l = torch.empty(world, rows, dtype=torch.float32, device=device)

    def gather(self) -> None:
        dist.all_gather_into_tensor(self.all_o.view(-1), self.part_o.view(-1), group=self.group)
        dist.all_gather_into_tensor(self.all_l.view(-1), self.part_l.view(-1), group=self.group)

    def merge(self, out_dtype=torch.bfloat16, out=None, out_lse=None,
              merge_fn: Callable | None = None):
        if merge_fn is None:
            from .ops import lse_merge
            merge_fn = lse_merge
        return merge_fn(self.all_o, self.all_l, out_dtype, out=out, out_lse=out_lse)

    def step(self, out_dtype=torch.bfloat16, out=None, out_lse=None, merge_fn: Callable | None = None):
        self.gather()
        return self.merge(out_dtype, out=out, out_lse=out_lse, merge_fn=merge_fn)
