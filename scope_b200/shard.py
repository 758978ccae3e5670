"""Sequence-sharded decode across GPUs: the shard plan and the one exchange step.

A physically partitioned KV cache puts a contiguous range of every sequence on
each GPU: GQA tokens [r*L/N, (r+1)*L/N) of every (sequence, kv-head) row, or
CSA compressed entries [r*nc/N, (r+1)*nc/N) of every sequence (a rank attends
to the ids of the global top-k list that fall in its range, rebased to its
local rows).  Each rank produces a normalised partial per query row, o fp32
and lse fp32; a rank whose range holds nothing of a row gives o = 0 and
lse = -inf.  The ranks then exchange the partials once and merge them by
log-sum-exp -- the merge the reference's runtimes do on the host
(system/qwenoffload.py:1606-1617, system/mixoffload.py:1456-1464) -- on the
device.  Three forms of that one exchange:

* PartialExchange: one NCCL all_gather of the blocks, then ws_lse_merge_strided
  on every rank (the result on every rank);
* PeerExchange: the blocks pushed into rank 0's slots over NVLink peer memory,
  merged there (the result on rank 0);
* ScatterExchange: each rank merges one share of the rows from its peers'
  copies and sends the merged share to rank 0 (the result on rank 0).

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


class PeerExchange:
    """The exchange over NVLink peer memory: rank 0 gathers, merges and holds
    the result (ws_peer_push / ws_peer_merge in include/scope_b200.h).

    Rank 0 allocates the buffer and broadcasts its CUDA IPC handle; the other
    ranks map it.  Before a step, a rank's decode writes its partial at
    ``slot()`` -- (o pointer, lse pointer): rank 0's own slot, or a local
    block on the other ranks -- then ``step()`` pushes the block into rank 0's
    slot and raises the rank's flag (ranks > 0, one launch) or waits for every
    flag, merges and returns (out, out_lse) (rank 0; None elsewhere).  Every
    rank must call ``step()`` once per step, in the same order.  The step
    counts live on the devices and the pointers never change, so the steps may
    be captured in a CUDA graph.
    """

    def __init__(self, rows: int, dim: int, world: int, rank: int, device, group=None):
        import ctypes

        from ._lib import check, lib
        self.rows, self.dim, self.world, self.rank, self.group = rows, dim, world, rank, group
        self.device = torch.device(device)
        L = lib()
        nbytes = L.ws_peer_exchange_bytes(world, rows, dim)
        if nbytes == 0:
            raise ValueError("PeerExchange: bad world / rows / dim")
        handle = ctypes.create_string_buffer(64)
        base = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            if rank == 0:
                check(L.ws_peer_buffer_create(nbytes, ctypes.byref(base), handle), "ws_peer_buffer_create")
            objs = [handle.raw if rank == 0 else None]
            dist.broadcast_object_list(objs, src=0, group=group)
            if rank != 0:
                check(L.ws_peer_buffer_open(ctypes.create_string_buffer(objs[0], 64), ctypes.byref(base)),
                      "ws_peer_buffer_open")
        self.base = base.value
        self._closed = False
        if rank != 0:
            # the decode writes here (local memory); ws_peer_push copies it into rank 0's slot
            n = -(-(rows * dim + rows) // 64) * 64
            self.block = torch.empty(n, dtype=torch.float32, device=self.device)
            self.state = torch.zeros(2, dtype=torch.int64, device=self.device)   # step count, CTA ticket

    def slot(self):
        """(o, lse) device addresses where this rank's decode writes its partial."""
        from ._lib import lib
        if self.rank != 0:
            o = self.block.data_ptr()
        else:
            o = self.base + lib().ws_peer_slot_offset(self.world, self.rows, self.dim, 0)
        return o, o + 4 * self.rows * self.dim

    def step(self, out=None, out_lse=None, out_dtype=torch.bfloat16):
        from . import _lib
        from ._lib import check, lib, stream_ptr
        with torch.cuda.device(self.device):
            st = stream_ptr(self.device)
            if self.rank == 0:
                if out is None:
                    out = torch.empty(self.rows, self.dim, dtype=out_dtype, device=self.device)
                if out_lse is None:
                    out_lse = torch.empty(self.rows, dtype=torch.float32, device=self.device)
                code = _lib.WS_DTYPE_BF16 if out.dtype == torch.bfloat16 else _lib.WS_DTYPE_F32
                check(lib().ws_peer_merge(self.base, self.world, self.rows, self.dim, out.data_ptr(), code,
                                          out_lse.data_ptr(), st), "ws_peer_merge")
                return out, out_lse
            check(lib().ws_peer_push(self.block.data_ptr(), self.base, self.world, self.rows, self.dim, self.rank,
                                     self.state.data_ptr(), st), "ws_peer_push")
        return None, None

    def close(self) -> None:
        """Collective: unmap on ranks > 0, then free on rank 0."""
        from ._lib import lib
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            if self.rank != 0:
                lib().ws_peer_buffer_close(self.base)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            if self.rank == 0:
                lib().ws_peer_buffer_free(self.base)
        self._closed = True


class ScatterExchange:
    """The exchange over NVLink peer memory in scatter-merge form
    (ws_peer_rs_scatter / ws_peer_rs_merge in include/scope_b200.h).

    Every rank allocates a buffer, the ranks all-gather their CUDA IPC handles
    and each maps every other rank's.  Each rank owns the share of rows
    ``shard_bounds(rows, world, rank)`` and merges it: its decode writes its
    whole partial at ``slot()`` (a local block), ``step()`` copies every
    peer's rows into that peer's buffer, waits for the peers' rows of its own
    share, merges them, and sends the merged share to rank 0 in ``out_dtype``.
    Rank 0 returns (out, out_lse) for all rows; the others (None, None).  A
    rank sends and receives (world - 1) / world of one block per step, against
    (world - 1) blocks into rank 0 for PeerExchange, so it pays when the
    partials are large (many query rows, wide latents) or world is large.
    Every rank calls ``step()`` once per step, in the same order; the step
    counts live on the devices, so the steps may be captured in a CUDA graph.
    """

    def __init__(self, rows: int, dim: int, world: int, rank: int, device, out_dtype=torch.bfloat16, group=None):
        import ctypes

        from ._lib import check, lib
        self.rows, self.dim, self.world, self.rank, self.group = rows, dim, world, rank, group
        self.device = torch.device(device)
        if out_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("ScatterExchange: out_dtype bf16 or fp32")
        self.out_dtype = out_dtype
        L = lib()
        nbytes = L.ws_peer_rs_bytes(world, rows, dim)
        if nbytes == 0:
            raise ValueError("ScatterExchange: bad world / rows / dim (world <= 32, dim % 4 == 0)")
        handle = ctypes.create_string_buffer(64)
        own = ctypes.c_void_p()
        self._closed = False
        with torch.cuda.device(self.device):
            check(L.ws_peer_buffer_create(nbytes, ctypes.byref(own), handle), "ws_peer_buffer_create")
            handles = [None] * world
            dist.all_gather_object(handles, handle.raw, group=group)
            ptrs, self._mapped = [], []
            for q in range(world):
                if q == rank:
                    ptrs.append(own.value)
                    continue
                b = ctypes.c_void_p()
                check(L.ws_peer_buffer_open(ctypes.create_string_buffer(handles[q], 64), ctypes.byref(b)),
                      "ws_peer_buffer_open")
                ptrs.append(b.value)
                self._mapped.append(b.value)
        self.own = own.value
        self.bases = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        n = -(-(rows * dim + rows) // 64) * 64
        self.block = torch.empty(n, dtype=torch.float32, device=self.device)   # this rank's partial, local
        self.state = torch.zeros(2, dtype=torch.int64, device=self.device)     # step count; ticket + failure mark

    def slot(self):
        """(o, lse) device addresses where this rank's decode writes its partial."""
        o = self.block.data_ptr()
        return o, o + 4 * self.rows * self.dim

    def step(self, out=None, out_lse=None):
        from . import _lib
        from ._lib import check, lib, stream_ptr
        code = _lib.WS_DTYPE_BF16 if self.out_dtype == torch.bfloat16 else _lib.WS_DTYPE_F32
        with torch.cuda.device(self.device):
            st = stream_ptr(self.device)
            if self.rank == 0:
                if out is None:
                    out = torch.empty(self.rows, self.dim, dtype=self.out_dtype, device=self.device)
                if out.dtype != self.out_dtype or out.numel() != self.rows * self.dim or not out.is_contiguous():
                    raise ValueError("ScatterExchange.step: out must be contiguous [rows, dim] of out_dtype")
                if out_lse is None:
                    out_lse = torch.empty(self.rows, dtype=torch.float32, device=self.device)
            L = lib()
            check(L.ws_peer_rs_scatter(self.block.data_ptr(), self.bases.data_ptr(), self.world, self.rows,
                                       self.dim, self.rank, self.state.data_ptr(), st), "ws_peer_rs_scatter")
            check(L.ws_peer_rs_merge(self.block.data_ptr(), self.bases.data_ptr(), self.world, self.rows, self.dim,
                                     self.rank, self.state.data_ptr(), out.data_ptr() if self.rank == 0 else None,
                                     code, out_lse.data_ptr() if self.rank == 0 else None, st), "ws_peer_rs_merge")
        return (out, out_lse) if self.rank == 0 else (None, None)

    def close(self) -> None:
        """Collective: unmap the peers' buffers, then free this rank's."""
        from ._lib import lib
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for b in self._mapped:
                lib().ws_peer_buffer_close(b)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            lib().ws_peer_buffer_free(self.own)
        self._closed = True
