"""GPU check of the exchange step's merge (ws_lse_merge_strided over the
gathered [o (R*D), lse (R)] blocks): the blocks of three entry shards of a CSA
cache, filled as one all_gather would leave them, must merge to the unsharded
result.  The collective itself is covered by the gloo tests and the N>1 bench."""
import pytest
import torch

import scope_b200
import scope_b200.csa_attn   # the submodule is imported on first use, not by the package
from scope_b200.shard import PartialExchange, shard_bounds

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_strided_merge_of_gathered_blocks():
    g = torch.Generator().manual_seed(81)
    bs, nH, nc, k, world = 3, 64, 3000, 700, 3
    q = torch.randn(bs, nH, 512, generator=g).bfloat16().to(DEV)
    kv = (torch.randn(bs, nc, 512, generator=g) * 32).round().clamp(-127, 127).to(torch.int8).to(DEV)
    sc = (torch.rand(bs, nc, generator=g) * 0.04 + 0.01).to(DEV)
    idx = torch.stack([torch.randperm(nc, generator=g)[:k].sort().values for _ in range(bs)]).int().to(DEV)
    full_o, full_l = scope_b200.csa_attn.csa_sparse_decode(q, kv, idx, 512 ** -0.5, sc, out_dtype=torch.float32)
    ex = PartialExchange(bs * nH, 512, world, DEV)
    for r in range(world):
        lo, hi = shard_bounds(nc, world, r)
        po, pl = scope_b200.csa_attn.csa_sparse_decode(q, kv[:, lo:hi].contiguous(), idx, 512 ** -0.5,
                                                       sc[:, lo:hi].contiguous(), shard_lo=lo,
                                                       idx_mode="sorted_shard", out_dtype=torch.float32)
        ex.all_o[r].copy_(po.view(-1, 512))
        ex.all_l[r].copy_(pl.view(-1))
    out, lse = ex.merge(torch.float32)
    assert (out - full_o.view(-1, 512)).abs().max().item() < 5e-3
    assert (lse - full_l.view(-1)).abs().max().item() < 1e-4
    ref_o, ref_l = scope_b200.lse_merge(ex.all_o.contiguous(), ex.all_l.contiguous(), torch.float32)
    assert torch.equal(out, ref_o) and torch.equal(lse, ref_l)
