"""The multi-GPU path's host logic on CPU: world-size-2 (and 3) gloo process
groups run the shard plan of scope_b200.shard, compute each rank's partial
with the float64 oracle, exchange the partials with PartialExchange (one
all_gather) and merge them; the result must equal the unsharded oracle.

Covered: GQA tokens sharded contiguously (cfg4's layout), CSA entries sharded
with the global sorted top-k list rebased per shard (cfg5's layout), a rank
whose shard holds no selected entry (lse = -inf), and a rank that raises
before the exchange (the others' collective ends with an error, not a hang).
"""
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from scope_b200.shard import PartialExchange, local_ids, shard_bounds


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_merge(all_o, all_l, out_dtype=None, out=None, out_lse=None):
    o, lse = oracle.lse_merge(all_o.numpy(), all_l.numpy())
    return torch.from_numpy(o), torch.from_numpy(lse)


def gqa_case(seed=4, B=2, Hkv=2, G=4, D=64, L=301):
    g = np.random.default_rng(seed)
    q = oracle.f32_to_bf16_bits(g.standard_normal((B * Hkv, G, D)).astype(np.float32))
    k = oracle.f32_to_bf16_bits(g.standard_normal((B * Hkv, L, D)).astype(np.float32))
    v = oracle.f32_to_bf16_bits(g.standard_normal((B * Hkv, L, D)).astype(np.float32))
    return q, k, v, D ** -0.5


def csa_case(seed=5, bs=2, nq=8, nc=400, k=120, skew=False):
    g = np.random.default_rng(seed)
    q = g.standard_normal((bs, nq, 512)).astype(np.float32)
    kv = np.clip(np.round(g.standard_normal((bs, nc, 512)) * 32), -127, 127).astype(np.int8)
    sc = (g.random((bs, nc)) * 0.04 + 0.01).astype(np.float32)
    hi = nc // 3 if skew else nc          # skew: every id in the first third (the last rank gets nothing)
    idx = np.stack([np.sort(g.choice(hi, size=k, replace=False)) for _ in range(bs)]).astype(np.int32)
    return q, kv, sc, idx, 512 ** -0.5


def worker(rank, world, port, kind, results):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        if kind == "gqa":
            q, k, v, sc = gqa_case()
            L = k.shape[1]
            lo, hi = shard_bounds(L, world, rank)
            o, m, s = oracle.gqa_decode(q, k[:, lo:hi], v[:, lo:hi], sc)
            rows, D = q.shape[0] * q.shape[1], q.shape[2]
            ex = PartialExchange(rows, D, world, "cpu")
            ex.part_o.copy_(torch.from_numpy(o.reshape(rows, D)))
            lse = np.where(s > 0, m + np.log(np.where(s > 0, s, 1.0)), -np.inf)
            ex.part_l.copy_(torch.from_numpy(lse.reshape(rows)))
        else:
            q, kv, scl, idx, sc = csa_case(skew=(kind == "csa_skew"))
            nc = kv.shape[1]
            lo, hi = shard_bounds(nc, world, rank)
            bs, nq, _ = q.shape
            ex = PartialExchange(bs * nq, 512, world, "cpu")
            for b in range(bs):
                ids = local_ids(torch.from_numpy(idx[b]), lo, hi).numpy().astype(np.int32)
                o, lse, bad = oracle.csa_attend(q[b:b + 1], kv[b:b + 1, lo:hi], sc, idx=ids[None, :],
                                                kv_scale=scl[b:b + 1, lo:hi])
                assert bad == 0
                ex.part_o[b * nq:(b + 1) * nq].copy_(torch.from_numpy(o[0]))
                ex.part_l[b * nq:(b + 1) * nq].copy_(torch.from_numpy(lse[0]))
        if kind == "raise" and rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        out, out_lse = ex.step(merge_fn=oracle_merge)
        results[rank] = (out.numpy(), out_lse.numpy(), ex.part_l.numpy())
        dist.destroy_process_group()
    except Exception:
        results[rank] = ("error", traceback.format_exc())


def failed(r):
    return isinstance(r[0], str) and r[0] == "error"


def run_world(world, kind):
    port = free_port()
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=worker, args=(r, world, port, kind, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            p.join()
    return dict(results)


@pytest.mark.parametrize("world", [2, 3])
def test_gqa_token_shards_merge_to_unsharded(world):
    res = run_world(world, "gqa")
    q, k, v, sc = gqa_case()
    o, m, s = oracle.gqa_decode(q, k, v, sc)
    rows = q.shape[0] * q.shape[1]
    for r in range(world):
        assert not failed(res[r]), res[r][1]
        assert np.abs(res[r][0] - o.reshape(rows, -1)).max() < 2e-6   # the exchanged partials are fp32
        assert np.abs(res[r][1] - (m + np.log(s)).reshape(rows)).max() < 2e-6   # the exchanged partials are fp32


@pytest.mark.parametrize("world", [2, 3])
def test_csa_entry_shards_merge_to_unsharded(world):
    res = run_world(world, "csa")
    q, kv, scl, idx, sc = csa_case()
    o, lse, _ = oracle.csa_attend(q, kv, sc, idx=idx, kv_scale=scl)
    for r in range(world):
        assert not failed(res[r]), res[r][1]
        assert np.abs(res[r][0] - o.reshape(-1, 512)).max() < 2e-6   # the exchanged partials are fp32
        assert np.abs(res[r][1] - lse.reshape(-1)).max() < 2e-6   # the exchanged partials are fp32


def test_csa_rank_without_entries():
    res = run_world(3, "csa_skew")
    q, kv, scl, idx, sc = csa_case(skew=True)
    o, lse, _ = oracle.csa_attend(q, kv, sc, idx=idx, kv_scale=scl)
    assert not failed(res[2]), res[2][1]
    assert np.all(np.isneginf(res[2][2]))                   # the last rank's partial is empty
    for r in range(3):
        assert np.abs(res[r][0] - o.reshape(-1, 512)).max() < 2e-6   # the exchanged partials are fp32


def test_failed_rank_ends_the_exchange_with_an_error():
    res = run_world(2, "raise")
    assert failed(res[1]) and "rank 1 fails" in res[1][1]
    assert failed(res[0])                                    # the survivor's all_gather errored, no hang


def test_shard_bounds_cover_exactly():
    for n in (0, 1, 7, 131072):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    ids = torch.tensor([3, 9, 10, 15, 40])
    assert local_ids(ids, 9, 16).tolist() == [0, 1, 6]
