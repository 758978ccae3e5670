"""Sequence-sharded decode across two GPUs over NCCL, checked on hardware.

Two processes (one per GPU, spawned, NCCL process group with a short
timeout) each hold a contiguous shard of every row: GQA tokens
[r*L/2, (r+1)*L/2) or CSA entries [r*nc/2, (r+1)*nc/2).  Each decodes its
shard with the CUDA kernel into the PartialExchange block, the partials are
exchanged with one all_gather and merged by ws_lse_merge_strided, and rank 0
compares the merged rows with the float64 oracle over the whole rows
(max-abs 2e-2 on bf16 outputs, 1e-3 on LSE).  Needs two GPUs; skipped
otherwise.
"""
import datetime
import multiprocessing as mp
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_OUT = 2e-2
TOL_LSE = 1e-3
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gqa_rank(rank, port, q, k, v, scale):
    import torch.distributed as dist

    import scope_b200
    from scope_b200 import _lib
    from scope_b200.shard import PartialExchange, shard_bounds
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=WORLD, rank=rank,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        scope_b200.build()
        rows, G, D = q.shape
        L = k.shape[1]
        lo, hi = shard_bounds(L, WORLD, rank)
        qd = q.to(dev)
        kd, vd = k[:, lo:hi].contiguous().to(dev), v[:, lo:hi].contiguous().to(dev)
        ex = PartialExchange(rows * G, D, WORLD, dev)
        L_ = _lib.lib()
        ws = torch.zeros(L_.ws_gqa_decode_workspace_size(rows, G, D, hi - lo), dtype=torch.uint8, device=dev)
        rc = L_.ws_gqa_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), kd.stride(0), kd.stride(1), vd.stride(0),
                              vd.stride(1), rows, G, D, D, hi - lo, scale, _lib.WS_DTYPE_BF16, _lib.WS_OUT_NORM_F32,
                              ex.part_o.data_ptr(), None, None, ex.part_l.data_ptr(), ws.data_ptr(), ws.numel(),
                              torch.cuda.current_stream().cuda_stream)
        assert rc == 0, L_.ws_last_error()
        out, lse = ex.step(torch.bfloat16)
        torch.cuda.synchronize()
        return out.float().cpu().numpy(), lse.cpu().numpy()
    finally:
        dist.destroy_process_group()


def _csa_rank(rank, port, q, kv, sc, idx, scale):
    import torch.distributed as dist

    import scope_b200
    import scope_b200.csa_attn as csa_attn
    from scope_b200.shard import PartialExchange, shard_bounds
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=WORLD, rank=rank,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        scope_b200.build_csa_attn()
        bs, nH, D = q.shape
        lo, hi = shard_bounds(kv.shape[1], WORLD, rank)
        po, pl = csa_attn.csa_sparse_decode(q.to(dev), kv[:, lo:hi].contiguous().to(dev), idx.to(dev), scale,
                                            sc[:, lo:hi].contiguous().to(dev), shard_lo=lo, idx_mode="sorted_shard",
                                            out_dtype=torch.float32)
        ex = PartialExchange(bs * nH, D, WORLD, dev)
        ex.part_o.copy_(po.view(-1, D))
        ex.part_l.copy_(pl.view(-1))
        out, lse = ex.step(torch.bfloat16)
        torch.cuda.synchronize()
        return out.float().cpu().numpy(), lse.cpu().numpy()
    finally:
        dist.destroy_process_group()


def _child(fn, rank, port, args, queue):
    try:
        queue.put((rank, "ok", fn(rank, port, *args)))
    except BaseException as e:   # reported to the parent, which fails the test
        queue.put((rank, "error", repr(e)))


def _run_two_ranks(fn, args):
    """Run fn(rank, port, *args) on ranks 0 and 1 (GPUs 0 and 1) in spawned
    processes; returns rank 0's result.  Bounded: a rank that does not report
    within the limit fails the test and its process is terminated."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_child, args=(fn, r, port, args, queue)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, status, payload = queue.get(timeout=240)
            results[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for r in range(WORLD):
        assert results[r][0] == "ok", f"rank {r}: {results[r][1]}"
    return results[0][1]


needs_two = pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")


@needs_two
@pytest.mark.parametrize("L", [8192, 4097])
def test_gqa_sharded_over_nccl(L):
    import oracle
    g = torch.Generator().manual_seed(31 + L)
    rows, G, D = 8, 8, 128
    q = torch.randn(rows, G, D, generator=g).bfloat16()
    k = torch.randn(rows, L, D, generator=g).bfloat16()
    v = torch.randn(rows, L, D, generator=g).bfloat16()
    scale = D ** -0.5
    out, lse = _run_two_ranks(_gqa_rank, (q, k, v, scale))
    ro, rm, rs = oracle.gqa_decode(oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v), scale)
    assert np.abs(out - ro.reshape(rows * G, D)).max() < TOL_OUT
    assert np.abs(lse - (rm + np.log(rs)).reshape(rows * G)).max() < TOL_LSE


@needs_two
def test_csa_sharded_over_nccl():
    import oracle
    g = torch.Generator().manual_seed(37)
    bs, nH, nc, kk = 4, 64, 8192, 1024
    q = torch.randn(bs, nH, 512, generator=g).bfloat16()
    kv = (torch.randn(bs, nc, 512, generator=g) * 32).round().clamp(-127, 127).to(torch.int8)
    sc = torch.rand(bs, nc, generator=g) * 0.04 + 0.01
    idx = torch.stack([torch.randperm(nc, generator=g)[:kk].sort().values for _ in range(bs)]).int()
    idx[0] = torch.arange(kk, dtype=torch.int32)   # sequence 0 selects only rank 0's entries: rank 1 sends -inf
    scale = 512 ** -0.5
    out, lse = _run_two_ranks(_csa_rank, (q, kv, sc, idx, scale))
    ro, rl, bad = oracle.csa_attend(oracle.bf16_bits(q), kv.numpy(), scale, idx=idx.numpy(), kv_scale=sc.numpy())
    assert bad == 0
    assert np.abs(out - ro.reshape(bs * nH, 512)).max() < TOL_OUT
    assert np.abs(lse - rl.reshape(bs * nH)).max() < TOL_LSE


def _cache_rank(rank, port, q, k4, v4, qp, qpe, c, p):
    """Both sharded caches at world 2: every rank is given all tokens, stores
    its half, and decode() runs the local kernel into the exchange block and
    the one exchange."""
    import torch.distributed as dist

    import scope_b200
    from scope_b200.kv_cache import ShardedKVCache, ShardedKVCacheCompressed
    from scope_b200.shard import PartialExchange
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=WORLD, rank=rank,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        scope_b200.build()
        B, H, D = q.shape
        Hkv, L = k4.shape[1], k4.shape[2]
        gq = ShardedKVCache(1, B, Hkv, L + 64, D, world=WORLD, rank=rank, device=dev)
        gq.append_4d(0, k4[:, :, :L - 1].to(dev), v4[:, :, :L - 1].to(dev))
        gq.append_4d(0, k4[:, :, L - 1:].to(dev), v4[:, :, L - 1:].to(dev))   # a decode step's new token
        out, lse = gq.decode(0, q.to(dev), D ** -0.5, exchange=PartialExchange(B * H, D, WORLD, dev))
        S = c.shape[1]
        mc = ShardedKVCacheCompressed(1, c.shape[0], S + 100, 512, 64, world=WORLD, rank=rank, device=dev)
        mc.append(0, c.to(dev), p.to(dev))
        mo, ml = mc.decode(0, qp.to(dev), qpe.to(dev), 192 ** -0.5,
                           exchange=PartialExchange(qp.shape[0], 512, WORLD, dev))
        torch.cuda.synchronize()
        return (out.float().cpu().numpy(), lse.cpu().numpy(), mo.float().cpu().numpy(), ml.cpu().numpy())
    finally:
        dist.destroy_process_group()


@needs_two
def test_sharded_caches_decode_over_nccl():
    import oracle
    g = torch.Generator().manual_seed(41)
    B, H, Hkv, D, L = 2, 32, 4, 128, 3001
    q = torch.randn(B, H, D, generator=g).bfloat16()
    k4 = torch.randn(B, Hkv, L, D, generator=g).bfloat16()
    v4 = torch.randn(B, Hkv, L, D, generator=g).bfloat16()
    Bm, nH, S = 2, 16, 1100
    qp = torch.randn(Bm * nH, 512, generator=g).bfloat16()
    qpe = torch.randn(Bm * nH, 64, generator=g).bfloat16()
    c = torch.randn(Bm, S, 512, generator=g).bfloat16()
    p = torch.randn(Bm, S, 64, generator=g).bfloat16()
    out, lse, mo, ml = _run_two_ranks(_cache_rank, (q, k4, v4, qp, qpe, c, p))
    G = H // Hkv
    ro, rm, rs = oracle.gqa_decode(oracle.bf16_bits(q.view(B * Hkv, G, D)),
                                   oracle.bf16_bits(k4.reshape(B * Hkv, L, D)),
                                   oracle.bf16_bits(v4.reshape(B * Hkv, L, D)), D ** -0.5)
    assert np.abs(out.reshape(B * H, D) - ro.reshape(B * H, D)).max() < TOL_OUT
    assert np.abs(lse.reshape(-1) - (rm + np.log(rs)).reshape(-1)).max() < TOL_LSE
    mro, mrm, mrs = oracle.mla_compressed(*(oracle.bf16_bits(t) for t in (qp, qpe, c, p)), 192 ** -0.5)
    assert np.abs(mo - mro / mrs[:, None]).max() < TOL_OUT
    assert np.abs(ml - (mrm + np.log(mrs))).max() < TOL_LSE


def _peer_rank(rank, port, qs, ks, vs, scale, kind="push", n_graph=3):
    """Steps of a sharded GQA decode whose partials go over NVLink peer memory
    (kind "push": PeerExchange, into rank 0's slots; "scatter": ScatterExchange,
    each rank merging its share of the rows): eager steps, then replays of a
    captured CUDA graph of decode + exchange; rank 0 returns every step's merge."""
    import torch.distributed as dist

    import scope_b200
    from scope_b200 import _lib
    from scope_b200.shard import PeerExchange, ScatterExchange, shard_bounds
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=WORLD, rank=rank,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        scope_b200.build()
        rows, G, D = qs[0].shape
        L = ks[0].shape[1]
        lo, hi = shard_bounds(L, WORLD, rank)
        ex = (PeerExchange(rows * G, D, WORLD, rank, dev) if kind == "push"
              else ScatterExchange(rows * G, D, WORLD, rank, dev))
        L_ = _lib.lib()
        ws = torch.zeros(L_.ws_gqa_decode_workspace_size(rows, G, D, hi - lo), dtype=torch.uint8, device=dev)
        outs = []
        # static buffers: the first steps run eagerly, the last ones replay a captured CUDA graph of the same
        # decode + exchange after their inputs are copied in (the exchange counts its steps on the devices)
        qd = torch.empty_like(qs[0], device=dev)
        kd = torch.empty(rows, hi - lo, D, dtype=torch.bfloat16, device=dev)
        vd = torch.empty_like(kd)
        out0 = torch.empty(rows * G, D, dtype=torch.bfloat16, device=dev)
        lse0 = torch.empty(rows * G, dtype=torch.float32, device=dev)

        def one_step():
            o_ptr, l_ptr = ex.slot()
            rc = L_.ws_gqa_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), kd.stride(0), kd.stride(1),
                                  vd.stride(0), vd.stride(1), rows, G, D, D, hi - lo, scale, _lib.WS_DTYPE_BF16,
                                  _lib.WS_OUT_NORM_F32, o_ptr, None, None, l_ptr, ws.data_ptr(), ws.numel(),
                                  torch.cuda.current_stream().cuda_stream)
            assert rc == 0, L_.ws_last_error()
            ex.step(out=out0 if rank == 0 else None, out_lse=lse0 if rank == 0 else None)

        n_eager = len(qs) - n_graph
        graph = None
        for s, (q, k, v) in enumerate(zip(qs, ks, vs)):
            qd.copy_(q)
            kd.copy_(k[:, lo:hi])
            vd.copy_(v[:, lo:hi])
            if s < n_eager:   # back to back on one stream, no host synchronisation between steps
                one_step()
            else:
                if graph is None:
                    torch.cuda.synchronize()
                    side = torch.cuda.Stream()
                    side.wait_stream(torch.cuda.current_stream())
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=side):
                        one_step()   # captured, not run
                    torch.cuda.synchronize()
                graph.replay()
            if rank == 0:
                outs.append((out0.float().clone(), lse0.clone()))
        torch.cuda.synchronize()
        status = scope_b200.status_take()
        ex.close()
        assert status == 0, status
        return [(o.cpu().numpy(), l_.cpu().numpy()) for o, l_ in outs]
    finally:
        dist.destroy_process_group()


@needs_two
@pytest.mark.parametrize("kind,rows,G", [("push", 8, 8), ("scatter", 8, 8), ("scatter", 35, 1)])
def test_peer_exchange_steps(kind, rows, G):
    """35 x 1 query rows split 17 / 18 between the scatter form's two shares."""
    import oracle
    g = torch.Generator().manual_seed(53)
    D, L, steps = 128, 6001, 7   # 4 eager steps, then 3 replays of a captured graph
    qs = [torch.randn(rows, G, D, generator=g).bfloat16() for _ in range(steps)]
    ks = [torch.randn(rows, L, D, generator=g).bfloat16() for _ in range(steps)]
    vs = [torch.randn(rows, L, D, generator=g).bfloat16() for _ in range(steps)]
    scale = D ** -0.5
    res = _run_two_ranks(_peer_rank, (qs, ks, vs, scale, kind))
    assert len(res) == steps
    for (out, lse), q, k, v in zip(res, qs, ks, vs):
        ro, rm, rs = oracle.gqa_decode(oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v), scale)
        assert np.abs(out - ro.reshape(rows * G, D)).max() < TOL_OUT
        assert np.abs(lse - (rm + np.log(rs)).reshape(rows * G)).max() < TOL_LSE
