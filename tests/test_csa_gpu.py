"""GPU parity of the CSA kernel (ws_csa_decode) and the int8 quantisers.

Against the reference's golden outputs (fused_csa_attn, fused_csa_attn_range,
indexer_attn_cpu, the bf16-query variants and the integer-score int8 family,
kernel/cpu_attn_ds4_ext/csa_attn.cpp) and against the float64 oracle on seeded
inputs.  Tolerances: normalised output max-abs 2e-2, LSE 1e-3 everywhere; the
quantisers and the gather are checked bit for bit.
"""
import numpy as np
import pytest
import torch

import oracle
import scope_b200
import scope_b200.csa_attn   # the submodule is imported on first use, not by the package

pytestmark = pytest.mark.gpu

TOL_OUT = 2e-2
TOL_LSE = 1e-3
DEV = "cuda:0"


@pytest.fixture(scope="module")
def csa():
    return scope_b200.build_csa_attn()


def bf16_dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def rand_case(bs, nq, nc, k, seed, int8=False, q_bf16=False, sorted_ids=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(bs, nq, 512, generator=g)
    if q_bf16:
        q = q.bfloat16()
    if int8:   # per sequence, to bound host memory at the benchmark size
        kv = torch.stack([(torch.randn(nc, 512, generator=g) * 32).round().clamp(-127, 127).to(torch.int8)
                          for _ in range(bs)])
        sc = torch.rand(bs, nc, generator=g) * 0.04 + 0.01
    else:
        kv = torch.randn(bs, nc, 512, generator=g).bfloat16()
        sc = None
    idx = None
    if k is not None:
        rows = []
        for _ in range(bs):
            r = torch.randperm(nc, generator=g)[:k]
            rows.append(r.sort().values if sorted_ids else r)
        idx = torch.stack(rows).int()
    return q, kv, sc, idx


def oracle_of(q, kv, sc, scale, idx=None, kv_range=None):
    qn = oracle.bf16_bits(q) if q.dtype == torch.bfloat16 else q.numpy()
    kvn = kv.numpy() if kv.dtype == torch.int8 else oracle.bf16_bits(kv)
    return oracle.csa_attend(qn, kvn, scale, idx=None if idx is None else idx.numpy(), kv_range=kv_range,
                             kv_scale=None if sc is None else sc.numpy())


def run_gather(q, kv, sc, idx, scale, out_dtype=torch.float32, **kw):
    out, lse = scope_b200.csa_attn.csa_sparse_decode(
        q.to(DEV), kv.to(DEV), idx.to(DEV), scale, None if sc is None else sc.to(DEV), out_dtype=out_dtype, **kw)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


# ------------------------------------------------------------ golden vectors
def test_golden_dense(csa, golden):
    g = golden("csa")
    q = torch.from_numpy(g["q"]).to(DEV)
    o, lse = csa.fused_csa_attn(q, bf16_dev(g["kv"]), float(g["scale"]))
    assert o.dtype == torch.float32 and o.shape == q.shape and lse.shape == q.shape[:-1]
    assert np.abs(o.cpu().numpy() - g["dense_o"]).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - g["dense_lse"]).max() < TOL_LSE


def test_golden_range(csa, golden):
    g = golden("csa")
    q = torch.from_numpy(g["q"]).to(DEV)
    o, lse = csa.fused_csa_attn_range(q, bf16_dev(g["kv"]), float(g["scale"]), int(g["range_s"]), int(g["range_e"]))
    assert np.abs(o.cpu().numpy() - g["range_o"]).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - g["range_lse"]).max() < TOL_LSE


def test_golden_gather(csa, golden):
    g = golden("csa")
    q = torch.from_numpy(g["q_gather"]).to(DEV)
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:-1], device=DEV)
    csa.indexer_attn_cpu(q, bf16_dev(g["kv"]), torch.from_numpy(g["idx"]).to(DEV), float(g["scale"]), o, lse)
    assert np.abs(o.cpu().numpy() - g["gather_o"]).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - g["gather_lse"]).max() < TOL_LSE


def test_golden_inplace_variants(csa, golden):
    """fp32-query in-place forms against the reference's fused_csa_attn output."""
    g = golden("csa")
    qf = torch.from_numpy(g["q"]).to(DEV)
    kv = bf16_dev(g["kv"])
    sc = float(g["scale"])
    for fn in (csa.fused_csa_attn_bsq, csa.fused_csa_attn_inplace):
        o = torch.full(qf.shape, float("nan"), device=DEV)
        lse = torch.full(qf.shape[:-1], float("nan"), device=DEV)
        fn(qf, kv, sc, o, lse)
        assert np.abs(o.cpu().numpy() - g["dense_o"]).max() < TOL_OUT, fn.__name__
        assert np.abs(lse.cpu().numpy() - g["dense_lse"]).max() < TOL_LSE, fn.__name__


@pytest.mark.parametrize("tag", ["h512", "h256"])
def test_golden_bf16_query_variants(csa, golden, tag):
    """_pool_bf16, _bsq_bf16, _fast_bf16 and _2pass_bf16 against the reference's
    own outputs on a bf16 query (csa_attn.cpp:379-474, :580-764, :885-1048,
    :1050-1173), at the full bar; hd 256 runs through the zero-padded path."""
    g = golden("csa_bf16q")
    q, kv, sc = bf16_dev(g[tag + "_q"]), bf16_dev(g[tag + "_kv"]), float(g[tag + "_scale"])
    o, lse = csa.fused_csa_attn_pool_bf16(q, kv, sc)
    assert o.dtype == torch.float32 and o.shape == q.shape
    assert np.abs(o.cpu().numpy() - g[tag + "_pool_o"]).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - g[tag + "_pool_lse"]).max() < TOL_LSE
    for name in ("bsq_bf16", "fast_bf16", "2pass_bf16"):
        o = torch.full(q.shape, float("nan"), device=DEV)
        lse = torch.full(q.shape[:-1], float("nan"), device=DEV)
        getattr(csa, "fused_csa_attn_" + name)(q, kv, sc, o, lse)
        assert np.abs(o.cpu().numpy() - g[f"{tag}_{name}_o"]).max() < TOL_OUT, name
        assert np.abs(lse.cpu().numpy() - g[f"{tag}_{name}_lse"]).max() < TOL_LSE, name


@pytest.mark.parametrize("tag", ["h512", "h256"])
def test_golden_int8_family(csa, golden, tag):
    """The reference's integer-score operators against its own outputs:
    _bsq_int8 (q and kv quantised inside the call), _bsq_int8_preq and
    _bsq_int8_full (csa_attn.cpp:766-883, :1235-1357, :1359-1483)."""
    g = golden("csa_int8")
    qn, kvn, sc = g[tag + "_q"], g[tag + "_kv"], float(g[tag + "_scale"])
    q, kv = torch.from_numpy(qn).to(DEV), bf16_dev(kvn)
    bs, nH, sq, hd = q.shape

    def fresh():
        return (torch.full(q.shape, float("nan"), device=DEV), torch.full(q.shape[:-1], float("nan"), device=DEV))

    o, lse = fresh()
    csa.fused_csa_attn_bsq_int8(q, kv, sc, o, lse)
    res = {"bsq": (o, lse)}
    ki8, ksc, ksm = csa.kv_quantize_bf16_to_int8(kv)
    qu8, qsc = csa.q_quantize_fp32_to_u8(q)
    o, lse = fresh()
    csa.fused_csa_attn_bsq_int8_preq(q, ki8, ksc, ksm, sc, o, lse)
    res["preq"] = (o, lse)
    o, lse = fresh()
    csa.fused_csa_attn_bsq_int8_full(qu8, qsc, ki8, ksc, ksm, kv, sc, o, lse)
    res["full"] = (o, lse)
    for name, (o, lse) in res.items():
        assert np.abs(o.cpu().numpy() - g[f"{tag}_{name}_o"]).max() < TOL_OUT, name
        assert np.abs(lse.cpu().numpy() - g[f"{tag}_{name}_lse"]).max() < TOL_LSE, name


@pytest.mark.parametrize("bs,nH,sq,nc,full", [(2, 64, 1, 2000, False), (2, 64, 1, 2000, True), (3, 16, 3, 777, False),
                                              (1, 128, 1, 4096, True), (2, 64, 1, 1, False),
                                              (76, 64, 1, 1100, False), (76, 64, 1, 1100, True)])
def test_int8_codes_random(csa, bs, nH, sq, nc, full):
    """Integer-score operators on seeded inputs against the oracle's integer
    restatement (several CTAs per sequence, ragged last tiles, several query
    groups, one entry; 76 sequences run one CTA each over 1100 entries, so a
    CTA crosses the 512-entry chunks its ids are resolved in)."""
    g = torch.Generator().manual_seed(1000 + nc + nH)
    q = torch.randn(bs, nH, sq, 512, generator=g)
    kv = torch.randn(bs, nc, 512, generator=g).bfloat16()
    sc = 512 ** -0.5
    qd, kvd = q.to(DEV), kv.to(DEV)
    ki8, ksc, ksm = csa.kv_quantize_bf16_to_int8(kvd)
    o = torch.empty(q.shape, device=DEV)
    lse = torch.empty(q.shape[:-1], device=DEV)
    if full:
        qu8, qsc = csa.q_quantize_fp32_to_u8(qd)
        csa.fused_csa_attn_bsq_int8_full(qu8, qsc, ki8, ksc, ksm, kvd, sc, o, lse)
    else:
        csa.fused_csa_attn_bsq_int8_preq(qd, ki8, ksc, ksm, sc, o, lse)
    torch.cuda.synchronize()
    qu8n, qscn = oracle.q_quantize_u8(q.numpy().reshape(bs, nH * sq, 512))
    ro, rl = oracle.csa_int8_codes(qu8n, qscn, ki8.cpu().numpy(), ksc.cpu().numpy(), ksm.cpu().numpy(), sc,
                                   kv_bf16=oracle.bf16_bits(kv) if full else None)
    assert np.abs(o.cpu().numpy().reshape(bs, -1, 512) - ro).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy().reshape(bs, -1) - rl).max() < TOL_LSE


@pytest.mark.parametrize("full", [False, True])
def test_int8_codes_gather_capi(full):
    """ws_csa_decode_qcodes with a top-k id list, through the C ABI."""
    from scope_b200 import _lib
    bs, nq, nc, k = 2, 64, 3000, 700
    g = torch.Generator().manual_seed(77)
    q = torch.randn(bs, nq, 512, generator=g)
    kv = torch.randn(bs, nc, 512, generator=g).bfloat16()
    idx = torch.stack([torch.randperm(nc, generator=g)[:k].sort().values for _ in range(bs)]).int()
    csa = scope_b200.build_csa_attn()
    kvd = kv.to(DEV)
    ki8, ksc, ksm = csa.kv_quantize_bf16_to_int8(kvd)
    qu8, qsc = csa.q_quantize_fp32_to_u8(q.to(DEV))
    o = torch.empty(bs, nq, 512, device=DEV)
    lse = torch.empty(bs, nq, device=DEV)
    L = _lib.lib()
    ws = torch.zeros(L.ws_csa_decode_workspace_size(bs, nq, _lib.WS_DTYPE_BF16), dtype=torch.uint8, device=DEV)
    idd = idx.to(DEV)
    rc = L.ws_csa_decode_qcodes(qu8.data_ptr(), qsc.data_ptr(), bs, nq, 512, ki8.data_ptr(), ksc.data_ptr(),
                                ksm.data_ptr(), kvd.data_ptr() if full else None, nc, 0, idd.data_ptr(), k,
                                _lib.WS_CSA_IDX_ALL, 0, nc, 512 ** -0.5, o.data_ptr(), _lib.WS_DTYPE_F32,
                                lse.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.ws_last_error()
    torch.cuda.synchronize()
    ro, rl = oracle.csa_int8_codes(qu8.cpu().numpy(), qsc.cpu().numpy(), ki8.cpu().numpy(), ksc.cpu().numpy(),
                                   ksm.cpu().numpy(), 512 ** -0.5, kv_bf16=oracle.bf16_bits(kv) if full else None,
                                   idx=idx.numpy())
    assert np.abs(o.cpu().numpy() - ro).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - rl).max() < TOL_LSE


def test_int8_exact_addition(csa, golden):
    """fused_csa_attn_int8_exact (no reference counterpart): int8 * scale
    entries with the query unquantised, against the oracle's exact arithmetic."""
    g = golden("csa")
    q = torch.from_numpy(g["q"]).to(DEV)
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:-1], device=DEV)
    csa.fused_csa_attn_int8_exact(q, torch.from_numpy(g["kv_i8"]).to(DEV), torch.from_numpy(g["kv_scales"]).to(DEV),
                                  float(g["scale"]), o, lse)
    bs, nH, sq, hd = q.shape
    ro, rl, _ = oracle.csa_attend(g["q"].reshape(bs, nH * sq, hd), g["kv_i8"], float(g["scale"]),
                                  kv_scale=g["kv_scales"])
    assert np.abs(o.cpu().numpy().reshape(bs, -1, hd) - ro).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy().reshape(bs, -1) - rl).max() < TOL_LSE


def test_golden_int8(csa, golden):
    """_bsq_int8_preq against the reference's own output (the first CSA fixture)."""
    g = golden("csa")
    q = torch.from_numpy(g["q"]).to(DEV)
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:-1], device=DEV)
    csa.fused_csa_attn_bsq_int8_preq(q, torch.from_numpy(g["kv_i8"]).to(DEV), torch.from_numpy(g["kv_scales"]).to(DEV),
                                     torch.from_numpy(g["kv_sums"]).to(DEV), float(g["scale"]), o, lse)
    bs, nH, sq, hd = q.shape
    on, ln = o.cpu().numpy().reshape(bs, -1, hd), lse.cpu().numpy().reshape(bs, -1)
    assert np.abs(on - g["int8_o"].reshape(bs, -1, hd)).max() < TOL_OUT
    assert np.abs(ln - g["int8_lse"].reshape(bs, -1)).max() < TOL_LSE


def test_quantisers_bit_exact_golden(csa, golden):
    g = golden("csa")
    i8, sc, sm = csa.kv_quantize_bf16_to_int8(bf16_dev(g["kv"]))
    assert np.array_equal(i8.cpu().numpy(), g["kv_i8"])
    assert np.array_equal(sc.cpu().numpy(), g["kv_scales"])
    assert np.array_equal(sm.cpu().numpy(), g["kv_sums"])
    u8, qs = csa.q_quantize_fp32_to_u8(torch.from_numpy(g["q"]).to(DEV))
    assert np.array_equal(u8.cpu().numpy(), g["q_u8"])
    assert np.array_equal(qs.cpu().numpy(), g["q_scales"])


@pytest.mark.parametrize("rows,hd", [(1, 512), (777, 512), (64, 128), (5, 8), (33, 1024)])
def test_quantisers_bit_exact_random(csa, rows, hd):
    g = torch.Generator().manual_seed(rows * 7 + hd)
    x = torch.randn(1, rows, hd, generator=g) * torch.rand(1, rows, 1, generator=g) * 10
    x[0, 0, :] = 0.0                      # an all-zero row hits the 1e-6 floor
    i8, sc, sm = csa.kv_quantize_bf16_to_int8(x.bfloat16().to(DEV))
    ri8, rsc, rsm = oracle.kv_quantize_s8(oracle.bf16_bits(x.bfloat16()))
    assert np.array_equal(i8.cpu().numpy(), ri8)
    assert np.array_equal(sc.cpu().numpy(), rsc)
    assert np.array_equal(sm.cpu().numpy(), rsm)
    u8, qs = csa.q_quantize_fp32_to_u8(x.to(DEV))
    ru8, rqs = oracle.q_quantize_u8(x.numpy())
    assert np.array_equal(u8.cpu().numpy(), ru8)
    assert np.array_equal(qs.cpu().numpy(), rqs)


# ------------------------------------------------------------ seeded shapes
@pytest.mark.parametrize("bs,nq,nc,k", [(1, 1, 64, 1), (2, 8, 300, 100), (3, 16, 1000, 128), (2, 17, 1000, 129),
                                        (1, 64, 4096, 2048), (2, 65, 3000, 700), (1, 33, 5000, 4097),
                                        (4, 128, 2000, 256), (160, 2, 300, 100), (20, 8, 600, 400)])
@pytest.mark.parametrize("int8", [False, True])
@pytest.mark.parametrize("q_bf16", [False, True])
def test_gather_random(bs, nq, nc, k, int8, q_bf16):
    q, kv, sc, idx = rand_case(bs, nq, nc, k, seed=bs * 100003 + nq * 101 + k, int8=int8, q_bf16=q_bf16)
    scale = 512 ** -0.5
    o, lse = run_gather(q, kv, sc, idx, scale)
    ro, rl, bad = oracle_of(q, kv, sc, scale, idx=idx)
    assert bad == 0
    assert np.abs(o - ro).max() < TOL_OUT
    assert np.abs(lse - rl).max() < TOL_LSE
    ob, _ = run_gather(q, kv, sc, idx, scale, out_dtype=torch.bfloat16)
    assert np.abs(ob - ro).max() < TOL_OUT


def test_gather_unsorted_duplicates():
    q, kv, sc, _ = rand_case(2, 24, 500, None, seed=11)
    g = torch.Generator().manual_seed(12)
    idx = torch.randint(0, 500, (2, 900), generator=g).int()     # unsorted, with repeats
    o, lse = run_gather(q, kv, sc, idx, 0.05)
    ro, rl, _ = oracle_of(q, kv, sc, 0.05, idx=idx)
    assert np.abs(o - ro).max() < TOL_OUT and np.abs(lse - rl).max() < TOL_LSE


def test_gather_rows_bit_exact():
    """One id per sequence and a unit (or power-of-two) value scale: the output
    is the gathered row itself, so any byte the gather moved wrongly shows."""
    g = torch.Generator().manual_seed(21)
    bs, nc = 40, 3000
    idx = torch.randint(0, nc, (bs, 1), generator=g).int()
    q = torch.randn(bs, 5, 512, generator=g)
    kv = torch.randn(bs, nc, 512, generator=g).bfloat16()
    o, _ = run_gather(q, kv, None, idx, 0.1)
    want = kv[torch.arange(bs), idx[:, 0].long()].float().numpy()
    assert np.array_equal(o, np.broadcast_to(want[:, None, :], o.shape))
    kv8 = torch.randint(-127, 128, (bs, nc, 512), generator=g).to(torch.int8)
    sc = torch.full((bs, nc), 0.03125)
    o, _ = run_gather(q, kv8, sc, idx, 0.1)
    want = kv8[torch.arange(bs), idx[:, 0].long()].float().numpy() * 0.03125
    assert np.array_equal(o, np.broadcast_to(want[:, None, :], o.shape))


def test_out_of_range_ids_are_skipped_and_reported():
    q, kv, sc, idx = rand_case(2, 8, 256, 64, seed=31)
    idx[0, 5] = -3
    idx[1, 60] = 256
    scope_b200.status_take()
    o, lse = run_gather(q, kv, sc, idx, 0.05)
    assert scope_b200.status_take() != 0
    ro, rl, bad = oracle_of(q, kv, sc, 0.05, idx=idx)
    assert bad == 2 * 8
    assert np.abs(o - ro).max() < TOL_OUT and np.abs(lse - rl).max() < TOL_LSE
    assert scope_b200.status_take() == 0


def test_empty_selection():
    q, kv, sc, _ = rand_case(2, 8, 100, None, seed=41)
    idx = torch.zeros(2, 0, dtype=torch.int32)
    o, lse = run_gather(q, kv, sc, idx, 0.05)
    assert np.all(o == 0) and np.all(np.isneginf(lse))


def test_dense_long_range(csa):
    """The dense form with many tiles per CTA (lazy rescale path) and fp32 q."""
    g = torch.Generator().manual_seed(51)
    q = torch.randn(2, 4, 3, 512, generator=g) * 3      # larger scores exercise the running max
    kv = torch.randn(2, 20000, 512, generator=g).bfloat16()
    o, lse = csa.fused_csa_attn(q.to(DEV), kv.to(DEV), 512 ** -0.5)
    ro, rl, _ = oracle_of(q.reshape(2, 12, 512), kv, None, 512 ** -0.5)
    assert np.abs(o.cpu().numpy().reshape(2, 12, 512) - ro).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy().reshape(2, 12) - rl).max() < TOL_LSE
    o, lse = csa.fused_csa_attn_range(q.to(DEV), kv.to(DEV), 512 ** -0.5, 1234, 17777)
    ro, rl, _ = oracle_of(q.reshape(2, 12, 512), kv, None, 512 ** -0.5, kv_range=(1234, 17777))
    assert np.abs(o.cpu().numpy().reshape(2, 12, 512) - ro).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy().reshape(2, 12) - rl).max() < TOL_LSE


def test_range_checks(csa):
    q = torch.zeros(1, 2, 1, 512, device=DEV)
    kv = torch.zeros(1, 10, 512, dtype=torch.bfloat16, device=DEV)
    for s, e in ((5, 5), (-1, 3), (2, 11)):
        with pytest.raises(RuntimeError, match="invalid kv range"):
            csa.fused_csa_attn_range(q, kv, 0.1, s, e)
    with pytest.raises(RuntimeError, match="fp32"):
        csa.fused_csa_attn(q.bfloat16(), kv, 0.1)


# ------------------------------------------------------------ shards
@pytest.mark.parametrize("mode", ["sorted_shard", "shard"])
@pytest.mark.parametrize("nshards", [2, 3, 8])
def test_sharded_merge_equals_unsharded(mode, nshards):
    """Entry-sharded cache: each shard attends to its own ids (rebased locally),
    and the log-sum-exp merge of the partials equals the unsharded result."""
    bs, nq, nc, k = 3, 64, 6000, 1500
    q, kv, sc, idx = rand_case(bs, nq, nc, k, seed=61 + nshards, int8=True, q_bf16=True,
                               sorted_ids=(mode == "sorted_shard"))
    scale = 512 ** -0.5
    qd, kvd, scd, idxd = q.to(DEV), kv.to(DEV), sc.to(DEV), idx.to(DEV)
    full_o, full_l = scope_b200.csa_attn.csa_sparse_decode(qd, kvd, idxd, scale, scd, out_dtype=torch.float32)
    bounds = [nc * s // nshards for s in range(nshards + 1)]
    parts_o, parts_l = [], []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        po, pl = scope_b200.csa_attn.csa_sparse_decode(qd, kvd[:, lo:hi].contiguous(), idxd, scale,
                                                       scd[:, lo:hi].contiguous(), shard_lo=lo, idx_mode=mode,
                                                       out_dtype=torch.float32)
        parts_o.append(po.reshape(bs * nq, 512))
        parts_l.append(pl.reshape(bs * nq))
    mo, ml = scope_b200.lse_merge(torch.stack(parts_o), torch.stack(parts_l), torch.float32)
    # both sides round their softmax weights to bf16 against different running maxima
    assert (mo - full_o.reshape(bs * nq, 512)).abs().max().item() < 5e-3
    assert (ml - full_l.reshape(bs * nq)).abs().max().item() < 1e-4
    ro, rl, _ = oracle_of(q, kv, sc, scale, idx=idx)
    assert np.abs(mo.cpu().numpy().reshape(bs, nq, 512) - ro).max() < TOL_OUT
    assert np.abs(ml.cpu().numpy().reshape(bs, nq) - rl).max() < TOL_LSE


def test_shard_without_entries_gives_neg_inf():
    q, kv, sc, idx = rand_case(2, 16, 1000, 50, seed=71)
    idx = idx.clamp(max=499)   # every id in the first half
    out, lse = scope_b200.csa_attn.csa_sparse_decode(q.to(DEV), kv[:, 500:].contiguous().to(DEV), idx.to(DEV),
                                                     0.05, shard_lo=500, idx_mode="sorted_shard",
                                                     out_dtype=torch.float32)
    assert torch.all(out == 0) and torch.all(torch.isneginf(lse))


# ------------------------------------------------------------ benchmark size
def test_cfg5_size():
    """The benchmark shape (bs=16, nH=64, nc=65536, k=2048, int8+scale, bf16 q):
    two sequences against the oracle, all against a 2-shard merge."""
    bs, nH, nc, k = 16, 64, 65536, 2048
    q, kv, sc, idx = rand_case(bs, nH, nc, k, seed=5, int8=True, q_bf16=True)
    scale = 512 ** -0.5
    qd, kvd, scd, idxd = q.to(DEV), kv.to(DEV), sc.to(DEV), idx.to(DEV)
    o, lse = scope_b200.csa_attn.csa_sparse_decode(qd, kvd, idxd, scale, scd)
    ro, rl, _ = oracle_of(q[:2], kv[:2], sc[:2], scale, idx=idx[:2])
    assert np.abs(o[:2].float().cpu().numpy() - ro).max() < TOL_OUT
    assert np.abs(lse[:2].cpu().numpy() - rl).max() < TOL_LSE
    parts = [scope_b200.csa_attn.csa_sparse_decode(qd, kvd[:, a:a + nc // 2].contiguous(), idxd, scale,
                                                   scd[:, a:a + nc // 2].contiguous(), shard_lo=a,
                                                   idx_mode="sorted_shard", out_dtype=torch.float32)
             for a in (0, nc // 2)]
    mo, ml = scope_b200.lse_merge(torch.stack([p[0].reshape(-1, 512) for p in parts]),
                                  torch.stack([p[1].reshape(-1) for p in parts]), torch.float32)
    assert (mo - o.float().reshape(-1, 512)).abs().max().item() < 2e-2
    assert (ml - lse.reshape(-1)).abs().max().item() < 1e-4


def test_workspace_pool_shared_with_gqa():
    """The CSA kernel's partials live past the counter header of the pooled
    workspace, so a GQA decode (whose merge tickets use that header) that
    follows a CSA call on the same stream stays exact."""
    ext = scope_b200.build()
    q, kv, sc, idx = rand_case(2, 64, 3000, 900, seed=91, int8=True, q_bf16=True)
    scope_b200.csa_attn.csa_sparse_decode(q.to(DEV), kv.to(DEV), idx.to(DEV), 0.05, sc.to(DEV))
    g = torch.Generator().manual_seed(92)
    qg = torch.randn(8, 4, 128, generator=g).bfloat16()
    k = torch.randn(8, 3000, 128, generator=g).bfloat16()
    v = torch.randn(8, 3000, 128, generator=g).bfloat16()
    for _ in range(2):
        o, m, s = ext.fused_cpu_attn_mla(qg.to(DEV), k.to(DEV), v.to(DEV), 128 ** -0.5)
        ro, rm, rs = oracle.gqa_decode(oracle.bf16_bits(qg), oracle.bf16_bits(k), oracle.bf16_bits(v), 128 ** -0.5)
        assert np.abs((o / s).cpu().numpy() - ro).max() < TOL_OUT
        scope_b200.csa_attn.csa_sparse_decode(q.to(DEV), kv.to(DEV), idx.to(DEV), 0.05, sc.to(DEV))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_split_merge_unaligned_output(out_dtype):
    """Split partials are merged inside the decode launch when the output rows
    take 16-byte stores; an output that starts off a 16-byte boundary goes
    through the separate merge grid instead.  Both against the oracle, with the
    workspace reused across the two."""
    from scope_b200 import _lib
    bs, nq, nc, k = 4, 64, 6000, 1500
    q, kv, sc, idx = rand_case(bs, nq, nc, k, seed=88, int8=True, q_bf16=True)
    L = _lib.lib()
    qd, kvd, scd, idd = q.to(DEV), kv.to(DEV), sc.to(DEV), idx.to(DEV)
    ro, rl, _ = oracle_of(q, kv, sc, 512 ** -0.5, idx=idx)
    esz = 4 if out_dtype == torch.float32 else 2
    for shift in (0, 1):   # elements: 0 -> aligned rows, 1 -> rows 4 or 2 bytes off a 16-byte boundary
        buf = torch.full((bs * nq * 512 + 8,), float("nan"), dtype=out_dtype, device=DEV)
        out = buf[shift:shift + bs * nq * 512]
        lse = torch.empty(bs, nq, device=DEV)
        ws = scope_b200._lib.workspaces.get(L.ws_csa_decode_workspace_size(bs, nq, _lib.WS_DTYPE_BF16), qd.device)
        rc = L.ws_csa_decode(qd.data_ptr(), _lib.WS_DTYPE_BF16, bs, nq, 512, kvd.data_ptr(), _lib.WS_DTYPE_I8,
                             scd.data_ptr(), nc, 0, idd.data_ptr(), k, _lib.WS_CSA_IDX_ALL, 0, 0, 512 ** -0.5,
                             out.data_ptr(), _lib.WS_DTYPE_F32 if esz == 4 else _lib.WS_DTYPE_BF16, lse.data_ptr(),
                             ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        if shift and rc != 0:   # the C ABI wants 16-byte aligned outputs: nothing to compare then
            assert rc == _lib.WS_ERR_INVALID_ARG
            continue
        assert rc == 0, L.ws_last_error()
        torch.cuda.synchronize()
        assert np.abs(out.float().cpu().numpy().reshape(bs, nq, 512) - ro).max() < TOL_OUT
        assert np.abs(lse.cpu().numpy() - rl).max() < TOL_LSE
    assert scope_b200.status_take() == 0
