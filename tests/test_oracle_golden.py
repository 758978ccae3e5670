"""Pin the CPU oracle (oracle/ws_oracle.c) to the reference's own outputs.

The fixtures in tests/golden/ were produced by the reference's AVX-512
extensions (see tests/golden/make_golden.py).  The oracle accumulates in
float64, the reference in fp32 with -ffast-math, so agreement is to fp32
rounding; the two lossy quantisers must agree bit for bit.
"""
import numpy as np
import pytest

import oracle

TOL_O = 2e-5      # fp32-level agreement on outputs of magnitude <= ~3
TOL_LSE = 5e-6


def f32(bits):
    return oracle.bits_to_f32(bits)


def test_gqa_qwen3_mla_form(golden):
    g = golden("gqa_qwen3_bf16")
    o, m, s = oracle.gqa_decode(g["q"], g["k"], g["v"], float(g["scale"]))
    ref_norm = g["mla_o"] / g["mla_sum"]
    assert np.abs(o - ref_norm).max() < TOL_O
    assert np.abs(m - g["mla_max"][..., 0]).max() < TOL_LSE
    ref_lse = g["mla_max"][..., 0] + np.log(g["mla_sum"][..., 0])
    assert np.abs((m + np.log(s)) - ref_lse).max() < TOL_LSE


def test_gqa_qwen3_public_bf16(golden):
    # fused_cpu_attn on bf16 returns bf16 out/max/sum (kernel/cpu_attn.cpp:631-634)
    g = golden("gqa_qwen3_bf16")
    o, m, s = oracle.gqa_decode(g["q"], g["k"], g["v"], float(g["scale"]))
    pub = f32(g["pub_out"])
    assert np.abs(pub - o).max() <= 2.0 ** -8 * np.abs(o).max() + 1e-6   # one bf16 rounding
    assert np.abs(f32(g["pub_max"])[..., 0] - m).max() <= 2.0 ** -8 * np.abs(m).max()
    assert np.allclose(f32(g["pub_sum"])[..., 0], s, rtol=2.0 ** -8)


def test_gqa_strided_view(golden):
    g = golden("gqa_strided_bf16")
    L, Hkv, D = g["k_cache"].shape
    o, m, s = oracle.gqa_decode_strided_buffer(g["q"], g["k_cache"], g["v_cache"], L,
                                               (D, Hkv * D), (D, Hkv * D), D, float(g["scale"]))
    assert np.abs(o - g["mla_o"] / g["mla_sum"]).max() < TOL_O
    assert np.abs(m + np.log(s) - (g["mla_max"][..., 0] + np.log(g["mla_sum"][..., 0]))).max() < TOL_LSE


def test_mla_nonabsorbed_192_128(golden):
    g = golden("mla_nonabsorbed_bf16")
    o, m, s = oracle.gqa_decode(g["q"], g["k"], g["v"], float(g["scale"]))
    assert np.abs(o - g["mla_o"] / g["mla_sum"]).max() < TOL_O
    assert np.abs(m - g["mla_max"][..., 0]).max() < TOL_LSE


def test_gqa_fp32(golden):
    g = golden("gqa_fp32")
    o, m, s = oracle.gqa_decode(g["q"], g["k"], g["v"], float(g["scale"]), kind="fp32")
    for pre in ("pub", "abl"):
        assert np.abs(o - g[pre + "_out"]).max() < TOL_O
        assert np.abs(m - g[pre + "_max"][..., 0]).max() < TOL_LSE
        assert np.allclose(s, g[pre + "_sum"][..., 0], rtol=1e-5)


def test_mla_compressed(golden):
    g = golden("mla_compressed")
    o, m, s = oracle.mla_compressed(g["q_proj"], g["q_pe"], g["c_kv"], g["k_pe"], float(g["scale"]))
    for pre in ("", "tile64_"):
        ro, rm, rs = g[pre + "o"], g[pre + "max"], g[pre + "sum"]
        assert np.abs(o / s[:, None] - ro / rs[:, None]).max() < TOL_O
        assert np.abs((m + np.log(s)) - (rm + np.log(rs))).max() < TOL_LSE
        assert np.abs(m - rm).max() < TOL_LSE


def test_csa_dense_range_gather(golden):
    g = golden("csa")
    q, kv, sc = g["q"], g["kv"], float(g["scale"])
    bs, nH, sq, hd = q.shape
    o, lse, bad = oracle.csa_attend(q.reshape(bs, nH * sq, hd), kv, sc)
    assert bad == 0
    assert np.abs(o - g["dense_o"].reshape(bs, -1, hd)).max() < TOL_O
    assert np.abs(lse - g["dense_lse"].reshape(bs, -1)).max() < TOL_LSE
    o, lse, _ = oracle.csa_attend(q.reshape(bs, nH * sq, hd), kv, sc,
                                  kv_range=(int(g["range_s"]), int(g["range_e"])))
    assert np.abs(o - g["range_o"].reshape(bs, -1, hd)).max() < TOL_O
    assert np.abs(lse - g["range_lse"].reshape(bs, -1)).max() < TOL_LSE
    o, lse, _ = oracle.csa_attend(g["q_gather"], kv, sc, idx=g["idx"])
    assert np.abs(o - g["gather_o"]).max() < TOL_O
    assert np.abs(lse - g["gather_lse"]).max() < TOL_LSE


def test_quantisers_bit_exact(golden):
    g = golden("csa")
    i8, sc, sm = oracle.kv_quantize_s8(g["kv"])
    assert np.array_equal(i8, g["kv_i8"])
    assert np.array_equal(sc, g["kv_scales"])
    assert np.array_equal(sm, g["kv_sums"])
    u8, qs = oracle.q_quantize_u8(g["q"])
    assert np.array_equal(u8, g["q_u8"])
    assert np.array_equal(qs, g["q_scales"])


def test_csa_int8_preq(golden):
    g = golden("csa")
    q = g["q"]
    bs, nH, sq, hd = q.shape
    o, lse = oracle.csa_int8_preq(q.reshape(bs, nH * sq, hd), g["kv_i8"], g["kv_scales"], g["kv_sums"],
                                  float(g["scale"]))
    assert np.abs(o - g["int8_o"].reshape(bs, -1, hd)).max() < TOL_O
    assert np.abs(lse - g["int8_lse"].reshape(bs, -1)).max() < TOL_LSE


def test_indexer_topk(golden):
    g = golden("indexer_topk")
    ids, scores = oracle.indexer_topk(g["q_idx"], g["kv_idx"], g["weights"], int(g["k"]))
    # same id sets (the reference's partial_sort leaves tie order unspecified)
    for b in range(ids.shape[0]):
        assert set(ids[b].tolist()) == set(g["ids"][b].tolist())
        # ordered by descending score
        assert np.all(np.diff(scores[b][ids[b]]) <= 0)


@pytest.mark.parametrize("tag", ["h512", "h256"])
def test_csa_int8_family(golden, tag):
    """_bsq_int8 (both quantisers inside the call), _int8_preq and _int8_full
    (csa_attn.cpp:766-883, :1235-1483) against the integer-score restatement."""
    g = golden("csa_int8")
    q, kv, sc = g[tag + "_q"], g[tag + "_kv"], float(g[tag + "_scale"])
    bs, nH, sq, hd = q.shape
    ki8, ksc, ksm = oracle.kv_quantize_s8(kv)
    qu8, qsc = oracle.q_quantize_u8(q.reshape(bs, nH * sq, hd))
    for name, vals in (("bsq", None), ("preq", None), ("full", kv)):
        o, lse = oracle.csa_int8_codes(qu8, qsc, ki8, ksc, ksm, sc, kv_bf16=vals)
        assert np.abs(o - g[f"{tag}_{name}_o"].reshape(bs, -1, hd)).max() < TOL_O, name
        assert np.abs(lse - g[f"{tag}_{name}_lse"].reshape(bs, -1)).max() < TOL_LSE, name


@pytest.mark.parametrize("tag", ["h512", "h256"])
def test_csa_bf16_query_variants(golden, tag):
    """_pool_bf16, _bsq_bf16, _fast_bf16 and _2pass_bf16 (csa_attn.cpp:379-474,
    :580-764, :885-1048, :1050-1173) on a bf16 query."""
    g = golden("csa_bf16q")
    q, kv, sc = g[tag + "_q"], g[tag + "_kv"], float(g[tag + "_scale"])
    bs, nH, sq, hd = q.shape
    o, lse, bad = oracle.csa_attend(q.reshape(bs, nH * sq, hd), kv, sc)
    assert bad == 0
    # _fast_bf16 takes exp from a degree-5 Taylor polynomial on a range-reduced
    # argument (csa_attn.cpp:85-103): relative error up to (ln 2)^6 / 720 ~ 1.6e-4
    # per weight, so its log-sum-exp may sit ~1.6e-4 off the exact one
    tol = {"fast_bf16": (2e-3, 3e-4)}
    for name in ("pool", "bsq_bf16", "fast_bf16", "2pass_bf16"):
        to, tl = tol.get(name, (TOL_O, TOL_LSE))
        assert np.abs(o - g[f"{tag}_{name}_o"].reshape(bs, -1, hd)).max() < to, name
        assert np.abs(lse - g[f"{tag}_{name}_lse"].reshape(bs, -1)).max() < tl, name


def indexer_large_inputs(seed, bs, nH, hd, nc):
    """The inputs tests/golden/make_golden.py drew for the large indexer fixture."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((bs, nH, hd), dtype=np.float32)
    kv = rng.standard_normal((bs, nc, hd), dtype=np.float32)
    w = rng.random((bs, nH), dtype=np.float32)
    return q, kv, w


def indexer_large_case(golden, i):
    """Regenerate case i of the large indexer fixture; returns (q, kv, w, k, ref_ids)."""
    g = golden("indexer_topk_large")
    seed, bs, nH, hd, nc, k = (int(x) for x in g[f"c{i}_shape"])
    q, kv, w = indexer_large_inputs(seed, bs, nH, hd, nc)
    chk = np.array([q.astype(np.float64).sum(), kv.astype(np.float64).sum(), w.astype(np.float64).sum()])
    assert np.array_equal(chk, g[f"c{i}_checksum"]), "numpy's generator no longer reproduces the fixture inputs"
    return q, kv, w, k, g[f"c{i}_ids"]


@pytest.mark.parametrize("i", [0, 1])
def test_indexer_topk_large_fp32_order(golden, i):
    """The reference's ranking at nc >= 20000, k = 2048 is the one its fp32
    scores give (16 FMA lanes, the AVX-512 reduction tree, unfused multiply
    then add): same id sets, same order up to runs of exactly equal scores."""
    q, kv, w, k, ref = indexer_large_case(golden, i)
    sc = oracle.indexer_scores_f32(q, kv, w, contract=False)
    ids = oracle.topk_from_scores(sc, k)
    agree = oracle.topk_agreement(ids, ref, sc)
    assert agree["set_diff"] == 0 and agree["order_diff"] == 0, agree


def test_lse_merge_matches_unsplit():
    rng = np.random.default_rng(0)
    B, G, D, L = 3, 4, 64, 257
    q = oracle.f32_to_bf16_bits(rng.standard_normal((B, G, D)).astype(np.float32))
    k = oracle.f32_to_bf16_bits(rng.standard_normal((B, L, D)).astype(np.float32))
    v = oracle.f32_to_bf16_bits(rng.standard_normal((B, L, D)).astype(np.float32))
    sc = D ** -0.5
    o, m, s = oracle.gqa_decode(q, k, v, sc)
    cuts = [0, 100, 101, 257]
    parts_o, parts_l = [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        po, pm, ps = oracle.gqa_decode(q, k[:, a:b], v[:, a:b], sc)
        parts_o.append(po.reshape(B * G, D))
        parts_l.append((pm + np.log(ps)).reshape(B * G))
    mo, ml = oracle.lse_merge(np.stack(parts_o), np.stack(parts_l))
    assert np.abs(mo - o.reshape(B * G, D)).max() < 1e-12
    assert np.abs(ml - (m + np.log(s)).reshape(B * G)).max() < 1e-12


def test_empty_share_gives_neg_inf():
    q = np.zeros((1, 2, 16), np.uint16)
    k = np.zeros((1, 0, 16), np.uint16)
    o, m, s = oracle.gqa_decode(q, k, k, 0.25)
    assert np.all(o == 0) and np.all(np.isneginf(m)) and np.all(s == 0)


@pytest.mark.ref
def test_oracle_matches_live_reference():
    """When the compiled reference is present, compare on fresh random inputs."""
    if not oracle.ref_available():
        pytest.skip("compiled reference not present")
    import torch
    ref = oracle.load_ref("cpu_attn_ext")
    torch.manual_seed(7)
    q = torch.randn(3, 8, 128).bfloat16()
    k = torch.randn(3, 517, 128).bfloat16()
    v = torch.randn(3, 517, 128).bfloat16()
    ro, rm, rs = ref.fused_cpu_attn_mla(q, k, v, 128 ** -0.5)
    o, m, s = oracle.gqa_decode(oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v), 128 ** -0.5)
    assert np.abs(o - (ro / rs).numpy()).max() < TOL_O
    assert np.abs(m - rm.numpy()[..., 0]).max() < TOL_LSE
