"""GPU parity of the GQA / MLA(non-absorbed) decode against the oracle and
the reference's golden outputs.

Tolerances (from the north star): bf16 outputs max-abs 2e-2, fp32 LSE 1e-3.
The kernels compute in fp32 from bf16 operands; the oracle in float64.
"""
import numpy as np
import pytest
import torch

import oracle
import scope_b200

pytestmark = pytest.mark.gpu

TOL_OUT = 2e-2
TOL_LSE = 1e-3
DEV = "cuda:0"


@pytest.fixture(scope="module")
def ext():
    return scope_b200.build()


def bits_to_bf16(bits, device=DEV):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def rand_bf16(*shape, gen):
    return torch.randn(*shape, generator=gen).bfloat16()


def oracle_of(q, k, v, scale):
    return oracle.gqa_decode(oracle.bf16_bits(q.cpu()), oracle.bf16_bits(k.cpu()), oracle.bf16_bits(v.cpu()), scale)


def test_golden_qwen3(ext, golden):
    g = golden("gqa_qwen3_bf16")
    q, k, v = (bits_to_bf16(g[n]) for n in ("q", "k", "v"))
    sc = float(g["scale"])
    o, m, s = ext.fused_cpu_attn_mla(q, k, v, sc)
    torch.cuda.synchronize()
    o, m, s = o.cpu().numpy(), m.cpu().numpy(), s.cpu().numpy()
    assert np.abs(o / s - g["mla_o"] / g["mla_sum"]).max() < TOL_OUT / 10
    assert np.abs((m + np.log(s)) - (g["mla_max"] + np.log(g["mla_sum"]))).max() < TOL_LSE
    po, pm, ps = ext.fused_cpu_attn(q, k, v, sc)
    assert po.dtype == torch.bfloat16 and pm.dtype == torch.bfloat16 and pm.shape == (4, 8, 1)
    ref_pub = oracle.bits_to_f32(g["pub_out"])
    assert np.abs(po.float().cpu().numpy() - ref_pub).max() < TOL_OUT


def test_golden_strided(ext, golden):
    g = golden("gqa_strided_bf16")
    q = bits_to_bf16(g["q"])
    kc, vc = bits_to_bf16(g["k_cache"]), bits_to_bf16(g["v_cache"])
    o, m, s = ext.fused_cpu_attn_mla(q, kc.permute(1, 0, 2), vc.permute(1, 0, 2), float(g["scale"]))
    o, s, m = o.cpu().numpy(), s.cpu().numpy(), m.cpu().numpy()
    assert np.abs(o / s - g["mla_o"] / g["mla_sum"]).max() < TOL_OUT / 10
    assert np.abs((m + np.log(s)) - (g["mla_max"] + np.log(g["mla_sum"]))).max() < TOL_LSE


def test_golden_mla_192_128(ext, golden):
    g = golden("mla_nonabsorbed_bf16")
    q, k, v = (bits_to_bf16(g[n]) for n in ("q", "k", "v"))
    o, m, s = ext.fused_cpu_attn_mla(q, k, v, float(g["scale"]))
    o, m, s = o.cpu().numpy(), m.cpu().numpy(), s.cpu().numpy()
    assert o.shape == (8, 1, 128)
    assert np.abs(o / s - g["mla_o"] / g["mla_sum"]).max() < TOL_OUT / 10
    assert np.abs((m + np.log(s)) - (g["mla_max"] + np.log(g["mla_sum"]))).max() < TOL_LSE


def test_golden_fp32(ext, golden):
    g = golden("gqa_fp32")
    q, k, v = (torch.from_numpy(g[n]).to(DEV) for n in ("q", "k", "v"))
    for fn, pre in ((ext.fused_cpu_attn, "pub"), (ext.fused_cpu_attn_fp32, "abl")):
        o, m, s = fn(q, k, v, float(g["scale"]))
        assert o.dtype == torch.float32
        assert np.abs(o.cpu().numpy() - g[pre + "_out"]).max() < 1e-4
        assert np.abs(m.cpu().numpy() - g[pre + "_max"]).max() < 1e-5
        assert np.allclose(s.cpu().numpy(), g[pre + "_sum"], rtol=1e-4)


@pytest.mark.parametrize("B,G,D,L", [
    (1, 8, 128, 4096),     # cfg1 shape (Qwen3-30B-A3B layer: 32 q heads / 4 kv heads -> B_kv = 4 rows)
    (4, 8, 128, 4096),
    (3, 8, 128, 1), (2, 8, 128, 15), (2, 8, 128, 16), (2, 8, 128, 63), (2, 8, 128, 64), (2, 8, 128, 65),
    (5, 4, 128, 1000), (7, 1, 128, 333), (2, 16, 128, 777), (3, 2, 64, 129), (300, 8, 128, 40),
    (2, 12, 128, 2049),
])
def test_random_shapes(ext, B, G, D, L):
    gen = torch.Generator().manual_seed(1000 + B * 7 + G * 13 + L)
    Bkv = B * (4 if (B, L) == (1, 4096) else 1)
    q = rand_bf16(Bkv, G, D, gen=gen)
    k = rand_bf16(Bkv, L, D, gen=gen)
    v = rand_bf16(Bkv, L, D, gen=gen)
    sc = D ** -0.5
    ro, rm, rs = oracle_of(q, k, v, sc)
    out, lse = scope_b200.cpu_attn.gqa_decode(q.to(DEV), k.to(DEV), v.to(DEV), sc)
    assert np.abs(out.float().cpu().numpy() - ro).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - (rm + np.log(rs))).max() < TOL_LSE
    o, m, s = ext.fused_cpu_attn_mla(q.to(DEV), k.to(DEV), v.to(DEV), sc)
    assert np.abs(m.cpu().numpy()[..., 0] - rm).max() < TOL_LSE
    assert np.allclose(s.cpu().numpy()[..., 0], rs, rtol=1e-3)


def test_token_major_cache_view(ext):
    """[L, Hkv, D] token-major buffer seen per head: strides (D, Hkv*D) on (b, t)."""
    gen = torch.Generator().manual_seed(5)
    L, Hkv, G, D = 3000, 4, 8, 128
    kc = rand_bf16(L, Hkv, D, gen=gen)
    vc = rand_bf16(L, Hkv, D, gen=gen)
    q = rand_bf16(Hkv, G, D, gen=gen)
    ro, rm, rs = oracle.gqa_decode_strided_buffer(oracle.bf16_bits(q), oracle.bf16_bits(kc), oracle.bf16_bits(vc),
                                                  L, (D, Hkv * D), (D, Hkv * D), D, D ** -0.5)
    out, lse = scope_b200.cpu_attn.gqa_decode(q.to(DEV), kc.to(DEV).permute(1, 0, 2), vc.to(DEV).permute(1, 0, 2),
                                              D ** -0.5)
    assert np.abs(out.float().cpu().numpy() - ro).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - (rm + np.log(rs))).max() < TOL_LSE


def test_empty_kv(ext):
    q = torch.randn(2, 8, 128, device=DEV).bfloat16()
    k = torch.empty(2, 0, 128, device=DEV, dtype=torch.bfloat16)
    o, m, s = ext.fused_cpu_attn_mla(q, k, k, 0.1)
    assert torch.all(o == 0) and torch.all(torch.isneginf(m)) and torch.all(s == 0)


def test_repeat_calls_reuse_workspace(ext):
    """Counters in the workspace reset themselves: many launches stay correct."""
    gen = torch.Generator().manual_seed(9)
    q = rand_bf16(4, 8, 128, gen=gen).to(DEV)
    k = rand_bf16(4, 8192, 128, gen=gen).to(DEV)
    v = rand_bf16(4, 8192, 128, gen=gen).to(DEV)
    first, lse0 = scope_b200.cpu_attn.gqa_decode(q, k, v, 0.088)
    for _ in range(20):
        out, lse = scope_b200.cpu_attn.gqa_decode(q, k, v, 0.088)
    assert torch.equal(out, first) and torch.equal(lse, lse0)


@pytest.mark.parametrize("layout", ["token_major", "head_major", "padded"])
def test_shares_ragged_two_way(ext, layout):
    """cfg2-style ragged batch, each sequence split into two physical shares,
    in the packed token-major, packed head-major and padded (reference cache) layouts."""
    gen = torch.Generator().manual_seed(2)
    B, Hkv, G, D = 5, 8, 4, 128
    lens = [1024, 77, 3000, 1, 2500]
    r = 0.25
    L0 = [int(r * L) for L in lens]
    q = rand_bf16(B, Hkv * G, D, gen=gen)
    ks = [rand_bf16(L, Hkv, D, gen=gen) for L in lens]
    vs = [rand_bf16(L, Hkv, D, gen=gen) for L in lens]

    def make(part):
        n = [b - a for a, b in part]
        if layout == "padded":
            cap = max(max(n), 1) + 3
            k = torch.full((B * Hkv, cap, D), float("nan")).bfloat16()   # unused capacity is never read
            v = torch.full((B * Hkv, cap, D), float("nan")).bfloat16()
            for bi, (a, b2) in enumerate(part):
                k[bi * Hkv:(bi + 1) * Hkv, :b2 - a] = ks[bi][a:b2].permute(1, 0, 2)
                v[bi * Hkv:(bi + 1) * Hkv, :b2 - a] = vs[bi][a:b2].permute(1, 0, 2)
            return scope_b200.Share(k.to(DEV), v.to(DEV), seqlens=torch.tensor(n, dtype=torch.int32).to(DEV))
        k = torch.cat([kk[a:b2] for kk, (a, b2) in zip(ks, part)], 0)
        v = torch.cat([vv[a:b2] for vv, (a, b2) in zip(vs, part)], 0)
        cu = torch.tensor([0] + list(np.cumsum(n)), dtype=torch.int32).to(DEV)
        if layout == "head_major":
            kd = k.permute(1, 0, 2).contiguous().to(DEV).permute(1, 0, 2)
            vd = v.permute(1, 0, 2).contiguous().to(DEV).permute(1, 0, 2)
            return scope_b200.Share(kd, vd, cu_seqlens=cu)
        return scope_b200.Share(k.to(DEV), v.to(DEV), cu_seqlens=cu)

    s0 = make([(0, a) for a in L0])
    s1 = make([(a, L) for a, L in zip(L0, lens)])
    out, lse = scope_b200.gqa_decode_shares(q.to(DEV), [s0, s1], D ** -0.5)
    out, lse = out.float().cpu().numpy(), lse.cpu().numpy()
    for b in range(B):
        qb = q[b].view(Hkv, G, D)
        kb = ks[b].permute(1, 0, 2)
        vb = vs[b].permute(1, 0, 2)
        ro, rm, rs = oracle_of(qb, kb.contiguous(), vb.contiguous(), D ** -0.5)
        assert np.abs(out[b].reshape(Hkv, G, D) - ro).max() < TOL_OUT, b
        assert np.abs(lse[b].reshape(Hkv, G) - (rm + np.log(rs))).max() < TOL_LSE, b


def _torch_ref(q, k, v, scale):
    """fp32 attention of q [G, D] over k, v [L, D] on the device: (out [G, D], lse [G])."""
    s = (q.float() @ k.float().T) * scale
    lse = torch.logsumexp(s, dim=1)
    return torch.softmax(s, dim=1) @ v.float(), lse


@pytest.mark.parametrize("B,nshare,max_len,seed", [(40, 3, 3000, 7), (64, 4, 700, 8), (16, 2, 32768, 2)])
def test_shares_many_segments(ext, B, nshare, max_len, seed):
    """Many short ragged segments per CTA (up to four shares per sequence, some empty), so a group's
    pieces come from several CTAs and shares and are merged by the deferred merge kernel; the last
    case is the cfg2 size.  Checked against an fp32 PyTorch reference on the device."""
    gen = torch.Generator().manual_seed(seed)
    Hkv, G, D = 8, 4, 128
    lens = torch.randint(1, max_len + 1, (B,), generator=gen)
    cuts = torch.sort(torch.randint(0, max_len + 1, (B, nshare - 1), generator=gen), dim=1).values
    bounds = torch.cat([torch.zeros(B, 1, dtype=torch.long), torch.minimum(cuts, lens[:, None]), lens[:, None]], 1)
    q = rand_bf16(B, Hkv * G, D, gen=gen).to(DEV)
    shares, full_k, full_v = [], [], []
    g2 = torch.Generator(device=DEV).manual_seed(seed)
    for b in range(B):
        full_k.append(torch.randn(Hkv, int(lens[b]), D, generator=g2, device=DEV).bfloat16())
        full_v.append(torch.randn(Hkv, int(lens[b]), D, generator=g2, device=DEV).bfloat16())
    for sh in range(nshare):
        n = (bounds[:, sh + 1] - bounds[:, sh]).tolist()
        cap = max(max(n), 1)
        k = torch.zeros(B * Hkv, cap, D, dtype=torch.bfloat16, device=DEV)
        v = torch.zeros(B * Hkv, cap, D, dtype=torch.bfloat16, device=DEV)
        for b in range(B):
            a0, a1 = int(bounds[b, sh]), int(bounds[b, sh + 1])
            k[b * Hkv:(b + 1) * Hkv, :a1 - a0] = full_k[b][:, a0:a1]
            v[b * Hkv:(b + 1) * Hkv, :a1 - a0] = full_v[b][:, a0:a1]
        shares.append(scope_b200.Share(k, v, seqlens=torch.tensor(n, dtype=torch.int32, device=DEV)))
    for rep in range(2):   # the workspace is reused: nothing may depend on a previous call's contents
        out, lse = scope_b200.gqa_decode_shares(q, shares, D ** -0.5)
        for b in range(B):
            for h in range(Hkv):
                ro, rl = _torch_ref(q[b, h * G:(h + 1) * G], full_k[b][h], full_v[b][h], D ** -0.5)
                assert (out[b, h * G:(h + 1) * G].float() - ro).abs().max().item() < TOL_OUT, (rep, b, h)
                assert (lse[b, h * G:(h + 1) * G] - rl).abs().max().item() < TOL_LSE, (rep, b, h)


def test_shares_one_empty_share(ext):
    """A sequence whose second share is empty, and a batch of all-empty rows."""
    gen = torch.Generator().manual_seed(3)
    B, Hkv, G, D = 2, 2, 8, 128
    q = rand_bf16(B, Hkv * G, D, gen=gen).to(DEV)
    k = rand_bf16(B * Hkv, 300, D, gen=gen)
    v = rand_bf16(B * Hkv, 300, D, gen=gen)
    sA = scope_b200.Share(k.to(DEV), v.to(DEV), seqlens=torch.tensor([300, 0], dtype=torch.int32, device=DEV))
    sB = scope_b200.Share(k.to(DEV), v.to(DEV), seqlens=torch.tensor([0, 0], dtype=torch.int32, device=DEV))
    out, lse = scope_b200.gqa_decode_shares(q, [sA, sB], D ** -0.5)
    ro, rm, rs = oracle_of(q[0].view(Hkv, G, D).cpu(), k[:Hkv], v[:Hkv], D ** -0.5)
    assert np.abs(out[0].float().cpu().numpy().reshape(Hkv, G, D) - ro).max() < TOL_OUT
    assert np.abs(lse[0].cpu().numpy().reshape(Hkv, G) - (rm + np.log(rs))).max() < TOL_LSE
    assert torch.all(out[1] == 0) and torch.all(torch.isneginf(lse[1]))


@pytest.mark.parametrize("P,R,D", [(3, 100, 128), (1, 7, 512), (9, 1024, 512), (32, 50, 512), (2, 10, 36),
                                   (33, 20, 64), (5, 9, 130)])
def test_lse_merge_kernel(P, R, D):
    """Both merge kernels: P <= 32 with D % 4 == 0 (lane-per-partial weights,
    all loads in flight) and the general one (P > 32 or D % 4 != 0)."""
    rng = np.random.default_rng(3 + P)
    o = rng.standard_normal((P, R, D))
    lse = rng.standard_normal((P, R)) * 3
    lse[P // 2, :5] = -np.inf
    lse[:, R // 2] = -np.inf
    ro, rl = oracle.lse_merge(o, lse)
    out, ol = scope_b200.lse_merge(torch.tensor(o, dtype=torch.float32, device=DEV),
                                   torch.tensor(lse, dtype=torch.float32, device=DEV), torch.float32)
    out, ol = out.cpu().numpy(), ol.cpu().numpy()
    assert np.abs(out - ro).max() < 1e-5
    fin = np.isfinite(rl)
    assert np.abs(ol[fin] - rl[fin]).max() < 1e-5
    assert np.all(np.isneginf(ol[~fin])) and np.all(out[~fin] == 0)


def test_split_merge_equals_unsplit_large(ext):
    """Size-independent property at a long context: attention over [0, L) equals
    the LSE merge of attention over [0, L/2) and [L/2, L)."""
    gen = torch.Generator(device=DEV).manual_seed(4)
    Bkv, G, D, L = 16, 8, 128, 131072
    q = torch.randn(Bkv, G, D, device=DEV, generator=gen).bfloat16()
    k = torch.randn(Bkv, L, D, device=DEV, generator=gen).bfloat16()
    v = torch.randn(Bkv, L, D, device=DEV, generator=gen).bfloat16()
    sc = D ** -0.5
    full_o, full_m, full_s = ext.fused_cpu_attn_mla(q, k, v, sc)
    parts = [ext.fused_cpu_attn_mla(q, k[:, a:a + L // 2], v[:, a:a + L // 2], sc) for a in (0, L // 2)]
    o_parts = torch.stack([(po / ps).view(-1, D) for po, pm, ps in parts])
    l_parts = torch.stack([(pm + ps.log()).view(-1) for po, pm, ps in parts])
    mo, ml = scope_b200.lse_merge(o_parts, l_parts, torch.float32)
    assert (mo - (full_o / full_s).view(-1, D)).abs().max().item() < 1e-4
    assert (ml - (full_m + full_s.log()).view(-1)).abs().max().item() < 1e-4
    # one row against the oracle at full length
    ro, rm, rs = oracle_of(q[:1].cpu(), k[:1].cpu(), v[:1].cpu(), sc)
    assert np.abs((full_o[:1] / full_s[:1]).cpu().numpy() - ro).max() < TOL_OUT
    assert np.abs((full_m[:1] + full_s[:1].log()).cpu().numpy()[..., 0] - (rm + np.log(rs))).max() < TOL_LSE


@pytest.mark.parametrize("B,G,Dk,Dv,L", [
    (3, 8, 32, 32, 500), (2, 4, 80, 80, 1300), (2, 8, 96, 96, 777), (2, 8, 256, 256, 1500),
    (3, 12, 256, 256, 900), (2, 4, 192, 192, 1000), (2, 10, 192, 192, 600), (2, 8, 64, 128, 900),
    (2, 12, 48, 112, 333), (2, 24, 128, 128, 2000), (2, 32, 128, 128, 700), (1, 40, 64, 64, 300)])
def test_head_sizes_and_groups(ext, B, G, Dk, Dv, L):
    """The head sizes and group counts the reference accepts (any D % 16 == 0,
    any G; kernel/cpu_attn.cpp:578-583): dims up to 256 run on the tile sizes
    rounded up to 64, G > 16 as chunks of 16 query heads over the same rows."""
    g = torch.Generator().manual_seed(B * 1000 + G * 10 + Dk + Dv + L)
    q = rand_bf16(B, G, Dk, gen=g)
    k = rand_bf16(B, L, Dk, gen=g)
    v = rand_bf16(B, L, Dv, gen=g)
    scale = Dk ** -0.5
    o, m, s = ext.fused_cpu_attn_mla(q.to(DEV), k.to(DEV), v.to(DEV), scale)
    torch.cuda.synchronize()
    ro, rm, rs = oracle_of(q, k, v, scale)
    o, m, s = o.cpu().numpy(), m.cpu().numpy()[..., 0], s.cpu().numpy()[..., 0]
    assert np.abs(o / s[..., None] - ro).max() < TOL_OUT
    assert np.abs((m + np.log(s)) - (rm + np.log(rs))).max() < TOL_LSE
    if Dk == Dv:   # the public bf16 form too (bf16 out, max, sum)
        po, pm, ps = ext.fused_cpu_attn(q.to(DEV), k.to(DEV), v.to(DEV), scale)
        torch.cuda.synchronize()
        assert np.abs(po.float().cpu().numpy() - ro).max() < TOL_OUT


def _f64_decode(q, k, v, scale):
    """float64 attention per row: q [B, G, D], k/v [B, L, D] -> (normalised out, lse)."""
    q, k, v = q.double(), k.double(), v.double()
    s = torch.einsum("bgd,bld->bgl", q, k) * scale
    lse = torch.logsumexp(s, dim=-1)
    return torch.einsum("bgl,bld->bgd", torch.softmax(s, dim=-1), v), lse


@pytest.mark.parametrize("B,G,D,L", [
    (3, 8, 128, 1), (2, 8, 128, 31), (2, 8, 128, 33), (4, 8, 128, 1000), (2, 16, 128, 2049), (3, 1, 64, 777),
    (2, 12, 256, 1500), (2, 16, 256, 300), (2, 8, 80, 500), (5, 3, 16, 64), (40, 8, 128, 3000),
    (2, 4, 192, 999), (2, 24, 128, 700), (1, 40, 64, 300),
])
@pytest.mark.parametrize("aligned", [True, False])
def test_fp32_path_shapes(ext, B, G, D, L, aligned):
    """The fp32 path of fused_cpu_attn: 16-byte aligned K/V rows run the tiled kernels (the register-blocked
    one for G <= 8 and D <= 128), rows that are not (a view starting one float into its buffer) the per-token
    kernel; more than 16 query heads per kv row run as launches of 16.  All against a float64 reference."""
    gen = torch.Generator().manual_seed(B * 31 + G * 7 + D + L)
    q = torch.randn(B, G, D, generator=gen)
    kb = torch.randn(B, L, D + 4, generator=gen)
    vb = torch.randn(B, L, D + 4, generator=gen)
    k, v = (kb[..., :D], vb[..., :D]) if aligned else (kb[..., 1:D + 1], vb[..., 1:D + 1])
    ro, rl = _f64_decode(q, k, v, D ** -0.5)
    kd, vd = kb.to(DEV), vb.to(DEV)
    kd, vd = (kd[..., :D], vd[..., :D]) if aligned else (kd[..., 1:D + 1], vd[..., 1:D + 1])
    o, m, s = ext.fused_cpu_attn(q.to(DEV), kd, vd, D ** -0.5)
    torch.cuda.synchronize()
    assert o.dtype == torch.float32
    assert (o.cpu().double() - ro).abs().max().item() < 1e-4
    assert ((m + s.log())[..., 0].cpu().double() - rl).abs().max().item() < 1e-4


def test_fp32_path_token_major_and_long(ext):
    """A token-major [L, Hkv, D] fp32 cache seen per head, and 16384-token rows split over many CTAs; repeated
    launches on one workspace give identical results."""
    gen = torch.Generator(device=DEV).manual_seed(12)
    L, Hkv, G, D = 16384, 4, 8, 128
    kc = torch.randn(L, Hkv, D, device=DEV, generator=gen)
    vc = torch.randn(L, Hkv, D, device=DEV, generator=gen)
    q = torch.randn(Hkv, G, D, device=DEV, generator=gen)
    o, m, s = ext.fused_cpu_attn(q, kc.permute(1, 0, 2), vc.permute(1, 0, 2), D ** -0.5)
    for _ in range(3):
        o2, m2, s2 = ext.fused_cpu_attn(q, kc.permute(1, 0, 2), vc.permute(1, 0, 2), D ** -0.5)
        assert torch.equal(o2, o) and torch.equal(m2, m) and torch.equal(s2, s)
    ro, rl = _f64_decode(q.cpu(), kc.permute(1, 0, 2).cpu(), vc.permute(1, 0, 2).cpu(), D ** -0.5)
    assert (o.cpu().double() - ro).abs().max().item() < 1e-4
    assert ((m + s.log())[..., 0].cpu().double() - rl).abs().max().item() < 1e-4
    assert scope_b200.status_take() == 0
