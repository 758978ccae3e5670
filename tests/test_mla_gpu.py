"""GPU parity of the absorbed-MLA decode (tcgen05) against the oracle and the
reference's golden outputs (fused_cpu_attn_mla_compressed,
kernel/cpu_attn.cpp:852-1022).  Tolerances: normalised output max-abs 2e-2,
LSE 1e-3, max 1e-3."""
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


def bits_to_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def rand_inputs(B, S, nH=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    qp = torch.randn(B * nH, 512, generator=g).bfloat16()
    qpe = torch.randn(B * nH, 64, generator=g).bfloat16()
    c = torch.randn(B, S, 512, generator=g).bfloat16()
    p = torch.randn(B, S, 64, generator=g).bfloat16()
    return qp, qpe, c, p


def check_against_oracle(ext, qp, qpe, c, p, scale):
    o, m, s = ext.fused_cpu_attn_mla_compressed(qp.to(DEV), qpe.to(DEV), c.to(DEV), p.to(DEV), scale)
    torch.cuda.synchronize()
    ro, rm, rs = oracle.mla_compressed(*(oracle.bf16_bits(t) for t in (qp, qpe, c, p)), scale)
    o, m, s = o.cpu().numpy(), m.cpu().numpy(), s.cpu().numpy()
    assert np.abs(o / s[:, None] - ro / rs[:, None]).max() < TOL_OUT
    assert np.abs((m + np.log(s)) - (rm + np.log(rs))).max() < TOL_LSE
    assert np.abs(m - rm).max() < TOL_LSE


def test_golden(ext, golden):
    g = golden("mla_compressed")
    qp, qpe, c, p = (bits_to_bf16(g[n]) for n in ("q_proj", "q_pe", "c_kv", "k_pe"))
    o, m, s = ext.fused_cpu_attn_mla_compressed(qp, qpe, c, p, float(g["scale"]))
    assert o.shape == (32, 512) and m.shape == (32,) and s.shape == (32,)
    assert o.dtype == torch.float32
    o, m, s = o.cpu().numpy(), m.cpu().numpy(), s.cpu().numpy()
    assert np.abs(o / s[:, None] - g["o"] / g["sum"][:, None]).max() < TOL_OUT / 10
    assert np.abs((m + np.log(s)) - (g["max"] + np.log(g["sum"]))).max() < TOL_LSE
    assert np.abs(m - g["max"]).max() < TOL_LSE


@pytest.mark.parametrize("B,S", [(2, 1), (2, 127), (2, 128), (2, 129), (3, 700), (1, 4096), (8, 2000),
                                 (300, 100), (37, 257)])
def test_random_shapes(ext, B, S):
    qp, qpe, c, p = rand_inputs(B, S, seed=B * 1000 + S)
    check_against_oracle(ext, qp, qpe, c, p, 192 ** -0.5)


def test_empty_sequence(ext):
    qp, qpe, c, p = rand_inputs(2, 0)
    o, m, s = ext.fused_cpu_attn_mla_compressed(qp.to(DEV), qpe.to(DEV), c.to(DEV), p.to(DEV), 0.07)
    assert torch.all(o == 0) and torch.all(torch.isneginf(m)) and torch.all(s == 0)


def test_normalised_bf16_path(ext):
    qp, qpe, c, p = rand_inputs(4, 1500, seed=7)
    out, lse = scope_b200.cpu_attn.mla_decode(qp.to(DEV), qpe.to(DEV), c.to(DEV), p.to(DEV), 192 ** -0.5)
    assert out.dtype == torch.bfloat16
    ro, rm, rs = oracle.mla_compressed(*(oracle.bf16_bits(t) for t in (qp, qpe, c, p)), 192 ** -0.5)
    assert np.abs(out.float().cpu().numpy() - ro / rs[:, None]).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - (rm + np.log(rs))).max() < TOL_LSE


def test_cfg3_size(ext):
    """The DeepSeek-V2-Lite benchmark shape (B=8, 16 heads, S=16384): two rows
    against the oracle, all rows against the split/merge property."""
    qp, qpe, c, p = rand_inputs(8, 16384, seed=3)
    sc = 192 ** -0.5
    qp_d, qpe_d, c_d, p_d = qp.to(DEV), qpe.to(DEV), c.to(DEV), p.to(DEV)
    o, m, s = ext.fused_cpu_attn_mla_compressed(qp_d, qpe_d, c_d, p_d, sc)
    ro, rm, rs = oracle.mla_compressed(*(oracle.bf16_bits(t) for t in (qp[:16], qpe[:16], c[:1], p[:1])), sc)
    on = (o / s[:, None]).cpu().numpy()
    assert np.abs(on[:16] - ro / rs[:, None]).max() < TOL_OUT
    assert np.abs((m + s.log()).cpu().numpy()[:16] - (rm + np.log(rs))).max() < TOL_LSE
    halves = [ext.fused_cpu_attn_mla_compressed(qp_d, qpe_d, c_d[:, a:a + 8192].contiguous(),
                                                p_d[:, a:a + 8192].contiguous(), sc) for a in (0, 8192)]
    parts_o = torch.stack([ho / hs[:, None] for ho, hm, hs in halves])
    parts_l = torch.stack([hm + hs.log() for ho, hm, hs in halves])
    mo, ml = scope_b200.lse_merge(parts_o, parts_l, torch.float32)
    assert (mo - o / s[:, None]).abs().max().item() < 1e-3
    assert (ml - (m + s.log())).abs().max().item() < 1e-3


# ------------------------------------------------ absorbed step with its projections
def absorbed_inputs(B, S, nop, vhd, nH=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    q_nope = torch.randn(B, nH, nop, generator=g).bfloat16()
    qpe = torch.randn(B * nH, 64, generator=g).bfloat16()
    c = torch.randn(B, S, 512, generator=g).bfloat16()
    p = torch.randn(B, S, 64, generator=g).bfloat16()
    w = (torch.randn(nH * (nop + vhd), 512, generator=g) * 0.05).bfloat16()   # kv_b_proj.weight
    return q_nope, qpe, c, p, w


@pytest.mark.parametrize("B,S,nop,vhd", [(1, 1, 128, 128), (2, 300, 128, 128), (8, 4096, 128, 128),
                                         (3, 129, 64, 96), (11, 257, 128, 128), (2, 0, 128, 128)])
def test_absorbed_step_matches_oracle(B, S, nop, vhd):
    """ws_mla_decode_absorbed (absorb GEMM, tcgen05 decode, merge fused with the up-projection) against
    the oracle of system/deepseek.py's absorbed decode branch, bf16 roundings included."""
    q_nope, qpe, c, p, w = absorbed_inputs(B, S, nop, vhd, seed=B * 131 + S)
    scale = 192 ** -0.5
    out, lse = scope_b200.cpu_attn.mla_decode_absorbed(q_nope.to(DEV), qpe.to(DEV), c.to(DEV), p.to(DEV),
                                                        w.to(DEV), scale, return_lse=True)
    assert out.dtype == torch.bfloat16 and tuple(out.shape) == (B, 16, vhd)
    w3 = w.view(16, nop + vhd, 512)
    ro, rl = oracle.mla_absorbed(oracle.bf16_bits(q_nope), oracle.bf16_bits(qpe), oracle.bf16_bits(c),
                                 oracle.bf16_bits(p), oracle.bf16_bits(w3[:, :nop].contiguous()),
                                 oracle.bf16_bits(w3[:, nop:].contiguous()), scale)
    o = out.float().cpu().numpy()
    assert np.abs(o - ro).max() < TOL_OUT
    lse = lse.cpu().numpy().reshape(-1)
    if S == 0:
        assert np.all(o == 0) and np.all(np.isneginf(lse))
    else:
        assert np.abs(lse - rl).max() < TOL_LSE


def test_absorbed_step_equals_unfused_composition():
    """The fused step against the reference's own order of operations on the GPU: bmm absorb (torch),
    the MLA decode, bf16 cast, bmm up-projection (torch)."""
    B, S, nop, vhd = 8, 16384, 128, 128
    q_nope, qpe, c, p, w = (t.to(DEV) for t in absorbed_inputs(B, S, nop, vhd, seed=7))
    scale = 192 ** -0.5
    out = scope_b200.cpu_attn.mla_decode_absorbed(q_nope, qpe, c, p, w, scale)
    w3 = w.view(16, nop + vhd, 512)
    w_uk, w_uv = w3[:, :nop], w3[:, nop:]
    qp = torch.bmm(q_nope.reshape(B * 16, 1, nop), w_uk.expand(B, 16, nop, 512).reshape(B * 16, nop, 512))
    o, _ = scope_b200.cpu_attn.mla_decode(qp.reshape(B * 16, 512).contiguous(), qpe, c, p, scale)
    ref = torch.bmm(o.view(B * 16, 1, 512),
                    w_uv.transpose(1, 2).expand(B, 16, 512, vhd).reshape(B * 16, 512, vhd)).view(B, 16, vhd)
    assert (out.float() - ref.float()).abs().max().item() < TOL_OUT


def test_decode_steps_after_appends_without_host_sync():
    """Decode steps on one stream, each right after the append of that step's token and with no host
    synchronisation in between: the decode is a programmatic dependent launch (its setup overlaps the
    previous grid), so its first latent load must still see the token the append just wrote."""
    from scope_b200.kv_cache import _append
    S0, steps, scale = 300, 6, 192 ** -0.5
    qp, qpe, c, p = rand_inputs(1, S0 + steps, seed=31)
    cd = torch.zeros(1, S0 + steps, 512, dtype=torch.bfloat16, device=DEV)
    pd = torch.zeros(1, S0 + steps, 64, dtype=torch.bfloat16, device=DEV)
    cd[:, :S0] = c[:, :S0].to(DEV)
    pd[:, :S0] = p[:, :S0].to(DEV)
    new_c, new_p = c[:, S0:].to(DEV).contiguous(), p[:, S0:].to(DEV).contiguous()
    qd, qped = qp.to(DEV), qpe.to(DEV)
    torch.cuda.synchronize()
    outs = []
    for s in range(steps):
        S = S0 + s + 1
        _append(cd, new_c[:, s:s + 1], S - 1)
        _append(pd, new_p[:, s:s + 1], S - 1)
        outs.append(scope_b200.cpu_attn.mla_decode(qd, qped, cd[:, :S], pd[:, :S], scale))
    torch.cuda.synchronize()
    for s, (out, lse) in enumerate(outs):
        S = S0 + s + 1
        ro, rm, rs = oracle.mla_compressed(*(oracle.bf16_bits(t) for t in (qp, qpe, c[:, :S], p[:, :S])), scale)
        assert np.abs(out.float().cpu().numpy() - ro / rs[:, None]).max() < TOL_OUT, s
        assert np.abs(lse.cpu().numpy() - (rm + np.log(rs))).max() < TOL_LSE, s


@pytest.mark.parametrize("nH,B,S", [(32, 3, 700), (128, 2, 1500), (8, 4, 300), (20, 2, 257)])
def test_head_counts(ext, nH, B, S):
    """Any heads per sequence (the reference takes nH = q_proj.size(0) / B,
    kernel/cpu_attn.cpp:858-862): multiples of 16 run as head groups that
    share the latent, other counts on zero-padded query rows."""
    check_against_oracle(ext, *rand_inputs(B, S, nH=nH, seed=nH + S), 192 ** -0.5)


def test_strided_latent_views(ext):
    """c_kv / k_pe as views of a larger cache ([B, cap, *] read for S tokens)
    are read in place through the batch stride."""
    from scope_b200.cpu_attn import mla_decode
    B, nH, S, cap = 3, 16, 900, 1280
    qp, qpe, c, p = rand_inputs(B, S, nH=nH, seed=5)
    cbuf = torch.zeros(B, cap, 512, dtype=torch.bfloat16, device=DEV)
    pbuf = torch.zeros(B, cap, 64, dtype=torch.bfloat16, device=DEV)
    cbuf[:, :S] = c.to(DEV)
    pbuf[:, :S] = p.to(DEV)
    cbuf[:, S:] = 30.0   # garbage past the filled tokens must not be read
    out, lse = mla_decode(qp.to(DEV), qpe.to(DEV), cbuf[:, :S], pbuf[:, :S], 192 ** -0.5)
    torch.cuda.synchronize()
    ro, rm, rs = oracle.mla_compressed(*(oracle.bf16_bits(t) for t in (qp, qpe, c, p)), 192 ** -0.5)
    assert np.abs(out.float().cpu().numpy() - ro / rs[:, None]).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy() - (rm + np.log(rs))).max() < TOL_LSE
