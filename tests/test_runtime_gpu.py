"""GPU parity of the runtime swap-in (scope_b200.runtime) against the oracle.

Mirrors the reference harness's correctness check
(roofline/bench_resident_kv.py:410-459): its three model shapes (qwen3: 4 kv
heads x 8 groups, 128/128; ds2: 16 heads x 1 group, 192/128; mixtral: 8 x 4,
128/128), B = 2, kv = 4096, and both splits -- kvlen (streamed gs = kv/4,
resident kv/4, CPU share the rest) and bkv (CPU rows, resident rows, streamed
rows).  The harness compares at atol = rtol = 2e-2 against torch on the whole
KV; here the reference is the float64 oracle, max-abs 2e-2 on the bf16
outputs.  The absorbed-MLA layer step (system/deepseek.py:326-407) is checked
over several decode steps with synthetic weights against the reference's
branch restated in fp32 torch.
"""
import numpy as np
import pytest
import torch

import oracle
import scope_b200
from scope_b200 import runtime
from scope_b200.kv_cache import ShardedKVCacheCompressed

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL_OUT = 2e-2
TOL_LSE = 1e-3

MODELS = {"qwen3": (4, 8, 128, 128), "ds2": (16, 1, 192, 128), "mixtral": (8, 4, 128, 128)}


def _case(model, B=2, kv=4096, seed=0):
    NH, G, QHD, VHD = MODELS[model]
    g = torch.Generator().manual_seed(seed)
    bkv = B * NH
    q = torch.randn(bkv, G, QHD, generator=g).bfloat16()
    k = torch.randn(bkv, kv, QHD, generator=g).bfloat16()
    v = torch.randn(bkv, kv, VHD, generator=g).bfloat16()
    return q, k, v, QHD ** -0.5


@pytest.mark.parametrize("model", sorted(MODELS))
def test_kvlen_split(model):
    scope_b200.build()
    B, kv = 2, 4096
    q, k, v, scale = _case(model, B, kv)
    gs = n_res = kv // 4
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    cuts = [(0, gs), (gs, gs + n_res), (gs + n_res, kv)]   # streamed, resident, CPU share
    out, lse = runtime.kvlen_decode(qd, [kd[:, a:b] for a, b in cuts], [vd[:, a:b] for a, b in cuts], scale, B=B,
                                    return_lse=True)
    torch.cuda.synchronize()
    NH, G, QHD, VHD = MODELS[model]
    assert out.shape == (B, NH * G, 1, VHD) and out.dtype == torch.bfloat16
    ro, rm, rs = oracle.gqa_decode(oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v), scale)
    assert np.abs(out.float().cpu().numpy().reshape(-1, VHD) - ro.reshape(-1, VHD)).max() < TOL_OUT
    assert np.abs(lse.cpu().numpy().reshape(-1) - (rm + np.log(rs)).reshape(-1)).max() < TOL_LSE


@pytest.mark.parametrize("model", sorted(MODELS))
def test_bkv_split(model):
    scope_b200.build()
    B, kv = 2, 4096
    q, k, v, scale = _case(model, B, kv, seed=1)
    NH, G, QHD, VHD = MODELS[model]
    bkv = B * NH
    b_cpu = bkv // 2
    n_res = max(1, b_cpu // 2)
    rows = [(0, b_cpu - n_res), (b_cpu - n_res, b_cpu), (b_cpu, bkv)]   # CPU rows, resident rows, streamed rows
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out = runtime.bkv_decode(qd, [(kd[a:b].contiguous(), vd[a:b].contiguous()) for a, b in rows], scale, B=B)
    torch.cuda.synchronize()
    ro, _, _ = oracle.gqa_decode(oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v), scale)
    assert np.abs(out.float().cpu().numpy().reshape(-1, VHD) - ro.reshape(-1, VHD)).max() < TOL_OUT


def test_kvlen_with_empty_shares():
    scope_b200.build()
    q, k, v, scale = _case("qwen3", 2, 1000, seed=2)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out = runtime.kvlen_decode(qd, [kd[:, :0], kd, kd[:, :0]], [vd[:, :0], vd, vd[:, :0]], scale, B=2)
    torch.cuda.synchronize()
    ro, _, _ = oracle.gqa_decode(oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v), scale)
    assert np.abs(out.float().cpu().numpy().reshape(-1, 128) - ro.reshape(-1, 128)).max() < TOL_OUT


def test_pairwise_merge_matches_whole():
    """The harness's (o, max, sum) merge (roofline/bench_resident_kv.py:141-148) on the device."""
    from scope_b200.cpu_attn import fused_cpu_attn_mla
    q, k, v, scale = _case("mixtral", 2, 3000, seed=3)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    o1, m1, s1 = fused_cpu_attn_mla(qd, kd[:, :1234], vd[:, :1234], scale)
    o2, m2, s2 = fused_cpu_attn_mla(qd, kd[:, 1234:], vd[:, 1234:], scale)
    o, m, s = runtime.pairwise_merge(o1, m1, s1, o2, m2, s2)
    torch.cuda.synchronize()
    ro, rm, rs = oracle.gqa_decode(oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v), scale)
    on = (o / s).cpu().numpy()
    assert np.abs(on - ro).max() < TOL_OUT
    assert np.abs((m + s.log()).cpu().numpy()[..., 0] - (rm + np.log(rs))).max() < TOL_LSE


def _reference_branch(q_nope, q_pe, c, p, w, nH, nop, vhd, scale):
    """The single-token branch of _mla_compressed_forward (system/deepseek.py:257-265,
    :326-407) restated in fp32 torch on the same inputs: absorb, scores over the
    whole cache, softmax, o_n = bf16(o / s), up-projection."""
    B = q_nope.shape[0]
    w3 = w.float().view(nH, nop + vhd, 512)
    w_uk, w_uv = w3[:, :nop], w3[:, nop:]
    qk = torch.einsum("bhn,hnc->bhc", q_nope.float().view(B, nH, nop), w_uk).bfloat16().float()   # bmm -> bf16
    sc = (torch.einsum("bhc,bsc->bhs", qk, c.float()) +
          torch.einsum("bhr,bsr->bhs", q_pe.float().view(B, nH, 64), p.float())) * scale
    m = sc.amax(-1, keepdim=True)
    e = torch.exp(sc - m)
    o = torch.einsum("bhs,bsc->bhc", e, c.float()) / e.sum(-1, keepdim=True)
    o_n = o.bfloat16().float()
    return torch.einsum("bhc,hvc->bhv", o_n, w_uv).reshape(B, 1, nH * vhd)


def test_mla_layer_decode_steps():
    """MlaDecodeLayer over a prefilled cache and then several decode steps (append the
    new token, attend over the cache in place), with synthetic kv_b_proj weights."""
    scope_b200.build()
    g = torch.Generator().manual_seed(9)
    B, nH, nop, vhd, prefill, steps = 2, 16, 128, 128, 3000, 4
    scale = (nop + 64) ** -0.5
    w = (torch.randn(nH * (nop + vhd), 512, generator=g) * 0.2).bfloat16()
    cache = ShardedKVCacheCompressed(1, B, prefill + 64, 512, 64, device=DEV)
    c0 = torch.randn(B, prefill, 512, generator=g).bfloat16()
    p0 = torch.randn(B, prefill, 64, generator=g).bfloat16()
    cache.append(0, c0.to(DEV), p0.to(DEV))
    layer = runtime.MlaDecodeLayer(cache, w.to(DEV), nH, nop, vhd, scale)
    cs, ps = [c0], [p0]
    for _ in range(steps):
        q_nope = torch.randn(B, nH, 1, nop, generator=g).bfloat16()
        q_pe = torch.randn(B, nH, 1, 64, generator=g).bfloat16()
        c1 = torch.randn(B, 1, 512, generator=g).bfloat16()
        p1 = torch.randn(B, 1, 64, generator=g).bfloat16()
        out = layer.step(0, q_nope.to(DEV), q_pe.to(DEV), c1.to(DEV), p1.to(DEV))
        cs.append(c1)
        ps.append(p1)
        torch.cuda.synchronize()
        want = _reference_branch(q_nope, q_pe, torch.cat(cs, 1), torch.cat(ps, 1), w, nH, nop, vhd, scale)
        assert out.shape == (B, 1, nH * vhd)
        # relative to the output's scale: bf16 rounding of o_n and of the output is ~4e-3 of it
        assert (out.float().cpu() - want).abs().max().item() < TOL_OUT * want.abs().max().item()
    assert cache.seq_len(0) == prefill + steps


def _ds4_case(seed, bsz=2, nH=16, hd=512, win=128, nc=700):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(bsz, 1, nH, hd, generator=g).bfloat16()
    kw = torch.randn(bsz, win, hd, generator=g).bfloat16()
    kc = torch.randn(bsz, nc, hd, generator=g).bfloat16()
    return q, kw, kc


def test_ds4_parallel_branch():
    """system/ds4offload.py:286-327 (the 'parallel' branch): window attention over the
    whole window cache, compressed attention over the first n_compress entries, merged
    by the pairwise formula -- restated here in float64 as the reference writes it."""
    scope_b200.build()
    q, kw, kc = _ds4_case(21)
    scale, n_compress = 512 ** -0.5, 650
    out, lse = runtime.ds4_window_compressed_decode(q.to(DEV), kw.to(DEV), kc.to(DEV), scale,
                                                    n_compress=n_compress, return_lse=True)
    torch.cuda.synchronize()
    qf, kwf, kcf = q.squeeze(1).double(), kw.double(), kc[:, :n_compress].double()

    def part(kv):
        sc = torch.einsum("bnh,bsh->bns", qf, kv) * scale
        m = sc.amax(-1, keepdim=True)
        e = torch.exp(sc - m)
        return torch.einsum("bns,bsh->bnh", e, kv), m, e.sum(-1, keepdim=True)

    o_c, m_c, s_c = part(kcf)
    o_w, m_w, s_w = part(kwf)
    m_g = torch.maximum(m_w, m_c)
    w_w, w_c = torch.exp(m_w - m_g), torch.exp(m_c - m_g)
    denom = w_w * s_w + w_c * s_c
    want = (o_w * w_w + o_c * w_c) / denom
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    assert (out.squeeze(1).double().cpu() - want).abs().max().item() < TOL_OUT
    assert (lse.double().cpu() - (m_g + denom.log())[..., 0]).abs().max().item() < TOL_LSE


def test_ds4_gather_branch_with_sink():
    """system/ds4offload.py:328-342: the valid window entries plus the indexer's
    compressed entries in one softmax, with a per-head sink logit in the denominator.
    Padding ids (-1) and ids past the cache are skipped."""
    scope_b200.build()
    q, kw, kc = _ds4_case(22)
    bsz, _, nH, hd = q.shape
    scale, window_len, k = 512 ** -0.5, 100, 256
    g = torch.Generator().manual_seed(23)
    ids = torch.stack([torch.randperm(kc.shape[1], generator=g)[:k] for _ in range(bsz)]).int()
    ids[:, -5:] = -1                       # padding
    ids[0, 0] = kc.shape[1] + 3            # past the cache
    sink = torch.randn(nH, generator=g) * 2.0
    out, lse = runtime.ds4_window_compressed_decode(q.to(DEV), kw.to(DEV), kc.to(DEV), scale, window_len=window_len,
                                                    topk_idxs=ids.to(DEV), attn_sink=sink.to(DEV), return_lse=True)
    torch.cuda.synchronize()
    for b in range(bsz):
        sel = ids[b][(ids[b] >= 0) & (ids[b] < kc.shape[1])].long()
        kv = torch.cat([kw[b, :window_len], kc[b, sel]]).double()            # [n, hd]
        sc = (q[b, 0].double() @ kv.T) * scale                                # [nH, n]
        logits = torch.cat([sc, sink.double()[:, None]], dim=1)              # the sink column carries no value
        p = torch.softmax(logits, dim=1)[:, :-1]
        want = p @ kv
        want_lse = torch.logsumexp(logits, dim=1)
        assert (out[b, 0].double().cpu() - want).abs().max().item() < TOL_OUT
        assert (lse[b].double().cpu() - want_lse).abs().max().item() < TOL_LSE
