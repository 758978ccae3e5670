"""GPU checks of the device-resident sharded KV caches (scope_b200.kv_cache):
appends are bit-exact copies (against the reference's InplaceKVCache
semantics: ``get`` returns every appended token in order), and the decode over
the cache -- one shard, or N shards emulated on one GPU and merged by LSE --
matches the float64 oracle over all tokens."""
import numpy as np
import pytest
import torch

import oracle
import scope_b200
from scope_b200.kv_cache import ShardedKVCache, ShardedKVCacheCompressed

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def steps_of(total, prefill):
    return [prefill] + [1] * (total - prefill)


def test_gqa_append_and_get_bit_exact():
    g = torch.Generator().manual_seed(1)
    B, Hkv, D, total = 2, 4, 128, 70
    cache = ShardedKVCache(2, B, Hkv, 100, D, device=DEV)
    ks, vs = [], []
    for n in steps_of(total, 33):
        k = torch.randn(B, Hkv, n, D, generator=g).bfloat16()
        v = torch.randn(B, Hkv, n, D, generator=g).bfloat16()
        cache.append_4d(1, k.to(DEV), v.to(DEV))
        ks.append(k)
        vs.append(v)
    kk, vv = cache.get(1)
    assert cache.seq_len(1) == total and kk.shape == (B * Hkv, total, D)
    assert torch.equal(kk.cpu(), torch.cat(ks, 2).reshape(B * Hkv, total, D))
    assert torch.equal(vv.cpu(), torch.cat(vs, 2).reshape(B * Hkv, total, D))
    assert cache.seq_len(0) == 0
    with pytest.raises(RuntimeError, match="full"):
        cache.append_4d(1, torch.zeros(B, Hkv, 31, D, dtype=torch.bfloat16, device=DEV),
                        torch.zeros(B, Hkv, 31, D, dtype=torch.bfloat16, device=DEV))


@pytest.mark.parametrize("world", [1, 2, 3])
def test_gqa_sharded_decode_matches_oracle(world):
    g = torch.Generator().manual_seed(10 + world)
    B, H, Hkv, D, total, max_seq = 2, 16, 4, 128, 300, 320
    caches = [ShardedKVCache(1, B, Hkv, max_seq, D, world=world, rank=r, device=DEV) for r in range(world)]
    ks, vs = [], []
    for n in steps_of(total, 200):
        k = torch.randn(B, Hkv, n, D, generator=g).bfloat16()
        v = torch.randn(B, Hkv, n, D, generator=g).bfloat16()
        for c in caches:
            c.append_4d(0, k.to(DEV), v.to(DEV))
        ks.append(k)
        vs.append(v)
    assert sum(c.local_len(0) for c in caches) == total
    q = torch.randn(B, H, D, generator=g).bfloat16()
    scale = D ** -0.5
    qv = q.reshape(B * Hkv, H // Hkv, D).to(DEV)
    parts_o, parts_l = [], []
    for c in caches:
        k, v = c.get(0)
        o, l = scope_b200.cpu_attn.gqa_decode(qv, k, v, scale, out_dtype=torch.float32)
        parts_o.append(o.reshape(B * H, D))
        parts_l.append(l.reshape(B * H))
    out, lse = scope_b200.lse_merge(torch.stack(parts_o), torch.stack(parts_l), torch.float32)
    K = torch.cat(ks, 2).reshape(B * Hkv, total, D)
    V = torch.cat(vs, 2).reshape(B * Hkv, total, D)
    ro, rm, rs = oracle.gqa_decode(oracle.bf16_bits(q.reshape(B * Hkv, H // Hkv, D)), oracle.bf16_bits(K),
                                   oracle.bf16_bits(V), scale)
    assert np.abs(out.cpu().numpy().reshape(B * Hkv, H // Hkv, D) - ro).max() < 2e-2
    assert np.abs(lse.cpu().numpy().reshape(B * Hkv, H // Hkv) - (rm + np.log(rs))).max() < 1e-3
    if world == 1:
        o1, l1 = caches[0].decode(0, q.to(DEV), scale)
        assert np.abs(o1.float().cpu().numpy().reshape(B * Hkv, H // Hkv, D) - ro).max() < 2e-2


@pytest.mark.parametrize("world", [1, 2])
def test_mla_compressed_cache(world):
    g = torch.Generator().manual_seed(20 + world)
    B, nH, total = 2, 16, 500
    caches = [ShardedKVCacheCompressed(1, B, 512, 512, 64, world=world, rank=r, device=DEV) for r in range(world)]
    cs, ps = [], []
    for n in steps_of(total, 400):
        c = torch.randn(B, n, 512, generator=g).bfloat16()
        p = torch.randn(B, n, 64, generator=g).bfloat16()
        for ca in caches:
            ca.append(0, c.to(DEV), p.to(DEV))
        cs.append(c)
        ps.append(p)
    C, P = torch.cat(cs, 1), torch.cat(ps, 1)
    if world == 1:
        cc, pp = caches[0].get(0)
        assert torch.equal(cc.cpu(), C) and torch.equal(pp.cpu(), P)
    qp = torch.randn(B * nH, 512, generator=g).bfloat16()
    qpe = torch.randn(B * nH, 64, generator=g).bfloat16()
    scale = 192 ** -0.5
    ext = scope_b200.build()
    parts_o, parts_l = [], []
    for ca in caches:
        cc, pp = ca.get(0)
        o, m, s = ext.fused_cpu_attn_mla_compressed(qp.to(DEV), qpe.to(DEV), cc.contiguous(), pp.contiguous(), scale)
        parts_o.append(o / s[:, None].clamp(min=1e-30))
        parts_l.append(torch.where(s > 0, m + s.clamp(min=1e-30).log(), torch.full_like(m, float("-inf"))))
    out, lse = scope_b200.lse_merge(torch.stack(parts_o), torch.stack(parts_l), torch.float32)
    ro, rm, rs = oracle.mla_compressed(*(oracle.bf16_bits(t) for t in (qp, qpe, C, P)), scale)
    assert np.abs(out.cpu().numpy() - ro / rs[:, None]).max() < 2e-2
    assert np.abs(lse.cpu().numpy() - (rm + np.log(rs))).max() < 1e-3


def test_mla_compressed_cache_decode():
    """ShardedKVCacheCompressed.decode at world 1: the cache buffers ([B, cap, *],
    cap > filled tokens) are read in place."""
    g = torch.Generator().manual_seed(29)
    B, nH, total = 2, 16, 700
    ca = ShardedKVCacheCompressed(1, B, 1024, 512, 64, device=DEV)
    cs, ps = [], []
    for n in steps_of(total, 300):
        c = torch.randn(B, n, 512, generator=g).bfloat16()
        p = torch.randn(B, n, 64, generator=g).bfloat16()
        ca.append(0, c.to(DEV), p.to(DEV))
        cs.append(c)
        ps.append(p)
    C, P = torch.cat(cs, 1), torch.cat(ps, 1)
    qp = torch.randn(B * nH, 512, generator=g).bfloat16()
    qpe = torch.randn(B * nH, 64, generator=g).bfloat16()
    out, lse = ca.decode(0, qp.to(DEV), qpe.to(DEV), 192 ** -0.5)
    torch.cuda.synchronize()
    ro, rm, rs = oracle.mla_compressed(*(oracle.bf16_bits(t) for t in (qp, qpe, C, P)), 192 ** -0.5)
    assert np.abs(out.float().cpu().numpy() - ro / rs[:, None]).max() < 2e-2
    assert np.abs(lse.cpu().numpy() - (rm + np.log(rs))).max() < 1e-3
