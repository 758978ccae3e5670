"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference's own AVX-512 extensions (compiled from the reference
sources into oracle/_ref by ``make -C oracle ref REF_DIR=<reference checkout>``)
on small seeded inputs and stores inputs + outputs as .npz.  The fixtures are
committed; this script is only re-run when a fixture is added.

    python tests/golden/make_golden.py                 # every fixture
    python tests/golden/make_golden.py csa_int8 ...    # the named sections only

Sections: base (the first seven fixtures), csa_int8, csa_bf16q, indexer_large.
indexer_large stores the reference's ids for inputs drawn from numpy's
``default_rng`` (platform-independent streams) rather than the inputs
themselves; tests regenerate them from the stored seed and check a checksum.

bf16 tensors are stored as their uint16 bit patterns.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def b(x):
    return oracle.bf16_bits(x)


def save(name, **arrs):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: (v.numpy() if torch.is_tensor(v) else np.asarray(v)) for k, v in arrs.items()})
    print("wrote", path, sum(os.path.getsize(path) for _ in [0]), "bytes")


def base():
    ref = oracle.load_ref("cpu_attn_ext")
    tile = oracle.load_ref("cpu_attn_tile_ext")
    csa = oracle.load_ref("csa_attn_kernel")
    ref.set_num_threads(4)

    # 1. GQA, Qwen3 layer shape (G=8, D=128), odd length, bf16 public + mla form
    g = torch.Generator().manual_seed(101)
    Bkv, G, D, L = 4, 8, 128, 203
    q = torch.randn(Bkv, G, D, generator=g).bfloat16()
    k = torch.randn(Bkv, L, D, generator=g).bfloat16()
    v = torch.randn(Bkv, L, D, generator=g).bfloat16()
    sc = D ** -0.5
    po, pm, ps = ref.fused_cpu_attn(q, k, v, sc)
    mo, mm, ms = ref.fused_cpu_attn_mla(q, k, v, sc)
    save("gqa_qwen3_bf16", q=b(q), k=b(k), v=b(v), scale=sc,
         pub_out=b(po), pub_max=b(pm), pub_sum=b(ps), mla_o=mo, mla_max=mm, mla_sum=ms)

    # 2. GQA with a strided KV view ([1, L, Hkv, D] token-major cache, per-head view)
    g = torch.Generator().manual_seed(102)
    Hkv, G, D, L = 4, 4, 128, 77
    q = torch.randn(Hkv, G, D, generator=g).bfloat16()
    kc = torch.randn(L, Hkv, D, generator=g).bfloat16()
    vc = torch.randn(L, Hkv, D, generator=g).bfloat16()
    kview, vview = kc.permute(1, 0, 2), vc.permute(1, 0, 2)
    mo, mm, ms = ref.fused_cpu_attn_mla(q, kview, vview, sc)
    save("gqa_strided_bf16", q=b(q), k_cache=b(kc), v_cache=b(vc), scale=sc,
         mla_o=mo, mla_max=mm, mla_sum=ms)

    # 3. DS2 non-absorbed MLA through fused_cpu_attn_mla (Dk=192, Dv=128, G=1)
    g = torch.Generator().manual_seed(103)
    Bkv, G, Dk, Dv, L = 8, 1, 192, 128, 150
    q = torch.randn(Bkv, G, Dk, generator=g).bfloat16()
    k = torch.randn(Bkv, L, Dk, generator=g).bfloat16()
    v = torch.randn(Bkv, L, Dv, generator=g).bfloat16()
    sc = Dk ** -0.5
    mo, mm, ms = ref.fused_cpu_attn_mla(q, k, v, sc)
    save("mla_nonabsorbed_bf16", q=b(q), k=b(k), v=b(v), scale=sc, mla_o=mo, mla_max=mm, mla_sum=ms)

    # 4. fp32 GQA (public fp32 path and the scalar ablation)
    g = torch.Generator().manual_seed(104)
    Bkv, G, D, L = 2, 8, 64, 300
    q = torch.randn(Bkv, G, D, generator=g)
    k = torch.randn(Bkv, L, D, generator=g)
    v = torch.randn(Bkv, L, D, generator=g)
    sc = D ** -0.5
    fo, fm, fs = ref.fused_cpu_attn(q, k, v, sc)
    so, sm, ss = ref.fused_cpu_attn_fp32(q, k, v, sc)
    save("gqa_fp32", q=q, k=k, v=v, scale=sc, pub_out=fo, pub_max=fm, pub_sum=fs,
         abl_out=so, abl_max=sm, abl_sum=ss)

    # 5. Absorbed MLA (DeepSeek-V2-Lite: 16 heads, latent 512 + rope 64)
    g = torch.Generator().manual_seed(105)
    B, nH, S = 2, 16, 130
    qp = torch.randn(B * nH, 512, generator=g).bfloat16()
    qpe = torch.randn(B * nH, 64, generator=g).bfloat16()
    c = torch.randn(B, S, 512, generator=g).bfloat16()
    p = torch.randn(B, S, 64, generator=g).bfloat16()
    sc = 192 ** -0.5
    o, m, s = ref.fused_cpu_attn_mla_compressed(qp, qpe, c, p, sc)
    os.environ["MLA_TILE"] = "64"
    to, tm, ts = tile.fused_cpu_attn_mla_compressed(qp, qpe, c, p, sc)
    del os.environ["MLA_TILE"]
    save("mla_compressed", q_proj=b(qp), q_pe=b(qpe), c_kv=b(c), k_pe=b(p), scale=sc,
         o=o, max=m, sum=s, tile64_o=to, tile64_max=tm, tile64_sum=ts)

    # 6. CSA: dense, range, gather (indexer_attn_cpu), int8 quantisers and int8_preq
    g = torch.Generator().manual_seed(106)
    bs, nH, sq, hd, nc, kk = 2, 4, 2, 512, 96, 32
    q = torch.randn(bs, nH, sq, hd, generator=g)
    kv = torch.randn(bs, nc, hd, generator=g).bfloat16()
    sc = hd ** -0.5
    do, dl = csa.fused_csa_attn(q, kv, sc)
    ro, rl = csa.fused_csa_attn_range(q, kv, sc, 10, 70)
    qg = torch.randn(bs, 8, hd, generator=g)
    idx = torch.stack([torch.randperm(nc, generator=g)[:kk].sort().values for _ in range(bs)]).int()
    go = torch.empty(bs, 8, hd)
    gl = torch.empty(bs, 8)
    csa.indexer_attn_cpu(qg, kv, idx, sc, go, gl, 2)
    ki8, ksc, ksm = csa.kv_quantize_bf16_to_int8(kv, 2)
    qu8, qsc = csa.q_quantize_fp32_to_u8(q, 2)
    io = torch.empty(bs, nH, sq, hd)
    il = torch.empty(bs, nH, sq)
    csa.fused_csa_attn_bsq_int8_preq(q, ki8, ksc, ksm, sc, io, il, 2)
    save("csa", q=q, kv=b(kv), scale=sc, dense_o=do, dense_lse=dl, range_o=ro, range_lse=rl,
         range_s=10, range_e=70, q_gather=qg, idx=idx, gather_o=go, gather_lse=gl,
         kv_i8=ki8, kv_scales=ksc, kv_sums=ksm, q_u8=qu8, q_scales=qsc, int8_o=io, int8_lse=il)

    # 7. Indexer top-k
    g = torch.Generator().manual_seed(107)
    bs, nH, hd, nc, k = 2, 4, 64, 200, 16
    qi = torch.randn(bs, nH, hd, generator=g)
    kvi = torch.randn(bs, nc, hd, generator=g)
    w = torch.rand(bs, nH, generator=g)
    ids = csa.indexer_topk_cpu(qi, kvi, w, k, 2)
    save("indexer_topk", q_idx=qi, kv_idx=kvi, weights=w, k=k, ids=ids)


def csa_int8():
    """The reference's integer-score operators: _bsq_int8 (both quantisers
    inside), _bsq_int8_preq and _bsq_int8_full, at hd 512 and hd 256."""
    csa = oracle.load_ref("csa_attn_kernel")
    g = torch.Generator().manual_seed(108)
    arrs = {}
    for tag, (bs, nH, sq, hd, nc) in (("h512", (2, 4, 2, 512, 96)), ("h256", (2, 3, 1, 256, 70))):
        q = torch.randn(bs, nH, sq, hd, generator=g)
        kv = torch.randn(bs, nc, hd, generator=g).bfloat16()
        sc = hd ** -0.5
        bo, bl = torch.empty(bs, nH, sq, hd), torch.empty(bs, nH, sq)
        csa.fused_csa_attn_bsq_int8(q, kv, sc, bo, bl, 2)
        ki8, ksc, ksm = csa.kv_quantize_bf16_to_int8(kv, 2)
        qu8, qsc = csa.q_quantize_fp32_to_u8(q, 2)
        po, pl = torch.empty(bs, nH, sq, hd), torch.empty(bs, nH, sq)
        csa.fused_csa_attn_bsq_int8_preq(q, ki8, ksc, ksm, sc, po, pl, 2)
        fo, fl = torch.empty(bs, nH, sq, hd), torch.empty(bs, nH, sq)
        csa.fused_csa_attn_bsq_int8_full(qu8, qsc, ki8, ksc, ksm, kv, sc, fo, fl, 2)
        arrs.update({f"{tag}_q": q, f"{tag}_kv": b(kv), f"{tag}_scale": sc, f"{tag}_bsq_o": bo, f"{tag}_bsq_lse": bl,
                     f"{tag}_preq_o": po, f"{tag}_preq_lse": pl, f"{tag}_full_o": fo, f"{tag}_full_lse": fl})
    save("csa_int8", **arrs)


def csa_bf16q():
    """The bf16-query dense variants (_pool_bf16, _bsq_bf16, _fast_bf16,
    _2pass_bf16) on bf16 q, at hd 512 and hd 256."""
    csa = oracle.load_ref("csa_attn_kernel")
    g = torch.Generator().manual_seed(109)
    arrs = {}
    for tag, (bs, nH, sq, hd, nc) in (("h512", (2, 8, 2, 512, 96)), ("h256", (2, 4, 1, 256, 50))):
        q = torch.randn(bs, nH, sq, hd, generator=g).bfloat16()
        kv = torch.randn(bs, nc, hd, generator=g).bfloat16()
        sc = hd ** -0.5
        po, pl = csa.fused_csa_attn_pool_bf16(q, kv, sc, 2)
        arrs.update({f"{tag}_q": b(q), f"{tag}_kv": b(kv), f"{tag}_scale": sc, f"{tag}_pool_o": po,
                     f"{tag}_pool_lse": pl})
        for name in ("bsq_bf16", "fast_bf16", "2pass_bf16"):
            o, l_ = torch.empty(bs, nH, sq, hd), torch.empty(bs, nH, sq)
            getattr(csa, "fused_csa_attn_" + name)(q, kv, sc, o, l_, 2)
            arrs[f"{tag}_{name}_o"] = o
            arrs[f"{tag}_{name}_lse"] = l_
    save("csa_bf16q", **arrs)


INDEXER_LARGE = ((1101, 2, 64, 128, 20000, 2048), (1102, 1, 16, 64, 65536, 2048))


def indexer_large_inputs(seed, bs, nH, hd, nc):
    """Inputs of one indexer_large case, from numpy's platform-independent generator."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((bs, nH, hd), dtype=np.float32)
    kv = rng.standard_normal((bs, nc, hd), dtype=np.float32)
    w = rng.random((bs, nH), dtype=np.float32)
    return q, kv, w


def indexer_large():
    """indexer_topk_cpu at nc >= 20000, k = 2048: the reference's ids."""
    csa = oracle.load_ref("csa_attn_kernel")
    arrs = {}
    for i, (seed, bs, nH, hd, nc, k) in enumerate(INDEXER_LARGE):
        q, kv, w = indexer_large_inputs(seed, bs, nH, hd, nc)
        ids = csa.indexer_topk_cpu(torch.from_numpy(q), torch.from_numpy(kv), torch.from_numpy(w), k, 4)
        arrs.update({f"c{i}_shape": np.array([seed, bs, nH, hd, nc, k]), f"c{i}_ids": ids,
                     f"c{i}_checksum": np.array([float(q.astype(np.float64).sum()), float(kv.astype(np.float64).sum()),
                                                 float(w.astype(np.float64).sum())])})
    save("indexer_topk_large", **arrs)


SECTIONS = {"base": base, "csa_int8": csa_int8, "csa_bf16q": csa_bf16q, "indexer_large": indexer_large}

if __name__ == "__main__":
    for name in (sys.argv[1:] or list(SECTIONS)):
        SECTIONS[name]()
