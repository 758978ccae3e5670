"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference's own AVX-512 extensions (compiled from the reference
sources into oracle/_ref by ``make -C oracle ref REF_DIR=<reference checkout>``)
on small seeded inputs and stores inputs + outputs as .npz.  The fixtures are
committed; this script is only re-run when a fixture is added.

    python tests/golden/make_golden.py

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


def main():
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


if __name__ == "__main__":
    main()
