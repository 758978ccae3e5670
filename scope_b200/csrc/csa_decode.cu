// CSA sparse decode (DeepSeek-V4 style): many query rows of one sequence
// attend over a shared 512-dim latent KV (K = V), either over the entries a
// top-k id list selects (gather) or over a contiguous id range (dense), with
// the KV stored bf16 or int8 with one fp32 scale per entry.
//
// Replaces indexer_attn_cpu (kernel/cpu_attn_ds4_ext/csa_attn.cpp:1819-1883),
// fused_csa_attn (:200-281) and fused_csa_attn_range (:1587-1656), and runs the
// int8-entry storage of the int8 family (values = int8 * scale, :1338-1344)
// without quantising the query.
//
// One thread-block cluster per (sequence, group of <= 64 query rows).  Its CS
// CTAs split the sequence's selected entries evenly; each CTA
//   * gathers its entries 128 at a time straight from global memory into a
//     128-byte-swizzled bf16 tile (int8 -> bf16 is exact for |v| <= 127; the
//     per-entry scale is folded into the scores and into P instead),
//   * S^T[128 x NQ] = K . Q^T and O^T[512 x NQ] += K^T . P^T on tcgen05 with
//     the accumulators in TMEM (the same smem tile read K-major, then MN-major),
//   * keeps a lazily updated running max per query row: O in TMEM is rescaled
//     only when a row's max grows by more than 2^8, which keeps P <= 256 and the
//     result exact because m, l and O always refer to the same max;
// then the cluster merges its CS partials through distributed shared memory:
// CTA r reduces query rows [r*NQ/CS, (r+1)*NQ/CS) by log-sum-exp over the
// peers' (m, l, O) and writes the output.  No workspace, one launch.
#include <cstdio>

#include "common.cuh"
#include "ws_internal.h"

namespace ws {
namespace csa {

constexpr int HD = 512;          // latent width
constexpr int TT = 128;          // entries per tile (MMA M of the first product)
constexpr int kThreads = 256;
constexpr int KBOX = TT * 128;   // 16 KB: 64 dims x 128 entries
constexpr float kLazy = 8.f;     // rescale O only when a row max grows by more than 2^8

// QSPLIT: an fp32 query is held as bf16 hi + lo parts (q - hi rounded again)
// and the first product runs on both, so the scores keep ~16 mantissa bits of
// the query instead of 8.
template <int NQ, bool QSPLIT>
struct Cfg {
    static constexpr int QBOX = NQ * 128;            // 64 dims x NQ query rows
    static constexpr int PBOX = NQ * 128;            // 64 entries x NQ rows
    static constexpr int OFF_K = 0;                  // 8 K boxes; reused for the O partial [NQ][512] fp32
    static constexpr int OFF_Q = 8 * KBOX;           // hi part, then (QSPLIT) lo part
    static constexpr int OFF_P = OFF_Q + (QSPLIT ? 2 : 1) * 8 * QBOX;
    static constexpr int OFF_MISC = OFF_P + 2 * PBOX;
    // misc: scale[TT], row[TT] (int), red[4][NQ], m_used, alpha, m_new, m_fin, l_fin [NQ each],
    //       lred[4][NQ], wgt[NQ][8], rinv[NQ], rlse[NQ]
    static constexpr int MISC_WORDS = 2 * TT + 4 * NQ + 5 * NQ + 4 * NQ + 8 * NQ + 2 * NQ;
    static constexpr size_t SMEM = 1024 + OFF_MISC + MISC_WORDS * 4 + 64;
    static constexpr int TMEM_COLS = NQ == 64 ? 512 : (NQ == 32 ? 256 : 128);
    static constexpr int S_COL = 0, O_COL = NQ;
    static_assert(NQ * HD * 4 <= 8 * KBOX, "O partial must fit in the K tile");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct Params {
    const void* q;
    int q_f32;
    int nq;                   // query rows per sequence (all groups)
    int ngroups;              // ceil(nq / NQ)
    const void* kv;
    int kv_i8;
    const float* kv_scales;   // [bs, nc_local] when kv_i8
    const int* idx;           // [bs, k] (gather) or null (dense)
    int k;
    int window;               // WS_CSA_IDX_* for the gather
    int64_t dense_begin, dense_end;   // dense: ids [begin, end), already clipped to the shard
    int64_t shard_lo, shard_hi;       // this buffer holds ids [shard_lo, shard_hi); row = id - shard_lo
    int64_t nc_local;
    float scale_log2;
    void* out;
    int out_f32;
    float* out_lse;
    int* status;
};

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// first position in ids[0, n) with ids[pos] >= v (ids sorted ascending)
__device__ __forceinline__ int lower_bound_ids(const int* ids, int n, int64_t v) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((int64_t)__ldg(ids + mid) < v) lo = mid + 1; else hi = mid;
    }
    return lo;
}

template <int NQ, bool QSPLIT>
__global__ void __launch_bounds__(kThreads, 1) csa_decode_kernel(const Params p) {
    using C = Cfg<NQ, QSPLIT>;
    constexpr int kMaxCs = 8;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* misc = reinterpret_cast<float*>(sm + C::OFF_MISC);
    float* s_scale = misc;                 // [TT]   per-entry value scale (1 for bf16)
    int* s_row = reinterpret_cast<int*>(s_scale + TT);   // [TT] local row, -1 = no entry
    float* s_red = reinterpret_cast<float*>(s_row + TT); // [4][NQ] per-warp tile max
    float* s_mused = s_red + 4 * NQ;       // [NQ]   running max (log2 units)
    float* s_alpha = s_mused + NQ;         // [NQ]   rescale factor of this tile
    float* s_mnew = s_alpha + NQ;          // [NQ]   running max after this tile
    float* s_mfin = s_mnew + NQ;           // [NQ]   this CTA's final (m, l)
    float* s_lfin = s_mfin + NQ;           // [NQ]
    float* s_lred = s_lfin + NQ;           // [4][NQ]
    float* s_wgt = s_lred + 4 * NQ;        // [NQ][8] merge weights of the peers
    float* s_rinv = s_wgt + 8 * NQ;        // [NQ]   1 / L
    float* s_rlse = s_rinv + NQ;           // [NQ]
    uint64_t* bars = reinterpret_cast<uint64_t*>(s_rlse + NQ);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2);
    int* s_flags = reinterpret_cast<int*>(tmem_holder + 1);   // [0] abort, [1] rescale

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = (int)cluster_ctarank(), CS = (int)cluster_nctarank();
    const int seq = blockIdx.y / p.ngroups, grp = blockIdx.y - seq * p.ngroups;
    const int row0 = grp * NQ;                                   // first query row of this group
    const int nrows = min(NQ, p.nq - row0);
    const int* ids = p.idx ? p.idx + (int64_t)seq * p.k : nullptr;
    const int64_t kv_seq = (int64_t)seq * p.nc_local;            // first row of this sequence

    // ---- this CTA's share of the sequence's entries: positions in ids (gather) or ids (dense)
    int64_t e_begin, e_end;
    {
        int64_t lo, hi;
        if (ids) {
            lo = 0;
            hi = p.k;
            if (p.window == WS_CSA_IDX_SORTED_SHARD) {
                lo = lower_bound_ids(ids, p.k, p.shard_lo);
                hi = lower_bound_ids(ids, p.k, p.shard_hi);
            }
        } else {
            lo = p.dense_begin;
            hi = p.dense_end;
        }
        const int64_t cnt = hi - lo;
        e_begin = lo + cnt * rank / CS;
        e_end = lo + cnt * (rank + 1) / CS;
    }
    const int ntiles = (int)((e_end - e_begin + TT - 1) / TT);

    const uint32_t kbase = smem_u32(sm + C::OFF_K), qbase = smem_u32(sm + C::OFF_Q), pbase = smem_u32(sm + C::OFF_P);
    if (tid == 0) {
        mbar_init(smem_u32(&bars[0]), 1);
        mbar_init(smem_u32(&bars[1]), 1);
        s_flags[0] = 0;
        s_flags[1] = 0;
        fence_mbar_init();
    }
    if (tid < NQ) s_mused[tid] = -INFINITY;
    // ---- queries -> K-major swizzled bf16 (rows past nrows are zero)
    for (int j = tid; j < NQ * (HD / 8); j += kThreads) {
        const int r = j / (HD / 8), c = j - r * (HD / 8);   // 8 dims per 16-byte chunk
        uint4 v = make_uint4(0, 0, 0, 0), vlo = make_uint4(0, 0, 0, 0);
        if (r < nrows) {
            const int64_t off = ((int64_t)seq * p.nq + row0 + r) * HD + c * 8;
            if (p.q_f32) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.q) + off));
                const float4 b = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.q) + off + 4));
                const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    hi[u] = pack_bf16(f[2 * u], f[2 * u + 1]);
                    const float h0 = __uint_as_float(hi[u] << 16), h1 = __uint_as_float(hi[u] & 0xffff0000u);
                    lo[u] = pack_bf16(f[2 * u] - h0, f[2 * u + 1] - h1);
                }
                v = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                vlo = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            } else {
                v = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.q) + off));
            }
        }
        *reinterpret_cast<uint4*>(sm + C::OFF_Q + (c >> 3) * C::QBOX + swz(r, c & 7)) = v;
        if (QSPLIT) *reinterpret_cast<uint4*>(sm + C::OFF_Q + (8 + (c >> 3)) * C::QBOX + swz(r, c & 7)) = vlo;
    }
    if (warp == 0) tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_holder;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    constexpr uint32_t id1 = idesc_bf16_f32(TT, NQ, false, false);
    constexpr uint32_t id2 = idesc_bf16_f32(128, NQ, true, false);

    float l_run[NQ];
#pragma unroll
    for (int h = 0; h < NQ; ++h) l_run[h] = 0.f;

    for (int t = 0; t < ntiles; ++t) {
        // ---- resolve this tile's entries to local rows
        const int64_t ebase = e_begin + (int64_t)t * TT;
        if (tid < TT) {
            const int64_t e = ebase + tid;
            int row = -1;
            float sc = 0.f;
            if (e < e_end) {
                const int64_t id = ids ? (int64_t)__ldg(ids + e) : e;
                if (id >= p.shard_lo && id < p.shard_hi) {
                    row = (int)(id - p.shard_lo);
                    sc = p.kv_i8 ? __ldg(p.kv_scales + kv_seq + row) : 1.f;
                } else if (p.window == WS_CSA_IDX_ALL) {
                    atomicExch(p.status, kDevBadIndex);   // skipped, and reported
                }
            }
            s_row[tid] = row;
            s_scale[tid] = sc;
        }
        __syncthreads();
        // ---- gather into the bf16 K tile (zero rows where there is no entry); all loads first
        if (p.kv_i8) {
            const int8_t* kv = static_cast<const int8_t*>(p.kv);
            const int c = tid & 31, rb = tid >> 5;               // 32 chunks of 16 int8 per row
            int4 raw[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int row = s_row[rb + 8 * i];
                raw[i] = row >= 0 ? __ldg(reinterpret_cast<const int4*>(kv + (kv_seq + row) * HD + c * 16))
                                  : make_int4(0, 0, 0, 0);
            }
            uint8_t* box = sm + C::OFF_K + (c >> 2) * KBOX;      // 16 dims per chunk; 64 dims per box
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int r = rb + 8 * i;
                const int8_t* b8 = reinterpret_cast<const int8_t*>(&raw[i]);
                uint32_t w[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) w[u] = pack_bf16((float)b8[2 * u], (float)b8[2 * u + 1]);
                *reinterpret_cast<uint4*>(box + swz(r, (c & 3) * 2)) = make_uint4(w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4*>(box + swz(r, (c & 3) * 2 + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
            }
        } else {
            const __nv_bfloat16* kv = static_cast<const __nv_bfloat16*>(p.kv);
            const int c = tid & 63, rb = tid >> 6;               // 64 chunks of 8 bf16 per row
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint4 v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int row = s_row[rb + 4 * (half * 16 + i)];
                    v[i] = row >= 0 ? __ldg(reinterpret_cast<const uint4*>(kv + (kv_seq + row) * HD + c * 8))
                                    : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    *reinterpret_cast<uint4*>(sm + C::OFF_K + (c >> 3) * KBOX + swz(rb + 4 * (half * 16 + i), c & 7)) =
                        v[i];
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- S^T = K . Q^T
        if (tid == 0) {
            for (int part = 0; part < (QSPLIT ? 2 : 1); ++part)
                for (int kb = 0; kb < 8; ++kb)
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16(tbase + C::S_COL, sdesc_sw128(kbase + kb * KBOX + kk * 32, 16, 1024),
                                  sdesc_sw128(qbase + (part * 8 + kb) * C::QBOX + kk * 32, 16, 1024), id1,
                                  (part | kb | kk) != 0);
            umma_commit(smem_u32(&bars[0]));
        }
        if (!mbar_wait_bounded(smem_u32(&bars[0]), t & 1)) {
            s_flags[0] = 1;
            atomicExch(p.status, kDevTimeout);
        }
        tc_fence_after();
        // ---- softmax over the tile (warps 0-3: thread = entry row)
        float x[NQ];
        float sc = 0.f;
        if (warp < 4) {
#pragma unroll
            for (int cb = 0; cb < NQ / 16; ++cb) tmem_ld16(tbase + lane_base + C::S_COL + cb * 16, x + cb * 16);
            tmem_wait_ld();
            const int r = warp * 32 + lane;
            sc = s_scale[r];
            const float f = sc * p.scale_log2;
            const bool valid = s_row[r] >= 0;
#pragma unroll
            for (int h = 0; h < NQ; ++h) {
                x[h] = valid ? x[h] * f : -INFINITY;
                float mx = x[h];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                if (lane == 0) s_red[warp * NQ + h] = mx;
            }
        }
        tc_fence_before();
        __syncthreads();
        // new running max per row (lazy), rescale factor, P
        if (warp < 4) {
            int need_any = 0;
#pragma unroll
            for (int h = 0; h < NQ; ++h) {
                const float mt = fmaxf(fmaxf(s_red[h], s_red[NQ + h]), fmaxf(s_red[2 * NQ + h], s_red[3 * NQ + h]));
                const float mo = s_mused[h];
                const bool need = mt > mo + kLazy;   // also true when mo == -inf and mt is finite
                const float mn = need ? mt : mo;
                const float alpha = need ? ex2(mo - mn) : 1.f;
                need_any |= (need && mo != -INFINITY) ? 1 : 0;
                const float pv = (mn == -INFINITY) ? 0.f : ex2(x[h] - mn);
                l_run[h] = l_run[h] * alpha + pv;
                x[h] = pv * sc;                     // the value scale folded into P
                if (tid == 0) {
                    s_alpha[h] = alpha;
                    s_mnew[h] = mn;
                }
            }
            // P^T, K-major: rows = query rows, 64 entries per 128-byte row, two boxes
            const int r = warp * 32 + lane;
            uint8_t* pb = sm + C::OFF_P + (r >> 6) * C::PBOX;
            const int kc = (r & 63) >> 3, ke = (r & 7) * 2;
#pragma unroll
            for (int h = 0; h < NQ; ++h)
                *reinterpret_cast<__nv_bfloat16*>(pb + h * 128 + ((kc ^ (h & 7)) << 4) + ke) = __float2bfloat16_rn(x[h]);
            if (tid == 0) s_flags[1] = need_any;
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (tid < NQ) s_mused[tid] = s_mnew[tid];
        if (s_flags[1] && t > 0 && warp < 4) {
            // O (previous tiles) *= alpha per query row; the previous second product has completed
            for (int mb = 0; mb < 4; ++mb)
#pragma unroll
                for (int cb = 0; cb < NQ / 16; ++cb) {
                    float v[16];
                    const uint32_t ta = tbase + lane_base + C::O_COL + mb * NQ + cb * 16;
                    tmem_ld16(ta, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int u = 0; u < 16; ++u) v[u] *= s_alpha[cb * 16 + u];
                    tmem_st16(ta, v);
                }
            tmem_wait_st();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- O^T += K^T . P^T
        if (tid == 0) {
            for (int mb = 0; mb < 4; ++mb)
                for (int ks = 0; ks < TT / 16; ++ks)
                    umma_bf16(tbase + C::O_COL + mb * NQ,
                              sdesc_sw128(kbase + (2 * mb) * KBOX + ks * 2048, KBOX, 1024),
                              sdesc_sw128(pbase + (ks >> 2) * C::PBOX + (ks & 3) * 32, 16, 1024), id2,
                              (t > 0 || ks > 0) ? 1u : 0u);
            umma_commit(smem_u32(&bars[1]));
        }
        if (!mbar_wait_bounded(smem_u32(&bars[1]), t & 1)) {
            s_flags[0] = 1;
            atomicExch(p.status, kDevTimeout);
        }
        tc_fence_after();
        __syncthreads();
        if (s_flags[0]) break;
    }

    // ---- this CTA's partial: (m, l) per row and O -> shared memory (over the K tile)
    if (warp < 4) {
#pragma unroll
        for (int h = 0; h < NQ; ++h) {
            float v = l_run[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) s_lred[warp * NQ + h] = v;
        }
    }
    __syncthreads();
    const bool have = ntiles > 0 && !s_flags[0];
    if (tid < NQ) {
        s_mfin[tid] = have ? s_mused[tid] : -INFINITY;
        s_lfin[tid] = have ? s_lred[tid] + s_lred[NQ + tid] + s_lred[2 * NQ + tid] + s_lred[3 * NQ + tid] : 0.f;
    }
    float* o_part = reinterpret_cast<float*>(sm + C::OFF_K);   // [NQ][512]
    if (have) {
        if (warp < 4)
            for (int mb = 0; mb < 4; ++mb)
#pragma unroll
                for (int cb = 0; cb < NQ / 16; ++cb) {
                    float v[16];
                    tmem_ld16(tbase + lane_base + C::O_COL + mb * NQ + cb * 16, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int u = 0; u < 16; ++u) o_part[(cb * 16 + u) * HD + mb * 128 + warp * 32 + lane] = v[u];
                }
    } else {
        for (int j = tid; j < NQ * HD; j += kThreads) o_part[j] = 0.f;
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();

    // ---- merge the cluster's partials: this CTA owns rows [rank*RPC, (rank+1)*RPC)
    const int RPC = NQ / CS;
    if (tid < RPC) {
        const int h = rank * RPC + tid;
        float M = -INFINITY;
        float mc[kMaxCs];
#pragma unroll
        for (int c = 0; c < kMaxCs; ++c) {
            mc[c] = c < CS ? dsmem_ld_f32(dsmem_addr(smem_u32(s_mfin + h), c)) : -INFINITY;
            M = fmaxf(M, mc[c]);
        }
        float L = 0.f;
#pragma unroll
        for (int c = 0; c < kMaxCs; ++c) {
            const float w = (mc[c] == -INFINITY) ? 0.f : ex2(mc[c] - M);
            s_wgt[tid * 8 + c] = w;
            if (w != 0.f) L += w * dsmem_ld_f32(dsmem_addr(smem_u32(s_lfin + h), c));
        }
        const bool empty = !(L > 0.f);
        s_rinv[tid] = empty ? 0.f : 1.f / L;
        s_rlse[tid] = empty ? -INFINITY : M * kLn2 + logf(L);
    }
    __syncthreads();
    for (int j = tid; j < RPC * (HD / 4); j += kThreads) {
        const int hl = j / (HD / 4), d4 = j - hl * (HD / 4);
        const int h = rank * RPC + hl;
        if (h >= nrows) continue;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < CS; ++c) {
            const float w = s_wgt[hl * 8 + c];
            if (w == 0.f) continue;
            const float4 v = dsmem_ld_f32x4(dsmem_addr(smem_u32(o_part + h * HD + d4 * 4), c));
            acc.x += w * v.x; acc.y += w * v.y; acc.z += w * v.z; acc.w += w * v.w;
        }
        const float inv = s_rinv[hl];
        const int64_t oi = ((int64_t)seq * p.nq + row0 + h) * HD + d4 * 4;
        if (p.out_f32) {
            *reinterpret_cast<float4*>(static_cast<float*>(p.out) + oi) =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        } else {
            __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + oi;
            *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
            *reinterpret_cast<__nv_bfloat162*>(o + 2) = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
        }
    }
    if (tid < RPC && rank * RPC + tid < nrows && p.out_lse)
        p.out_lse[(int64_t)seq * p.nq + row0 + rank * RPC + tid] = s_rlse[tid];
    // peers keep their shared memory until every CTA of the cluster has read it
    cluster_sync();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tbase, C::TMEM_COLS);
}

template <int NQ, bool QSPLIT>
static int launch(const Params& p, int bs, int cs, cudaStream_t st) {
    auto kfn = csa_decode_kernel<NQ, QSPLIT>;
    static int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg<NQ, QSPLIT>::SMEM) !=
            cudaSuccess)
            return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for csa_decode_kernel");
        configured_dev = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs, (unsigned)(bs * p.ngroups), 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg<NQ, QSPLIT>::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, p);
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace csa

int csa_cluster_size(int64_t entries_per_seq) {
    int cs = 1;
    while (cs < 8 && entries_per_seq > (int64_t)cs * 256) cs *= 2;
    return cs;
}

int csa_launch(const CsaLaunch& a) {
    using namespace csa;
    Params p;
    memset(&p, 0, sizeof(p));
    p.q = a.q;
    p.q_f32 = a.q_f32;
    p.nq = a.nq;
    // query rows per cluster: 64 for a bf16 query, 32 for an fp32 query (its hi/lo parts)
    const int NQ = a.nq <= 16 ? 16 : (a.nq <= 32 || a.q_f32 ? 32 : 64);
    p.ngroups = (a.nq + NQ - 1) / NQ;
    if ((int64_t)a.bs * p.ngroups > 65535) return set_error(WS_ERR_UNSUPPORTED, "csa_decode: bs * ceil(nq/64) > 65535");
    p.kv = a.kv;
    p.kv_i8 = a.kv_i8;
    p.kv_scales = a.kv_scales;
    p.idx = a.idx;
    p.k = a.k;
    p.window = a.window;
    p.shard_lo = a.shard_lo;
    p.shard_hi = a.shard_lo + a.nc_local;
    p.dense_begin = std::max(a.dense_begin, p.shard_lo);
    p.dense_end = std::max(p.dense_begin, std::min(a.dense_end, p.shard_hi));
    p.nc_local = a.nc_local;
    p.scale_log2 = a.scale * kLog2e;
    p.out = a.out;
    p.out_f32 = a.out_f32;
    p.out_lse = a.out_lse;
    p.status = device_status_word();
    // CTAs per sequence: about 256 entries each, at most 8 (one portable cluster)
    const int cs = csa_cluster_size(a.idx ? (int64_t)a.k : p.dense_end - p.dense_begin);
    cudaStream_t st = static_cast<cudaStream_t>(a.stream);
    if (a.q_f32) return NQ == 16 ? launch<16, true>(p, a.bs, cs, st) : launch<32, true>(p, a.bs, cs, st);
    if (NQ == 16) return launch<16, false>(p, a.bs, cs, st);
    if (NQ == 32) return launch<32, false>(p, a.bs, cs, st);
    return launch<64, false>(p, a.bs, cs, st);
}

}  // namespace ws
