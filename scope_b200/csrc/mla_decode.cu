// Absorbed-MLA decode on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces fused_cpu_attn_mla_compressed (kernel/cpu_attn.cpp:852-1022):
//   score(h, t) = scale * (q_proj[h] . c[t] + q_pe[h] . p[t])   (576-dim dot)
//   o[h]        = sum_t softmax(score)[h, t] * c[t]              (V = the 512 latent)
// for nH heads of one sequence sharing one latent KV.
//
// One persistent CTA per SM walks an even share of the flattened (batch,
// token tile) space.  Warp roles (352 threads):
//   warp 8      producer: TMA loads of each tile (128 tokens; 64 with
//               WS_MLA_TILE=64) -- the latent as four "pairs" (two 64-dim
//               SWIZZLE_128B boxes) through a 5-slot ring (11 for 64-token
//               tiles), the 64-dim rope box through a 2-slot ring, and the
//               batch's queries (576 x nH) when a new batch starts;
//   warps 9-10  one thread each issues the MMAs (warp 9 the first product of
//               every tile, warp 10 the second); warp 9 owns the TMEM allocation:
//                 S^T[tile x nH]     = [C | P](tile) . [Q_proj | Q_pe]^T  (A K-major)
//                 O^T[512 x nH]      = C(tile)^T . P^T                   (A MN-major:
//                 the same swizzled latent tile, read along the other axis)
//               S and O are double-buffered in TMEM (10*nH of 256 columns);
//   warps 0-3   softmax: lanes 0-15 of each warp = a token (the M=64 TMEM
//               layout puts tile row 16w+r in lane 32w+r); per-head tile max by warp
//               shuffles + shared memory, online rescale factors, P in bf16
//               written K-major (swizzled) for the second MMA;
//   warps 4-7   correction: thread = latent dim (TMEM lane) x 4 blocks; loads
//               each tile's fresh O^T from TMEM and accumulates
//               acc = acc * alpha + O in registers.
// At a batch boundary the CTA files one piece (o, m, l) per head into
// workspace slot cta + batch; mla_merge_kernel (launched as a programmatic
// dependent) merges a batch's pieces by log-sum-exp into the outputs.
// Every mbarrier wait is bounded (2 s) and a timeout aborts the CTA cleanly
// (status word set, TMEM freed).
#include <cstdio>

#include "common.cuh"
#include "ws_internal.h"

namespace ws {

namespace mla {

constexpr int NH = 16;          // heads per sequence (MMA N)
constexpr int CLR = 512;        // latent (kv_lora_rank)
constexpr int QRD = 64;         // rope dims
#ifndef WS_MLA_TILE
#define WS_MLA_TILE 128
#endif
constexpr int TT = WS_MLA_TILE;  // tokens per tile (MMA M of the first product: 64 or 128)
static_assert(TT == 64 || TT == 128, "MLA tile must be 64 or 128 tokens");
constexpr int NP = TT == 64 ? 11 : 5;   // latent pair slots (4 per tile)
constexpr int NE = TT == 64 ? 3 : 2;    // rope slots
constexpr int BOX_BYTES = TT * 128;         // 8 KB: 64 dims x 64 tokens
constexpr int PAIR_BYTES = 2 * BOX_BYTES;   // 16 KB: 128 latent dims x 64 tokens
constexpr int QBOX_BYTES = NH * 128;        // 2 KB
constexpr int PBUF_BYTES = (TT / 64) * NH * 128;   // P^T of one tile: one K-box per 64 tokens
constexpr int TMEM_COLS = 256;
constexpr int S_COL = 0;                    // S[j] at j*NH
constexpr int O_COL = 2 * NH;               // O[j] at O_COL + j*4*NH
constexpr int kThreads = 352;
constexpr int SLOT_FLOATS = NH * CLR + 2 * NH;

constexpr int OFF_PAIRS = 0;
constexpr int OFF_PE = OFF_PAIRS + NP * PAIR_BYTES;
constexpr int OFF_Q = OFF_PE + NE * BOX_BYTES;
constexpr int OFF_P = OFF_Q + 9 * QBOX_BYTES;
constexpr int OFF_MISC = OFF_P + 2 * PBUF_BYTES;
// barriers
constexpr int B_PAIR_FULL = 0, B_PAIR_EMPTY = NP, B_PE_FULL = 2 * NP, B_PE_EMPTY = 2 * NP + NE,
              B_Q_FULL = 2 * NP + 2 * NE, B_Q_EMPTY = B_Q_FULL + 1, B_S_FULL = B_Q_EMPTY + 1,
              B_S_EMPTY = B_S_FULL + 2, B_P_FULL = B_S_EMPTY + 2, B_P_EMPTY = B_P_FULL + 2,
              B_O_FULL = B_P_EMPTY + 2, B_O_EMPTY = B_O_FULL + 2, B_ALPHA = B_O_EMPTY + 2,
              B_ST_FULL = B_ALPHA + 4, B_ST_EMPTY = B_ST_FULL + 1, B_RED = B_ST_EMPTY + 1, B_LRED = B_RED + 2,
              B_DONE = B_LRED + 1, B_DONE2 = B_DONE + 1, NBARS = B_DONE2 + 1;
constexpr int MISC_BYTES = NBARS * 8 + (2 * 4 * NH + 4 * NH + 2 * NH + 4 * NH) * 4 + 64;
constexpr size_t SMEM_BYTES = 1024 + OFF_MISC + MISC_BYTES;
static_assert(SMEM_BYTES <= 227 * 1024, "MLA shared-memory plan exceeds 227 KB");

struct Maps {
    CUtensorMap c;     // c_kv  [B, S, 512]   dims (512, S, B)
    CUtensorMap pe;    // k_pe  [B, S, 64]    dims (64, S, B)
    CUtensorMap q;     // q_proj [B*nH, 512]  dims (512, B*nH, 1)
    CUtensorMap qpe;   // q_pe   [B*nH, 64]   dims (64, B*nH, 1)
};

struct Params {
    int B, S, tpb;          // query sequences (head groups of NH heads), tokens, tiles per sequence
    int hg;                 // head groups per latent sequence: query sequence b reads latent row b / hg
    float scale_log2;       // softmax scale * log2(e)
    int c_tok_in_dim2, pe_tok_in_dim2;   // tensor-map axis order (see make_kv_map)
    float* ws_part;         // pieces, slot = cta + batch
    int kv_after_primary;   // launched as a programmatic dependent of a grid that may write the latent cache
    int* status;
};

struct Smem {
    uint8_t* base;
    uint64_t* bars;
    float* red;      // [2][4][NH] per-warp tile maxima
    float* alpha;    // [4][NH] per-tile rescale factors for the correction warps
    float* stats;    // [2][NH] segment (m, l)
    float* lred;     // [4][NH] per-warp partial sums
    uint32_t* tmem_holder;
    volatile int* abort_flag;
};

__device__ __forceinline__ uint32_t bar(const Smem& s, int i) { return smem_u32(&s.bars[i]); }

// Bounded wait that also gives up as soon as another role aborted the CTA.
__device__ __forceinline__ bool wait_bar(const Smem& s, uint32_t b, uint32_t parity, int* status) {
    if (mbar_try_wait(b, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(b, parity)) return true;
        if (*s.abort_flag) return false;
        if (globaltimer_ns() - t0 > 2000000000ull) {
            *s.abort_flag = 1;
            atomicExch(status, kDevTimeout);
            return false;
        }
    }
}

// 16 per-thread values -> each lane ends with the warp-wide max (or sum) of every entry.
__device__ __forceinline__ void warp_allmax16(float* v) {
#pragma unroll
    for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v[h] = fmaxf(v[h], __shfl_xor_sync(0xffffffffu, v[h], o));
}
__device__ __forceinline__ void warp_allsum16(float* v) {
#pragma unroll
    for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v[h] += __shfl_xor_sync(0xffffffffu, v[h], o);
}

__global__ void __launch_bounds__(kThreads, 1)
mla_decode_kernel(const __grid_constant__ Maps maps, const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    Smem s;
    s.base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    s.bars = reinterpret_cast<uint64_t*>(s.base + OFF_MISC);
    s.red = reinterpret_cast<float*>(s.bars + NBARS);
    s.alpha = s.red + 2 * 4 * NH;
    s.stats = s.alpha + 4 * NH;
    s.lred = s.stats + 2 * NH;
    s.tmem_holder = reinterpret_cast<uint32_t*>(s.lred + 4 * NH);
    s.abort_flag = reinterpret_cast<volatile int*>(s.tmem_holder + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x;
    const int64_t total = (int64_t)p.B * p.tpb;
    const int nctas = total < 1 ? 1 : (total < (int64_t)gridDim.x ? (int)total : (int)gridDim.x);
    const int64_t t_begin = cta < nctas ? split_start(cta, total, nctas) : total;
    const int64_t t_end = cta < nctas ? split_start(cta + 1, total, nctas) : total;

    const uint32_t pairs = smem_u32(s.base + OFF_PAIRS), pes = smem_u32(s.base + OFF_PE);
    const uint32_t qs = smem_u32(s.base + OFF_Q), ps = smem_u32(s.base + OFF_P);

    // Producer state (lane 0 of warp 8 issues every TMA load).  It initialises the barriers and issues
    // the first tile's loads before the setup barrier, so they are in flight during the TMEM allocation.
    int seg = -1, qn = 0;
    int64_t pi = 0;   // tiles whose loads were issued (on a failed wait: the tile being issued)
    int pb = (int)(t_begin / p.tpb);
    int ptl = (int)(t_begin - (int64_t)pb * p.tpb);
    auto issue_tile = [&]() -> bool {
        const int64_t i = pi;
        const bool new_seg = pb != seg;   // this tile starts a sequence: its q follows the tile's latent
        const int lb = pb / p.hg;         // the latent sequence this query sequence's heads read
        for (int pr = 0; pr < 4; ++pr) {
            const int64_t n = 4 * i + pr;
            const int sl = (int)(n % NP);
            const uint32_t u = (uint32_t)(n / NP);
            if (u > 0 && !wait_bar(s, bar(s, B_PAIR_EMPTY + sl), (u - 1) & 1, p.status)) return false;
            mbar_arrive_expect_tx(bar(s, B_PAIR_FULL + sl), PAIR_BYTES);
            const int c1 = p.c_tok_in_dim2 ? lb : ptl * TT, c2 = p.c_tok_in_dim2 ? ptl * TT : lb;
            tma_load_3d(pairs + sl * PAIR_BYTES, &maps.c, bar(s, B_PAIR_FULL + sl), 128 * pr, c1, c2);
            tma_load_3d(pairs + sl * PAIR_BYTES + BOX_BYTES, &maps.c, bar(s, B_PAIR_FULL + sl), 128 * pr + 64,
                        c1, c2);
        }
        if (new_seg) {
            if (qn > 0 && !wait_bar(s, bar(s, B_Q_EMPTY), (qn - 1) & 1, p.status)) return false;
            // q may come from the previous grid on the stream (the absorb GEMM, launched as its
            // programmatic dependent); without one this returns at once
            if (qn == 0) pdl_wait_primary();
            mbar_arrive_expect_tx(bar(s, B_Q_FULL), 9 * QBOX_BYTES);
            for (int kb = 0; kb < 8; ++kb)
                tma_load_3d(qs + kb * QBOX_BYTES, &maps.q, bar(s, B_Q_FULL), kb * 64, pb * NH, 0);
            tma_load_3d(qs + 8 * QBOX_BYTES, &maps.qpe, bar(s, B_Q_FULL), 0, pb * NH, 0);
            ++qn;
            seg = pb;
        }
        const int e = (int)(i % NE);
        const uint32_t ue = (uint32_t)(i / NE);
        if (ue > 0 && !wait_bar(s, bar(s, B_PE_EMPTY + e), (ue - 1) & 1, p.status)) return false;
        mbar_arrive_expect_tx(bar(s, B_PE_FULL + e), BOX_BYTES);
        tma_load_3d(pes + e * BOX_BYTES, &maps.pe, bar(s, B_PE_FULL + e), 0, p.pe_tok_in_dim2 ? lb : ptl * TT,
                    p.pe_tok_in_dim2 ? ptl * TT : lb);
        if (++ptl == p.tpb) {
            ptl = 0;
            ++pb;
        }
        ++pi;
        return true;
    };

    bool pok = true;
    if (warp == 8 && lane == 0) {
        for (int i = 0; i < NP; ++i) {
            mbar_init(bar(s, B_PAIR_FULL + i), 1);
            mbar_init(bar(s, B_PAIR_EMPTY + i), 1);
        }
        for (int i = 0; i < NE; ++i) {
            mbar_init(bar(s, B_PE_FULL + i), 1);
            mbar_init(bar(s, B_PE_EMPTY + i), 1);
        }
        mbar_init(bar(s, B_Q_FULL), 1);
        mbar_init(bar(s, B_Q_EMPTY), 1);
        for (int j = 0; j < 2; ++j) {
            mbar_init(bar(s, B_S_FULL + j), 1);
            mbar_init(bar(s, B_S_EMPTY + j), 4);
            mbar_init(bar(s, B_P_FULL + j), 4);
            mbar_init(bar(s, B_P_EMPTY + j), 1);
            mbar_init(bar(s, B_O_FULL + j), 1);
            mbar_init(bar(s, B_O_EMPTY + j), 4);
        }
        for (int j = 0; j < 4; ++j) mbar_init(bar(s, B_ALPHA + j), 1);
        mbar_init(bar(s, B_ST_FULL), 1);
        mbar_init(bar(s, B_ST_EMPTY), 4);
        mbar_init(bar(s, B_RED), 4);
        mbar_init(bar(s, B_RED + 1), 4);
        mbar_init(bar(s, B_LRED), 4);
        mbar_init(bar(s, B_DONE), 1);
        mbar_init(bar(s, B_DONE2), 1);
        *s.abort_flag = 0;
        fence_mbar_init();
        if (t_begin < t_end) {
            tma_prefetch_desc(&maps.c);
            tma_prefetch_desc(&maps.pe);
            tma_prefetch_desc(&maps.q);
            tma_prefetch_desc(&maps.qpe);
            // a programmatic dependent launch of a grid that may append to the cache waits for it before
            // its first latent load; after the absorb GEMM (which writes only q_proj) it waits only for q
            if (p.kv_after_primary) pdl_wait_primary();
            pok = issue_tile();   // the first tile waits on no barrier
        }
    }
    if (warp == 9) tmem_alloc(smem_u32(s.tmem_holder), TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *s.tmem_holder;
    pdl_launch_dependents();

    if (warp == 8) {
        // ------------------------------------------------------------ producer
        if (lane == 0 && t_begin < t_end) {
            while (pok && t_begin + pi < t_end) pok = issue_tile();
            if (*s.abort_flag) {
                // leave no bulk copy in flight into this CTA's shared memory:
                // wait (bounded) for the last load issued into every slot
                const int64_t np_issued = 4 * pi + 4, ne_issued = pi + 1;
                for (int sl = 0; sl < NP; ++sl) {
                    int64_t n = np_issued - 1 - ((np_issued - 1 - sl) % NP + NP) % NP;
                    if (n >= 0) mbar_wait_bounded(bar(s, B_PAIR_FULL + sl), (uint32_t)(n / NP) & 1, 200000000ull);
                }
                for (int e = 0; e < NE; ++e) {
                    int64_t n = ne_issued - 1 - ((ne_issued - 1 - e) % NE + NE) % NE;
                    if (n >= 0) mbar_wait_bounded(bar(s, B_PE_FULL + e), (uint32_t)(n / NE) & 1, 200000000ull);
                }
                if (qn > 0) mbar_wait_bounded(bar(s, B_Q_FULL), (qn - 1) & 1, 200000000ull);
            }
        }
    } else if (warp == 9 || warp == 10) {
        // ------------------------------------------------------------- MMA issue
        // Two issuing threads: warp 9 runs the first product of every tile,
        // warp 10 the second, so freeing a tile's ring slots (after its second
        // product) never waits behind the next tile's loads.
        if (lane == 0 && t_begin < t_end) {
            const uint32_t id1 = idesc_bf16_f32(TT, NH, false, false);
            const uint32_t id2 = idesc_bf16_f32(128, NH, true, false);
            const int64_t n_tiles = t_end - t_begin;
            int q_seg = -1, qn = 0;
            bool ok = true;
            auto gemm1 = [&](int64_t i) -> bool {
                const int64_t t = t_begin + i;
                const int b = (int)(t / p.tpb), tl = (int)(t - (int64_t)b * p.tpb);
                const int j = (int)(i & 1);
                const uint32_t us = (uint32_t)(i >> 1);
                if (b != q_seg) {
                    if (!wait_bar(s, bar(s, B_Q_FULL), qn & 1, p.status)) return false;
                    ++qn;
                    q_seg = b;
                }
                if (us > 0 && !wait_bar(s, bar(s, B_S_EMPTY + j), (us - 1) & 1, p.status)) return false;
                tc_fence_after();
                // S^T = [C | P] . [Q_proj | Q_pe]^T  (K = 576 in 36 steps of 16)
                for (int pr = 0; pr < 4; ++pr) {
                    const int64_t n = 4 * i + pr;
                    const int sl = (int)(n % NP);
                    if (!wait_bar(s, bar(s, B_PAIR_FULL + sl), (uint32_t)(n / NP) & 1, p.status)) return false;
                    tc_fence_after();
                    for (int half = 0; half < 2; ++half)
                        for (int kk = 0; kk < 4; ++kk)
                            umma_bf16(tbase + S_COL + j * NH,
                                      sdesc_sw128(pairs + sl * PAIR_BYTES + half * BOX_BYTES + kk * 32, 16, 1024),
                                      sdesc_sw128(qs + (2 * pr + half) * QBOX_BYTES + kk * 32, 16, 1024), id1,
                                      (pr | half | kk) != 0);
                }
                const int e = (int)(i % NE);
                if (!wait_bar(s, bar(s, B_PE_FULL + e), (uint32_t)(i / NE) & 1, p.status)) return false;
                tc_fence_after();
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16(tbase + S_COL + j * NH, sdesc_sw128(pes + e * BOX_BYTES + kk * 32, 16, 1024),
                              sdesc_sw128(qs + 8 * QBOX_BYTES + kk * 32, 16, 1024), id1, 1);
                umma_commit(bar(s, B_S_FULL + j));
                umma_commit(bar(s, B_PE_EMPTY + e));
                if (t + 1 == t_end || tl + 1 == p.tpb) umma_commit(bar(s, B_Q_EMPTY));
                return true;
            };
            auto gemm2 = [&](int64_t i) -> bool {
                const int j = (int)(i & 1);
                const uint32_t us = (uint32_t)(i >> 1);
                // O^T = C^T . P^T  (M = 512 in 4 blocks of 128, K = 64 tokens in 4 steps)
                if (!wait_bar(s, bar(s, B_P_FULL + j), us & 1, p.status)) return false;
                if (us > 0 && !wait_bar(s, bar(s, B_O_EMPTY + j), (us - 1) & 1, p.status)) return false;
                tc_fence_after();
                for (int mb = 0; mb < 4; ++mb) {
                    const int sl = (int)((4 * i + mb) % NP);
                    for (int ks = 0; ks < TT / 16; ++ks)
                        umma_bf16(tbase + O_COL + j * 4 * NH + mb * NH,
                                  sdesc_sw128(pairs + sl * PAIR_BYTES + ks * 2048, BOX_BYTES, 1024),
                                  sdesc_sw128(ps + j * PBUF_BYTES + (ks >> 2) * (NH * 128) + (ks & 3) * 32, 16, 1024),
                                  id2, ks > 0);
                    umma_commit(bar(s, B_PAIR_EMPTY + sl));
                }
                umma_commit(bar(s, B_O_FULL + j));
                umma_commit(bar(s, B_P_EMPTY + j));
                return true;
            };
            if (warp == 9) {
                for (int64_t i = 0; ok && i < n_tiles; ++i) ok = gemm1(i);
            } else {
                for (int64_t i = 0; ok && i < n_tiles; ++i) ok = gemm2(i);
            }
            // every MMA this thread issued has finished before TMEM is freed
            const uint32_t done = bar(s, warp == 9 ? B_DONE : B_DONE2);
            umma_commit(done);
            mbar_wait_bounded(done, 0, 1000000000ull);
        }
    } else if (warp < 4) {
        // ------------------------------------------------------------- softmax
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        float m_run[NH], l_run[NH];
#pragma unroll
        for (int h = 0; h < NH; ++h) {
            m_run[h] = -INFINITY;
            l_run[h] = 0.f;
        }
        int sn = 0;
        int64_t i = 0;
        int b = (int)(t_begin / (p.tpb > 0 ? p.tpb : 1));
        int tl = (int)(t_begin - (int64_t)b * p.tpb);
        for (int64_t t = t_begin; t < t_end; ++t, ++i) {
            const int j = (int)(i & 1);
            const uint32_t us = (uint32_t)(i >> 1);
            if (!wait_bar(s, bar(s, B_S_FULL + j), us & 1, p.status)) break;
            tc_fence_after();
            float x[NH];
            tmem_ld16(tbase + lane_base + S_COL + j * NH, x);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(s, B_S_EMPTY + j));
            // M=128: tile row r sits in TMEM lane r.  M=64: tile row 16*warp + r
            // sits in lane 32*warp + r (lanes 16-31 of each warp are unused).
            const int k = TT == 128 ? warp * 32 + lane : warp * 16 + (lane & 15);   // token within the tile
            const bool valid = (TT == 128 || lane < 16) && tl * TT + k < p.S;
            float mx[NH];
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                x[h] = valid ? x[h] * p.scale_log2 : -INFINITY;
                mx[h] = x[h];
            }
            warp_allmax16(mx);
            // exchange the four warps' maxima through shared memory; the
            // exchange barrier is an mbarrier so that its wait is bounded too
            float* red = s.red + (int)(i & 1) * 4 * NH;
            if (lane == 0)
#pragma unroll
                for (int h = 0; h < NH; ++h) red[warp * NH + h] = mx[h];
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(s, B_RED + (int)(i & 1)));
            if (!wait_bar(s, bar(s, B_RED + (int)(i & 1)), us & 1, p.status)) break;
            float alpha[NH], pv[NH];
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                const float mt = fmaxf(fmaxf(red[h], red[NH + h]), fmaxf(red[2 * NH + h], red[3 * NH + h]));
                const float mn = fmaxf(m_run[h], mt);
                const float mu = (mn == -INFINITY) ? 0.f : mn;
                alpha[h] = ex2(m_run[h] - mu);
                pv[h] = ex2(x[h] - mu);
                l_run[h] = l_run[h] * alpha[h] + pv[h];
                m_run[h] = mn;
            }
            if (us > 0 && !wait_bar(s, bar(s, B_P_EMPTY + j), (us - 1) & 1, p.status)) break;
            // P^T for the second MMA: K-major (rows = heads, the tile's 64 tokens per 128-B row)
            if (TT == 128 || lane < 16) {
                uint8_t* pb = s.base + OFF_P + j * PBUF_BYTES + (k >> 6) * (NH * 128);
                const int kc = (k & 63) >> 3, ke = (k & 7) * 2;
#pragma unroll
                for (int h = 0; h < NH; ++h)
                    *reinterpret_cast<__nv_bfloat16*>(pb + h * 128 + ((kc ^ (h & 7)) << 4) + ke) =
                        __float2bfloat16_rn(pv[h]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(s, B_P_FULL + j));
            if (warp == 0 && lane == 0) {
#pragma unroll
                for (int h = 0; h < NH; ++h) s.alpha[(i & 3) * NH + h] = alpha[h];
                mbar_arrive(bar(s, B_ALPHA + (int)(i & 3)));
            }
            const bool seg_end = (t + 1 == t_end) || (tl + 1 == p.tpb);
            if (seg_end) {
                float lsum[NH];
#pragma unroll
                for (int h = 0; h < NH; ++h) lsum[h] = l_run[h];
                warp_allsum16(lsum);
                if (lane == 0)
#pragma unroll
                    for (int h = 0; h < NH; ++h) s.lred[warp * NH + h] = lsum[h];
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(s, B_LRED));
                if (!wait_bar(s, bar(s, B_LRED), sn & 1, p.status)) break;
                if (warp == 0 && lane == 0) {
                    if (sn > 0 && !wait_bar(s, bar(s, B_ST_EMPTY), (sn - 1) & 1, p.status)) {
                    } else {
#pragma unroll
                        for (int h = 0; h < NH; ++h) {
                            s.stats[h] = m_run[h];
                            s.stats[NH + h] = s.lred[h] + s.lred[NH + h] + s.lred[2 * NH + h] + s.lred[3 * NH + h];
                        }
                        mbar_arrive(bar(s, B_ST_FULL));
                    }
                }
                ++sn;
#pragma unroll
                for (int h = 0; h < NH; ++h) {
                    m_run[h] = -INFINITY;
                    l_run[h] = 0.f;
                }
            }
            if (++tl == p.tpb) {
                tl = 0;
                ++b;
            }
        }
    } else {
        // ---------------------------------------------------------- correction
        const int q4 = warp - 4;
        const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
        float acc[4][NH];
#pragma unroll
        for (int mb = 0; mb < 4; ++mb)
#pragma unroll
            for (int h = 0; h < NH; ++h) acc[mb][h] = 0.f;
        int sn = 0;
        int64_t i = 0;
        int b = (int)(t_begin / (p.tpb > 0 ? p.tpb : 1));
        int tl = (int)(t_begin - (int64_t)b * p.tpb);
        for (int64_t t = t_begin; t < t_end; ++t, ++i) {
            const int j = (int)(i & 1);
            const uint32_t us = (uint32_t)(i >> 1);
            if (!wait_bar(s, bar(s, B_O_FULL + j), us & 1, p.status)) break;
            tc_fence_after();
            float o[4][NH];
#pragma unroll
            for (int mb = 0; mb < 4; ++mb) tmem_ld16(tbase + lane_base + O_COL + j * 4 * NH + mb * NH, o[mb]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(s, B_O_EMPTY + j));
            if (!wait_bar(s, bar(s, B_ALPHA + (int)(i & 3)), (uint32_t)(i >> 2) & 1, p.status)) break;
            const float* al = s.alpha + (i & 3) * NH;
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                const float a = al[h];
#pragma unroll
                for (int mb = 0; mb < 4; ++mb) acc[mb][h] = fmaf(acc[mb][h], a, o[mb][h]);
            }
            const bool seg_end = (t + 1 == t_end) || (tl + 1 == p.tpb);
            if (seg_end) {
                if (!wait_bar(s, bar(s, B_ST_FULL), sn & 1, p.status)) break;
                float* part = p.ws_part + (int64_t)(cta + b) * SLOT_FLOATS;
#pragma unroll
                for (int h = 0; h < NH; ++h)
#pragma unroll
                    for (int mb = 0; mb < 4; ++mb) part[h * CLR + mb * 128 + q4 * 32 + lane] = acc[mb][h];
                if (q4 == 0 && lane < NH) {
                    part[NH * CLR + lane] = s.stats[lane];
                    part[NH * CLR + NH + lane] = s.stats[NH + lane];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(s, B_ST_EMPTY));
                ++sn;
#pragma unroll
                for (int mb = 0; mb < 4; ++mb)
#pragma unroll
                    for (int h = 0; h < NH; ++h) acc[mb][h] = 0.f;
            }
            if (++tl == p.tpb) {
                tl = 0;
                ++b;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 9) tmem_dealloc(tbase, TMEM_COLS);
}

struct MergeParams {
    int B, S, tpb, nctas;
    const float* ws_part;
    int out_mode;
    void* out;
    float* out_max;
    float* out_sum;
    float* out_lse;
    int early_trigger;   // let the next grid on the stream be scheduled as soon as this one starts
};

__device__ __forceinline__ void write_row_stats(const MergeParams& p, int row, float L, float M) {
    const bool empty = !(L > 0.f);
    const float mnat = empty ? -INFINITY : M * kLn2;
    if (p.out_max) p.out_max[row] = mnat;
    if (p.out_sum) p.out_sum[row] = empty ? 0.f : L;
    if (p.out_lse) p.out_lse[row] = empty ? -INFINITY : mnat + logf(L);
}

// Log-sum-exp merge of a row's pieces.  One warp per (batch, head, 32 latent dims), so the reads spread
// over many SMs: lane k takes piece k's (m, l) and lane d accumulates latent dim d over the pieces.
// Up to 64 pieces are read in one round trip (the common case: a sequence spans ~20 CTAs); more take
// batches of 64.
constexpr int kMlaMergeBatch = 64;
__global__ void __launch_bounds__(256) mla_merge_kernel(const MergeParams p) {
    pdl_wait_primary();
    if (p.early_trigger) pdl_launch_dependents();   // a following decode may start its setup meanwhile
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wid = blockIdx.x * 8 + warp;
    if (wid >= p.B * NH * (CLR / 32)) return;
    const int row = wid / (CLR / 32), chunk = wid - row * (CLR / 32);
    const int b = row / NH, h = row - b * NH;
    int c0 = 0, npc = 0;
    if (p.tpb > 0) {
        const int64_t total = (int64_t)p.B * p.tpb;
        const int64_t t0 = (int64_t)b * p.tpb;
        c0 = (int)split_owner(t0, total, p.nctas);
        npc = (int)split_owner(t0 + p.tpb - 1, total, p.nctas) - c0 + 1;
    }
    const float* base = p.ws_part + (int64_t)(c0 + b) * SLOT_FLOATS;   // piece k at base + k * SLOT_FLOATS
    const int d = chunk * 32 + lane;
    const float* col = base + h * CLR + d;
    // a batch's (m, l) loads are issued together with its values: one round trip per 64 pieces
    float M = -INFINITY, L = 0.f, acc = 0.f;
    for (int k0 = 0; k0 < npc; k0 += kMlaMergeBatch) {
        float v[kMlaMergeBatch], mk[2], lk[2];
#pragma unroll
        for (int u = 0; u < kMlaMergeBatch; ++u)
            v[u] = k0 + u < npc ? __ldg(col + (int64_t)(k0 + u) * SLOT_FLOATS) : 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int k = k0 + lane + 32 * r;
            const float* pp = base + (int64_t)k * SLOT_FLOATS + NH * CLR;
            mk[r] = k < npc ? __ldg(pp + h) : -INFINITY;
            lk[r] = k < npc ? __ldg(pp + NH + h) : 0.f;
        }
        float Mb = fmaxf(mk[0], mk[1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Mb = fmaxf(Mb, __shfl_xor_sync(0xffffffffu, Mb, o));
        const float Mn = fmaxf(M, Mb);
        const float Mu = (Mn == -INFINITY) ? 0.f : Mn;
        const float a = (M == -INFINITY) ? 0.f : ex2(M - Mu);   // rescale of the earlier batches
        float w[2], Lb = 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            w[r] = mk[r] == -INFINITY ? 0.f : ex2(mk[r] - Mu);
            Lb += w[r] * lk[r];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Lb += __shfl_xor_sync(0xffffffffu, Lb, o);
        float ab = 0.f;
#pragma unroll
        for (int u = 0; u < kMlaMergeBatch; ++u) ab = fmaf(__shfl_sync(0xffffffffu, w[u >> 5], u & 31), v[u], ab);
        acc = acc * a + ab;
        L = L * a + Lb;
        M = Mn;
    }
    const bool empty = !(L > 0.f);
    const int64_t oi = (int64_t)row * CLR + d;
    if (p.out_mode == WS_OUT_UNNORM_F32) {
        static_cast<float*>(p.out)[oi] = empty ? 0.f : acc;
    } else {
        const float o = empty ? 0.f : acc / L;
        if (p.out_mode == WS_OUT_NORM_F32) static_cast<float*>(p.out)[oi] = o;
        else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(o);
    }
    if (lane == 0 && chunk == 0) write_row_stats(p, row, L, M);
}

// The up-projection of the absorbed form (system/deepseek.py:405-407): out[b, h, v] = sum_c o_n[b, h, c] *
// w_uv[h][v][c], o_n the merged output rounded to bf16 (as the reference rounds it before its bmm).
// CTA (h, 32 outputs v): the 32 weight rows (32 KB, contiguous) and the B rows o_n[:, h, :] are staged in
// shared memory with every 16-byte load issued at once; thread (b, v) then accumulates in fp32.
// A programmatic dependent launch of the merge.
constexpr int kUpV = 32;
__global__ void __launch_bounds__(256) mla_up_kernel(const __nv_bfloat16* __restrict__ o_n, int B,
                                                     const __nv_bfloat16* __restrict__ w_uv, int64_t w_head_stride,
                                                     int vhd, __nv_bfloat16* __restrict__ out) {
    __shared__ __align__(16) __nv_bfloat16 s_w[kUpV * CLR];   // 32 KB
    __shared__ __align__(16) __nv_bfloat16 s_o[8 * CLR];      // 8 KB: eight batches at a time
    const int h = blockIdx.x, v0 = blockIdx.y * kUpV, tid = threadIdx.x;
    const int nv = min(kUpV, vhd - v0);
    const __nv_bfloat16* wh = w_uv + (size_t)h * w_head_stride + (size_t)v0 * CLR;
    // the weights do not depend on the merge: requested first (asynchronous copies, all in flight)
    for (int i = tid; i < nv * CLR / 8; i += 256) cp_async16(smem_u32(s_w + 8 * i), wh + 8 * i, true);
    pdl_wait_primary();   // o_n is written by the merge
    for (int b0 = 0; b0 < B; b0 += 8) {
        const int nb = min(8, B - b0);
        __syncthreads();
        for (int i = tid; i < nb * CLR / 8; i += 256) {
            const int bb = i / (CLR / 8), q = i - bb * (CLR / 8);
            cp_async16(smem_u32(s_o + bb * CLR + 8 * q), o_n + ((size_t)(b0 + bb) * NH + h) * CLR + 8 * q, true);
        }
        cp_async_wait_all();
        __syncthreads();
        const int bb = tid / kUpV, v = tid - bb * kUpV;   // 8 batches x 32 outputs
        if (bb < nb && v < nv) {
            const __nv_bfloat16* wr = s_w + v * CLR;
            const __nv_bfloat16* orow = s_o + bb * CLR;
            float acc = 0.f;
#pragma unroll 4
            for (int c = 0; c < CLR; c += 8) {
                // rotate the start by v so the 32 threads of a warp read different banks of s_w
                const int cc = (c + v * 8) & (CLR - 1);
                const uint4 w8 = *reinterpret_cast<const uint4*>(wr + cc);
                const uint4 o8 = *reinterpret_cast<const uint4*>(orow + cc);
                const uint32_t ww[4] = {w8.x, w8.y, w8.z, w8.w}, oo[4] = {o8.x, o8.y, o8.z, o8.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    acc = fmaf(__uint_as_float(oo[u] << 16), __uint_as_float(ww[u] << 16), acc);
                    acc = fmaf(__uint_as_float(oo[u] & 0xffff0000u), __uint_as_float(ww[u] & 0xffff0000u), acc);
                }
            }
            out[((size_t)(b0 + bb) * NH + h) * vhd + v0 + v] = __float2bfloat16_rn(acc);
        }
    }
}

// The absorb step of the absorbed form (system/deepseek.py:257-265): q_proj[b, h, :] = q_nope[b, h, :] . w_uk[h]
// (q_nope [B, NH, nop], w_uk[h] [nop, 512] at head stride w_head_stride, both bf16; fp32 accumulation, bf16
// q_proj [B * NH, 512]).  CTA (h, 128 latent columns): the weight block (nop x 128, 16-byte loads all
// issued at once) and eight batches' q rows at a time in shared memory; thread = latent column.
__global__ void __launch_bounds__(128) mla_absorb_kernel(const __nv_bfloat16* __restrict__ q_nope,
                                                         const __nv_bfloat16* __restrict__ w_uk, int64_t w_head_stride,
                                                         int B, int nop, __nv_bfloat16* __restrict__ q_proj) {
    extern __shared__ __align__(16) __nv_bfloat16 s_w[];   // nop rows of 128 columns (<= 64 KB, dynamic)
    __shared__ __align__(16) float s_q[8][256];
    pdl_launch_dependents();   // the decode grid may start streaming the latent cache now
    const int h = blockIdx.x, c0 = blockIdx.y * 128, tid = threadIdx.x;
    const __nv_bfloat16* wb = w_uk + (size_t)h * w_head_stride + c0;
    for (int i = tid; i < nop * 16; i += 128) {   // row k: 16 copies of 8 columns, all in flight
        const int k = i >> 4, q = i & 15;
        cp_async16(smem_u32(s_w + k * 128 + 8 * q), wb + (size_t)k * CLR + 8 * q, true);
    }
    cp_async_wait_all();
    for (int b0 = 0; b0 < B; b0 += 8) {
        const int nb = min(8, B - b0);
        __syncthreads();
        float qv[16];   // every load issued before the first store (nb * nop <= 2048)
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int i = tid + r * 128, bb = i / nop, k = i - bb * nop;
            qv[r] = i < nb * nop ? __bfloat162float(q_nope[((size_t)(b0 + bb) * NH + h) * nop + k]) : 0.f;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int i = tid + r * 128, bb = i / nop, k = i - bb * nop;
            if (i < nb * nop) s_q[bb][k] = qv[r];
        }
        __syncthreads();
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
        for (int k = 0; k < nop; k += 4) {   // four k per step: the loads of a step are independent
            float w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) w[u] = __bfloat162float(s_w[(k + u) * 128 + tid]);
#pragma unroll
            for (int bb = 0; bb < 8; ++bb) {
                const float4 q4 = *reinterpret_cast<const float4*>(&s_q[bb][k]);
                acc[bb] = fmaf(q4.x, w[0], acc[bb]);
                acc[bb] = fmaf(q4.y, w[1], acc[bb]);
                acc[bb] = fmaf(q4.z, w[2], acc[bb]);
                acc[bb] = fmaf(q4.w, w[3], acc[bb]);
            }
        }
        for (int bb = 0; bb < nb; ++bb)
            q_proj[((size_t)(b0 + bb) * NH + h) * CLR + c0 + tid] = __float2bfloat16_rn(acc[bb]);
    }
}

}  // namespace mla

size_t mla_workspace_bytes(int B, int nH, int S) {
    (void)S;
    const int nsm = device_sm_count();
    const int hg = std::max(1, (nH + mla::NH - 1) / mla::NH);   // query sequences per latent sequence
    return kCounterHeaderBytes + size_t(nsm + (size_t)B * hg) * mla::SLOT_FLOATS * 4;
}

int mla_launch(const void* q_proj, const void* q_pe, const void* c_kv, const void* k_pe, int B, int nH, int S,
               float scale, int out_mode, void* out, float* out_max, float* out_sum, float* out_lse, void* workspace,
               size_t workspace_bytes, cudaStream_t st, bool after_primary, bool kv_after_primary,
               int64_t c_bstride, int64_t pe_bstride) {
    using namespace mla;
    // nH = hg * 16 heads per sequence run as hg query sequences of 16 heads that read the same latent
    // sequence (query rows b*nH + h are already laid out that way: query sequence b*hg + h/16)
    if (nH < NH || nH % NH) return set_error(WS_ERR_UNSUPPORTED, "mla_decode: heads per sequence must be a multiple of 16");
    if (B < 0 || S < 0) return set_error(WS_ERR_INVALID_ARG, "mla_decode: bad shape");
    if (B == 0) return WS_OK;
    const int hg = nH / NH;
    if (c_bstride < 0) c_bstride = (int64_t)S * CLR;
    if (pe_bstride < 0) pe_bstride = (int64_t)S * QRD;
    if (c_bstride < (int64_t)S * CLR || pe_bstride < (int64_t)S * QRD || c_bstride % 8 || pe_bstride % 8)
        return set_error(WS_ERR_INVALID_ARG, "mla_decode: batch strides must cover S tokens and be 16-byte multiples");
    const int BL = B;   // latent sequences
    B *= hg;            // query sequences from here on
    const int tpb = (S + TT - 1) / TT;
    const int64_t total = (int64_t)B * tpb;
    const int nsm = device_sm_count();
    const int nctas = (int)std::max<int64_t>(1, std::min<int64_t>(nsm, total));
    const size_t need = kCounterHeaderBytes + size_t(nctas + B) * SLOT_FLOATS * 4;
    if (workspace_bytes < need || !workspace)
        return set_error(WS_ERR_WORKSPACE, "mla_decode: workspace too small (see ws_mla_decode_workspace_size)");
    if (reinterpret_cast<uintptr_t>(workspace) % 16)
        return set_error(WS_ERR_WORKSPACE, "mla_decode: workspace must be 16-byte aligned");
    float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterHeaderBytes);
    if (total > 0) {
        Maps maps;
        memset(&maps, 0, sizeof(maps));
        int fc = 0, fpe = 0, fq = 0, rc;
        if ((rc = make_kv_map(&maps.c, c_kv, CLR, c_bstride, CLR, S, BL, TT, &fc)) != WS_OK) return rc;
        if ((rc = make_kv_map(&maps.pe, k_pe, QRD, pe_bstride, QRD, S, BL, TT, &fpe)) != WS_OK) return rc;
        if ((rc = make_kv_map(&maps.q, q_proj, CLR, (int64_t)B * NH * CLR, CLR, (int64_t)B * NH, 1, NH, &fq)) != WS_OK)
            return rc;
        if (fq) return set_error(WS_ERR_INVALID_ARG, "mla_decode: unexpected query layout");
        if ((rc = make_kv_map(&maps.qpe, q_pe, QRD, (int64_t)B * NH * QRD, QRD, (int64_t)B * NH, 1, NH, &fq)) != WS_OK)
            return rc;
        if (fq) return set_error(WS_ERR_INVALID_ARG, "mla_decode: unexpected query layout");
        Params prm;
        prm.c_tok_in_dim2 = fc;
        prm.pe_tok_in_dim2 = fpe;
        prm.B = B;
        prm.hg = hg;
        prm.S = S;
        prm.tpb = tpb;
        prm.scale_log2 = scale * kLog2e;
        prm.ws_part = part;
        prm.kv_after_primary = after_primary && kv_after_primary;
        prm.status = device_status_word();
        static int configured_dev = -1;
        int dev = 0;
        cudaGetDevice(&dev);
        if (configured_dev != dev) {
            if (cudaFuncSetAttribute(mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)SMEM_BYTES) != cudaSuccess)
                return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for mla_decode_kernel");
            configured_dev = dev;
        }
        cudaLaunchConfig_t dcfg = {};
        dcfg.gridDim = dim3((unsigned)nctas);
        dcfg.blockDim = dim3(kThreads);
        dcfg.dynamicSmemBytes = SMEM_BYTES;
        dcfg.stream = st;
        cudaLaunchAttribute dattr[1];
        dattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        dattr[0].val.programmaticStreamSerializationAllowed = 1;
        dcfg.attrs = dattr;
        dcfg.numAttrs = after_primary ? 1 : 0;
        cudaError_t e = cudaLaunchKernelEx(&dcfg, mla_decode_kernel, maps, prm);
        if (e != cudaSuccess) return set_error(WS_ERR_CUDA, cudaGetErrorString(e));
    }
    MergeParams mp;
    mp.B = B;
    mp.S = S;
    mp.tpb = tpb;
    mp.nctas = nctas;
    mp.ws_part = part;
    mp.out_mode = out_mode;
    mp.out = out;
    mp.out_max = out_max;
    mp.out_sum = out_sum;
    mp.out_lse = out_lse;
    // plain decode steps: the next step's decode (a programmatic dependent) overlaps this merge with its
    // setup.  Not after the absorb path's decode: there the up-projection follows, and letting it start
    // early measured slower (58 against 51 us per absorbed step)
    mp.early_trigger = kv_after_primary ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((B * NH * (CLR / 32) + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = total > 0 ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, mla_merge_kernel, mp);
    if (e != cudaSuccess) return set_error(WS_ERR_CUDA, cudaGetErrorString(e));
    return WS_OK;
}

size_t mla_absorbed_workspace_bytes(int B, int nH, int S) {
    // the decode's own part, then q_proj and o_n (bf16 [B * 16, 512] each)
    return align_up(mla_workspace_bytes(B, nH, S), 256) + 2 * align_up((size_t)std::max(B, 1) * mla::NH * mla::CLR * 2, 256);
}

int mla_absorbed_launch(const void* q_nope, const void* w_uk, int64_t w_uk_head_stride, const void* q_pe,
                        const void* c_kv, const void* k_pe, const void* w_uv, int64_t w_uv_head_stride, int B, int nH,
                        int S, int nop, int vhd, float scale, void* out, float* out_lse, void* workspace,
                        size_t workspace_bytes, cudaStream_t st, int64_t c_bstride, int64_t pe_bstride) {
    using namespace mla;
    if (nH != NH) return set_error(WS_ERR_UNSUPPORTED, "mla_decode_absorbed: this build supports 16 heads per sequence");
    if (B < 0 || S < 0 || nop < 4 || nop > 256 || nop % 4 || vhd < 1 || w_uk_head_stride < (int64_t)nop * CLR ||
        w_uv_head_stride < (int64_t)vhd * CLR)
        return set_error(WS_ERR_INVALID_ARG, "mla_decode_absorbed: bad shape or head stride");
    if (B == 0) return WS_OK;
    if (!workspace || workspace_bytes < mla_absorbed_workspace_bytes(B, nH, S))
        return set_error(WS_ERR_WORKSPACE, "mla_decode_absorbed: workspace too small (see ws_mla_decode_absorbed_workspace_size)");
    if (reinterpret_cast<uintptr_t>(workspace) % 16)
        return set_error(WS_ERR_WORKSPACE, "mla_decode_absorbed: workspace must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(w_uk) % 16 || reinterpret_cast<uintptr_t>(w_uv) % 16 || w_uk_head_stride % 8 ||
        w_uv_head_stride % 8)
        return set_error(WS_ERR_INVALID_ARG, "mla_decode_absorbed: weights and head strides must be 16-byte aligned");
    const size_t dec = align_up(mla_workspace_bytes(B, nH, S), 256);
    const size_t rowbuf = align_up((size_t)B * NH * CLR * 2, 256);
    __nv_bfloat16* q_proj = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + dec);
    __nv_bfloat16* o_n = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + dec + rowbuf);
    const int smem = nop * 128 * 2;
    static int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(mla_absorb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 256 * 128 * 2) !=
            cudaSuccess)
            return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for mla_absorb_kernel");
        configured_dev = dev;
    }
    mla_absorb_kernel<<<dim3(NH, CLR / 128), 128, smem, st>>>(static_cast<const __nv_bfloat16*>(q_nope),
                                                              static_cast<const __nv_bfloat16*>(w_uk), w_uk_head_stride,
                                                              B, nop, q_proj);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(WS_ERR_CUDA, cudaGetErrorString(e));
    int rc = mla_launch(q_proj, q_pe, c_kv, k_pe, B, nH, S, scale, WS_OUT_NORM_BF16, o_n, nullptr, nullptr, out_lse,
                        workspace, dec, st, /*after_primary=*/true, /*kv_after_primary=*/false, c_bstride, pe_bstride);
    if (rc != WS_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(NH, (unsigned)((vhd + kUpV - 1) / kUpV));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, mla_up_kernel, static_cast<const __nv_bfloat16*>(o_n), B,
                           static_cast<const __nv_bfloat16*>(w_uv), w_uv_head_stride, vhd,
                           static_cast<__nv_bfloat16*>(out));
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace ws
