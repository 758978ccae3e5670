// fp32 GQA decode on the CUDA cores.
//
// The fp32 branch of fused_cpu_attn (kernel/cpu_attn.cpp:620-629, run_kernel
// <false,false>) and the scalar ablation fused_cpu_attn_fp32
// (kernel/cpu_attn.cpp:674-848).  fp32 operands are kept in fp32 end to end
// (tf32 tensor cores would not meet the 1e-3 LSE bar), on the CUDA cores.
//
// Grid (B_kv, splits).  Each block takes a contiguous token range of one row.
// When every K and V row is 16-byte aligned, tiles of TT tokens are staged in
// shared memory by 16-byte cp.async copies through a 3-stage ring:
//   * gqa_f32_rb_kernel (G <= 8, D <= 128) reads every K and V element of a
//     tile from shared memory once: scores with lane = (token, float4 chunk)
//     over all heads and a 3-shuffle sum, the online softmax with warp = head,
//     P.V with lane = 4 value dims of every head over a share of the tokens;
//   * gqa_f32_tile_kernel (other sizes): scores with thread = (token, heads),
//     P.V with thread = (head, 4 value dims).
// Otherwise gqa_f32_kernel: 4 warps interleave tokens, lanes own head dims,
// and the warps' states are merged in shared memory.  When a row has several
// splits the block that files the last split (atomic ticket) merges them.
#include "common.cuh"
#include "ws_internal.h"

namespace ws {

constexpr int kF32MaxG = 16;
constexpr int kF32MaxDPerLane = 8;   // D <= 256

struct F32Params {
    const float* q;
    const float* k;
    const float* v;
    int64_t k_sb, k_st, v_sb, v_st;
    int G, D, L, splits;
    int GR;          // query heads per kv row in q and the outputs (this launch takes G of them, G <= GR)
    float scale;
    int out_mode;
    void* out;
    void* out_max;
    void* out_sum;
    float* out_lse;
    float* ws_part;
    int* ws_cnt;
};

__device__ __forceinline__ void f32_store(const F32Params& p, int row, int g, int d, float o_un, float m, float l) {
    const bool empty = !(l > 0.f);
    const int64_t oi = ((int64_t)row * p.GR + g) * p.D + d;
    float* out = static_cast<float*>(p.out);
    out[oi] = empty ? 0.f : (p.out_mode == WS_OUT_UNNORM_F32 ? o_un : o_un / l);
    if (d == 0) {
        const int64_t mi = (int64_t)row * p.GR + g;
        if (p.out_max) {
            static_cast<float*>(p.out_max)[mi] = empty ? -INFINITY : m;
            static_cast<float*>(p.out_sum)[mi] = empty ? 0.f : l;
        }
        if (p.out_lse) p.out_lse[mi] = empty ? -INFINITY : m + logf(l);
    }
}

template <int DPL>
__global__ void __launch_bounds__(128) gqa_f32_kernel(const F32Params p) {
    __shared__ float s_m[4][kF32MaxG], s_l[4][kF32MaxG];
    __shared__ int s_last;
    extern __shared__ float s_o[];   // [4][G][D]
    const int row = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = (p.L + p.splits - 1) / p.splits;
    const int t0 = split * per, t1 = min(p.L, t0 + per);

    float qr[kF32MaxG][DPL], o[kF32MaxG][DPL], m[kF32MaxG], l[kF32MaxG];
#pragma unroll
    for (int g = 0; g < kF32MaxG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            qr[g][i] = (g < p.G && d < p.D) ? p.q[((int64_t)row * p.GR + g) * p.D + d] : 0.f;
            o[g][i] = 0.f;
        }
    }
    for (int t = t0 + warp; t < t1; t += 4) {
        const float* kr = p.k + (int64_t)row * p.k_sb + (int64_t)t * p.k_st;
        const float* vr = p.v + (int64_t)row * p.v_sb + (int64_t)t * p.v_st;
        float kx[DPL], vx[DPL];
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            kx[i] = d < p.D ? __ldg(kr + d) : 0.f;
            vx[i] = d < p.D ? __ldg(vr + d) : 0.f;
        }
#pragma unroll
        for (int g = 0; g < kF32MaxG; ++g) {
            if (g >= p.G) break;
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < DPL; ++i) s = fmaf(qr[g][i], kx[i], s);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            s *= p.scale;
            const float nm = fmaxf(m[g], s);
            const float eo = ex2((m[g] - nm) * kLog2e), en = ex2((s - nm) * kLog2e);
            l[g] = eo * l[g] + en;
            m[g] = nm;
#pragma unroll
            for (int i = 0; i < DPL; ++i) o[g][i] = fmaf(eo, o[g][i], en * vx[i]);
        }
    }
    // merge the 4 warps
#pragma unroll
    for (int g = 0; g < kF32MaxG; ++g) {
        if (g >= p.G) break;
        if (lane == 0) {
            s_m[warp][g] = m[g];
            s_l[warp][g] = l[g];
        }
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            if (d < p.D) s_o[(warp * p.G + g) * p.D + d] = o[g][i];
        }
    }
    __syncthreads();
    const int slot_floats = p.G * p.D + 2 * p.G;
    float* part = p.ws_part + ((int64_t)row * p.splits + split) * slot_floats;
    for (int e = threadIdx.x; e < p.G * p.D; e += blockDim.x) {
        const int g = e / p.D, d = e - g * p.D;
        float M = -INFINITY;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][g]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float acc = 0.f, L = 0.f;
        for (int w = 0; w < 4; ++w) {
            const float wt = ex2((s_m[w][g] - Mu) * kLog2e);
            acc += wt * s_o[(w * p.G + g) * p.D + d];
            L += wt * s_l[w][g];
        }
        if (p.splits == 1) {
            f32_store(p, row, g, d, acc, M, L);
        } else {
            part[g * p.D + d] = acc;
            if (d == 0) {
                part[p.G * p.D + g] = M;
                part[p.G * p.D + p.G + g] = L;
            }
        }
    }
    if (p.splits == 1) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(p.ws_cnt + row, 1) == p.splits - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int e = threadIdx.x; e < p.G * p.D; e += blockDim.x) {
        const int g = e / p.D, d = e - g * p.D;
        float M = -INFINITY;
        for (int s = 0; s < p.splits; ++s)
            M = fmaxf(M, __ldcg(p.ws_part + ((int64_t)row * p.splits + s) * slot_floats + p.G * p.D + g));
        const float Mu = M == -INFINITY ? 0.f : M;
        float acc = 0.f, L = 0.f;
        for (int s = 0; s < p.splits; ++s) {
            const float* pp = p.ws_part + ((int64_t)row * p.splits + s) * slot_floats;
            const float wt = ex2((__ldcg(pp + p.G * p.D + g) - Mu) * kLog2e);
            acc += wt * __ldcg(pp + g * p.D + d);
            L += wt * __ldcg(pp + p.G * p.D + p.G + g);
        }
        f32_store(p, row, g, d, acc, M, L);
    }
    if (threadIdx.x == 0) p.ws_cnt[row] = 0;
}

// ------------------------------------------------------------------ tiled forms
// TT tokens x DMAX dims per operand and stage (TT * DMAX = 4096 floats): TT = 32 for D <= 128, 16 for D <= 256.
constexpr int kF32Threads = 256;
constexpr int kF32Stages = 3;
constexpr int kF32RbHeads = 8;   // heads of the register-blocked form

template <int DMAX>
struct F32Tile {
    static constexpr int TT = 4096 / DMAX;
    static constexpr int KS = DMAX + 4;   // K row stride: consecutive lanes' rows start on distinct bank groups
    static constexpr int STAGE_FLOATS = TT * KS + TT * DMAX;
    // the ring, then q [G][D], scores / probabilities [G][TT], the heads' alpha, max and sum
    static size_t smem(int G, int D) {
        return size_t(kF32Stages) * STAGE_FLOATS * 4 + size_t(G) * D * 4 + size_t(G) * TT * 4 + 3 * kF32MaxG * 4 + 16;
    }
};

// register-blocked form: the ring, q [G][D], scores [8][TT], probabilities [TT][8], alpha, max, sum
inline size_t f32_rb_smem(int G, int D) {
    using T = F32Tile<128>;
    return size_t(kF32Stages) * T::STAGE_FLOATS * 4 + size_t(G) * D * 4 +
           size_t(2 * kF32RbHeads * T::TT + 3 * kF32RbHeads) * 4 + 16;
}

// Tile of TT tokens starting at tb into a ring stage: 16-byte cp.async copies spread over the threads (K rows at
// stride KS, V rows at stride VS), one commit group per tile; rows at or past the split's end t1 are zero-filled
// and never read from global memory.  Called by every thread.
template <int TT, int KS, int VS>
__device__ __forceinline__ void f32_issue_tile(const F32Params& p, float* ks, float* vs, const float* kbase,
                                               const float* vbase, int tb, int t1, int tid) {
    const int D4 = p.D / 4;
    for (int c = tid; c < TT * D4; c += kF32Threads) {
        const int r = c / D4, d = (c - r * D4) * 4;
        const bool ok = tb + r < t1;
        const int64_t tok = ok ? tb + r : 0;   // not read when !ok
        cp_async16(smem_u32(ks + r * KS + d), kbase + tok * p.k_st + d, ok);
        cp_async16(smem_u32(vs + r * VS + d), vbase + tok * p.v_st + d, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits until tile i (of `issued` tiles whose copies were committed) has landed for every thread.
__device__ __forceinline__ void f32_wait_tile(int i, int issued) {
    static_assert(kF32Stages == 3, "at most two tiles in flight");
    if (issued - i - 1 >= 1) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();   // tile i landed; tile i - 1's stage and probabilities are free
}

// The CTA's result: o(g, d) un-normalised against the running max mx2[g] (log2 units) with sum l[g]; written as
// the output when the row has one split, else as this split's piece, and the split that files the last piece
// merges the row's pieces.
template <typename OF>
__device__ __forceinline__ void f32_finish(const F32Params& p, int row, int split, int tid, const float* mx2,
                                           const float* lsum, OF o_of) {
    __shared__ int s_last;
    const int G = p.G, D = p.D;
    const int slot_floats = G * D + 2 * G;
    float* part = p.ws_part + ((int64_t)row * p.splits + split) * slot_floats;
    for (int e = tid; e < G * D; e += kF32Threads) {
        const int g = e / D, d = e - g * D;
        const float M = mx2[g] == -INFINITY ? -INFINITY : mx2[g] * kLn2, L = lsum[g];
        const float acc = o_of(g, d);
        if (p.splits == 1) {
            f32_store(p, row, g, d, acc, M, L);
        } else {
            part[g * D + d] = acc;
            if (d == 0) {
                part[G * D + g] = M;
                part[G * D + G + g] = L;
            }
        }
    }
    if (p.splits == 1) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(p.ws_cnt + row, 1) == p.splits - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int e = tid; e < G * D; e += kF32Threads) {
        const int g = e / D, d = e - g * D;
        float M = -INFINITY;
        for (int sp = 0; sp < p.splits; ++sp)
            M = fmaxf(M, __ldcg(p.ws_part + ((int64_t)row * p.splits + sp) * slot_floats + G * D + g));
        const float Mu = M == -INFINITY ? 0.f : M;
        float acc = 0.f, L = 0.f;
        for (int sp = 0; sp < p.splits; ++sp) {
            const float* pp = p.ws_part + ((int64_t)row * p.splits + sp) * slot_floats;
            const float wt = ex2((__ldcg(pp + G * D + g) - Mu) * kLog2e);
            acc += wt * __ldcg(pp + g * D + d);
            L += wt * __ldcg(pp + G * D + G + g);
        }
        f32_store(p, row, g, d, acc, M, L);
    }
    if (tid == 0) p.ws_cnt[row] = 0;
}

// One head of the online softmax over a tile, warp = head, lane = token (TT <= 32): x is this lane's score in
// log2 units (-inf past the tile's valid tokens).  Returns the lane's probability; lane 0 updates the head's
// running max and sum and publishes the rescale factor.
__device__ __forceinline__ float f32_softmax_head(float x, int lane, float* alpha, float* mx2, float* lsum) {
    float mx = x;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_old = *mx2;
    const float m_new = fmaxf(m_old, mx);
    const float mu = m_new == -INFINITY ? 0.f : m_new;
    const float pe = ex2(x - mu);
    float sum = pe;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float a = ex2(m_old - mu);
    __syncwarp();
    if (lane == 0) {
        *alpha = a;
        *mx2 = m_new;
        *lsum = *lsum * a + sum;
    }
    return pe;
}

// Register-blocked form for G <= 8 and D <= 128 (tiles of F32Tile<128>): every K and V element of a tile is read
// from shared memory once, where the head-per-thread form reads it once per head.
//   scores:  warp w takes tokens 4w .. 4w+3; lane l (token 4w + l/8, chunk l%8) accumulates every head over the
//            float4 columns chunk, chunk + 8, ... of its token's K row, the 8 lanes of a token add their sums
//            with three shuffles, and lane c keeps head c;
//   softmax: warp = head, lane = token; probabilities stored token-major;
//   P.V:     warp w takes tokens w, w + 8, w + 16, w + 24 of every tile, lane c owns value dims 4c .. 4c+3 of
//            every head; the eight warps' partial outputs are added once, after the last tile.
__global__ void __launch_bounds__(kF32Threads, 2) gqa_f32_rb_kernel(const F32Params p) {
    using T = F32Tile<128>;
    constexpr int TT = T::TT, KS = T::KS, GB = kF32RbHeads;
    static_assert(TT == 32 && kF32Threads == 256, "lane = token in the softmax, 8 warps x 4 tokens");
    extern __shared__ float4 smem4[];
    float* sm = reinterpret_cast<float*>(smem4);
    float* s_q = sm + kF32Stages * T::STAGE_FLOATS;   // [G][D]
    float* s_s = s_q + p.G * p.D;                     // [GB][TT] scores (log2 units)
    float* s_pt = s_s + GB * TT;                      // [TT][GB] probabilities, token-major
    float* s_alpha = s_pt + TT * GB;                  // [GB]
    float* s_mx = s_alpha + GB;                       // [GB] running max (log2 units)
    float* s_sum = s_mx + GB;                         // [GB] running sum
    const int row = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int per = (p.L + p.splits - 1) / p.splits;
    const int t0 = min(p.L, split * per), t1 = min(p.L, t0 + per);
    const int ntiles = (t1 - t0 + TT - 1) / TT;
    const int D = p.D, D4 = p.D / 4, G = p.G;
    const float sl2 = p.scale * kLog2e;
    const float* kbase = p.k + (int64_t)row * p.k_sb;
    const float* vbase = p.v + (int64_t)row * p.v_sb;
    auto load_tile = [&](int i) {
        float* ks = sm + (i % kF32Stages) * T::STAGE_FLOATS;
        f32_issue_tile<TT, KS, 128>(p, ks, ks + TT * KS, kbase, vbase, t0 + i * TT, t1, tid);
    };
    int issued = min(ntiles, kF32Stages - 1);
    for (int i = 0; i < issued; ++i) load_tile(i);
    for (int e = tid; e < G * D; e += kF32Threads) s_q[e] = p.q[(int64_t)row * p.GR * D + e];
    for (int e = tid; e < TT * GB; e += kF32Threads) s_pt[e] = 0.f;   // heads >= G stay 0
    if (tid < GB) {
        s_alpha[tid] = 0.f;
        s_mx[tid] = -INFINITY;
        s_sum[tid] = 0.f;
    }

    float4 o[GB];
#pragma unroll
    for (int h = 0; h < GB; ++h) o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int tq = warp * 4 + (lane >> 3), ch = lane & 7;   // score step: token, float4 chunk
    for (int i = 0; i < ntiles; ++i) {
        f32_wait_tile(i, issued);
        if (issued < ntiles) load_tile(issued++);
        const float* ks = sm + (i % kF32Stages) * T::STAGE_FLOATS;
        const float* vs = ks + TT * KS;
        const int nvalid = min(TT, t1 - (t0 + i * TT));
        {
            float acc[GB];
#pragma unroll
            for (int h = 0; h < GB; ++h) acc[h] = 0.f;
            const float* kr = ks + tq * KS;
            for (int f = ch; f < D4; f += 8) {
                const float4 kv = *reinterpret_cast<const float4*>(kr + 4 * f);
#pragma unroll
                for (int h = 0; h < GB; ++h) {
                    if (h < G) {
                        const float4 qv = *reinterpret_cast<const float4*>(s_q + h * D + 4 * f);
                        acc[h] = fmaf(qv.x, kv.x, acc[h]);
                        acc[h] = fmaf(qv.y, kv.y, acc[h]);
                        acc[h] = fmaf(qv.z, kv.z, acc[h]);
                        acc[h] = fmaf(qv.w, kv.w, acc[h]);
                    }
                }
            }
            float mine = 0.f;
#pragma unroll
            for (int h = 0; h < GB; ++h) {
                acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
                acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
                acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 4);
                if (ch == h) mine = acc[h];
            }
            if (ch < G) s_s[ch * TT + tq] = tq < nvalid ? mine * sl2 : -INFINITY;
        }
        __syncthreads();
        if (warp < G) s_pt[lane * GB + warp] = f32_softmax_head(s_s[warp * TT + lane], lane, s_alpha + warp,
                                                                s_mx + warp, s_sum + warp);
        __syncthreads();
        if (lane < D4) {   // P . V: tokens warp, warp + 8, ..., value dims 4 lane .. 4 lane + 3, every head
            const float4 a0 = *reinterpret_cast<const float4*>(s_alpha);
            const float4 a1 = *reinterpret_cast<const float4*>(s_alpha + 4);
            const float al[GB] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
            for (int h = 0; h < GB; ++h) {
                o[h].x *= al[h]; o[h].y *= al[h]; o[h].z *= al[h]; o[h].w *= al[h];
            }
#pragma unroll
            for (int u = 0; u < TT / 8; ++u) {
                const int t = warp + 8 * u;
                const float4 vv = *reinterpret_cast<const float4*>(vs + t * 128 + 4 * lane);
                const float4 p0 = *reinterpret_cast<const float4*>(s_pt + t * GB);
                const float4 p1 = *reinterpret_cast<const float4*>(s_pt + t * GB + 4);
                const float pt[GB] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                for (int h = 0; h < GB; ++h) {
                    o[h].x = fmaf(pt[h], vv.x, o[h].x);
                    o[h].y = fmaf(pt[h], vv.y, o[h].y);
                    o[h].z = fmaf(pt[h], vv.z, o[h].z);
                    o[h].w = fmaf(pt[h], vv.w, o[h].w);
                }
            }
        }
    }
    __syncthreads();
    // the eight warps' partial outputs, added in the (now idle) ring: red[warp][head][128]
    float* red = sm;
    if (lane < D4)
#pragma unroll
        for (int h = 0; h < GB; ++h)
            if (h < G) *reinterpret_cast<float4*>(red + (warp * GB + h) * 128 + 4 * lane) = o[h];
    __syncthreads();
    f32_finish(p, row, split, tid, s_mx, s_sum, [&](int g, int d) {
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) acc += red[(w * GB + g) * 128 + d];
        return acc;
    });
}

// Head-per-thread form (any G <= 16, D <= DMAX): scores with thread = (token tq, heads gq, gq + NGQ, ...), the
// online softmax with warp = head, P.V with thread = (head, 4 value dims).
template <int DMAX>
__global__ void __launch_bounds__(kF32Threads, 2) gqa_f32_tile_kernel(const F32Params p) {
    using T = F32Tile<DMAX>;
    constexpr int TT = T::TT, KS = T::KS;
    constexpr int NGQ = kF32Threads / TT;                     // head groups of the score step
    constexpr int HPT = (kF32MaxG + NGQ - 1) / NGQ;           // heads per thread in the score step
    constexpr int NPT = kF32MaxG * (DMAX / 4) / kF32Threads;  // (head, 4 dims) outputs per thread, at most
    extern __shared__ float4 smem4[];
    float* sm = reinterpret_cast<float*>(smem4);
    float* s_q = sm + kF32Stages * T::STAGE_FLOATS;           // [G][D]
    float* s_p = s_q + p.G * p.D;                             // [G][TT] scores, then probabilities
    float* s_alpha = s_p + p.G * TT;                          // [kF32MaxG]
    float* s_mx = s_alpha + kF32MaxG;                         // [kF32MaxG] running max (log2 units)
    float* s_sum = s_mx + kF32MaxG;                           // [kF32MaxG] running sum
    const int row = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int per = (p.L + p.splits - 1) / p.splits;
    const int t0 = min(p.L, split * per), t1 = min(p.L, t0 + per);
    const int ntiles = (t1 - t0 + TT - 1) / TT;
    const int D = p.D, D4 = p.D / 4;
    const float sl2 = p.scale * kLog2e;
    const float* kbase = p.k + (int64_t)row * p.k_sb;
    const float* vbase = p.v + (int64_t)row * p.v_sb;
    auto load_tile = [&](int i) {
        float* ks = sm + (i % kF32Stages) * T::STAGE_FLOATS;
        f32_issue_tile<TT, KS, DMAX>(p, ks, ks + TT * KS, kbase, vbase, t0 + i * TT, t1, tid);
    };
    int issued = min(ntiles, kF32Stages - 1);
    for (int i = 0; i < issued; ++i) load_tile(i);
    for (int e = tid; e < p.G * D; e += kF32Threads) s_q[e] = p.q[(int64_t)row * p.GR * D + e];
    if (tid < kF32MaxG) {
        s_alpha[tid] = 0.f;
        s_mx[tid] = -INFINITY;
        s_sum[tid] = 0.f;
    }

    float4 o[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int tq = tid % TT, gq = tid / TT;   // score step: token, first head
    for (int i = 0; i < ntiles; ++i) {
        f32_wait_tile(i, issued);
        if (issued < ntiles) load_tile(issued++);
        const float* ks = sm + (i % kF32Stages) * T::STAGE_FLOATS;
        const float* vs = ks + TT * KS;
        const int nvalid = min(TT, t1 - (t0 + i * TT));
        {
            float acc[HPT];
#pragma unroll
            for (int h = 0; h < HPT; ++h) acc[h] = 0.f;
            const float4* kr = reinterpret_cast<const float4*>(ks + tq * KS);
            for (int d4 = 0; d4 < D4; ++d4) {
                const float4 kv = kr[d4];
#pragma unroll
                for (int h = 0; h < HPT; ++h) {
                    const int g = gq + h * NGQ;
                    if (g < p.G) {
                        const float4 qv = reinterpret_cast<const float4*>(s_q + g * D)[d4];
                        acc[h] = fmaf(qv.x, kv.x, acc[h]);
                        acc[h] = fmaf(qv.y, kv.y, acc[h]);
                        acc[h] = fmaf(qv.z, kv.z, acc[h]);
                        acc[h] = fmaf(qv.w, kv.w, acc[h]);
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < HPT; ++h) {
                const int g = gq + h * NGQ;
                if (g < p.G) s_p[g * TT + tq] = tq < nvalid ? acc[h] * sl2 : -INFINITY;
            }
        }
        __syncthreads();
        for (int g = warp; g < p.G; g += kF32Threads / 32) {   // online softmax: warp = head, lane = token
            const float pe = f32_softmax_head(lane < TT ? s_p[g * TT + lane] : -INFINITY, lane, s_alpha + g,
                                              s_mx + g, s_sum + g);
            if (lane < TT) s_p[g * TT + lane] = pe;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < NPT; ++j) {   // P . V: thread = (head, 4 value dims)
            const int e = tid + j * kF32Threads, g = e / D4, c = e - g * D4;
            if (g < p.G) {
                const float a = s_alpha[g];
                float4 acc = make_float4(o[j].x * a, o[j].y * a, o[j].z * a, o[j].w * a);
                const float* pr = s_p + g * TT;
                const float4* vc = reinterpret_cast<const float4*>(vs) + c;
#pragma unroll 8
                for (int t = 0; t < TT; ++t) {
                    const float pt = pr[t];
                    const float4 vv = vc[t * (DMAX / 4)];
                    acc.x = fmaf(pt, vv.x, acc.x);
                    acc.y = fmaf(pt, vv.y, acc.y);
                    acc.z = fmaf(pt, vv.z, acc.z);
                    acc.w = fmaf(pt, vv.w, acc.w);
                }
                o[j] = acc;
            }
        }
    }
    __syncthreads();
    // each (head, 4 dims) output lives in one thread's registers: stage them in the (now idle) ring
    float* red = sm;
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int e = tid + j * kF32Threads, g = e / D4, c = e - g * D4;
        if (g < p.G) *reinterpret_cast<float4*>(red + g * D + 4 * c) = o[j];
    }
    __syncthreads();
    f32_finish(p, row, split, tid, s_mx, s_sum, [&](int g, int d) { return red[g * D + d]; });
}

static int gqa_f32_heads(const void* q, const void* k, const void* v, int64_t k_sb, int64_t k_st, int64_t v_sb,
                         int64_t v_st, int B_kv, int G, int GR, int g0, int D, int L, float scale, int out_mode,
                         void* out, void* out_max, void* out_sum, float* out_lse, void* workspace,
                         size_t workspace_bytes, cudaStream_t st);

int gqa_f32_launch(const void* q, const void* k, const void* v, int64_t k_sb, int64_t k_st, int64_t v_sb,
                      int64_t v_st, int B_kv, int G, int D, int L, float scale, int out_mode, void* out,
                      void* out_max, void* out_sum, float* out_lse, void* workspace, size_t workspace_bytes,
                      cudaStream_t st) {
    if (D > 32 * kF32MaxDPerLane) return set_error(WS_ERR_UNSUPPORTED, "fp32 path: head_dim must be <= 256");
    if (G > kF32MaxG) {
        // more query heads per kv row than one launch takes: launches of 16 heads over the same rows, q and
        // the outputs addressed through their rows of G heads (the kv rows are read once per launch)
        for (int g0 = 0; g0 < G; g0 += kF32MaxG) {
            const int rc = gqa_f32_heads(q, k, v, k_sb, k_st, v_sb, v_st, B_kv, std::min(kF32MaxG, G - g0), G, g0, D, L,
                                         scale, out_mode, out, out_max, out_sum, out_lse, workspace, workspace_bytes, st);
            if (rc != WS_OK) return rc;
        }
        return WS_OK;
    }
    return gqa_f32_heads(q, k, v, k_sb, k_st, v_sb, v_st, B_kv, G, G, 0, D, L, scale, out_mode, out, out_max, out_sum,
                         out_lse, workspace, workspace_bytes, st);
}

// One launch over heads g0 .. g0 + G - 1 of rows that hold GR heads each.
static int gqa_f32_heads(const void* q, const void* k, const void* v, int64_t k_sb, int64_t k_st, int64_t v_sb,
                         int64_t v_st, int B_kv, int G, int GR, int g0, int D, int L, float scale, int out_mode,
                         void* out, void* out_max, void* out_sum, float* out_lse, void* workspace,
                         size_t workspace_bytes, cudaStream_t st) {
    F32Params p;
    p.q = static_cast<const float*>(q) + (int64_t)g0 * D;
    p.k = static_cast<const float*>(k);
    p.v = static_cast<const float*>(v);
    p.k_sb = k_sb; p.k_st = k_st; p.v_sb = v_sb; p.v_st = v_st;
    p.G = G; p.GR = GR; p.D = D; p.L = L; p.scale = scale; p.out_mode = out_mode;
    p.out = static_cast<float*>(out) + (int64_t)g0 * D;
    p.out_max = out_max ? static_cast<float*>(out_max) + g0 : nullptr;
    p.out_sum = out_sum ? static_cast<float*>(out_sum) + g0 : nullptr;
    p.out_lse = out_lse ? out_lse + g0 : nullptr;
    const int DPL = (D + 31) / 32 <= 4 ? 4 : 8;
    const int slot_floats = G * D + 2 * G;
    // splits: enough blocks to cover the SMs twice, at most one per 256 tokens
    const int nsm = device_sm_count();
    int splits = std::max(1, std::min((L + 255) / 256, (2 * nsm + B_kv - 1) / B_kv));
    if (B_kv > kMaxGroupsPerLaunch) return set_error(WS_ERR_UNSUPPORTED, "fp32 path: more than 65536 rows in one launch");
    const size_t cnt_bytes = kCounterHeaderBytes;
    const size_t slots_fit = workspace_bytes > cnt_bytes ? (workspace_bytes - cnt_bytes) / (size_t(slot_floats) * 4) : 0;
    while (splits > 1 && size_t(B_kv) * splits > slots_fit) --splits;
    if (splits > 1 && !workspace) splits = 1;
    p.ws_cnt = static_cast<int*>(workspace);
    p.ws_part = workspace ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + cnt_bytes) : nullptr;
    // the tiled forms when every K and V row starts 16-byte aligned (16-byte cp.async copies)
    const bool aligned = reinterpret_cast<uintptr_t>(k) % 16 == 0 && reinterpret_cast<uintptr_t>(v) % 16 == 0 &&
                         k_sb % 4 == 0 && k_st % 4 == 0 && v_sb % 4 == 0 && v_st % 4 == 0 && D % 4 == 0;
    if (aligned) {
        const bool wide = D > 128, rb = !wide && G <= kF32RbHeads;
        const size_t smem = rb ? f32_rb_smem(G, D) : wide ? F32Tile<256>::smem(G, D) : F32Tile<128>::smem(G, D);
        const int tt = wide ? F32Tile<256>::TT : F32Tile<128>::TT;
        auto kfn = rb ? gqa_f32_rb_kernel : wide ? gqa_f32_tile_kernel<256> : gqa_f32_tile_kernel<128>;
        if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for the tiled fp32 decode");
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kF32Threads, smem) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        // one wave: every row split over the resident CTAs it can have, each split at least two tiles
        int sp = std::max(1, std::min((L + 2 * tt - 1) / (2 * tt), nsm * per_sm / std::max(B_kv, 1)));
        while (sp > 1 && size_t(B_kv) * sp > slots_fit) --sp;
        if (sp > 1 && !workspace) sp = 1;
        p.splits = sp;
        kfn<<<dim3(B_kv, sp), kF32Threads, smem, st>>>(p);
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
    }
    p.splits = splits;
    dim3 grid(B_kv, splits);
    const size_t smem = size_t(4) * G * D * sizeof(float);
    if (DPL == 4) {
        cudaFuncSetAttribute(gqa_f32_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        gqa_f32_kernel<4><<<grid, 128, smem, st>>>(p);
    } else {
        cudaFuncSetAttribute(gqa_f32_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        gqa_f32_kernel<8><<<grid, 128, smem, st>>>(p);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace ws
