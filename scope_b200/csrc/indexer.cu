// Indexer top-k of the DeepSeek-V4 CSA path: which compressed entries each
// sequence's sparse decode attends to.
//
// Replaces indexer_topk_cpu / indexer_topk_cpu_par
// (kernel/cpu_attn_ds4_ext/csa_attn.cpp:1658-1817):
//   score[b, j] = sum_h w[b, h] * relu(q[b, h] . kv[b, j])       (fp32 products and sums)
//   ids[b, :]   = the k entries with the largest scores, in descending score
//                 order (the reference's partial_sort leaves ties unordered;
//                 here the lower id comes first), or in ascending id order.
// Two launches:
//   indexer_score_kernel  -- thread = entry, the sequence's q in shared memory,
//                            fp32 on the CUDA cores in the reference's own
//                            order of operations (identical scores);
//                            (bf16 inputs: indexer_score_tc_kernel, tcgen05);
//   indexer_select_split_kernel -- several CTAs per sequence: a threshold placed
//                            from a sample of the scores, candidates appended to
//                            a workspace buffer, and the last CTA of the sequence
//                            (a ticket) selects: a bucket select over the
//                            candidates that leaves the k winners ordered, with a
//                            radix select (four 8-bit passes) plus merge sort
//                            when buckets overflow or the sample misjudges;
//   indexer_select_kernel -- the same with one CTA per sequence and the
//                            candidates in shared memory (no workspace, or
//                            many sequences).
#include "common.cuh"
#include "ws_internal.h"

namespace ws {
namespace idx {

constexpr int kScoreThreads = 128;   // entries per scoring CTA
constexpr int kMaxHeads = 64;
constexpr int kChunk = 16;           // dims of kv held in registers at a time
constexpr int kSelThreads = 1024;
constexpr int kMaxK = 4096;

// float -> uint32 with the same order (larger float <-> larger key)
__device__ __forceinline__ uint32_t ordered_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <bool BF16>
__global__ void __launch_bounds__(kScoreThreads) indexer_score_kernel(const void* __restrict__ q,
                                                                      const void* __restrict__ kv,
                                                                      const float* __restrict__ w, int nH, int hd,
                                                                      int64_t nc, float* __restrict__ scores) {
    extern __shared__ float s_q[];   // [nH][hd] fp32, then w [nH]
    const int b = blockIdx.y;
    const int64_t j = (int64_t)blockIdx.x * kScoreThreads + threadIdx.x;
    float* s_w = s_q + nH * hd;
    for (int i = threadIdx.x; i < nH * hd; i += kScoreThreads) {
        const int64_t off = (int64_t)b * nH * hd + i;
        s_q[i] = BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(q)[off]) : static_cast<const float*>(q)[off];
    }
    for (int i = threadIdx.x; i < nH; i += kScoreThreads) s_w[i] = w[(int64_t)b * nH + i];
    __syncthreads();
    if (j >= nc) return;
    const int64_t row = ((int64_t)b * nc + j) * hd;
    if constexpr (!BF16) {
        // fp32: the reference's own arithmetic (csa_attn.cpp:1706-1724), so the scores and hence the ranking
        // equal indexer_topk_cpu's bit for bit: per head 16 lane accumulators (lane l takes dims l, l+16, ...
        // by fused multiply-add), reduced pairwise as the AVX-512 horizontal add does (8-lane halves, 4-lane
        // halves, lanes {0+2, 1+3}, last add), then s = s + relu(dot) * w[h], multiply and add each rounded.
        // Rows of up to kRegDims dims are held in registers; longer rows are re-read per head (L1).
        constexpr int kRegDims = 128;
        const float* kvr = static_cast<const float*>(kv) + row;
        float xr[kRegDims];
        const bool inreg = hd <= kRegDims;
        if (inreg) {
#pragma unroll
            for (int c = 0; c < kRegDims / 16; ++c) {
                if (c * 16 < hd) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 v = __ldg(reinterpret_cast<const float4*>(kvr + c * 16) + u);
                        xr[c * 16 + 4 * u] = v.x; xr[c * 16 + 4 * u + 1] = v.y;
                        xr[c * 16 + 4 * u + 2] = v.z; xr[c * 16 + 4 * u + 3] = v.w;
                    }
                }
            }
        }
        float s = 0.f;
        for (int h = 0; h < nH; ++h) {
            const float* qh = s_q + h * hd;
            float a[16];
#pragma unroll
            for (int l = 0; l < 16; ++l) a[l] = 0.f;
            auto lanes = [&](const float (&x)[16], int d0) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 qq = reinterpret_cast<const float4*>(qh + d0)[u];
                    a[4 * u] = fmaf(qq.x, x[4 * u], a[4 * u]);
                    a[4 * u + 1] = fmaf(qq.y, x[4 * u + 1], a[4 * u + 1]);
                    a[4 * u + 2] = fmaf(qq.z, x[4 * u + 2], a[4 * u + 2]);
                    a[4 * u + 3] = fmaf(qq.w, x[4 * u + 3], a[4 * u + 3]);
                }
            };
            if (inreg) {
#pragma unroll
                for (int c = 0; c < kRegDims / 16; ++c) {
                    if (c * 16 < hd) {
                        float x[16];
#pragma unroll
                        for (int l = 0; l < 16; ++l) x[l] = xr[c * 16 + l];
                        lanes(x, c * 16);
                    }
                }
            } else {
                for (int d0 = 0; d0 < hd; d0 += 16) {
                    float x[16];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 v = __ldg(reinterpret_cast<const float4*>(kvr + d0) + u);
                        x[4 * u] = v.x; x[4 * u + 1] = v.y; x[4 * u + 2] = v.z; x[4 * u + 3] = v.w;
                    }
                    lanes(x, d0);
                }
            }
            float t3[8], t6[4];
#pragma unroll
            for (int i = 0; i < 8; ++i) t3[i] = __fadd_rn(a[i + 8], a[i]);
#pragma unroll
            for (int i = 0; i < 4; ++i) t6[i] = __fadd_rn(t3[i + 4], t3[i]);
            const float dot = __fadd_rn(__fadd_rn(t6[0], t6[2]), __fadd_rn(t6[1], t6[3]));
            s = __fadd_rn(s, __fmul_rn(dot > 0.f ? dot : 0.f, s_w[h]));
        }
        scores[(int64_t)b * nc + j] = s;
        return;
    }
    float acc[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) acc[h] = 0.f;
    for (int d0 = 0; d0 < hd; d0 += kChunk) {
        float x[kChunk];
        if (BF16) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(kv) + row + d0);
#pragma unroll
            for (int u = 0; u < kChunk / 8; ++u) {
                const uint4 a = __ldg(src + u);
                const uint32_t wds[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    x[8 * u + 2 * e] = __uint_as_float(wds[e] << 16);
                    x[8 * u + 2 * e + 1] = __uint_as_float(wds[e] & 0xffff0000u);
                }
            }
        } else {
            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(kv) + row + d0);
#pragma unroll
            for (int u = 0; u < kChunk / 4; ++u) {
                const float4 a = __ldg(src + u);
                x[4 * u] = a.x; x[4 * u + 1] = a.y; x[4 * u + 2] = a.z; x[4 * u + 3] = a.w;
            }
        }
#pragma unroll
        for (int h = 0; h < kMaxHeads; ++h) {
            if (h >= nH) break;
            const float4* qh = reinterpret_cast<const float4*>(s_q + h * hd + d0);
            float a = acc[h];
#pragma unroll
            for (int u = 0; u < kChunk / 4; ++u) {
                const float4 qq = qh[u];
                a = fmaf(qq.x, x[4 * u], a);
                a = fmaf(qq.y, x[4 * u + 1], a);
                a = fmaf(qq.z, x[4 * u + 2], a);
                a = fmaf(qq.w, x[4 * u + 3], a);
            }
            acc[h] = a;
        }
    }
    float s = 0.f;
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
        if (h >= nH) break;
        s = fmaf(fmaxf(acc[h], 0.f), s_w[h], s);
    }
    scores[(int64_t)b * nc + j] = s;
}

// Block-wide exclusive prefix sum of one int per thread (kSelThreads threads); returns the total in *total.
__device__ __forceinline__ int block_scan(int v, int* s_warp, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int t = s_warp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        s_warp[lane] = t;   // inclusive over warps
    }
    __syncthreads();
    const int before = (warp > 0 ? s_warp[warp - 1] : 0) + x - v;
    *total = s_warp[31];
    __syncthreads();
    return before;
}

constexpr int kBatch = 16;     // global scores per thread per step: four independent 16-byte loads in flight
constexpr int kEqCap = 2048;   // ties at the threshold gathered in one pass (more: ordered scan)
constexpr int kCand = 8192;    // candidates kept in shared memory
constexpr int kSample = 1024;  // sampled scores that place the candidate threshold

// The kBatch scores of step j0 this thread owns: ids j0 + 4 * (u * kSelThreads + tid) + e for u < 4, e < 4
// (16-byte loads when the row is 16-byte aligned); keys past nc are returned as 0 with valid = false.
__device__ __forceinline__ void load_keys(const float* sc, int64_t nc, int64_t j0, bool vec, uint32_t (&key)[kBatch],
                                          int64_t (&id)[kBatch]) {
#pragma unroll
    for (int u = 0; u < kBatch / 4; ++u) {
        const int64_t j = j0 + 4 * ((int64_t)u * kSelThreads + threadIdx.x);
        float v[4];
        if (vec && j + 3 < nc) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(sc + j));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = j + e < nc ? __ldcg(sc + j + e) : 0.f;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            id[4 * u + e] = j + e < nc ? j + e : -1;
            key[4 * u + e] = ordered_key(v[e]);
        }
    }
}

// The keys of load_keys without the ids (0 past nc; callers test the position).
__device__ __forceinline__ void load_keys_only(const float* sc, int64_t nc, int64_t j0, bool vec,
                                               uint32_t (&key)[kBatch]) {
#pragma unroll
    for (int u = 0; u < kBatch / 4; ++u) {
        const int64_t j = j0 + 4 * ((int64_t)u * kSelThreads + threadIdx.x);
        float v[4];
        if (vec && j + 3 < nc) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(sc + j));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = j + e < nc ? __ldcg(sc + j + e) : 0.f;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) key[4 * u + e] = j + e < nc ? ordered_key(v[e]) : 0u;
    }
}

// Sources of keys for the select passes: each thread takes KB keys per step of kSelThreads * KB
// positions (ids past the end come back as -1).
struct GlobalKeys {   // a sequence's scores in global memory (L2: just written by the scoring kernel)
    static constexpr int KB = kBatch;
    const float* sc;
    int64_t n;
    bool vec;
    __device__ __forceinline__ void load(int64_t j0, uint32_t (&key)[KB], int64_t (&id)[KB]) const {
        load_keys(sc, n, j0, vec, key, id);
    }
};
template <int KB_>
struct SharedKeys {   // keys in shared memory with their ids alongside, or (id == nullptr) the position
    static constexpr int KB = KB_;
    const uint32_t* key;
    const int32_t* id;
    int n;
    __device__ __forceinline__ void load(int64_t j0, uint32_t (&k)[KB], int64_t (&i)[KB]) const {
#pragma unroll
        for (int u = 0; u < KB; ++u) {
            const int64_t j = j0 + (int64_t)u * kSelThreads + threadIdx.x;
            const bool ok = j < n;
            k[u] = ok ? key[j] : 0u;
            i[u] = ok ? (id ? (int64_t)id[j] : j) : -1;
        }
    }
};


constexpr int kBuckets = 4096;   // linear buckets of the bucket select (four per thread)
constexpr int kBucketCap = 64;   // largest bucket among the winners the bucket select ranks (more: radix select)
static_assert(kBuckets == 4 * kSelThreads, "bucket_count gives each thread four buckets");
static_assert(kSample == kSelThreads, "sample_threshold gives each thread one sample");

struct SelectSmem {   // the select kernels' dynamic shared memory
    uint32_t ckey[kCand];   // candidates (before them: the samples; after them: the sort's scratch)
    int32_t cid[kCand];
    uint32_t key[kMaxK + kBucketCap];   // the k winners (bucket select: bucket order, up to a bucket past k)
    int32_t id[kMaxK + kBucketCap];
    int32_t eq[kEqCap];     // ids of keys equal to the threshold
    int whist[32][256];     // warp-private histograms of a radix pass
    int bstart[kBuckets + 1];   // bucket select: keys in the buckets above each bucket, then the count
    int bcur[kBuckets];         // bucket counts, then the scatter cursors
    int hist[256];
    int warp[32];
    uint32_t wlo[32], whi[32];
    uint32_t prefix, mask;
    int remaining, ngt, neq, ncand, flag, dstar, gbase, last;
};

// Radix select, 8 bits per pass from the top: the r-th largest key (1 <= r <= n) of the source is left in
// s.prefix, and s.remaining = how many keys equal to it belong to the r largest.
template <class Src>
__device__ void radix_select(const Src& src, int64_t n, int r, SelectSmem& s) {
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid == 0) {
        s.prefix = 0;
        s.mask = 0;
        s.remaining = r;
    }
    __syncthreads();
    const int warp = tid >> 5;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 32 * 256; i += kSelThreads) (&s.whist[0][0])[i] = 0;
        __syncthreads();
        const uint32_t prefix = s.prefix, mask = s.mask;
        for (int64_t j0 = 0; j0 < n; j0 += (int64_t)kSelThreads * Src::KB) {   // warp-uniform trip count
            uint32_t key[Src::KB];
            int64_t id[Src::KB];
            src.load(j0, key, id);
#pragma unroll
            for (int u = 0; u < Src::KB; ++u) {
                const bool hit = id[u] >= 0 && (key[u] & mask) == prefix;
                if (!__any_sync(0xffffffffu, hit)) continue;   // later passes: most warps hold no key of the prefix
                const int bin = hit ? (int)((key[u] >> shift) & 255) : 256;
                // the lowest lane of each distinct bin adds the count to this warp's own histogram
                // (keys of similar magnitude share a few bins: a block-wide histogram would serialise)
                const uint32_t same = __match_any_sync(0xffffffffu, bin);
                if (hit && lane == __ffs(same) - 1) s.whist[warp][bin] += __popc(same);
            }
        }
        __syncthreads();
        for (int i = tid; i < 256; i += kSelThreads) {
            int t = 0;
#pragma unroll 8
            for (int w = 0; w < 32; ++w) t += s.whist[w][i];
            s.hist[i] = t;
        }
        __syncthreads();
        if (tid < 32) {   // the bin of the remaining-th largest: lane l sums bins 255-8l .. 248-8l
            const int rem = s.remaining;
            int c[8], tot = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                c[e] = s.hist[255 - 8 * lane - e];
                tot += c[e];
            }
            int incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const int excl = incl - tot;
            const uint32_t hitm = __ballot_sync(0xffffffffu, excl < rem && incl >= rem);
            if (lane == (hitm ? __ffs(hitm) - 1 : 31)) {
                int r2 = rem - excl, bin = 255 - 8 * lane - 7;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    if (c[e] >= r2) {
                        bin = 255 - 8 * lane - e;
                        break;
                    }
                    r2 -= c[e];
                }
                s.remaining = r2;   // keys of this bin (among those with the prefix) still to take
                s.prefix = prefix | ((uint32_t)bin << shift);
                s.mask = mask | (255u << shift);
            }
        }
        __syncthreads();
    }
}

// Every key above thr into s.key / s.id (s.ngt of them, at most kMaxK kept), and the ids of keys equal
// to it into s.eq (s.neq of them, at most kEqCap kept).
template <class Src>
__device__ void collect_above(const Src& src, int64_t n, uint32_t thr, SelectSmem& s) {
    if (threadIdx.x == 0) {
        s.ngt = 0;
        s.neq = 0;
    }
    __syncthreads();
    for (int64_t j0 = 0; j0 < n; j0 += (int64_t)kSelThreads * Src::KB) {
        uint32_t key[Src::KB];
        int64_t id[Src::KB];
        src.load(j0, key, id);
#pragma unroll
        for (int u = 0; u < Src::KB; ++u) {
            const int64_t j = id[u];
            if (j < 0) continue;
            if (key[u] > thr) {
                const int slot = atomicAdd(&s.ngt, 1);
                if (slot < kMaxK) {
                    s.key[slot] = key[u];
                    s.id[slot] = (int32_t)j;
                }
            } else if (key[u] == thr) {
                const int slot = atomicAdd(&s.neq, 1);
                if (slot < kEqCap) s.eq[slot] = (int32_t)j;
            }
        }
    }
    __syncthreads();
}

// Sorts the k winners into descending order of v, where v = key << 32 | ~id (descending key, then
// ascending id) or v = ~id (ascending id); v is unique per winner.  Padded to N = 1024 E with values
// below every winner's.  Each warp sorts a run of 32 E in registers (bitonic network: a pair at
// stride s < E within a thread, else across lanes by shuffles), then the runs are merged pairwise in
// shared memory, log2(32) levels: thread t finds where its E outputs start with one merge-path search
// and takes them in order.  The winners' ids, in order, go to ids_out[0, k).
template <int E>
__device__ void merge_sort_desc(const uint32_t* key, const int32_t* id, int k, int by_id, uint64_t* A, uint64_t* B,
                                int32_t* ids_out) {
    constexpr int N = kSelThreads * E, R0 = 32 * E;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint64_t v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int j = warp * R0 + E * lane + e;
        const uint64_t nid = (uint64_t)(uint32_t)~(j < k ? id[j] : 0x7fffffff);
        v[e] = (j < k && !by_id) ? ((uint64_t)key[j] << 32 | nid) : nid;   // padding: ~0x7fffffff, below all
    }
    for (int size = 2; size <= R0; size <<= 1) {
        for (int s = size >> 1; s > 0; s >>= 1) {
            if (s < E) {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    if (e & s) continue;
                    const bool up = ((E * lane + e) & size) == 0;   // up: the larger first
                    if ((v[e] > v[e + s]) != up) {
                        const uint64_t t = v[e]; v[e] = v[e + s]; v[e + s] = t;
                    }
                }
            } else {
                const int ls = s / E;
                const bool lower = (lane & ls) == 0;
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, v[e], ls);
                    const bool up = ((E * lane + e) & size) == 0;
                    const bool lower_first = lower ? v[e] > o : o > v[e];
                    if (lower_first != up) v[e] = o;   // keep own exactly when lower_first == up
                }
            }
        }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) A[warp * R0 + E * lane + e] = v[e];
    __syncthreads();
    for (int L = R0; L < N; L <<= 1) {
        const int o0 = E * tid, base = o0 / (2 * L) * (2 * L), op = o0 - base;
        const uint64_t* a = A + base;
        const uint64_t* b = A + base + L;
        int lo = max(0, op - L), hi = min(op, L);
        while (lo < hi) {   // A elements among the first op outputs (ties, padding only: to B first)
            const int mid = (lo + hi) >> 1;
            if (a[mid] > b[op - mid - 1]) lo = mid + 1; else hi = mid;
        }
        int i = lo, j = op - lo;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const bool take_a = i < L && (j >= L || a[i] > b[j]);
            B[base + op + e] = take_a ? a[i] : b[j];
            if (take_a) ++i; else ++j;
        }
        __syncthreads();
        uint64_t* t = A; A = B; B = t;
    }
    for (int j = tid; j < k; j += kSelThreads) ids_out[j] = (int32_t)~(uint32_t)A[j];   // A: the merged run
    __syncthreads();
}

// Block-wide min and max of per-thread partials, one barrier; every thread gets the result.
__device__ __forceinline__ void block_range(uint32_t& lo, uint32_t& hi, SelectSmem& s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (lane == 0) {
        s.wlo[warp] = lo;
        s.whi[warp] = hi;
    }
    __syncthreads();
    lo = s.wlo[lane];
    hi = s.whi[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
}

// kBuckets equal-width buckets over the keys [lo, hi], numbered from the top (bucket 0 holds the
// largest keys): a key's bucket is its offset above lo shifted right until the range fits 12 bits.
struct Buckets {
    uint32_t lo;
    int shift;
    __device__ __forceinline__ Buckets(uint32_t lo_, uint32_t hi_) : lo(lo_) {
        const int bits = 32 - __clz(hi_ - lo_);   // 0 when lo == hi
        shift = max(0, bits - 12);
    }
    __device__ __forceinline__ int of(uint32_t key) const { return kBuckets - 1 - (int)((key - lo) >> shift); }
    __device__ __forceinline__ uint32_t lower_edge(int d) const { return lo + ((uint32_t)(kBuckets - 1 - d) << shift); }
};

// Zeroes the bucket counts and the overflow flag (a barrier must follow before bucket_count).
__device__ __forceinline__ void bucket_clear(SelectSmem& s) {
    for (int i = threadIdx.x; i < kBuckets; i += kSelThreads) s.bcur[i] = 0;
    if (threadIdx.x == 0) s.flag = 0;
}

// Counts the n keys (shared memory) per bucket: s.bstart[d] = keys in the buckets above d,
// s.bstart[kBuckets] = n, s.bcur = s.bstart; s.dstar = the bucket of the r-th largest key (1 <= r <= n);
// s.flag = 1 when a bucket that starts before r holds more than cap keys.  Expects bucket_clear and a
// barrier since; three barriers.
__device__ void bucket_count(const uint32_t* key, int n, const Buckets& bk, int r, int cap, SelectSmem& s) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < n; i += kSelThreads) atomicAdd(&s.bcur[bk.of(key[i])], 1);
    __syncthreads();
    int c[4], tot = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        c[e] = s.bcur[4 * tid + e];
        tot += c[e];
    }
    int x = tot;   // inclusive scan over the warp's threads
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s.warp[warp] = x;
    __syncthreads();
    int wx = s.warp[lane];   // every warp scans the 32 warp totals itself
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, wx, o);
        if (lane >= o) wx += y;
    }
    const int wbefore = __shfl_sync(0xffffffffu, wx, (warp + 31) & 31);
    const int total = __shfl_sync(0xffffffffu, wx, 31);
    int st = (warp > 0 ? wbefore : 0) + x - tot;
    bool over = false;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        s.bstart[4 * tid + e] = st;
        s.bcur[4 * tid + e] = st;
        if (st < r && st + c[e] >= r) s.dstar = 4 * tid + e;
        over |= st < r && c[e] > cap;
        st += c[e];
    }
    if (over) s.flag = 1;
    if (tid == 0) s.bstart[kBuckets] = total;
    __syncthreads();
}

// The candidate threshold of a sequence with nc > kCand scores: the lower edge of the bucket that holds
// the r-th largest of kSample evenly spaced scores (r = k's share plus six standard deviations plus 16),
// so at least r samples lie at or above it.  Uses s.ckey [0, kSample).
__device__ uint32_t sample_threshold(const float* sc, int64_t nc, int k, SelectSmem& s) {
    const int tid = threadIdx.x;
    const uint32_t key = ordered_key(__ldcg(sc + (int64_t)tid * nc / kSample));
    s.ckey[tid] = key;
    bucket_clear(s);
    uint32_t lo = key, hi = key;
    block_range(lo, hi, s);
    const double base = (double)k * kSample / (double)nc;
    const int r = min(kSample, (int)ceil(base + 6.0 * sqrt(base) + 16.0));
    const Buckets bk(lo, hi);
    bucket_count(s.ckey, kSample, bk, r, kSample, s);
    return bk.lower_edge(s.dstar);
}

// The k largest of the n candidates in s.ckey / s.cid (k <= n <= kCand; keys within [lo, hi]), in
// descending key order and ascending id among equal keys, into s.ckey / s.cid [0, k): count the
// candidates per bucket, place the keys of every bucket that starts before k in bucket order, and rank
// each inside its bucket.  Returns false, with the candidates untouched, when one of those buckets holds
// more than kBucketCap keys (heavy ties, or a few keys far above the rest).  Expects bucket_clear and a
// barrier since.
__device__ bool bucket_select(int n, int k, uint32_t lo, uint32_t hi, SelectSmem& s) {
    const int tid = threadIdx.x;
    const Buckets bk(lo, hi);
    bucket_count(s.ckey, n, bk, k, kBucketCap, s);
    if (s.flag) return false;
    for (int i = tid; i < n; i += kSelThreads) {
        const uint32_t key = s.ckey[i];
        const int d = bk.of(key);
        if (s.bstart[d] < k) {   // positions stay below k - 1 + kBucketCap
            const int pos = atomicAdd(&s.bcur[d], 1);
            s.key[pos] = key;
            s.id[pos] = s.cid[i];
        }
    }
    __syncthreads();
    const int filled = s.bstart[s.dstar + 1];
    for (int p = tid; p < filled; p += kSelThreads) {
        const uint32_t key = s.key[p];
        const int32_t id = s.id[p];
        const int d = bk.of(key);
        const int b0 = s.bstart[d], b1 = s.bstart[d + 1];
        int rank = 0;
        for (int q = b0; q < b1; ++q) {
            const uint32_t kq = s.key[q];
            rank += (kq > key || (kq == key && s.id[q] < id)) ? 1 : 0;
        }
        const int f = b0 + rank;
        if (f < k) {
            s.ckey[f] = key;
            s.cid[f] = id;
        }
    }
    __syncthreads();
    return true;
}

// Orders the k winners in s.key / s.id (descending key then ascending id, or ascending id) into s.id;
// the candidate buffers, free by now, hold the merge buffers (ckey + cid: 64 KB = 2 x 4096 values).
__device__ __forceinline__ void sort_winners(int k, int by_id, SelectSmem& s) {
    uint64_t* mA = reinterpret_cast<uint64_t*>(s.ckey);
    if (k <= 2048) merge_sort_desc<2>(s.key, s.id, k, by_id, mA, mA + 4096, s.id);
    else merge_sort_desc<4>(s.key, s.id, k, by_id, mA, mA + 4096, s.id);
}

// The k winners among the n keys of src by radix select, the ties at the threshold in id order, then
// ordered: their ids into s.id [0, k).  sc / nc: the sequence's scores, for the ordered scan that takes
// very many ties.
template <class Src>
__device__ void radix_path(const Src& src, int64_t n, int k, int by_id, const float* sc, int64_t nc,
                           SelectSmem& s) {
    const int tid = threadIdx.x;
    radix_select(src, n, k, s);
    collect_above(src, n, s.prefix, s);
    const uint32_t thr = s.prefix;       // the k-th largest key
    const int need_eq = s.remaining;     // keys equal to it that belong to the top k
    const int ngt = min(s.ngt, k);
    const int neq = s.neq;
    if (neq <= kEqCap) {
        // the ties, lowest ids first: sort the gathered ids ascending and take need_eq of them
        int m2 = 1;
        while (m2 < neq) m2 <<= 1;
        for (int i = neq + tid; i < m2; i += kSelThreads) s.eq[i] = 0x7fffffff;
        __syncthreads();
        for (int size = 2; size <= m2; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < m2 / 2; i += kSelThreads) {
                    const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                    const bool up = (lo & size) == 0;
                    const int32_t a = s.eq[lo], c = s.eq[hi];
                    if ((a < c) != up && a != c) {
                        s.eq[lo] = c;
                        s.eq[hi] = a;
                    }
                }
                __syncthreads();
            }
        for (int i = tid; i < need_eq; i += kSelThreads) {
            s.key[ngt + i] = thr;
            s.id[ngt + i] = s.eq[i];
        }
    } else {
        // very many ties: take them in id order with a block-wide scan over all scores
        int taken = 0;
        for (int64_t j0 = 0; j0 < nc && taken < need_eq; j0 += kSelThreads) {
            const int64_t j = j0 + tid;
            const int eq = (j < nc && ordered_key(__ldcg(sc + j)) == thr) ? 1 : 0;
            int total = 0;
            const int before = block_scan(eq, s.warp, &total);
            if (eq && taken + before < need_eq) {
                s.key[ngt + taken + before] = thr;
                s.id[ngt + taken + before] = (int32_t)j;
            }
            taken += total;   // uniform across the block
        }
    }
    __syncthreads();
    sort_winners(k, by_id, s);
}

// The selection of a sequence once its candidates (ncand of them, keys within [lo, hi]) sit in
// s.ckey / s.cid: the bucket select when k <= ncand <= kCand, else (or when a bucket overflows) the
// radix path over the candidates or over all scores.  Returns the array holding the k ids in order.
__device__ const int32_t* select_candidates(int ncand, int k, int by_id, uint32_t lo, uint32_t hi,
                                           const GlobalKeys& all, SelectSmem& s) {
    const int tid = threadIdx.x;
    if (ncand >= k && ncand <= kCand) {
        if (bucket_select(ncand, k, lo, hi, s)) {
            if (!by_id) return s.cid;
            for (int i = tid; i < k; i += kSelThreads) {
                s.key[i] = s.ckey[i];
                s.id[i] = s.cid[i];
            }
            __syncthreads();
            sort_winners(k, by_id, s);
            return s.id;
        }
        radix_path(SharedKeys<4>{s.ckey, s.cid, ncand}, ncand, k, by_id, all.sc, all.n, s);
    } else {
        radix_path(all, all.n, k, by_id, all.sc, all.n, s);
    }
    return s.id;
}

// Candidate pass over the scores [lo, hi) of one sequence: every key >= the threshold (from thr(),
// called while the first step's loads are in flight) goes, with its id, to emit(slot, key, id) at a slot
// from take(count) (block-uniform; called by one thread per step with the step's total).  Sixteen keys
// per thread per step, all loads in flight together.  Clears the buckets for the final select.
template <class Thr, class Take, class Emit>
__device__ __forceinline__ void candidate_pass(const float* sc, int64_t lo, int64_t hi, bool vec, Thr thr,
                                               SelectSmem& s, Take take, Emit emit) {
    const int tid = threadIdx.x, lane = tid & 31;
    uint32_t key[kBatch];
    load_keys_only(sc, hi, lo, vec, key);
    const uint32_t t_lo = thr();
    bucket_clear(s);   // for the final select
    if (tid == 0) s.ncand = 0;
    __syncthreads();
    for (int64_t j0 = lo; j0 < hi; j0 += (int64_t)kSelThreads * kBatch) {
        if (j0 != lo) load_keys_only(sc, hi, j0, vec, key);
        auto pos = [&](int u) { return j0 + 4 * ((int64_t)(u >> 2) * kSelThreads + tid) + (u & 3); };
        int cnt = 0;
#pragma unroll
        for (int u = 0; u < kBatch; ++u) cnt += (pos(u) < hi && key[u] >= t_lo) ? 1 : 0;
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int wbase = 0;
        if (lane == 31 && incl > 0) wbase = atomicAdd(&s.ncand, incl);
        __syncthreads();
        if (tid == 0) {
            s.gbase = take(s.ncand);
            s.ncand = 0;
        }
        __syncthreads();
        int slot = s.gbase + __shfl_sync(0xffffffffu, wbase, 31) + incl - cnt;
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            if (pos(u) < hi && key[u] >= t_lo) {
                emit(slot, key[u], (int32_t)pos(u));
                ++slot;
            }
        }
    }
}

// One CTA per sequence: candidates against the sampled threshold into shared memory, then the select.
__global__ void __launch_bounds__(kSelThreads) indexer_select_kernel(const float* __restrict__ scores, int64_t nc,
                                                                     int k, int by_id, int32_t* __restrict__ out) {
    extern __shared__ __align__(16) uint8_t sel_smem[];
    SelectSmem& s = *reinterpret_cast<SelectSmem*>(sel_smem);
    const int b = blockIdx.x, tid = threadIdx.x;
    const float* sc = scores + (int64_t)b * nc;
    const GlobalKeys all{sc, nc, (reinterpret_cast<uintptr_t>(sc) & 15) == 0};
    pdl_wait_primary();   // the scores come from the previous grid
    // every key passes when all scores fit the buffer; else a sampled threshold keeps (for any but
    // adversarial orders) between k and kCand of them
    int total = 0;
    uint32_t klo = 0xffffffffu, khi = 0;   // range of the stored candidates
    candidate_pass(
        sc, 0, nc, all.vec, [&] { return nc > kCand ? sample_threshold(sc, nc, k, s) : 0u; }, s,
        [&](int n) {
            const int base = total;
            total += n;
            return base;
        },
        [&](int slot, uint32_t key, int32_t id) {
            if (slot < kCand) {
                s.ckey[slot] = key;
                s.cid[slot] = id;
                klo = min(klo, key);
                khi = max(khi, key);
            }
        });
    if (tid == 0) s.ncand = total;
    block_range(klo, khi, s);
    const int32_t* ids = select_candidates(s.ncand, k, by_id, klo, khi, all, s);
    for (int i = tid; i < k; i += kSelThreads) out[(int64_t)b * k + i] = ids[i];
}

// `parts` CTAs per sequence (blockIdx.x; blockIdx.y = sequence), each over `chunk` of its scores: the
// same sampled threshold in every CTA, candidates appended to the sequence's global buffer (cand, kCand
// per sequence).  counters[b] packs the candidate count (low 32 bits, slots taken by atomic adds) and a
// ticket (high 32 bits): the CTA that takes the last ticket learns the total from it, reads the
// candidates back, returns the counter to zero and selects.
__global__ void __launch_bounds__(kSelThreads) indexer_select_split_kernel(const float* __restrict__ scores,
                                                                           int64_t nc, int k, int by_id,
                                                                           int64_t chunk, int parts, uint2* cand,
                                                                           unsigned long long* counters,
                                                                           int32_t* __restrict__ out) {
    extern __shared__ __align__(16) uint8_t sel_smem[];
    SelectSmem& s = *reinterpret_cast<SelectSmem*>(sel_smem);
    const int part = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const float* sc = scores + (int64_t)b * nc;
    const GlobalKeys all{sc, nc, (reinterpret_cast<uintptr_t>(sc) & 15) == 0};
    unsigned long long* counter = counters + b;
    uint2* gc = cand + (int64_t)b * kCand;
    const int64_t lo = (int64_t)part * chunk, hi = min(nc, lo + chunk);
    pdl_wait_primary();   // the scores come from the previous grid
    candidate_pass(
        sc, lo, hi, all.vec, [&] { return sample_threshold(sc, nc, k, s); }, s,
        [&](int n) { return n > 0 ? (int)(uint32_t)atomicAdd(counter, (unsigned long long)n) : 0; },
        [&](int slot, uint32_t key, int32_t id) {
            if (slot < kCand) gc[slot] = make_uint2(key, (uint32_t)id);
        });
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned long long old = atomicAdd(counter, 1ull << 32);
        s.last = (int)(old >> 32) == parts - 1;
        s.ncand = (int)(uint32_t)old;   // every CTA's slots were taken before its ticket
        if (s.last) *reinterpret_cast<volatile unsigned long long*>(counter) = 0ull;
    }
    __syncthreads();
    if (!s.last) return;
    __threadfence();
    const int ncand = s.ncand;
    uint32_t klo = 0xffffffffu, khi = 0;
    if (ncand >= k && ncand <= kCand) {
        for (int i = tid; i < ncand; i += kSelThreads) {
            const uint2 c = __ldcg(gc + i);
            s.ckey[i] = c.x;
            s.cid[i] = (int32_t)c.y;
            klo = min(klo, c.x);
            khi = max(khi, c.x);
        }
    }
    block_range(klo, khi, s);
    const int32_t* ids = select_candidates(ncand, k, by_id, klo, khi, all, s);
    for (int i = tid; i < k; i += kSelThreads) out[(int64_t)b * k + i] = ids[i];
}

// ---------------------------------------------------------------- bf16 scoring on tcgen05
// D[128 entries x 64 heads] = KV_tile . Q^T (M=128, N=64, K=hd) in TMEM, two D buffers; the
// sequence's q (zero rows past nH) sits in shared memory, KV tiles stream through a TMA ring.
// Warp 0: TMA producer; warp 1: MMA issuer (and TMEM owner); warps 2-5: epilogue
// (thread = entry: score = sum_h w_h * relu(D[entry, h])).  One sequence per CTA, CTAs of a
// sequence split its tiles evenly.
namespace tc {
constexpr int TT = 128, NHP = 64;                // entries per tile, heads padded
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int BOX = TT * 128;                    // 64 dims x 128 entries bf16 = 16 KB
constexpr int QBOX = NHP * 128;                  // 64 dims x 64 heads = 8 KB
enum { B_FULL = 0, B_EMPTY = kMaxStages, B_DFULL = 2 * kMaxStages, B_DEMPTY = 2 * kMaxStages + 2,
       NBARS = 2 * kMaxStages + 4 };

struct TcParams {
    int nH, kb, stages, ctas_per_seq, kv_tok_in_dim2;
    int64_t nc;
    float* scores;
    int* status;
};

__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* status) {
    if (*abort) return false;
    if (mbar_wait_bounded(bar, parity)) return true;
    *abort = 1;
    atomicExch(status, kDevTimeout);
    return false;
}

__global__ void __launch_bounds__(kThreads, 2) indexer_score_tc_kernel(const __grid_constant__ CUtensorMap map_kv,
                                                                       const __nv_bfloat16* __restrict__ q,
                                                                       const float* __restrict__ w,
                                                                       const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int KB = p.kb, ST = p.stages;
    const int stage_bytes = KB * BOX;
    uint8_t* s_q = sm;                                   // KB boxes of 8 KB
    uint8_t* s_ring = sm + KB * QBOX;                    // ST stages
    float* s_w = reinterpret_cast<float*>(s_ring + ST * stage_bytes);   // [64]
    uint64_t* bars = reinterpret_cast<uint64_t*>(s_w + NHP);
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + NBARS);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
    const uint32_t bar0 = smem_u32(bars);
#define TB(i) (bar0 + 8u * (uint32_t)(i))

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.x / p.ctas_per_seq, part = blockIdx.x - b * p.ctas_per_seq;
    const int64_t ntl = (p.nc + TT - 1) / TT;
    const int64_t t_begin = ntl * part / p.ctas_per_seq, t_end = ntl * (part + 1) / p.ctas_per_seq;
    const int n = (int)(t_end - t_begin);

    if (tid == 0) {
        for (int i = 0; i < kMaxStages; ++i) {
            mbar_init(TB(B_FULL + i), 1);
            mbar_init(TB(B_EMPTY + i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(TB(B_DFULL + i), 1);
            mbar_init(TB(B_DEMPTY + i), 4);
        }
        *s_abort = 0;
        fence_mbar_init();
    }
    // the producer (thread 0) issues the loads of the first ring-full of tiles at once: they wait on no
    // barrier and are in flight while q is staged and TMEM allocated
    const int first = n < ST ? n : ST;
    auto issue = [&](int i) {
        const int s = i % ST;
        mbar_arrive_expect_tx(TB(B_FULL + s), stage_bytes);
        const int tok = (int)((t_begin + i) * TT);
        for (int kb = 0; kb < KB; ++kb)
            tma_load_3d(smem_u32(s_ring + s * stage_bytes + kb * BOX), &map_kv, TB(B_FULL + s), kb * 64,
                        p.kv_tok_in_dim2 ? b : tok, p.kv_tok_in_dim2 ? tok : b);
    };
    if (tid == 0) {
        tma_prefetch_desc(&map_kv);
        for (int i = 0; i < first; ++i) issue(i);
    }
    // q of this sequence -> K-major swizzled bf16 [64 rows x hd] (zero rows past nH); weights (0 past nH)
    const int hd = KB * 64;
    for (int j = tid; j < NHP * (hd / 8); j += kThreads) {
        const int r = j / (hd / 8), c = j - r * (hd / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < p.nH) v = __ldg(reinterpret_cast<const uint4*>(q + ((int64_t)b * p.nH + r) * hd + c * 8));
        *reinterpret_cast<uint4*>(s_q + (c >> 3) * QBOX + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = v;
    }
    if (tid < NHP) s_w[tid] = tid < p.nH ? w[(int64_t)b * p.nH + tid] : 0.f;
    if (warp == 1) tmem_alloc(smem_u32(s_tmem), 128);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch_dependents();   // the select's CTAs may take SMs as this grid's CTAs finish
    const uint32_t tbase = *s_tmem;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        int i = first;
        if (lane == 0) {
            for (; i < n; ++i) {
                const int s = i % ST;
                if (!tc_wait(TB(B_EMPTY + s), ((i / ST) - 1) & 1, s_abort, p.status)) break;
                issue(i);
            }
            if (*s_abort) {   // leave no bulk copy in flight: wait (bounded) for the last load of every slot
                for (int s = 0; s < ST; ++s) {
                    const int last = i - 1 - ((i - 1 - s) % ST + ST) % ST;
                    if (last >= 0) mbar_wait_bounded(TB(B_FULL + s), (uint32_t)(last / ST) & 1, 200000000ull);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        const uint32_t id = idesc_bf16_f32(TT, NHP, false, false);
        for (int i = 0; i < n; ++i) {
            const int s = i % ST, d = i & 1;
            bool ok = tc_wait(TB(B_FULL + s), (i / ST) & 1, s_abort, p.status);
            if (ok && i >= 2) ok = tc_wait(TB(B_DEMPTY + d), ((i >> 1) - 1) & 1, s_abort, p.status);
            if (!ok) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t a0 = smem_u32(s_ring + s * stage_bytes), b0 = smem_u32(s_q);
                for (int kb = 0; kb < KB; ++kb)
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16(tbase + d * NHP, sdesc_sw128(a0 + kb * BOX + kk * 32, 16, 1024),
                                  sdesc_sw128(b0 + kb * QBOX + kk * 32, 16, 1024), id, (kb | kk) != 0);
                umma_commit(TB(B_EMPTY + s));
                umma_commit(TB(B_DFULL + d));
            }
            __syncwarp();
        }
    } else {
        // ---------------------------------------------------------------- epilogue (thread = entry)
        const int quad = warp & 3;                        // TMEM lane quadrant this warp may read
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        for (int i = 0; i < n; ++i) {
            const int d = i & 1;
            if (!tc_wait(TB(B_DFULL + d), (i >> 1) & 1, s_abort, p.status)) break;
            tc_fence_after();
            float x[NHP];
#pragma unroll
            for (int c = 0; c < NHP / 16; ++c) tmem_ld16(tbase + lane_base + d * NHP + c * 16, x + c * 16);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(TB(B_DEMPTY + d));
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int h = 0; h < NHP; h += 2) {
                s0 = fmaf(fmaxf(x[h], 0.f), s_w[h], s0);
                s1 = fmaf(fmaxf(x[h + 1], 0.f), s_w[h + 1], s1);
            }
            const int64_t j = (t_begin + i) * TT + quad * 32 + lane;
            if (j < p.nc) p.scores[(int64_t)b * p.nc + j] = s0 + s1;
        }
    }
#undef TB
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tbase, 128);
}
}  // namespace tc

}  // namespace idx

// Candidate buffer of the split select: after the counter header and the scores.
static size_t cand_offset(int bs, int64_t nc) {
    return kCounterHeaderBytes + align_up((size_t)std::max(bs, 1) * (size_t)std::max<int64_t>(nc, 1) * 4, 256);
}

size_t indexer_workspace_bytes(int bs, int64_t nc) {
    return cand_offset(bs, nc) + align_up((size_t)std::max(bs, 1) * idx::kCand * sizeof(uint2), 256);
}

// The select: `parts` CTAs per sequence when a workspace holds the candidate buffer and fewer than
// half the SMs would otherwise work (the split kernel), else one CTA per sequence.
static int select_launch(const float* scores, int64_t nc, int k, int by_id, int32_t* out, int bs, void* workspace,
                         size_t workspace_bytes, cudaStream_t st) {
    using namespace idx;
    const int smem = (int)sizeof(SelectSmem);
    static int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(indexer_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
                cudaSuccess ||
            cudaFuncSetAttribute(indexer_select_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
                cudaSuccess)
            return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for the indexer select kernels");
        configured_dev = dev;
    }
    int parts = 1;
    int64_t chunk = nc;
    const bool have_ws = workspace && workspace_bytes >= indexer_workspace_bytes(bs, nc) &&
                         (size_t)bs * sizeof(unsigned long long) <= kCounterHeaderBytes;
    if (have_ws && nc > kCand) {
        const int target = std::min(16, device_sm_count() / std::max(bs, 1));
        if (target >= 2) {
            const int64_t grain = 4 * kSelThreads;   // one 16-byte load per thread (keeps chunks 16-byte aligned)
            chunk = (nc + target - 1) / target;
            chunk = (chunk + grain - 1) / grain * grain;
            parts = (int)((nc + chunk - 1) / chunk);
        }
    }
    // a programmatic dependent of the scoring kernel: launched while it drains, waits for its scores
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kSelThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (parts >= 2) {
        uint8_t* base = static_cast<uint8_t*>(workspace);
        cfg.gridDim = dim3((unsigned)parts, (unsigned)bs);
        e = cudaLaunchKernelEx(&cfg, indexer_select_split_kernel, scores, nc, k, by_id, chunk, parts,
                               reinterpret_cast<uint2*>(base + cand_offset(bs, nc)),
                               reinterpret_cast<unsigned long long*>(base), out);
    } else {
        cfg.gridDim = dim3((unsigned)bs);
        e = cudaLaunchKernelEx(&cfg, indexer_select_kernel, scores, nc, k, by_id, out);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

int indexer_topk_launch(const void* q, const void* kv, int bf16, const float* w, int bs, int nH, int hd, int64_t nc,
                        int k, int by_id, int32_t* out_ids, float* out_scores, void* workspace,
                        size_t workspace_bytes, cudaStream_t st) {
    using namespace idx;
    if (nH < 1) return set_error(WS_ERR_INVALID_ARG, "indexer_topk: nH >= 1");
    if (hd < kChunk || hd % kChunk) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: hd % 16 == 0");
    // bf16 inputs: up to 64 heads and hd <= 256 (tensor-core tiles, per-head accumulators); fp32 inputs: any
    // shape whose query block fits in shared memory
    if (bf16 && (nH > kMaxHeads || hd > 256))
        return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: bf16 inputs take 1..64 heads and hd <= 256");
    if (((size_t)nH * hd + nH) * sizeof(float) > 220 * 1024)
        return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: nH * hd * 4 bytes must fit in 220 KB of shared memory");
    if (k > kMaxK) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: k <= 4096");
    if (nc > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: nc > 2^31 - 1");
    float* scores = out_scores;
    if (!scores) {
        if (!workspace || workspace_bytes < indexer_workspace_bytes(bs, nc))
            return set_error(WS_ERR_WORKSPACE, "indexer_topk: workspace missing or too small");
        scores = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterHeaderBytes);
    }
    if (bf16 && hd % 64 == 0 && hd <= 256) {
        // tensor-core scoring: one sequence per CTA group, the CTAs of a sequence split its tiles
        using namespace tc;
        TcParams tp;
        tp.nH = nH;
        tp.kb = hd / 64;
        const size_t fixed = 1024 + (size_t)tp.kb * QBOX + NHP * 4 + NBARS * 8 + 16;
        // Two CTAs per SM, each with a two-stage ring, when the shared memory allows it (hd <= 128): their
        // pipelines cover each other's per-tile hand-offs, which one CTA with a deeper ring does not (the
        // bench's idx step went from 66.6 to 64.2 us; a ring of 3 instead of 5 stages at one CTA per SM
        // measured the same as 5).  Otherwise one CTA per SM with the deepest ring that fits.
        int per_sm = 2;
        tp.stages = (int)std::min<size_t>(kMaxStages, (112 * 1024 - fixed) / ((size_t)tp.kb * BOX));
        if (tp.stages < 2) {
            per_sm = 1;
            tp.stages = (int)std::min<size_t>(kMaxStages, (200 * 1024 - fixed) / ((size_t)tp.kb * BOX));
        }
        tp.nc = nc;
        tp.scores = scores;
        tp.status = device_status_word();
        const int sms = device_sm_count();
        const int64_t tiles = (nc + TT - 1) / TT;
        tp.ctas_per_seq = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)sms * per_sm / std::max(bs, 1)));
        CUtensorMap map;
        int tok_in_dim2 = 0;
        int rc = make_kv_map(&map, kv, hd, nc * hd, hd, nc, bs, TT, &tok_in_dim2);
        if (rc != WS_OK) return rc;
        tp.kv_tok_in_dim2 = tok_in_dim2;
        const size_t smem = fixed + (size_t)tp.stages * tp.kb * BOX;
        static int configured_dev = -1;
        int dev = 0;
        cudaGetDevice(&dev);
        if (configured_dev != dev) {
            if (cudaFuncSetAttribute(indexer_score_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024 + 1024) != cudaSuccess)
                return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for indexer_score_tc_kernel");
            configured_dev = dev;
        }
        const int64_t grid = (int64_t)bs * tp.ctas_per_seq;
        if (grid > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: too many sequences");
        indexer_score_tc_kernel<<<(unsigned)grid, kThreads, smem, st>>>(
            map, static_cast<const __nv_bfloat16*>(q), w, tp);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return set_error(WS_ERR_CUDA, cudaGetErrorString(e));
        return k > 0 ? select_launch(scores, nc, k, by_id, out_ids, bs, workspace, workspace_bytes, st) : WS_OK;
    }
    const size_t smem = ((size_t)nH * hd + nH) * sizeof(float);
    auto kfn = bf16 ? indexer_score_kernel<true> : indexer_score_kernel<false>;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for indexer_score_kernel");
    const dim3 grid((unsigned)((nc + kScoreThreads - 1) / kScoreThreads), (unsigned)bs);
    kfn<<<grid, kScoreThreads, smem, st>>>(q, kv, w, nH, hd, nc, scores);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(WS_ERR_CUDA, cudaGetErrorString(e));
    return k > 0 ? select_launch(scores, nc, k, by_id, out_ids, bs, workspace, workspace_bytes, st) : WS_OK;
}

}  // namespace ws
