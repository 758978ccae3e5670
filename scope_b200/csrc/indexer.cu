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
//                            fp32 FMA on the CUDA cores (exact fp32 products);
//   indexer_select_kernel -- one CTA per sequence: radix select of the k-th
//                            largest score (four 8-bit passes over the scores,
//                            which stay in L2), collection of the k winners
//                            (ties at the threshold taken in id order), and a
//                            bitonic sort in shared memory.
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
    float acc[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) acc[h] = 0.f;
    const int64_t row = ((int64_t)b * nc + j) * hd;
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

__global__ void __launch_bounds__(kSelThreads) indexer_select_kernel(const float* __restrict__ scores, int64_t nc,
                                                                     int k, int by_id, int32_t* __restrict__ out) {
    __shared__ int s_hist[256];
    __shared__ int s_warp[32];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_remaining, s_ngt;
    __shared__ uint32_t s_key[kMaxK];
    __shared__ int32_t s_id[kMaxK];
    const int b = blockIdx.x, tid = threadIdx.x;
    const float* sc = scores + (int64_t)b * nc;
    if (tid == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_remaining = k;
    }
    __syncthreads();
    // ---- radix select: the k-th largest key, 8 bits per pass from the top
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kSelThreads) s_hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int64_t j0 = 0; j0 < nc; j0 += kSelThreads) {   // warp-uniform trip count (for __match_any_sync)
            const int64_t j = j0 + tid;
            const uint32_t key = j < nc ? ordered_key(__ldcg(sc + j)) : 0u;
            const bool hit = j < nc && (key & mask) == prefix;
            const int bin = hit ? (int)((key >> shift) & 255) : 256;
            // one atomic per distinct bin in the warp: scores of similar magnitude share a few bins
            const uint32_t same = __match_any_sync(0xffffffffu, bin);
            if (hit && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&s_hist[bin], __popc(same));
        }
        __syncthreads();
        if (tid == 0) {
            int rem = s_remaining, bin = 0;
            for (int d = 255; d >= 0; --d) {
                if (s_hist[d] >= rem) {
                    bin = d;
                    break;
                }
                rem -= s_hist[d];
            }
            s_remaining = rem;   // keys of this bin (among those with the prefix) still to take
            s_prefix = prefix | ((uint32_t)bin << shift);
            s_mask = mask | (255u << shift);
        }
        __syncthreads();
    }
    const uint32_t thr = s_prefix;       // the k-th largest key
    const int need_eq = s_remaining;     // keys equal to it that belong to the top k
    if (tid == 0) s_ngt = 0;
    __syncthreads();
    // ---- collect: every key above the threshold, then the first need_eq keys equal to it, in id order
    for (int64_t j = tid; j < nc; j += kSelThreads) {
        const uint32_t key = ordered_key(__ldcg(sc + j));
        if (key > thr) {
            const int slot = atomicAdd(&s_ngt, 1);
            if (slot < kMaxK) {
                s_key[slot] = key;
                s_id[slot] = (int32_t)j;
            }
        }
    }
    __syncthreads();
    const int ngt = min(s_ngt, k);
    int taken = 0;
    for (int64_t j0 = 0; j0 < nc && taken < need_eq; j0 += kSelThreads) {
        const int64_t j = j0 + tid;
        const int eq = (j < nc && ordered_key(__ldcg(sc + j)) == thr) ? 1 : 0;
        int total = 0;
        const int before = block_scan(eq, s_warp, &total);
        if (eq && taken + before < need_eq) {
            s_key[ngt + taken + before] = thr;
            s_id[ngt + taken + before] = (int32_t)j;
        }
        taken += total;   // uniform across the block
    }
    __syncthreads();
    // ---- bitonic sort of the k winners (padded to a power of two): descending key, then ascending id;
    //      or ascending id
    int n2 = 1;
    while (n2 < k) n2 <<= 1;
    for (int i = k + tid; i < n2; i += kSelThreads) {
        s_key[i] = 0u;           // below every real key
        s_id[i] = 0x7fffffff;
    }
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < n2 / 2; i += kSelThreads) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;   // this run sorts into the final order
                const uint32_t ka = s_key[lo], kb = s_key[hi];
                const int32_t ia = s_id[lo], ib = s_id[hi];
                // "a before b" in the final order
                const bool a_first = by_id ? (ia < ib) : (ka > kb || (ka == kb && ia < ib));
                if (a_first != up) {
                    s_key[lo] = kb; s_key[hi] = ka;
                    s_id[lo] = ib;  s_id[hi] = ia;
                }
            }
            __syncthreads();
        }
    }
    for (int i = tid; i < k; i += kSelThreads) out[(int64_t)b * k + i] = s_id[i];
}

}  // namespace idx

size_t indexer_workspace_bytes(int bs, int64_t nc) {
    return kCounterHeaderBytes + align_up((size_t)std::max(bs, 1) * (size_t)std::max<int64_t>(nc, 1) * 4, 256);
}

int indexer_topk_launch(const void* q, const void* kv, int bf16, const float* w, int bs, int nH, int hd, int64_t nc,
                        int k, int by_id, int32_t* out_ids, float* out_scores, void* workspace,
                        size_t workspace_bytes, cudaStream_t st) {
    using namespace idx;
    if (nH < 1 || nH > kMaxHeads) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: 1..64 heads");
    if (hd < kChunk || hd % kChunk || hd > 256) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: hd % 16 == 0, <= 256");
    if (k > kMaxK) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: k <= 4096");
    if (nc > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: nc > 2^31 - 1");
    float* scores = out_scores;
    if (!scores) {
        if (!workspace || workspace_bytes < indexer_workspace_bytes(bs, nc))
            return set_error(WS_ERR_WORKSPACE, "indexer_topk: workspace missing or too small");
        scores = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterHeaderBytes);
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
    if (k > 0) {
        indexer_select_kernel<<<bs, kSelThreads, 0, st>>>(scores, nc, k, by_id, out_ids);
        e = cudaGetLastError();
        if (e != cudaSuccess) return set_error(WS_ERR_CUDA, cudaGetErrorString(e));
    }
    return WS_OK;
}

}  // namespace ws
