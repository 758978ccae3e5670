// Log-sum-exp merge of P partial attention results.
//
// The cross-GPU combine of a sequence-sharded KV cache, the combine of a CSA
// decode split over several CTAs, and the GPU form of the runtime merges of
// the reference (system/qwenoffload.py:1606-1617, system/mixoffload.py:1456-1464,
// system/deepseek.py:397-404):
//   M = max_p lse_p ;  L = M + log(sum_p exp(lse_p - M)) ;
//   o = sum_p exp(lse_p - L) * o_p
// A partial whose lse is -inf has weight 0 and its o row is never read.
#include "common.cuh"
#include "ws_internal.h"

namespace ws {
namespace {

// P <= PB (8, 16 or 32), D % 4 == 0: one warp per (row, 128-column chunk).  Lane p holds partial p's
// log-sum-exp; every partial's 16-byte load of the lane's four columns is issued together with them,
// so the merge costs one round trip to memory.
template <bool PDL, int PB>
__global__ void lse_merge_vec_kernel(const float* __restrict__ o_parts, int64_t os, const float* __restrict__ lse_parts,
                                     int64_t ls, int P, int64_t R, int D, void* __restrict__ out, int out_dtype,
                                     float* __restrict__ out_lse) {
    if (PDL) pdl_wait_primary();   // the partials are written by the previous grid
    const int nchunk = (D + 127) / 128;
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (item >= R * nchunk) return;
    const int64_t row = item / nchunk;
    const int chunk = (int)(item - row * nchunk);
    const int d = chunk * 128 + lane * 4;
    const bool dv = d < D;
    float4 v[PB];
#pragma unroll
    for (int u = 0; u < PB; ++u)
        v[u] = (u < P && dv) ? __ldg(reinterpret_cast<const float4*>(o_parts + (int64_t)u * os + row * D + d))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
    const float lp = lane < P ? __ldg(lse_parts + (int64_t)lane * ls + row) : -INFINITY;
    float M = lp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float e = (M == -INFINITY || lp == -INFINITY) ? 0.f : ex2((lp - M) * kLog2e);
    float S = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    const float w = S > 0.f ? e / S : 0.f;   // exp(lse_p - L); 0 for an empty partial, whose o is never used
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < PB; ++u) {
        const float wu = __shfl_sync(0xffffffffu, w, u & 31);
        if (wu != 0.f) {   // an empty partial may hold anything (even NaN): skip it
            acc.x = fmaf(wu, v[u].x, acc.x); acc.y = fmaf(wu, v[u].y, acc.y);
            acc.z = fmaf(wu, v[u].z, acc.z); acc.w = fmaf(wu, v[u].w, acc.w);
        }
    }
    if (dv) {
        if (out_dtype == WS_DTYPE_F32) {
            *reinterpret_cast<float4*>(static_cast<float*>(out) + row * D + d) = acc;
        } else {
            __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out) + row * D + d;
            *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(acc.x, acc.y);
            *reinterpret_cast<__nv_bfloat162*>(o + 2) = __floats2bfloat162_rn(acc.z, acc.w);
        }
    }
    if (lane == 0 && chunk == 0 && out_lse) out_lse[row] = (S > 0.f) ? M + logf(S) : -INFINITY;
}

// Any P and D: one warp per row, partials in sequence.
template <bool PDL>
__global__ void lse_merge_kernel(const float* __restrict__ o_parts, int64_t os, const float* __restrict__ lse_parts,
                                 int64_t ls, int P, int64_t R, int D, void* __restrict__ out, int out_dtype,
                                 float* __restrict__ out_lse) {
    if (PDL) pdl_wait_primary();
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= R) return;
    float M = -INFINITY;
    for (int p = 0; p < P; ++p) M = fmaxf(M, __ldg(lse_parts + (int64_t)p * ls + row));
    float S = 0.f;
    if (M != -INFINITY)
        for (int p = 0; p < P; ++p) S += ex2((__ldg(lse_parts + (int64_t)p * ls + row) - M) * kLog2e);
    const float L = (M == -INFINITY) ? -INFINITY : M + logf(S);
    for (int d = lane; d < D; d += 32) {
        float acc = 0.f;
        if (M != -INFINITY)
            for (int p = 0; p < P; ++p) {
                const float w = ex2((__ldg(lse_parts + (int64_t)p * ls + row) - L) * kLog2e);
                if (w == 0.f) continue;
                acc += w * __ldg(o_parts + (int64_t)p * os + row * D + d);
            }
        if (out_dtype == WS_DTYPE_F32) static_cast<float*>(out)[row * D + d] = acc;
        else static_cast<__nv_bfloat16*>(out)[row * D + d] = __float2bfloat16_rn(acc);
    }
    if (lane == 0 && out_lse) out_lse[row] = L;
}

}  // namespace

// Partial p's o rows start at o_parts + p * os, its lse values at lse_parts + p * ls.
int lse_merge_launch(const float* o_parts, int64_t os, const float* lse_parts, int64_t ls, int P, int64_t R, int D,
                     void* out, int out_dtype, float* out_lse, cudaStream_t st, bool after_primary) {
    if (R == 0) return WS_OK;
    const int warps = 4;   // small blocks: the whole grid of a decode-sized merge is resident at once
    const bool vec = P <= 32 && (D % 4 == 0) && (os % 4 == 0) && (reinterpret_cast<uintptr_t>(o_parts) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(out) % (out_dtype == WS_DTYPE_F32 ? 16 : 8) == 0);
    const int64_t items = vec ? R * ((D + 127) / 128) : R;
    const int64_t blocks = (items + warps - 1) / warps;
    if (blocks > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "lse_merge: too many rows");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(warps * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = after_primary ? 1 : 0;
    cudaError_t e;
    if (vec) {
        auto kv = after_primary ? (P <= 8 ? lse_merge_vec_kernel<true, 8>
                                          : P <= 16 ? lse_merge_vec_kernel<true, 16> : lse_merge_vec_kernel<true, 32>)
                                : (P <= 8 ? lse_merge_vec_kernel<false, 8>
                                          : P <= 16 ? lse_merge_vec_kernel<false, 16> : lse_merge_vec_kernel<false, 32>);
        e = cudaLaunchKernelEx(&cfg, kv, o_parts, os, lse_parts, ls, P, R, D, out, out_dtype, out_lse);
    } else
        e = after_primary ? cudaLaunchKernelEx(&cfg, lse_merge_kernel<true>, o_parts, os, lse_parts, ls, P, R, D, out,
                                               out_dtype, out_lse)
                          : cudaLaunchKernelEx(&cfg, lse_merge_kernel<false>, o_parts, os, lse_parts, ls, P, R, D, out,
                                               out_dtype, out_lse);
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace ws
