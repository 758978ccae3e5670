// Log-sum-exp merge of P partial attention results.
//
// The cross-GPU combine of a sequence-sharded KV cache, and the GPU form of
// the runtime merges of the reference (system/qwenoffload.py:1606-1617,
// system/mixoffload.py:1456-1464, system/deepseek.py:397-404):
//   M = max_p lse_p ;  L = M + log(sum_p exp(lse_p - M)) ;
//   o = sum_p exp(lse_p - L) * o_p
// One warp per output row; o_p rows are read with 16-byte loads when D % 4 == 0.
#include "common.cuh"
#include "ws_internal.h"

namespace ws {

// Partial p's o rows start at o_parts + p * os, its lse values at lse_parts + p * ls.
template <bool VEC>
__global__ void lse_merge_kernel(const float* __restrict__ o_parts, int64_t os, const float* __restrict__ lse_parts,
                                 int64_t ls, int P, int64_t R, int D, void* __restrict__ out, int out_dtype,
                                 float* __restrict__ out_lse) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= R) return;
    float M = -INFINITY;
    for (int p = 0; p < P; ++p) M = fmaxf(M, __ldg(lse_parts + (int64_t)p * ls + row));
    float S = 0.f;
    if (M != -INFINITY)
        for (int p = 0; p < P; ++p) S += ex2((__ldg(lse_parts + (int64_t)p * ls + row) - M) * kLog2e);
    const float L = (M == -INFINITY) ? -INFINITY : M + logf(S);
    if (VEC) {
        for (int d = lane * 4; d < D; d += 128) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (M != -INFINITY)
                for (int p = 0; p < P; ++p) {
                    const float w = ex2((__ldg(lse_parts + (int64_t)p * ls + row) - L) * kLog2e);
                    if (w == 0.f) continue;
                    const float4 v = __ldg(reinterpret_cast<const float4*>(o_parts + (int64_t)p * os + row * D + d));
                    acc.x += w * v.x; acc.y += w * v.y; acc.z += w * v.z; acc.w += w * v.w;
                }
            if (out_dtype == WS_DTYPE_F32) {
                *reinterpret_cast<float4*>(static_cast<float*>(out) + row * D + d) = acc;
            } else {
                __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
                __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out) + row * D + d;
                *reinterpret_cast<__nv_bfloat162*>(o) = lo;
                *reinterpret_cast<__nv_bfloat162*>(o + 2) = hi;
            }
        }
    } else {
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
    }
    if (lane == 0 && out_lse) out_lse[row] = L;
}

int lse_merge_launch(const float* o_parts, int64_t os, const float* lse_parts, int64_t ls, int P, int64_t R, int D,
                     void* out, int out_dtype, float* out_lse, cudaStream_t st) {
    const int warps = 8;
    const int64_t blocks = (R + warps - 1) / warps;
    if (blocks > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "lse_merge: too many rows");
    const bool vec = (D % 4 == 0) && (os % 4 == 0) && (reinterpret_cast<uintptr_t>(o_parts) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(out) % (out_dtype == WS_DTYPE_F32 ? 16 : 8) == 0);
    if (vec)
        lse_merge_kernel<true><<<(unsigned)blocks, warps * 32, 0, st>>>(o_parts, os, lse_parts, ls, P, R, D, out,
                                                                          out_dtype, out_lse);
    else
        lse_merge_kernel<false><<<(unsigned)blocks, warps * 32, 0, st>>>(o_parts, os, lse_parts, ls, P, R, D, out,
                                                                           out_dtype, out_lse);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace ws
