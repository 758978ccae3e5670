// Per-row quantisers of the CSA int8 family, bit-exact with the reference:
//   kv_quantize_bf16_to_int8 (kernel/cpu_attn_ds4_ext/csa_attn.cpp:1203-1233,
//   row kernel quantize_bf16_to_s8 :729-764) and q_quantize_fp32_to_u8
//   (:1175-1201, row kernel :704-727).
// Per row: maxv = max(max |x|, 1e-6); scale = maxv * (1/127) (the reference
// is built with -ffast-math, which turns maxv / 127 into that product);
// inv = 127 / maxv (IEEE division); q = rne(x * inv), saturated to int8, or
// rne(x * inv) + 128 saturated to uint8.  The int8 form also returns the
// row sum of the quantised values (int32).
// One warp per row, 8 elements per lane per step (rows up to 512 wide are held
// in registers and read once); HBM-bound.
#include "common.cuh"
#include "ws_internal.h"

namespace ws {
namespace {

constexpr int kRowsPerBlock = 8;   // one warp per row

__device__ __forceinline__ float row_scale_inv(float maxv, float* scale) {
    maxv = fmaxf(maxv, 1e-6f);
    *scale = __fmul_rn(maxv, 1.0f / 127.0f);
    return __fdiv_rn(127.0f, maxv);
}

__global__ void __launch_bounds__(32 * kRowsPerBlock) kv_quant_s8_kernel(const __nv_bfloat16* __restrict__ kv,
                                                                        int64_t rows, int hd, int8_t* __restrict__ out,
                                                                        float* __restrict__ scales,
                                                                        int32_t* __restrict__ sums) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
    if (row >= rows) return;
    const __nv_bfloat16* x = kv + row * hd;
    auto absmax8 = [](const uint4& v, float m) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float2 f = __bfloat1622float2(h[u]);
            m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
        return m;
    };
    auto quant8 = [&](const uint4& v, float inv, int d, int32_t& sum) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float2 f = __bfloat1622float2(h[u]);
            const int a = max(-128, min(127, __float2int_rn(__fmul_rn(f.x, inv))));
            const int b = max(-128, min(127, __float2int_rn(__fmul_rn(f.y, inv))));
            sum += a + b;
            packed[u >> 1] |= ((uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8)) << ((u & 1) * 16);
        }
        *reinterpret_cast<uint2*>(out + row * hd + d) = make_uint2(packed[0], packed[1]);
    };
    float maxv = 0.f, sc, inv;
    int32_t sum = 0;
    if (hd <= 512) {
        // the row stays in registers: two 16-byte loads per lane, issued together, read once
        const int d0 = lane * 8, d1 = lane * 8 + 256;
        const uint4 v0 = d0 < hd ? __ldg(reinterpret_cast<const uint4*>(x + d0)) : make_uint4(0, 0, 0, 0);
        const uint4 v1 = d1 < hd ? __ldg(reinterpret_cast<const uint4*>(x + d1)) : make_uint4(0, 0, 0, 0);
        maxv = absmax8(v1, absmax8(v0, 0.f));   // zero padding leaves the max unchanged
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) maxv = fmaxf(maxv, __shfl_xor_sync(0xffffffffu, maxv, o));
        inv = row_scale_inv(maxv, &sc);
        if (d0 < hd) quant8(v0, inv, d0, sum);
        if (d1 < hd) quant8(v1, inv, d1, sum);
    } else {
        for (int d = lane * 8; d < hd; d += 256) maxv = absmax8(__ldg(reinterpret_cast<const uint4*>(x + d)), maxv);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) maxv = fmaxf(maxv, __shfl_xor_sync(0xffffffffu, maxv, o));
        inv = row_scale_inv(maxv, &sc);
        for (int d = lane * 8; d < hd; d += 256) quant8(__ldg(reinterpret_cast<const uint4*>(x + d)), inv, d, sum);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
        scales[row] = sc;
        sums[row] = sum;
    }
}

__global__ void __launch_bounds__(32 * kRowsPerBlock) q_quant_u8_kernel(const float* __restrict__ q, int64_t rows,
                                                                       int hd, uint8_t* __restrict__ out,
                                                                       float* __restrict__ scales) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float* x = q + row * hd;
    float maxv = 0.f;
    for (int d = lane * 8; d < hd; d += 256) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(x + d));
        const float4 b = __ldg(reinterpret_cast<const float4*>(x + d + 4));
        maxv = fmaxf(maxv, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
        maxv = fmaxf(maxv, fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) maxv = fmaxf(maxv, __shfl_xor_sync(0xffffffffu, maxv, o));
    float sc;
    const float inv = row_scale_inv(maxv, &sc);
    for (int d = lane * 8; d < hd; d += 256) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(x + d));
        const float4 b = __ldg(reinterpret_cast<const float4*>(x + d + 4));
        const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int v = max(0, min(255, __float2int_rn(__fmul_rn(f[u], inv)) + 128));
            packed[u >> 2] |= (uint32_t)v << ((u & 3) * 8);
        }
        *reinterpret_cast<uint2*>(out + row * hd + d) = make_uint2(packed[0], packed[1]);
    }
    if (lane == 0) scales[row] = sc;
}

}  // namespace

int csa_kv_quantize_launch(const void* kv, int64_t rows, int hd, void* out, float* scales, int32_t* sums,
                           cudaStream_t st) {
    if (rows == 0) return WS_OK;
    const unsigned grid = (unsigned)((rows + kRowsPerBlock - 1) / kRowsPerBlock);
    kv_quant_s8_kernel<<<grid, 32 * kRowsPerBlock, 0, st>>>(static_cast<const __nv_bfloat16*>(kv), rows, hd,
                                                             static_cast<int8_t*>(out), scales, sums);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

int csa_q_quantize_launch(const float* q, int64_t rows, int hd, void* out, float* scales, cudaStream_t st) {
    if (rows == 0) return WS_OK;
    const unsigned grid = (unsigned)((rows + kRowsPerBlock - 1) / kRowsPerBlock);
    q_quant_u8_kernel<<<grid, 32 * kRowsPerBlock, 0, st>>>(q, rows, hd, static_cast<uint8_t*>(out), scales);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace ws
