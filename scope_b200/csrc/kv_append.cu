// Append new tokens to a device-resident KV cache: the write side of the
// physically partitioned cache (the reference's InplaceKVCache.append_4d,
// system/qwenoffload.py:97-122, and InplaceKVCacheCompressed.append,
// system/deepseek.py:171-194, which copy into pinned host buffers).
//   dst element (row, t0 + i, d) at dst + row * dst_row + (t0 + i) * dst_tok + d
//   src element (row, i, d)      at src + row * src_row + i * src_tok + d
// for row < rows, i < n_new, d < D (strides in elements).  One warp per
// (row, token), 16-byte copies when every address and D allow it.  HBM-bound.
#include "common.cuh"
#include "ws_internal.h"

namespace ws {
namespace {

template <bool VEC>
__global__ void kv_append_kernel(uint8_t* __restrict__ dst, int64_t dst_row, int64_t dst_tok,
                                 const uint8_t* __restrict__ src, int64_t src_row, int64_t src_tok, int64_t rows,
                                 int64_t n_new, int64_t row_bytes, int64_t t0) {
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);   // (row, token) pair
    const int lane = threadIdx.x & 31;
    if (item >= rows * n_new) return;
    const int64_t row = item / n_new, i = item - row * n_new;
    uint8_t* d = dst + row * dst_row + (t0 + i) * dst_tok;
    const uint8_t* s = src + row * src_row + i * src_tok;
    if (VEC) {
        for (int64_t b = (int64_t)lane * 16; b < row_bytes; b += 32 * 16)
            *reinterpret_cast<uint4*>(d + b) = __ldg(reinterpret_cast<const uint4*>(s + b));
    } else {
        for (int64_t b = lane; b < row_bytes; b += 32) d[b] = s[b];
    }
}

}  // namespace

int kv_append_launch(void* dst, int64_t dst_row, int64_t dst_tok, const void* src, int64_t src_row, int64_t src_tok,
                     int64_t rows, int64_t n_new, int D, int elem_bytes, int64_t t0, cudaStream_t st) {
    if (rows == 0 || n_new == 0) return WS_OK;
    const int64_t eb = elem_bytes;
    const int64_t row_bytes = (int64_t)D * eb;
    const bool vec = row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(dst) % 16) == 0 &&
                     (reinterpret_cast<uintptr_t>(src) % 16) == 0 && (dst_row * eb) % 16 == 0 &&
                     (dst_tok * eb) % 16 == 0 && (src_row * eb) % 16 == 0 && (src_tok * eb) % 16 == 0 &&
                     (t0 * dst_tok * eb) % 16 == 0;
    const int warps = 8;
    const int64_t blocks = (rows * n_new + warps - 1) / warps;
    if (blocks > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "kv_append: too many rows");
    auto kfn = vec ? kv_append_kernel<true> : kv_append_kernel<false>;
    kfn<<<(unsigned)blocks, warps * 32, 0, st>>>(static_cast<uint8_t*>(dst), dst_row * eb, dst_tok * eb,
                                                  static_cast<const uint8_t*>(src), src_row * eb, src_tok * eb, rows,
                                                  n_new, row_bytes, t0);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace ws
