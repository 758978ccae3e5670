// ws_gqa_decode_noalloc: the bf16 GQA decode of ws_gqa_decode without a
// caller-supplied workspace.
//
// Who needs it: callers that can hand us their inputs and outputs but cannot
// give us any other device memory.  Typical cases are a serving process whose
// memory manager reserved the GPU's free HBM for its KV-cache pool at start-up
// (a further cudaMalloc would fail, or would have to be carved out of that
// pool, which the caller's plugin interface does not expose), and plugin or
// FFI hosts that pass only tensors across the boundary.  cudaMalloc also
// synchronises the device, which a decode loop cannot afford per step.
//
// How: the split-KV kernel's scratch (per-piece partials and the merge
// counters) lives in one file-scope __device__ array of kScratchBytes, which
// every GPU that loads this library holds until the process exits.  Its device
// address is looked up once per device with cudaGetSymbolAddress -- in host
// code the array's name only stands in for it -- on the first call made with
// that device current; make that first call before any stream capture.
//
// Rules for callers:
//   * requests whose scratch would exceed kScratchBytes are rejected with
//     WS_ERR_WORKSPACE (the message gives both sizes);
//   * every call on a device shares the one array, so calls that may overlap on
//     the GPU (different streams without ordering between them) race and give
//     wrong results -- serialise them on one stream;
//   * the merge counters are cleared with cudaMemsetAsync on the caller's
//     stream before each launch; the partials need no clearing.
// Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
#include <atomic>
#include <cstdio>

#include "common.cuh"
#include "ws_internal.h"

namespace ws {

constexpr size_t kScratchBytes = size_t(4) << 20;   // 4 MiB per device

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

// Device address of g_noalloc_scratch for the current device (nullptr on failure), looked up on the first
// call per device and kept in an atomic slot, so calls from several host threads read it safely (two threads
// racing on the first call both store the same address).  A cudaDeviceReset() discards the module and with
// it this address: a process that resets a device must not call this entry point on it afterwards.
static void* scratch_address() {
    static std::atomic<void*> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    void* ptr = cache[dev].load(std::memory_order_acquire);
    if (!ptr) {
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess) return nullptr;
        cache[dev].store(ptr, std::memory_order_release);
    }
    return ptr;
}

}  // namespace ws

using namespace ws;

extern "C" {

size_t ws_gqa_decode_noalloc_max_scratch(void) { return kScratchBytes; }

int ws_gqa_decode_noalloc(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_t,
                          int64_t v_stride_b, int64_t v_stride_t, int B_kv, int G, int Dk, int Dv, int L, float scale,
                          int out_mode, void* out, void* out_max, void* out_sum, float* out_lse, void* stream) {
    if (B_kv < 0 || G < 1 || L < 0 || Dk < 1 || Dv < 1) return set_error(WS_ERR_INVALID_ARG, "bad shape");
    if (B_kv == 0) return WS_OK;
    if (!q || !out || (L > 0 && (!k || !v))) return set_error(WS_ERR_INVALID_ARG, "null pointer");
    if (out_mode < WS_OUT_NORM_BF16 || out_mode > WS_OUT_NORM_F32) return set_error(WS_ERR_INVALID_ARG, "bad out_mode");
    if ((out_max == nullptr) != (out_sum == nullptr)) return set_error(WS_ERR_INVALID_ARG, "out_max/out_sum: both or neither");
    const size_t need = ws_gqa_decode_workspace_size(B_kv, G, Dv, L);
    if (need > kScratchBytes) {
        char buf[200];
        snprintf(buf, sizeof(buf),
                 "ws_gqa_decode_noalloc: this shape needs %zu bytes of scratch, the built-in scratch holds %zu; "
                 "use ws_gqa_decode with a workspace", need, kScratchBytes);
        return set_error(WS_ERR_WORKSPACE, buf);
    }
    void* scratch = scratch_address();
    if (!scratch) return set_error(WS_ERR_CUDA, "ws_gqa_decode_noalloc: cudaGetSymbolAddress failed");
    // the merge counters (one int per output row group) must start at zero
    const size_t counters = std::min(align_up(size_t(B_kv) * 4, 256), kCounterHeaderBytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(scratch, 0, counters, st) != cudaSuccess)
        return set_error(WS_ERR_CUDA, "ws_gqa_decode_noalloc: clearing the scratch counters failed");
    return ws_gqa_decode(q, k, v, k_stride_b, k_stride_t, v_stride_b, v_stride_t, B_kv, G, Dk, Dv, L, scale,
                         WS_DTYPE_BF16, out_mode, out, out_max, out_sum, out_lse, scratch, kScratchBytes, stream);
}

}  // extern "C"
