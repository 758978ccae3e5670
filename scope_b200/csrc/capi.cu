// extern "C" entry points of libscope_b200.so: argument checks, tensor-map
// encoding and launch.  Declarations and contracts: include/scope_b200.h.
#include <cudaTypedefs.h>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "ws_internal.h"

namespace ws {

static thread_local char g_err[512] = "";

int set_error(int code, const char* msg) {
    snprintf(g_err, sizeof(g_err), "%s", msg ? msg : "");
    return code;
}

int device_sm_count() {
    static int cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// Kernel-side failure word (bounded waits that gave up).  One per device.
__device__ int g_status_word;

int* device_status_word() {
    static int* cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    if (!cache[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_status_word) != cudaSuccess) return nullptr;
        cache[dev] = static_cast<int*>(ptr);
    }
    return cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D bf16 tensor map over a KV buffer whose element (tok, row, d) sits at
// base + tok*stride_tok + row*stride_row + d.  The box is 64 dims x box_tok
// tokens x 1 row, 128-byte swizzled; the two outer dimensions are ordered by
// increasing stride, and *tok_in_dim2 says where the token axis ended up.
int make_kv_map(CUtensorMap* map, const void* base, int64_t stride_tok, int64_t stride_row, int D, int64_t n_tok,
                int64_t n_rows, int box_tok, int* tok_in_dim2) {
    auto fn = encode_fn();
    if (!fn) return set_error(WS_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
    if (reinterpret_cast<uintptr_t>(base) % 16) return set_error(WS_ERR_INVALID_ARG, "KV base must be 16-byte aligned");
    // strides of size-1 axes are irrelevant: normalise them so that ordering works
    if (n_rows == 1) stride_row = stride_tok * n_tok;
    if (n_tok == 1) stride_tok = (n_rows == 1 ? D : stride_row * n_rows);
    if (stride_tok <= 0 || stride_row <= 0) return set_error(WS_ERR_INVALID_ARG, "KV strides must be positive");
    if ((stride_tok * 2) % 16 || (stride_row * 2) % 16)
        return set_error(WS_ERR_INVALID_ARG, "KV strides must be multiples of 8 elements (16 bytes)");
    cuuint64_t dims[3];
    cuuint64_t strides[2];
    cuuint32_t box[3];
    const cuuint32_t es[3] = {1, 1, 1};
    dims[0] = (cuuint64_t)D;
    box[0] = 64;
    if (stride_tok <= stride_row) {
        *tok_in_dim2 = 0;
        dims[1] = n_tok; dims[2] = n_rows;
        strides[0] = stride_tok * 2; strides[1] = stride_row * 2;
        box[1] = box_tok; box[2] = 1;
    } else {
        *tok_in_dim2 = 1;
        dims[1] = n_rows; dims[2] = n_tok;
        strides[0] = stride_row * 2; strides[1] = stride_tok * 2;
        box[1] = 1; box[2] = box_tok;
    }
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
        return set_error(WS_ERR_INVALID_ARG, buf);
    }
    return WS_OK;
}

}  // namespace ws

using namespace ws;

extern "C" {

const char* ws_last_error(void) { return g_err; }

int ws_version(void) { return 100; }

int ws_status_take(void* stream) {
    int* w = device_status_word();
    if (!w) return set_error(WS_ERR_CUDA, "status word unavailable");
    int h = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&h, w, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemsetAsync(w, 0, sizeof(int), st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
        return set_error(WS_ERR_CUDA, "status word read failed");
    return h == 0 ? WS_OK : WS_ERR_DEVICE;
}

size_t ws_gqa_decode_workspace_size(int B_kv, int G, int Dv, int L) {
    B_kv = std::min(B_kv, kMaxGroupsPerLaunch);   // larger calls run in chunks of rows
    G = std::min(G, kMaxHeadsPerLaunch);          // and of 16 query heads
    const int64_t tiles = (int64_t)B_kv * ((L + 63) / 64);
    const int nsm = device_sm_count();
    const int nctas = (int)std::min<int64_t>(nsm, std::max<int64_t>(tiles, 1));
    // the fp32 path (same entry, WS_DTYPE_F32) splits each row over up to 2 x SMs / rows blocks of >= 256
    // tokens, one slot of G x Dv + 2G floats each: size for that too, so its split is not cut short
    const int64_t f32_splits = std::max<int64_t>(1, std::min<int64_t>((L + 255) / 256, (2 * nsm + B_kv - 1) / B_kv));
    const size_t f32 = kCounterHeaderBytes + (size_t)B_kv * f32_splits * ((size_t)G * Dv + 2 * G) * sizeof(float);
    return std::max(gqa_workspace_bytes(G, Dv, B_kv, B_kv, nctas), f32);
}

int ws_gqa_decode(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_t,
                  int64_t v_stride_b, int64_t v_stride_t, int B_kv, int G, int Dk, int Dv, int L, float scale,
                  int dtype, int out_mode, void* out, void* out_max, void* out_sum, float* out_lse, void* workspace,
                  size_t workspace_bytes, void* stream) {
    if (B_kv < 0 || G < 1 || L < 0 || Dk < 1 || Dv < 1) return set_error(WS_ERR_INVALID_ARG, "bad shape");
    if (B_kv == 0) return WS_OK;
    if (!q || !out || (L > 0 && (!k || !v))) return set_error(WS_ERR_INVALID_ARG, "null pointer");
    if (out_mode < WS_OUT_NORM_BF16 || out_mode > WS_OUT_NORM_F32) return set_error(WS_ERR_INVALID_ARG, "bad out_mode");
    if ((out_max == nullptr) != (out_sum == nullptr)) return set_error(WS_ERR_INVALID_ARG, "out_max/out_sum: both or neither");
    if (dtype == WS_DTYPE_F32) {
        if (out_mode == WS_OUT_NORM_BF16) return set_error(WS_ERR_INVALID_ARG, "fp32 inputs cannot use WS_OUT_NORM_BF16");
        if (Dk != Dv) return set_error(WS_ERR_UNSUPPORTED, "fp32 path needs Dk == Dv");
        return gqa_f32_launch(q, k, v, k_stride_b, k_stride_t, v_stride_b, v_stride_t, B_kv, G, Dk, L, scale, out_mode,
                              out, out_max, out_sum, out_lse, workspace, workspace_bytes,
                              static_cast<cudaStream_t>(stream));
    }
    if (dtype != WS_DTYPE_BF16) return set_error(WS_ERR_INVALID_ARG, "dtype must be bf16 or fp32");
    if (B_kv > kMaxGroupsPerLaunch) {
        // rows are independent: run them in chunks that fit the counter header
        const size_t ob = out_mode == WS_OUT_NORM_BF16 ? 2 : 4;
        for (int r0 = 0; r0 < B_kv; r0 += kMaxGroupsPerLaunch) {
            const int n = std::min(kMaxGroupsPerLaunch, B_kv - r0);
            const int rc = ws_gqa_decode(
                static_cast<const uint16_t*>(q) + (int64_t)r0 * G * Dk,
                static_cast<const uint16_t*>(k) + (int64_t)r0 * k_stride_b,
                static_cast<const uint16_t*>(v) + (int64_t)r0 * v_stride_b, k_stride_b, k_stride_t, v_stride_b,
                v_stride_t, n, G, Dk, Dv, L, scale, dtype, out_mode,
                static_cast<uint8_t*>(out) + (size_t)r0 * G * Dv * ob,
                out_max ? static_cast<uint8_t*>(out_max) + (size_t)r0 * G * ob : nullptr,
                out_sum ? static_cast<uint8_t*>(out_sum) + (size_t)r0 * G * ob : nullptr,
                out_lse ? out_lse + (size_t)r0 * G : nullptr, workspace, workspace_bytes, stream);
            if (rc != WS_OK) return rc;
        }
        return WS_OK;
    }
    // more than 16 query heads per kv row: chunks of 16 heads, each a launch over the same rows (the kv rows
    // are read once per chunk); the chunks address q and the outputs through their row strides
    const size_t ob = out_mode == WS_OUT_NORM_BF16 ? 2 : 4;
    for (int g0 = 0; g0 < G; g0 += kMaxHeadsPerLaunch) {
        const int gc = std::min(kMaxHeadsPerLaunch, G - g0);
        GqaLaunch a;
        memset(&a, 0, sizeof(a));
        a.q = static_cast<const uint16_t*>(q) + (int64_t)g0 * Dk;
        a.q_row_stride = (int64_t)G * Dk;
        a.G = gc; a.Dk = Dk; a.Dv = Dv; a.scale = scale;
        a.varlen = 0;
        a.n_rows = B_kv; a.L = L;
        a.nshare = 1;
        a.shares[0].k = k; a.shares[0].v = v;
        a.shares[0].n_tok = L; a.shares[0].n_rows = B_kv;
        a.shares[0].k_stride_tok = k_stride_t; a.shares[0].k_stride_row = k_stride_b;
        a.shares[0].v_stride_tok = v_stride_t; a.shares[0].v_stride_row = v_stride_b;
        a.out_mode = out_mode;
        a.out = static_cast<uint8_t*>(out) + (size_t)g0 * Dv * ob;
        a.out_max = out_max ? static_cast<uint8_t*>(out_max) + (size_t)g0 * ob : nullptr;
        a.out_sum = out_sum ? static_cast<uint8_t*>(out_sum) + (size_t)g0 * ob : nullptr;
        a.out_lse = out_lse ? out_lse + g0 : nullptr;
        a.out_row_stride = (int64_t)G * Dv; a.ml_row_stride = G;
        a.workspace = workspace; a.workspace_bytes = workspace_bytes;
        a.status = device_status_word();
        a.stream = stream;
        const int rc = gqa_launch(a);
        if (rc != WS_OK) return rc;
    }
    return WS_OK;
}

size_t ws_gqa_decode_shares_workspace_size(int B, int Hkv, int G, int Dv, int n_shares) {
    return gqa_workspace_bytes(G, Dv, B * Hkv * n_shares, B * Hkv, device_sm_count()) + gqa_varlen_extra_bytes(B);
}

int ws_gqa_decode_shares(const void* q, int B, int Hkv, int G, int Dk, int Dv, float scale, const ws_kv_share* shares,
                         int n_shares, void* out, float* out_lse, void* workspace, size_t workspace_bytes,
                         void* stream) {
    if (B < 0 || Hkv < 1 || G < 1 || n_shares < 1 || n_shares > 4) return set_error(WS_ERR_INVALID_ARG, "bad shape");
    if (B == 0) return WS_OK;
    if (!q || !out || !shares) return set_error(WS_ERR_INVALID_ARG, "null pointer");
    GqaLaunch a;
    memset(&a, 0, sizeof(a));
    a.q = q;
    a.q_row_stride = (int64_t)G * Dk;
    a.G = G; a.Dk = Dk; a.Dv = Dv; a.scale = scale;
    a.varlen = 1;
    a.B = B; a.Hkv = Hkv;
    a.nshare = n_shares;
    for (int s = 0; s < n_shares; ++s) {
        const bool padded = shares[s].seqlens != nullptr;
        if (!padded && !shares[s].cu_seqlens)
            return set_error(WS_ERR_INVALID_ARG, "share needs cu_seqlens (packed) or seqlens (padded)");
        if (padded && shares[s].cu_seqlens)
            return set_error(WS_ERR_INVALID_ARG, "share: give cu_seqlens or seqlens, not both");
        if (shares[s].n_tok > 0 && (!shares[s].k || !shares[s].v)) return set_error(WS_ERR_INVALID_ARG, "share without k/v");
        if (shares[s].n_tok > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "share longer than 2^31 tokens");
        a.shares[s].k = shares[s].k; a.shares[s].v = shares[s].v;
        a.shares[s].cu_seqlens = shares[s].cu_seqlens;
        a.shares[s].seqlens = shares[s].seqlens;
        a.shares[s].n_tok = shares[s].n_tok; a.shares[s].n_rows = padded ? (int64_t)B * Hkv : Hkv;
        a.shares[s].k_stride_tok = shares[s].k_stride_t; a.shares[s].k_stride_row = shares[s].k_stride_h;
        a.shares[s].v_stride_tok = shares[s].v_stride_t; a.shares[s].v_stride_row = shares[s].v_stride_h;
    }
    a.out_mode = WS_OUT_NORM_BF16;
    a.out = out; a.out_max = nullptr; a.out_sum = nullptr; a.out_lse = out_lse;
    a.out_row_stride = (int64_t)G * Dv; a.ml_row_stride = G;
    a.workspace = workspace; a.workspace_bytes = workspace_bytes;
    a.status = device_status_word();
    a.stream = stream;
    return gqa_launch(a);
}

size_t ws_mla_decode_workspace_size(int B, int nH, int S) { return mla_workspace_bytes(B, nH, S); }

int ws_mla_decode(const void* q_proj, const void* q_pe, const void* c_kv, const void* k_pe, int B, int nH, int S,
                  float scale, int out_mode, void* out, float* out_max, float* out_sum, float* out_lse,
                  void* workspace, size_t workspace_bytes, void* stream) {
    if (B < 0 || nH < 1 || S < 0) return set_error(WS_ERR_INVALID_ARG, "mla_decode: bad shape");
    if (B == 0) return WS_OK;
    if (!q_proj || !q_pe || !out || (S > 0 && (!c_kv || !k_pe))) return set_error(WS_ERR_INVALID_ARG, "null pointer");
    if (out_mode < WS_OUT_NORM_BF16 || out_mode > WS_OUT_NORM_F32) return set_error(WS_ERR_INVALID_ARG, "bad out_mode");
    // a programmatic dependent launch: the decode's setup overlaps the previous grid on the stream, and it
    // waits for that grid before reading q or the latent cache
    return mla_launch(q_proj, q_pe, c_kv, k_pe, B, nH, S, scale, out_mode, out, out_max, out_sum, out_lse, workspace,
                      workspace_bytes, static_cast<cudaStream_t>(stream), /*after_primary=*/true,
                      /*kv_after_primary=*/true);
}

int ws_mla_decode_strided(const void* q_proj, const void* q_pe, const void* c_kv, int64_t c_batch_stride,
                          const void* k_pe, int64_t pe_batch_stride, int B, int nH, int S, float scale, int out_mode,
                          void* out, float* out_max, float* out_sum, float* out_lse, void* workspace,
                          size_t workspace_bytes, void* stream) {
    if (B < 0 || nH < 1 || S < 0) return set_error(WS_ERR_INVALID_ARG, "mla_decode: bad shape");
    if (B == 0) return WS_OK;
    if (!q_proj || !q_pe || !out || (S > 0 && (!c_kv || !k_pe))) return set_error(WS_ERR_INVALID_ARG, "null pointer");
    if (out_mode < WS_OUT_NORM_BF16 || out_mode > WS_OUT_NORM_F32) return set_error(WS_ERR_INVALID_ARG, "bad out_mode");
    if (c_batch_stride < 0 || pe_batch_stride < 0) return set_error(WS_ERR_INVALID_ARG, "mla_decode: negative stride");
    return mla_launch(q_proj, q_pe, c_kv, k_pe, B, nH, S, scale, out_mode, out, out_max, out_sum, out_lse, workspace,
                      workspace_bytes, static_cast<cudaStream_t>(stream), /*after_primary=*/true,
                      /*kv_after_primary=*/true, c_batch_stride, pe_batch_stride);
}

size_t ws_mla_decode_absorbed_workspace_size(int B, int nH, int S) { return mla_absorbed_workspace_bytes(B, nH, S); }

int ws_mla_decode_absorbed(const void* q_nope, const void* w_uk, int64_t w_uk_head_stride, const void* q_pe,
                           const void* c_kv, const void* k_pe, const void* w_uv, int64_t w_uv_head_stride, int B,
                           int nH, int S, int nop, int vhd, float scale, void* out, float* out_lse, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (B < 0 || nH < 1 || S < 0) return set_error(WS_ERR_INVALID_ARG, "mla_decode_absorbed: bad shape");
    if (B == 0) return WS_OK;
    if (!q_nope || !w_uk || !q_pe || !w_uv || !out || (S > 0 && (!c_kv || !k_pe)))
        return set_error(WS_ERR_INVALID_ARG, "null pointer");
    return mla_absorbed_launch(q_nope, w_uk, w_uk_head_stride, q_pe, c_kv, k_pe, w_uv, w_uv_head_stride, B, nH, S, nop,
                               vhd, scale, out, out_lse, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int ws_mla_decode_absorbed_strided(const void* q_nope, const void* w_uk, int64_t w_uk_head_stride, const void* q_pe,
                                   const void* c_kv, int64_t c_batch_stride, const void* k_pe, int64_t pe_batch_stride,
                                   const void* w_uv, int64_t w_uv_head_stride, int B, int nH, int S, int nop, int vhd,
                                   float scale, void* out, float* out_lse, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    if (B < 0 || nH < 1 || S < 0 || c_batch_stride < 0 || pe_batch_stride < 0)
        return set_error(WS_ERR_INVALID_ARG, "mla_decode_absorbed: bad shape");
    if (B == 0) return WS_OK;
    if (!q_nope || !w_uk || !q_pe || !w_uv || !out || (S > 0 && (!c_kv || !k_pe)))
        return set_error(WS_ERR_INVALID_ARG, "null pointer");
    return mla_absorbed_launch(q_nope, w_uk, w_uk_head_stride, q_pe, c_kv, k_pe, w_uv, w_uv_head_stride, B, nH, S, nop,
                               vhd, scale, out, out_lse, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                               c_batch_stride, pe_batch_stride);
}

size_t ws_csa_decode_workspace_size(int bs, int nq, int q_dtype) {
    return csa_workspace_bytes(std::max(bs, 0), std::max(nq, 1), q_dtype == WS_DTYPE_F32);
}

int ws_csa_decode(const void* q, int q_dtype, int bs, int nq, int hd, const void* kv, int kv_dtype,
                  const float* kv_scales, int64_t nc, int64_t shard_lo, const int32_t* idx, int k, int idx_mode,
                  int64_t kv_begin, int64_t kv_end, float scale, void* out, int out_dtype, float* out_lse,
                  void* workspace, size_t workspace_bytes, void* stream) {
    if (bs < 0 || nq < 1 || nc < 0 || shard_lo < 0) return set_error(WS_ERR_INVALID_ARG, "csa_decode: bad shape");
    if (hd != 512) return set_error(WS_ERR_UNSUPPORTED, "csa_decode: this build supports a 512-wide latent");
    if (q_dtype != WS_DTYPE_F32 && q_dtype != WS_DTYPE_BF16) return set_error(WS_ERR_INVALID_ARG, "csa_decode: q dtype");
    if (kv_dtype != WS_DTYPE_BF16 && kv_dtype != WS_DTYPE_I8) return set_error(WS_ERR_INVALID_ARG, "csa_decode: kv dtype");
    if (out_dtype != WS_DTYPE_F32 && out_dtype != WS_DTYPE_BF16) return set_error(WS_ERR_INVALID_ARG, "csa_decode: out dtype");
    if (idx && (k < 0 || idx_mode < WS_CSA_IDX_ALL || idx_mode > WS_CSA_IDX_SHARD))
        return set_error(WS_ERR_INVALID_ARG, "csa_decode: bad k or idx_mode");
    if (!idx && kv_end < kv_begin) return set_error(WS_ERR_INVALID_ARG, "csa_decode: kv_end < kv_begin");
    if (nc > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "csa_decode: nc > 2^31 - 1");
    if (bs == 0) return WS_OK;
    if (!q || !out || (nc > 0 && !kv) || (kv_dtype == WS_DTYPE_I8 && nc > 0 && !kv_scales))
        return set_error(WS_ERR_INVALID_ARG, "csa_decode: null pointer");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv) | reinterpret_cast<uintptr_t>(out)) % 16)
        return set_error(WS_ERR_INVALID_ARG, "csa_decode: q, kv and out must be 16-byte aligned");
    CsaLaunch a;
    memset(&a, 0, sizeof(a));
    a.q = q;
    a.q_f32 = q_dtype == WS_DTYPE_F32;
    a.bs = bs;
    a.nq = nq;
    a.kv = kv;
    a.kv_i8 = kv_dtype == WS_DTYPE_I8;
    a.kv_scales = kv_scales;
    a.nc_local = nc;
    a.shard_lo = shard_lo;
    a.idx = idx;
    a.k = idx ? k : 0;
    a.window = idx_mode;
    a.dense_begin = kv_begin;
    a.dense_end = kv_end;
    a.scale = scale;
    a.out = out;
    a.out_f32 = out_dtype == WS_DTYPE_F32;
    a.out_lse = out_lse;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes;
    a.stream = stream;
    return csa_launch(a);
}

int ws_csa_decode_qcodes(const uint8_t* q_u8, const float* q_scales, int bs, int nq, int hd, const int8_t* kv_i8,
                         const float* kv_scales, const int32_t* kv_sums, const void* kv_bf16, int64_t nc,
                         int64_t shard_lo, const int32_t* idx, int k, int idx_mode, int64_t kv_begin, int64_t kv_end,
                         float scale, void* out, int out_dtype, float* out_lse, void* workspace,
                         size_t workspace_bytes, void* stream) {
    if (bs < 0 || nq < 1 || nc < 0 || shard_lo < 0) return set_error(WS_ERR_INVALID_ARG, "csa_decode_qcodes: bad shape");
    if (hd != 512) return set_error(WS_ERR_UNSUPPORTED, "csa_decode_qcodes: this build supports a 512-wide latent");
    if (out_dtype != WS_DTYPE_F32 && out_dtype != WS_DTYPE_BF16)
        return set_error(WS_ERR_INVALID_ARG, "csa_decode_qcodes: out dtype");
    if (idx && (k < 0 || idx_mode < WS_CSA_IDX_ALL || idx_mode > WS_CSA_IDX_SHARD))
        return set_error(WS_ERR_INVALID_ARG, "csa_decode_qcodes: bad k or idx_mode");
    if (!idx && kv_end < kv_begin) return set_error(WS_ERR_INVALID_ARG, "csa_decode_qcodes: kv_end < kv_begin");
    if (nc > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "csa_decode_qcodes: nc > 2^31 - 1");
    if (bs == 0) return WS_OK;
    if (!q_u8 || !q_scales || !out || (nc > 0 && (!kv_i8 || !kv_scales || !kv_sums)))
        return set_error(WS_ERR_INVALID_ARG, "csa_decode_qcodes: null pointer");
    if ((reinterpret_cast<uintptr_t>(q_u8) | reinterpret_cast<uintptr_t>(kv_i8) | reinterpret_cast<uintptr_t>(kv_bf16) |
         reinterpret_cast<uintptr_t>(out)) % 16)
        return set_error(WS_ERR_INVALID_ARG, "csa_decode_qcodes: q_u8, kv_i8, kv_bf16 and out must be 16-byte aligned");
    CsaLaunch a;
    memset(&a, 0, sizeof(a));
    a.q = q_u8;
    a.q_u8 = 1;
    a.q_scales = q_scales;
    a.kv_sums = kv_sums;
    a.kv_val = kv_bf16;
    a.bs = bs;
    a.nq = nq;
    a.kv = kv_i8;
    a.kv_i8 = 1;
    a.kv_scales = kv_scales;
    a.nc_local = nc;
    a.shard_lo = shard_lo;
    a.idx = idx;
    a.k = idx ? k : 0;
    a.window = idx_mode;
    a.dense_begin = kv_begin;
    a.dense_end = kv_end;
    a.scale = scale;
    a.out = out;
    a.out_f32 = out_dtype == WS_DTYPE_F32;
    a.out_lse = out_lse;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes;
    a.stream = stream;
    return csa_launch(a);
}

int ws_csa_kv_quantize_s8(const void* kv, int64_t rows, int hd, void* out, float* scales, int32_t* sums,
                          void* stream) {
    if (rows < 0 || hd < 8 || hd % 8) return set_error(WS_ERR_INVALID_ARG, "csa_kv_quantize: bad shape");
    if (rows == 0) return WS_OK;
    if (!kv || !out || !scales || !sums) return set_error(WS_ERR_INVALID_ARG, "csa_kv_quantize: null pointer");
    if ((reinterpret_cast<uintptr_t>(kv) | reinterpret_cast<uintptr_t>(out)) % 16)
        return set_error(WS_ERR_INVALID_ARG, "csa_kv_quantize: kv and out must be 16-byte aligned");
    return csa_kv_quantize_launch(kv, rows, hd, out, scales, sums, static_cast<cudaStream_t>(stream));
}

int ws_csa_q_quantize_u8(const float* q, int64_t rows, int hd, void* out, float* scales, void* stream) {
    if (rows < 0 || hd < 8 || hd % 8) return set_error(WS_ERR_INVALID_ARG, "csa_q_quantize: bad shape");
    if (rows == 0) return WS_OK;
    if (!q || !out || !scales) return set_error(WS_ERR_INVALID_ARG, "csa_q_quantize: null pointer");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) % 16)
        return set_error(WS_ERR_INVALID_ARG, "csa_q_quantize: q and out must be 16-byte aligned");
    return csa_q_quantize_launch(q, rows, hd, out, scales, static_cast<cudaStream_t>(stream));
}

size_t ws_indexer_topk_workspace_size(int bs, int64_t nc) { return indexer_workspace_bytes(bs, nc); }

int ws_indexer_topk(const void* q, const void* kv, int dtype, const float* w, int bs, int nH, int hd, int64_t nc,
                    int k, int order, int32_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes,
                    void* stream) {
    if (bs < 0 || nH < 1 || hd < 1 || nc < 0 || k < 0) return set_error(WS_ERR_INVALID_ARG, "indexer_topk: bad shape");
    if (bs > 65535) return set_error(WS_ERR_UNSUPPORTED, "indexer_topk: bs > 65535");
    if (dtype != WS_DTYPE_F32 && dtype != WS_DTYPE_BF16) return set_error(WS_ERR_INVALID_ARG, "indexer_topk: dtype");
    if (order != WS_TOPK_BY_SCORE && order != WS_TOPK_BY_ID) return set_error(WS_ERR_INVALID_ARG, "indexer_topk: order");
    k = (int)std::min<int64_t>(k, nc);   // as the reference: k = min(k, nc)
    if (bs == 0 || nc == 0) return WS_OK;
    if (!q || !kv || !w || (k > 0 && !out_ids)) return set_error(WS_ERR_INVALID_ARG, "indexer_topk: null pointer");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv)) % 16)
        return set_error(WS_ERR_INVALID_ARG, "indexer_topk: q and kv must be 16-byte aligned");
    return indexer_topk_launch(q, kv, dtype == WS_DTYPE_BF16, w, bs, nH, hd, nc, k, order == WS_TOPK_BY_ID, out_ids,
                               out_scores, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int ws_kv_append(void* dst, int64_t dst_stride_row, int64_t dst_stride_tok, int64_t capacity, const void* src,
                 int64_t src_stride_row, int64_t src_stride_tok, int64_t rows, int64_t n_new, int D, int dtype,
                 int64_t t0, void* stream) {
    if (rows < 0 || n_new < 0 || D < 1 || t0 < 0 || capacity < 0) return set_error(WS_ERR_INVALID_ARG, "kv_append: bad shape");
    if (t0 + n_new > capacity) return set_error(WS_ERR_INVALID_ARG, "kv_append: the cache is full");
    const int eb = dtype == WS_DTYPE_BF16 ? 2 : dtype == WS_DTYPE_F32 ? 4 : dtype == WS_DTYPE_I8 ? 1 : 0;
    if (!eb) return set_error(WS_ERR_INVALID_ARG, "kv_append: dtype");
    if (rows == 0 || n_new == 0) return WS_OK;
    if (!dst || !src) return set_error(WS_ERR_INVALID_ARG, "kv_append: null pointer");
    if (dst_stride_row < 0 || dst_stride_tok < D || src_stride_row < 0 || src_stride_tok < 0)
        return set_error(WS_ERR_INVALID_ARG, "kv_append: bad strides");
    return kv_append_launch(dst, dst_stride_row, dst_stride_tok, src, src_stride_row, src_stride_tok, rows, n_new, D,
                            eb, t0, static_cast<cudaStream_t>(stream));
}

int ws_lse_merge(const float* o_parts, const float* lse_parts, int P, int64_t R, int D, void* out, int out_dtype,
                 float* out_lse, void* stream) {
    if (P < 1 || R < 0 || D < 1) return set_error(WS_ERR_INVALID_ARG, "bad shape");
    if (R == 0) return WS_OK;
    if (!o_parts || !lse_parts || !out) return set_error(WS_ERR_INVALID_ARG, "null pointer");
    if (out_dtype != WS_DTYPE_BF16 && out_dtype != WS_DTYPE_F32) return set_error(WS_ERR_INVALID_ARG, "bad out dtype");
    return lse_merge_launch(o_parts, R * D, lse_parts, R, P, R, D, out, out_dtype, out_lse,
                            static_cast<cudaStream_t>(stream));
}

int ws_lse_merge_strided(const float* o_parts, int64_t o_part_stride, const float* lse_parts,
                         int64_t lse_part_stride, int P, int64_t R, int D, void* out, int out_dtype, float* out_lse,
                         void* stream) {
    if (P < 1 || R < 0 || D < 1) return set_error(WS_ERR_INVALID_ARG, "bad shape");
    if (o_part_stride < R * D || lse_part_stride < R) return set_error(WS_ERR_INVALID_ARG, "part strides too small");
    if (R == 0) return WS_OK;
    if (!o_parts || !lse_parts || !out) return set_error(WS_ERR_INVALID_ARG, "null pointer");
    if (out_dtype != WS_DTYPE_BF16 && out_dtype != WS_DTYPE_F32) return set_error(WS_ERR_INVALID_ARG, "bad out dtype");
    return lse_merge_launch(o_parts, o_part_stride, lse_parts, lse_part_stride, P, R, D, out, out_dtype, out_lse,
                            static_cast<cudaStream_t>(stream));
}

}  // extern "C"
