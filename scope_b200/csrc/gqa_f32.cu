// fp32 GQA decode on the CUDA cores.
//
// The fp32 branch of fused_cpu_attn (kernel/cpu_attn.cpp:620-629, run_kernel
// <false,false>) and the scalar ablation fused_cpu_attn_fp32
// (kernel/cpu_attn.cpp:674-848).  fp32 operands are kept in fp32 end to end
// (tf32 tensor cores would not meet the 1e-3 LSE bar), so this path is
// FMA-bound rather than HBM-bound; it exists for API completeness.
//
// Grid (B_kv, splits).  Each block takes a contiguous token range of one row;
// its 4 warps interleave tokens, lanes own head dims.  Warp states are merged
// in shared memory; when a row has several splits the block that files the
// last split (atomic ticket) merges them.
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
    const int64_t oi = ((int64_t)row * p.G + g) * p.D + d;
    float* out = static_cast<float*>(p.out);
    out[oi] = empty ? 0.f : (p.out_mode == WS_OUT_UNNORM_F32 ? o_un : o_un / l);
    if (d == 0) {
        const int64_t mi = (int64_t)row * p.G + g;
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
            qr[g][i] = (g < p.G && d < p.D) ? p.q[((int64_t)row * p.G + g) * p.D + d] : 0.f;
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

int gqa_f32_launch(const void* q, const void* k, const void* v, int64_t k_sb, int64_t k_st, int64_t v_sb,
                      int64_t v_st, int B_kv, int G, int D, int L, float scale, int out_mode, void* out,
                      void* out_max, void* out_sum, float* out_lse, void* workspace, size_t workspace_bytes,
                      cudaStream_t st) {
    if (G > kF32MaxG) return set_error(WS_ERR_UNSUPPORTED, "fp32 path: groups must be <= 16");
    if (D > 32 * kF32MaxDPerLane) return set_error(WS_ERR_UNSUPPORTED, "fp32 path: head_dim must be <= 256");
    F32Params p;
    p.q = static_cast<const float*>(q);
    p.k = static_cast<const float*>(k);
    p.v = static_cast<const float*>(v);
    p.k_sb = k_sb; p.k_st = k_st; p.v_sb = v_sb; p.v_st = v_st;
    p.G = G; p.D = D; p.L = L; p.scale = scale; p.out_mode = out_mode;
    p.out = out; p.out_max = out_max; p.out_sum = out_sum; p.out_lse = out_lse;
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
    p.splits = splits;
    p.ws_cnt = static_cast<int*>(workspace);
    p.ws_part = workspace ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + cnt_bytes) : nullptr;
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
