// Exchange of sequence-shard partials over NVLink peer memory: the root-gather
// form (peer_push_kernel / peer_merge_kernel) and, further down, the
// scatter-merge form (rs_scatter_kernel / rs_merge_kernel).
//
// The reference's runtimes merge the partials of their KV shares on the host
// (system/qwenoffload.py:1606-1617, system/mixoffload.py:1456-1464); across
// GPUs of one box the merge input is each rank's (o fp32, lse fp32) block.
// Instead of an all_gather collective, rank 0's buffer is mapped into every
// rank's address space with CUDA IPC, and per step:
//   * every rank's decode writes its block: rank 0 straight into its own slot,
//     the other ranks into a local block;
//   * ranks 1..N-1 run peer_push_kernel: wait (bounded) until rank 0 has merged
//     the previous step (its slot is free again), copy the block into rank 0's
//     slot with 16-byte stores over NVLink, fence at system scope, and the CTA
//     that takes the last ticket stores this step's epoch into rank 0's flag
//     word for the rank with release semantics;
//   * rank 0 runs peer_merge_kernel: each CTA waits (bounded, acquire loads)
//     for every rank's flag to reach the epoch, merges its rows by log-sum-exp
//     from the slots, and the CTA that takes the last ticket publishes the
//     epoch as consumed.
// The epochs live on the devices -- each rank's push counts its own steps in
// its state word, rank 0's merge counts through `consumed` -- and every
// pointer is fixed, so a captured CUDA graph may replay the steps.  Both
// kernels are programmatic dependent launches: their polls of the other
// ranks' words run while the decode before them drains.
// Buffer layout (rank 0's allocation): a 1 KB control block -- flags[64]
// (int64, one per rank), consumed (int64), the merge's CTA ticket (int32), the
// last epoch whose merge gave up (int64) -- then `world` slots of slot_floats
// floats each, slot r holding o [rows, dim] then lse [rows].
// Every wait gives up after kWaitNs, records kDevTimeout in the status word
// and skips its work; the exchange is then unusable and must be rebuilt.
// No cluster multicast and no multimem: plain stores and loads only.
#include <cstdio>
#include <type_traits>

#include "common.cuh"
#include "ws_internal.h"

namespace ws {
namespace peer {

constexpr int kMaxRanks = 64;
constexpr size_t kCtrlBytes = 1024;
constexpr int kConsumed = kMaxRanks;            // int64 index of the consumed word
constexpr int kTicketByte = (kMaxRanks + 1) * 8;
constexpr int kFailed = kMaxRanks + 2;          // int64 index: the last epoch a merge CTA gave up in
constexpr uint64_t kWaitNs = 2000000000ull;     // 2 s
constexpr int kRowsPerCta = 8;                  // one warp per row

__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
    asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
    int64_t v;
    asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// A launch that may start while the previous grid on the stream drains (programmatic stream serialization);
// the kernel calls griddepcontrol.wait before it reads anything that grid writes.
inline void pdl_config(cudaLaunchConfig_t& cfg, cudaLaunchAttribute (&attr)[1], dim3 grid, dim3 block,
                       cudaStream_t st) {
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
}

// slot floats: o [rows, dim] + lse [rows], rounded up to 64 floats (256 bytes) so every slot and its o
// block start 16-byte aligned
inline int64_t slot_floats(int64_t rows, int dim) { return (int64_t)align_up((size_t)(rows * dim + rows), 64); }

// Ranks > 0, one launch per step: wait until rank 0 has consumed the previous step (the slot is free), copy
// this rank's block (written locally by its decode) into rank 0's slot with 16-byte stores spread over the
// grid, then the CTA that takes the last ticket advances this rank's epoch and publishes it as the rank's
// flag (not when a CTA gave up waiting).  state: [0] this rank's epoch (int64), [1] the CTA ticket and the
// last epoch a CTA gave up in (int32 each).  Keeping the decode's own stores
// local matters: its merge tickets fence every prior store, and a fence behind stores to another GPU waits
// for the NVLink round trip.
__global__ void __launch_bounds__(256) peer_push_kernel(const float4* __restrict__ src, float4* dst, int64_t n16,
                                                        int64_t* root_ctrl, int64_t* state, int rank, int* status) {
    __shared__ int s_go;
    int* ticket = reinterpret_cast<int*>(state + 1);   // [0] the CTA ticket, [1] the last step a CTA gave up in
    // A programmatic dependent of the decode: the wait for rank 0 to free the slot (a read over NVLink) runs
    // while the decode finishes.  The step count read before griddepcontrol.wait is a guess (a previous push
    // may still be in flight when the grid before this one started early); it is read again after the wait
    // and the slot wait repeated if it changed.
    const int64_t guess = *reinterpret_cast<volatile int64_t*>(state) + 1;
    auto slot_free = [&](int64_t e, uint64_t t0) {
        while (ld_acquire_sys(root_ctrl + kConsumed) < e - 1) {
            if (globaltimer_ns() - t0 > kWaitNs) {
                atomicExch(status, kDevTimeout);
                atomicExch(ticket + 1, (int)e);
                return 0;
            }
            __nanosleep(128);
        }
        return 1;
    };
    int go = 1;
    const uint64_t t0 = globaltimer_ns();
    if (threadIdx.x == 0) go = slot_free(guess, t0);
    pdl_wait_primary();   // the decode's block (and every grid before it) is complete
    // the last CTA advances the count only after every CTA has read it
    const int64_t epoch = *reinterpret_cast<volatile int64_t*>(state) + 1;
    if (threadIdx.x == 0) {
        if (go && epoch != guess) go = slot_free(epoch, t0);
        else if (!go) atomicExch(ticket + 1, (int)epoch);
        s_go = go;
    }
    __syncthreads();
    if (s_go) {   // four 16-byte loads in flight per thread, then their stores
        const int64_t nth = (int64_t)gridDim.x * blockDim.x;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += 4 * nth) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i + u * nth < n16) v[u] = __ldcg(src + i + u * nth);
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i + u * nth < n16) dst[i + u * nth] = v[u];
        }
    }
    __threadfence_system();   // every thread's copies are performed before its CTA takes the ticket
    __syncthreads();
    if (threadIdx.x != 0) return;
    if (atomicAdd(ticket, 1) != (int)gridDim.x - 1) return;
    atomicExch(ticket, 0);
    state[0] = epoch;   // advanced even after a failed wait, so the ranks' step counts stay in line
    if (atomicAdd(ticket + 1, 0) == (int)epoch) return;   // a CTA gave up: its share was not copied
    __threadfence_system();
    st_release_sys(root_ctrl + rank, epoch);
}

template <bool OUT_BF16>
__global__ void __launch_bounds__(32 * kRowsPerCta) peer_merge_kernel(const float* __restrict__ slots,
                                                                      int64_t slot_stride, int P, int64_t R, int D,
                                                                      int64_t* ctrl, void* out, float* out_lse,
                                                                      int* status) {
    __shared__ int s_ok;
    // A programmatic dependent of rank 0's decode: the waits for the other ranks' flags run while that decode
    // finishes; its own slot is read only after griddepcontrol.wait.  This step's epoch is one past the last
    // consumed one (the last CTA advances `consumed` only after every CTA has read it); the value read before
    // the wait is a guess, read again after it, and the flag waits are repeated if it changed.
    const int64_t guess = *reinterpret_cast<volatile int64_t*>(ctrl + kConsumed) + 1;
    auto flags_up = [&](int64_t e, uint64_t t0) {
        for (int r = 1; r < P; ++r) {
            while (ld_acquire_sys(ctrl + r) < e) {
                if (globaltimer_ns() - t0 > kWaitNs) {
                    atomicExch(status, kDevTimeout);
                    atomicExch(reinterpret_cast<unsigned long long*>(ctrl + kFailed), (unsigned long long)e);
                    return 0;
                }
                __nanosleep(64);
            }
        }
        return 1;
    };
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    if (threadIdx.x == 0) ok = flags_up(guess, t0);
    pdl_wait_primary();
    const int64_t epoch = *reinterpret_cast<volatile int64_t*>(ctrl + kConsumed) + 1;
    if (threadIdx.x == 0) {
        if (ok && epoch != guess) ok = flags_up(epoch, t0);
        else if (!ok) atomicExch(reinterpret_cast<unsigned long long*>(ctrl + kFailed), (unsigned long long)epoch);
        s_ok = ok;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + warp;
    if (s_ok && row < R) {
        // lane p < P holds partial p's lse (P <= 32); the weights follow from the row's log-sum-exp
        const float lp = lane < P ? __ldcg(slots + lane * slot_stride + R * D + row) : -INFINITY;
        float M = lp;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float w = (M == -INFINITY || lp == -INFINITY) ? 0.f : expf(lp - M);
        float s = w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float lse = M == -INFINITY ? -INFINITY : M + logf(s);
        const float wp = M == -INFINITY ? 0.f : w / s;   // exp(lp - lse)
        for (int c = lane * 4; c < D; c += 128) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p0 = 0; p0 < P; p0 += 8) {   // eight partials' loads in flight, then their sums
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (p0 + u < P)
                        v[u] = __ldcg(reinterpret_cast<const float4*>(slots + (p0 + u) * slot_stride + row * D + c));
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const float e = __shfl_sync(0xffffffffu, wp, (p0 + u) & 31);
                    if (p0 + u >= P || e == 0.f) continue;   // an empty partial may hold anything: skipped
                    acc.x = fmaf(e, v[u].x, acc.x);
                    acc.y = fmaf(e, v[u].y, acc.y);
                    acc.z = fmaf(e, v[u].z, acc.z);
                    acc.w = fmaf(e, v[u].w, acc.w);
                }
            }
            if (OUT_BF16) {
                uint2 pk = make_uint2(pack_bf16(acc.x, acc.y), pack_bf16(acc.z, acc.w));
                *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + row * D + c) = pk;
            } else {
                *reinterpret_cast<float4*>(static_cast<float*>(out) + row * D + c) = acc;
            }
        }
        if (lane == 0 && out_lse) out_lse[row] = lse;
    }
    // the last CTA to finish publishes the epoch as consumed (its slots may be overwritten from now on)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        int* ticket = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ctrl) + kTicketByte);
        if (atomicAdd(ticket, 1) == (int)gridDim.x - 1) {
            atomicExch(ticket, 0);
            // publish only when no CTA of this launch gave up waiting
            if (atomicAdd(reinterpret_cast<unsigned long long*>(ctrl + kFailed), 0ull) != (unsigned long long)epoch) {
                __threadfence_system();
                st_release_sys(ctrl + kConsumed, epoch);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------------
// Scatter-merge form.  Gathering every block on rank 0 puts world - 1 blocks through rank 0's inbound links;
// here every rank owns one contiguous share of the rows and merges it, so each rank sends and receives
// (world - 1) / world of one block, and only the merged shares (out dtype, no lse weights) go to rank 0.
// Every rank allocates a buffer of ws_peer_rs_bytes and maps every other rank's:
//   control block (2 KB, int64 words): flags[64] -- flag[r] = the last step rank r scattered into this
//   buffer; gflags[64] (rank 0's buffer) -- gflag[q] = the last step rank q stored its merged share;
//   consumed -- the last step whose slots this rank's merge has read; gconsumed (rank 0's buffer) -- the
//   last step whose gathered shares rank 0 has copied out; the merge's CTA ticket; the last step a merge
//   CTA gave up in.
//   then `world` slots: slot r holds rank r's partial of this rank's share, o [share, dim] then lse [share];
//   then the gather area (used in rank 0's buffer): out [rows, dim] in the out dtype, lse [rows] at a fixed
//   offset of rows * dim floats.
// Per step, every rank: rs_scatter_kernel (wait until each peer has read the previous step's slot, copy
// the peer's rows of this rank's block into it, release flag[rank] in the peer's buffer), then
// rs_merge_kernel (wait for every flag, merge this rank's share from the slots and its own block; rank 0
// writes its rows to out, the others store theirs in rank 0's gather area and release their gflag after
// a bounded wait for rank 0 to have copied out the previous step; rank 0 then waits for every gflag and
// copies the gathered rows to out).
namespace rs {

constexpr size_t kCtrl = 2048;
constexpr int kFlags = 0, kGFlags = 64, kConsumedW = 128, kGConsumed = 129, kTicketW = 130, kFailedW = 131;

__host__ __device__ inline int64_t share_lo(int64_t rows, int world, int q) { return rows * q / world; }
__host__ __device__ inline int64_t slot_floats(int64_t rows, int world, int dim) {
    const int64_t sm = (rows + world - 1) / world;   // the largest share
    return (sm * dim + sm + 63) / 64 * 64;
}
__host__ __device__ inline int64_t area_offset(int64_t rows, int world, int dim) {
    return (int64_t)kCtrl + (int64_t)world * slot_floats(rows, world, dim) * 4;
}

// Bounded wait of one lane for *p >= v; false (and the status recorded) when it gives up.
__device__ __forceinline__ bool wait_at_least(const int64_t* p, int64_t v, uint64_t t0, int* status) {
    while (ld_acquire_sys(p) < v) {
        if (globaltimer_ns() - t0 > kWaitNs) {
            atomicExch(status, kDevTimeout);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

__global__ void __launch_bounds__(256) rs_scatter_kernel(const float* __restrict__ block,
                                                         const int64_t* __restrict__ bases, int world, int64_t rows,
                                                         int dim, int rank, int64_t* state, int* status) {
    __shared__ int s_go;
    const int64_t epoch = state[0] + 1;   // the last CTA advances it only after every CTA has read it
    int* ticket = reinterpret_cast<int*>(state + 1);   // [0] the CTA ticket, [1] the last step a CTA gave up in
    const int64_t sf = slot_floats(rows, world, dim);
    if (threadIdx.x < 32) {   // lane q: peer q has read its slots of the previous step
        const int q = threadIdx.x;
        bool ok = true;
        if (q < world && q != rank)
            ok = wait_at_least(reinterpret_cast<const int64_t*>(bases[q]) + kConsumedW, epoch - 1, globaltimer_ns(),
                               status);
        ok = __all_sync(0xffffffffu, ok);
        if (q == 0) {
            if (!ok) atomicExch(ticket + 1, (int)epoch);
            s_go = ok;
        }
    }
    __syncthreads();
    if (s_go) {
        const int64_t nth = (int64_t)gridDim.x * blockDim.x;
        const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
        for (int p = 1; p < world; ++p) {
            const int q = (rank + p) % world;   // the ranks start on different peers
            const int64_t lo = share_lo(rows, world, q), n = share_lo(rows, world, q + 1) - lo;
            float* slot = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bases[q]) + kCtrl) + (int64_t)rank * sf;
            const float4* src = reinterpret_cast<const float4*>(block + lo * dim);
            float4* dst = reinterpret_cast<float4*>(slot);
            const int64_t n16 = n * dim / 4;
            for (int64_t i = t; i < n16; i += nth) dst[i] = __ldcg(src + i);
            for (int64_t i = t; i < n; i += nth) slot[n * dim + i] = __ldcg(block + rows * dim + lo + i);
        }
    }
    __threadfence_system();   // every thread's stores are performed before its CTA takes the ticket
    __syncthreads();
    if (threadIdx.x != 0) return;
    if (atomicAdd(ticket, 1) != (int)gridDim.x - 1) return;
    atomicExch(ticket, 0);
    state[0] = epoch;   // advanced even after a failed wait, so the ranks' step counts stay in line
    if (atomicAdd(ticket + 1, 0) == (int)epoch) return;
    __threadfence_system();
    for (int p = 1; p < world; ++p) {
        const int q = (rank + p) % world;
        st_release_sys(reinterpret_cast<int64_t*>(bases[q]) + kFlags + rank, epoch);
    }
}

template <bool OUT_BF16>
__global__ void __launch_bounds__(32 * kRowsPerCta) rs_merge_kernel(const float* __restrict__ block,
                                                                    const int64_t* __restrict__ bases, int world,
                                                                    int64_t rows, int dim, int rank,
                                                                    const int64_t* state, void* out, float* out_lse,
                                                                    int* status) {
    using OutT = typename std::conditional<OUT_BF16, __nv_bfloat16, float>::type;
    __shared__ int s_ok;
    const int64_t epoch = *reinterpret_cast<const volatile int64_t*>(state);   // advanced by this step's scatter
    int64_t* ctrl = reinterpret_cast<int64_t*>(bases[rank]);
    int64_t* root = reinterpret_cast<int64_t*>(bases[0]);
    const int64_t sf = slot_floats(rows, world, dim);
    const float* slots = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(ctrl) + kCtrl);
    const int64_t lo = share_lo(rows, world, rank), n = share_lo(rows, world, rank + 1) - lo;
    uint8_t* area = reinterpret_cast<uint8_t*>(root) + area_offset(rows, world, dim);   // rank 0's gather area
    OutT* area_o = reinterpret_cast<OutT*>(area);
    float* area_l = reinterpret_cast<float*>(area) + rows * dim;
    if (threadIdx.x < 32) {   // lane q: flag q reached this step; lane `rank` (> 0): rank 0 copied out the last one
        const int q = threadIdx.x;
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        if (q < world && q != rank) ok = wait_at_least(ctrl + kFlags + q, epoch, t0, status);
        if (q == rank && rank != 0) ok = wait_at_least(root + kGConsumed, epoch - 1, t0, status);
        ok = __all_sync(0xffffffffu, ok);
        if (q == 0) {
            if (!ok) atomicExch(reinterpret_cast<unsigned long long*>(ctrl + kFailedW), (unsigned long long)epoch);
            s_ok = ok;
        }
    }
    __syncthreads();
    const bool ok1 = s_ok;   // read once by every thread: s_ok is written again below
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * kRowsPerCta + warp;   // row within this rank's share
    if (ok1 && r < n) {
        // lane p < world holds partial p's lse; this rank's own partial is read from its block
        const float lp = lane < world ? __ldcg(lane == rank ? block + rows * dim + lo + r : slots + lane * sf + n * dim + r)
                                      : -INFINITY;
        float M = lp;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float w = (M == -INFINITY || lp == -INFINITY) ? 0.f : expf(lp - M);
        float s = w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float lse = M == -INFINITY ? -INFINITY : M + logf(s);
        const float wp = M == -INFINITY ? 0.f : w / s;   // exp(lp - lse)
        OutT* dst = (rank == 0 ? static_cast<OutT*>(out) : area_o) + (lo + r) * dim;
        for (int c = lane * 4; c < dim; c += 128) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p0 = 0; p0 < world; p0 += 8) {   // eight partials' loads in flight, then their sums
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int p = p0 + u;
                    if (p < world) {
                        const float* src = p == rank ? block + (lo + r) * dim : slots + p * sf + r * dim;
                        v[u] = __ldcg(reinterpret_cast<const float4*>(src + c));
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const float e = __shfl_sync(0xffffffffu, wp, (p0 + u) & 31);
                    if (p0 + u >= world || e == 0.f) continue;
                    acc.x = fmaf(e, v[u].x, acc.x);
                    acc.y = fmaf(e, v[u].y, acc.y);
                    acc.z = fmaf(e, v[u].z, acc.z);
                    acc.w = fmaf(e, v[u].w, acc.w);
                }
            }
            if (OUT_BF16)
                *reinterpret_cast<uint2*>(dst + c) = make_uint2(pack_bf16(acc.x, acc.y), pack_bf16(acc.z, acc.w));
            else
                *reinterpret_cast<float4*>(dst + c) = acc;
        }
        if (lane == 0) {
            if (rank != 0) area_l[lo + r] = lse;
            else if (out_lse) out_lse[lo + r] = lse;
        }
    }
    if (rank == 0 && world > 1 && ok1) {
        // the other ranks' merged rows [share_lo(1), rows) arrive in the gather area; copy them to out
        __syncthreads();   // every thread has read s_ok before it is written again
        if (threadIdx.x < 32) {
            const int q = threadIdx.x;
            bool ok = true;
            if (q >= 1 && q < world) ok = wait_at_least(ctrl + kGFlags + q, epoch, globaltimer_ns(), status);
            ok = __all_sync(0xffffffffu, ok);
            if (q == 0) {
                if (!ok)
                    atomicExch(reinterpret_cast<unsigned long long*>(ctrl + kFailedW), (unsigned long long)epoch);
                s_ok = ok;
            }
        }
        __syncthreads();
        if (s_ok) {
            const int64_t r1 = share_lo(rows, world, 1);
            const int64_t nth = (int64_t)gridDim.x * blockDim.x;
            const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
            // rows * dim elements of 2 or 4 bytes with dim % 4 == 0: 8-byte units from any row start
            const uint2* src = reinterpret_cast<const uint2*>(area_o + r1 * dim);
            uint2* dst = reinterpret_cast<uint2*>(static_cast<OutT*>(out) + r1 * dim);
            const int64_t n8 = (rows - r1) * dim * (int64_t)sizeof(OutT) / 8;
            for (int64_t i = t; i < n8; i += nth) dst[i] = __ldcg(src + i);
            if (out_lse)
                for (int64_t i = t; i < rows - r1; i += nth) out_lse[r1 + i] = __ldcg(area_l + r1 + i);
        }
    }
    // the last CTA publishes this step: slots read (consumed); rank 0: gathered rows copied out; the others:
    // the merged share stored in rank 0's gather area (gflag)
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        int* ticket = reinterpret_cast<int*>(ctrl + kTicketW);
        if (atomicAdd(ticket, 1) == (int)gridDim.x - 1) {
            atomicExch(ticket, 0);
            if (atomicAdd(reinterpret_cast<unsigned long long*>(ctrl + kFailedW), 0ull) != (unsigned long long)epoch) {
                __threadfence_system();
                st_release_sys(ctrl + kConsumedW, epoch);
                if (rank == 0) st_release_sys(ctrl + kGConsumed, epoch);
                else st_release_sys(root + kGFlags + rank, epoch);
            }
        }
    }
}

}  // namespace rs
}  // namespace peer
}  // namespace ws

using namespace ws;
using namespace ws::peer;

extern "C" {

size_t ws_peer_exchange_bytes(int world, int64_t rows, int dim) {
    if (world < 1 || world > kMaxRanks || rows < 0 || dim < 1) return 0;
    return kCtrlBytes + (size_t)world * (size_t)slot_floats(rows, dim) * sizeof(float);
}

size_t ws_peer_slot_offset(int world, int64_t rows, int dim, int rank) {
    (void)world;
    return kCtrlBytes + (size_t)rank * (size_t)slot_floats(rows, dim) * sizeof(float);
}

int ws_peer_buffer_create(size_t bytes, void** dev_ptr, void* ipc_handle) {
    if (!dev_ptr || !ipc_handle || bytes < kCtrlBytes) return set_error(WS_ERR_INVALID_ARG, "peer_buffer_create: bad argument");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();   // zeroed before any peer maps it
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return set_error(WS_ERR_CUDA, cudaGetErrorString(e));
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *dev_ptr = p;
    return WS_OK;
}

int ws_peer_buffer_open(const void* ipc_handle, void** dev_ptr) {
    if (!ipc_handle || !dev_ptr) return set_error(WS_ERR_INVALID_ARG, "peer_buffer_open: bad argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

int ws_peer_buffer_close(void* dev_ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

int ws_peer_buffer_free(void* dev_ptr) {
    const cudaError_t e = cudaFree(dev_ptr);
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

int ws_peer_push(const float* block, void* root_base, int world, int64_t rows, int dim, int rank, int64_t* state,
                 void* stream) {
    if (!block || !root_base || !state || rank < 1 || rank >= world || world > kMaxRanks || rows < 0 || dim < 1)
        return set_error(WS_ERR_INVALID_ARG, "peer_push: bad argument");
    if (reinterpret_cast<uintptr_t>(block) % 16 || reinterpret_cast<uintptr_t>(state) % 8)
        return set_error(WS_ERR_INVALID_ARG, "peer_push: block must be 16-byte and state 8-byte aligned");
    const int64_t n16 = (rows * dim + rows + 3) / 4;   // the block and the slot are rounded up to 64 floats
    float4* dst = reinterpret_cast<float4*>(static_cast<uint8_t*>(root_base) + ws_peer_slot_offset(world, rows, dim, rank));
    const int ctas = (int)std::max<int64_t>(1, std::min<int64_t>(128, (n16 + 255) / 256));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    pdl_config(cfg, attr, dim3(ctas), dim3(256), static_cast<cudaStream_t>(stream));
    const cudaError_t e = cudaLaunchKernelEx(&cfg, peer_push_kernel, reinterpret_cast<const float4*>(block), dst, n16,
                                             static_cast<int64_t*>(root_base), state, rank, device_status_word());
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

int ws_peer_merge(void* root_base, int world, int64_t rows, int dim, void* out, int out_dtype, float* out_lse,
                  void* stream) {
    if (!root_base || world < 1 || world > 32 || rows < 0 || dim < 4 || dim % 4 || (rows > 0 && !out))
        return set_error(WS_ERR_INVALID_ARG, "peer_merge: bad argument (world <= 32, dim % 4 == 0)");
    if (out_dtype != WS_DTYPE_BF16 && out_dtype != WS_DTYPE_F32)
        return set_error(WS_ERR_INVALID_ARG, "peer_merge: out dtype");
    if (reinterpret_cast<uintptr_t>(out) % 16) return set_error(WS_ERR_INVALID_ARG, "peer_merge: out must be 16-byte aligned");
    const int64_t sf = slot_floats(rows, dim);
    const float* slots = reinterpret_cast<const float*>(static_cast<uint8_t*>(root_base) + kCtrlBytes);
    const int64_t ctas = std::max<int64_t>(1, (rows + kRowsPerCta - 1) / kRowsPerCta);
    if (ctas > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "peer_merge: too many rows");
    int64_t* ctrl = static_cast<int64_t*>(root_base);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    pdl_config(cfg, attr, dim3((unsigned)ctas), dim3(32 * kRowsPerCta), static_cast<cudaStream_t>(stream));
    const cudaError_t e =
        out_dtype == WS_DTYPE_BF16
            ? cudaLaunchKernelEx(&cfg, peer_merge_kernel<true>, slots, sf, world, rows, dim, ctrl, out, out_lse,
                                 device_status_word())
            : cudaLaunchKernelEx(&cfg, peer_merge_kernel<false>, slots, sf, world, rows, dim, ctrl, out, out_lse,
                                 device_status_word());
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

size_t ws_peer_rs_bytes(int world, int64_t rows, int dim) {
    if (world < 1 || world > 32 || rows < 0 || dim < 4 || dim % 4) return 0;
    return (size_t)rs::area_offset(rows, world, dim) + align_up((size_t)(rows * dim + rows), 64) * sizeof(float);
}

int ws_peer_rs_scatter(const float* block, const int64_t* bases, int world, int64_t rows, int dim, int rank,
                       int64_t* state, void* stream) {
    if (!block || !bases || !state || world < 1 || world > 32 || rank < 0 || rank >= world || rows < 0 || dim < 4 ||
        dim % 4)
        return set_error(WS_ERR_INVALID_ARG, "peer_rs_scatter: bad argument (world <= 32, dim % 4 == 0)");
    if (reinterpret_cast<uintptr_t>(block) % 16 || reinterpret_cast<uintptr_t>(bases) % 8 ||
        reinterpret_cast<uintptr_t>(state) % 8)
        return set_error(WS_ERR_INVALID_ARG, "peer_rs_scatter: block must be 16-byte, bases and state 8-byte aligned");
    // (world - 1) / world of the block leaves this rank: one 16-byte copy per thread per pass
    const int64_t n16 = (rows - rows / std::max(world, 1)) * dim / 4 + 1;
    const int ctas = (int)std::max<int64_t>(1, std::min<int64_t>(128, (n16 + 255) / 256));
    rs::rs_scatter_kernel<<<ctas, 256, 0, static_cast<cudaStream_t>(stream)>>>(block, bases, world, rows, dim, rank,
                                                                             state, device_status_word());
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

int ws_peer_rs_merge(const float* block, const int64_t* bases, int world, int64_t rows, int dim, int rank,
                     const int64_t* state, void* out, int out_dtype, float* out_lse, void* stream) {
    if (!block || !bases || !state || world < 1 || world > 32 || rank < 0 || rank >= world || rows < 0 || dim < 4 ||
        dim % 4 || (rank == 0 && rows > 0 && !out))
        return set_error(WS_ERR_INVALID_ARG, "peer_rs_merge: bad argument (world <= 32, dim % 4 == 0, out on rank 0)");
    if (out_dtype != WS_DTYPE_BF16 && out_dtype != WS_DTYPE_F32)
        return set_error(WS_ERR_INVALID_ARG, "peer_rs_merge: out dtype");
    if (reinterpret_cast<uintptr_t>(block) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return set_error(WS_ERR_INVALID_ARG, "peer_rs_merge: block and out must be 16-byte aligned");
    const int64_t share = (rows + world - 1) / world;
    // rank 0 also copies the gathered rows out: at least 64 CTAs there, and the same grid on every rank
    const int64_t ctas = std::max<int64_t>(64, (share + kRowsPerCta - 1) / kRowsPerCta);
    if (ctas > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "peer_rs_merge: too many rows");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (out_dtype == WS_DTYPE_BF16)
        rs::rs_merge_kernel<true><<<(unsigned)ctas, 32 * kRowsPerCta, 0, st>>>(block, bases, world, rows, dim, rank,
                                                                            state, out, out_lse, device_status_word());
    else
        rs::rs_merge_kernel<false><<<(unsigned)ctas, 32 * kRowsPerCta, 0, st>>>(block, bases, world, rows, dim, rank,
                                                                             state, out, out_lse, device_status_word());
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
