// CSA sparse decode (DeepSeek-V4 style): the query rows of one sequence
// attend over a shared 512-wide latent KV (K = V), either over the entries a
// top-k id list selects (gather) or over a contiguous id range (dense), with
// the KV stored bf16 or int8 with one fp32 scale per entry.
//
// Replaces indexer_attn_cpu (kernel/cpu_attn_ds4_ext/csa_attn.cpp:1819-1883),
// fused_csa_attn (:200-281) and fused_csa_attn_range (:1587-1656), and runs the
// int8-entry storage (values = int8 * scale, :1338-1344) with an unquantised
// query.
//
// Query-code mode (QM > 0) reproduces the reference's int8 operators
// (fused_csa_attn_bsq_int8 :766-883, _bsq_int8_preq :1235-1357, _bsq_int8_full
// :1359-1483): the query arrives as u8 codes with one fp32 scale per row, the
// entries as s8 codes with a scale and a code sum each, and the score is the
// reference's integer form
//     ((sum_d u8[d] * s8[d]) - 128 * ksum) * q_scale * k_scale * scale.
// u8 and s8 codes are exact in fp16 and every partial sum of the first product
// is an integer below 2^24, so the fp16 tensor-core product gives the same
// integer dot as the reference's VNNI dpbusd.  Values are int8 * k_scale
// (QM = 1) or a separate bf16 entry buffer (QM = 2, the _full operator: the
// codes tile feeds the first product and the bf16 tile the second, so the ring
// holds one tile of each instead of two tiles).
//
// One CTA per (sequence, group of query rows, split): the `splits` CTAs of a
// (sequence, group) divide its selected entries evenly, with splits chosen so
// that the whole grid is one wave over the SMs.  Inside a CTA, warp roles:
//   * gather warps (3): resolve entry ids to rows of this buffer (512 at a
//     time), load each 64-entry tile's rows straight from global memory into
//     registers (two tiles in flight for int8) and write them as a
//     128-byte-swizzled bf16 tile into a 2-slot ring (int8 -> bf16 is exact;
//     the per-entry scale is folded into the scores and into P instead);
//   * MMA warp (1): S[heads x 64] = Q . K^T (M=64, heads on TMEM lanes, two S
//     buffers) and O^T[512 x heads] += K^T . P^T (M=128), tcgen05 with the
//     accumulators in TMEM;
//   * softmax warps (4): one thread per head owns that head's running max and
//     sum and reads its 64 scores from its own TMEM lane, so the per-tile max
//     and sum need no cross-thread reduction; the max is updated lazily (O is
//     rescaled in TMEM only when a head's max grows by more than 2^8, which
//     keeps P <= 256 and is exact because m, l and O always share one max).
// All eight warps then write the CTA's normalised O rows and log-sum-exp:
// the output itself when splits == 1, else partial `split` of the workspace
// (fp32, L2-resident), which the log-sum-exp merge kernel (merge.cu, launched
// as a programmatic dependent of this grid) combines into the output.
//
// Every wait is bounded: a wait that gives up records kDevTimeout in the
// status word and sets a CTA-wide abort flag, after which the remaining waits
// return at once and no more products are issued, so every role still reaches
// the final barriers.
#include <cstdio>

#include "common.cuh"
#include "ws_internal.h"

namespace ws {
namespace csa {

constexpr int HD = 512;                  // latent width
constexpr int TT = 64;                   // entries per tile
constexpr int KBOX = TT * 128;           // 8 KB: 64 dims x 64 entries, 128-byte swizzled
constexpr int KSLOT = 8 * KBOX;          // 64 KB: one bf16 tile of 512 dims
constexpr int CHUNK = 512;               // entries resolved to rows at a time (8 tiles)
// 8 warps (two per SM sub-partition, so up to 255 registers a thread)
constexpr int kSmWarps = 4, kGaWarps = 3;
constexpr int kGaThreads = 32 * kGaWarps;
constexpr int kMmaWarp = kSmWarps + kGaWarps;
constexpr int kThreads = 32 * (kMmaWarp + 1);   // 256
constexpr int kGaRows = (TT + kGaWarps - 1) / kGaWarps;   // tile rows per gather warp (22)
constexpr int kResolve = (CHUNK + kGaThreads - 1) / kGaThreads;   // entries per gather thread per chunk
constexpr float kLazy = 8.f;             // rescale O only when a head's max grows by more than 2^8
constexpr int kMaxSplit = 32;          // CTAs one (sequence, group) is split over, at most
// named barriers (0 is __syncthreads); BAR_Q: the softmax warps arrive once the query tile is in
// shared memory, the gather and MMA warps wait on it before they first use it
constexpr int BAR_SOFTMAX = 1, BAR_GATHER = 2, BAR_Q = 3;

// mbarriers
// two of each: K slot full / empty, S buffer full / empty, P buffer full / empty (P empty: the second
// product that read the buffer, and every product issued before it, has finished)
enum { B_KFULL = 0, B_KEMPTY = 2, B_SFULL = 4, B_SEMPTY = 6, B_PFULL = 8, B_PEMPTY = 10, NBARS = 12 };

// QSPLIT: an fp32 query is held as bf16 hi + lo parts (lo = q - hi, rounded
// again) and the first product runs on both, so the scores keep ~16 mantissa
// bits of the query; 32 query rows per group then.  A bf16 query: 64 rows.
template <bool QSPLIT>
struct Cfg {
    static constexpr int NQ = QSPLIT ? 32 : 64;
    static constexpr int QBOX = NQ * 128;                  // 64 dims x NQ rows
    static constexpr int OFF_K = 0;                        // K ring; the O partial [NQ][512] fp32 at the end
    static constexpr int OFF_Q = 2 * KSLOT;
    static constexpr int QBYTES = (QSPLIT ? 2 : 1) * 8 * QBOX;
    // the M=64 product reads 64 rows from each box start: for 32-row boxes the
    // extra rows are the next box (garbage rows of S nobody reads); the last
    // box reads into this pad
    static constexpr int QPAD = QSPLIT ? 4096 : 0;
    static constexpr int OFF_P = OFF_Q + QBYTES + QPAD;    // 2 x P [NQ rows x 64 entries], K-major
    static constexpr int PBYTES = NQ * 128;
    static constexpr int OFF_MISC = OFF_P + 2 * PBYTES;
    // misc, in 4-byte words
    static constexpr int W_CROW = 0;                       // [CHUNK] local row of each entry, -1 = none
    static constexpr int W_CSC = W_CROW + CHUNK;           // [CHUNK] value scale of each entry
    static constexpr int W_F = W_CSC + CHUNK;              // [2][TT] score factor: scale * softmax scale * log2(e)
    static constexpr int W_BIAS = W_F + 2 * TT;            // [2][TT] 0, or -inf where there is no entry
    static constexpr int W_PSC = W_BIAS + 2 * TT;          // [2][TT] value scale folded into P
    static constexpr int W_CKS = W_PSC + 2 * TT;           // [CHUNK] code sum of each entry (query-code mode)
    static constexpr int W_COR = W_CKS + CHUNK;            // [2][TT] -128 * code sum (query-code mode)
    static constexpr int W_ALPHA = W_COR + 2 * TT;         // [2][64] per-head rescale factor, by tile parity
    static constexpr int W_NEED = W_ALPHA + 128;           // [2][4] per-warp "some head rescales"
    static constexpr int W_RINV = W_NEED + 8;              // [64] 2^eref / l: normalises a head's O row
    static constexpr int W_RLSE = W_RINV + 64;             // [64] log-sum-exp of a head, -inf when empty
    static constexpr int W_QEXP = W_RLSE + 64;             // [64] per-head query exponent (fp16 products)
    static constexpr int W_TEXP = W_QEXP + 64;             // [2] value-scale exponent of the tile in each slot
    static constexpr int W_WMAX = W_TEXP + 2;              // [4] per-gather-warp max value scale of a chunk
    static constexpr int W_FLAGS = W_WMAX + 4;             // [0] abort, [1] TMEM base
    static constexpr int W_BARS = W_FLAGS + 4;
    static constexpr int MISC_WORDS = W_BARS + 2 * NBARS;
    static constexpr size_t SMEM = 1024 + OFF_MISC + MISC_WORDS * 4;
    static constexpr int S_COL = 0;                        // two S buffers of TT columns
    static constexpr int O_COL = 2 * TT;                   // O^T: 4 blocks of NQ columns (128 dims each)
    static constexpr int TMEM_COLS = 512;
    static_assert(O_COL + 4 * NQ <= TMEM_COLS, "TMEM budget");
    static_assert(NQ * HD * 4 <= 2 * KSLOT, "O partial must fit in the K ring");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert((W_BARS & 1) == 0, "mbarrier alignment");
};

struct Params {
    const void* q;
    int q_f32;
    int nq;                   // query rows per sequence (all groups)
    int ngroups;              // ceil(nq / NQ)
    const void* kv;
    int kv_i8;
    const float* kv_scales;   // [bs, nc_local] when kv_i8
    const float* q_scales;    // query-code mode: [bs * nq] u8 query scales
    const int* kv_sums;       //                  [bs, nc_local] s8 code sums
    const void* kv_val;       //                  QM = 2: bf16 values [bs, nc_local, 512]
    const int* idx;           // [bs, k] (gather) or null (dense)
    int k;
    int window;               // WS_CSA_IDX_* for the gather
    int64_t dense_begin, dense_end;   // dense: ids [begin, end), already clipped to the shard
    int64_t shard_lo, shard_hi;       // this buffer holds ids [shard_lo, shard_hi); row = id - shard_lo
    int64_t nc_local;
    float scale_log2;
    void* out;
    int out_f32;
    int out_aligned;          // out is 16-byte aligned: rows are written with bulk copies
    float* out_lse;
    float* part_o;            // splits > 1: [splits][bs * nq][512] normalised partial outputs
    float* part_lse;          //             [splits][bs * nq] their log-sum-exp
    int* status;
};

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// first position in ids[0, n) with ids[pos] >= v (ids sorted ascending)
__device__ __forceinline__ int lower_bound_ids(const int* ids, int n, int64_t v) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((int64_t)__ldg(ids + mid) < v) lo = mid + 1; else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ void wait_bar(uint32_t bar, uint32_t parity, volatile int* abort, int* status) {
    if (*abort) return;
    if (!mbar_wait_bounded(bar, parity)) {
        *abort = 1;
        atomicExch(status, kDevTimeout);
    }
}

// KV_I8: int8 entries; both products then run in fp16 (int8 -> fp16 is exact
// and takes two byte permutes and one packed subtract per four values).  The
// query is scaled per head by a power of two so its largest element sits in
// [2^14, 2^15) (no fp16 overflow, elements above 2^-28 of it exact), and the
// value scales folded into P are scaled per 512-entry chunk by a power of two
// so that P <= 256.  bf16 entries: bf16 products, no scaling.
// QM: 0 = float query; 1 = u8 query codes, values int8 * scale; 2 = u8 query
// codes, bf16 values from p.kv_val (both need KV_I8 and a 64-row group).
template <bool KV_I8, bool QSPLIT, int QM>
__global__ void __launch_bounds__(kThreads, 1) csa_decode_kernel(const Params p) {
    static_assert(QM == 0 || (KV_I8 && !QSPLIT), "query codes need int8 entries and 64-row groups");
    using C = Cfg<QSPLIT>;
    constexpr int NQ = C::NQ;
    constexpr bool P_F16 = KV_I8 && QM != 2;   // P (and the second product's operands) fp16, else bf16
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint32_t* misc = reinterpret_cast<uint32_t*>(sm + C::OFF_MISC);
    int* s_crow = reinterpret_cast<int*>(misc + C::W_CROW);
    float* s_csc = reinterpret_cast<float*>(misc + C::W_CSC);
    float* s_f = reinterpret_cast<float*>(misc + C::W_F);
    float* s_bias = reinterpret_cast<float*>(misc + C::W_BIAS);
    float* s_psc = reinterpret_cast<float*>(misc + C::W_PSC);
    int* s_cks = reinterpret_cast<int*>(misc + C::W_CKS);
    float* s_cor = reinterpret_cast<float*>(misc + C::W_COR);
    float* s_alpha = reinterpret_cast<float*>(misc + C::W_ALPHA);
    int* s_need = reinterpret_cast<int*>(misc + C::W_NEED);
    float* s_rinv = reinterpret_cast<float*>(misc + C::W_RINV);
    float* s_rlse = reinterpret_cast<float*>(misc + C::W_RLSE);
    int* s_qexp = reinterpret_cast<int*>(misc + C::W_QEXP);
    int* s_texp = reinterpret_cast<int*>(misc + C::W_TEXP);
    float* s_wmax = reinterpret_cast<float*>(misc + C::W_WMAX);
    volatile int* s_abort = reinterpret_cast<volatile int*>(misc + C::W_FLAGS);
    uint32_t* s_tmem = misc + C::W_FLAGS + 1;
    uint64_t* bars = reinterpret_cast<uint64_t*>(misc + C::W_BARS);
    const uint32_t bar0 = smem_u32(bars);
#define BAR(i) (bar0 + 8u * (uint32_t)(i))

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, splits = gridDim.x;
    const int seq = blockIdx.y / p.ngroups, grp = blockIdx.y - seq * p.ngroups;
    const int row0 = grp * NQ;                       // first query row of this group
    const int nrows = min(NQ, p.nq - row0);
    const int* ids = p.idx ? p.idx + (int64_t)seq * p.k : nullptr;
    const int64_t kv_seq = (int64_t)seq * p.nc_local;   // first row of this sequence

    // ---- this CTA's share of the sequence's entries: positions in ids (gather) or ids (dense)
    int64_t e_begin, e_end;
    {
        int64_t lo, hi;
        if (ids) {
            lo = 0;
            hi = p.k;
            if (p.window == WS_CSA_IDX_SORTED_SHARD) {
                lo = lower_bound_ids(ids, p.k, p.shard_lo);
                hi = lower_bound_ids(ids, p.k, p.shard_hi);
            }
        } else {
            lo = p.dense_begin;
            hi = p.dense_end;
        }
        const int64_t cnt = hi - lo;
        e_begin = lo + cnt * split / splits;
        e_end = lo + cnt * (split + 1) / splits;
    }
    const int ntiles = (int)((e_end - e_begin + TT - 1) / TT);

    // ---- entry ids -> local rows and value scales, CHUNK entries at a time (gather warps)
    const int gtid = tid - 32 * kSmWarps;   // 0..95 in the gather warps
    // resolve_rows: ids -> local rows (s_crow) and the value-scale loads issued; finish_scales: the
    // scales and the chunk's largest scale (s_csc, s_wmax).  Between the two, the rows are known and
    // the first tile's row loads can be in flight with the scale loads.
    int64_t id[kResolve];   // issue_ids -> resolve_rows: the chunk's ids in flight
    float sc_pend[kResolve];
    int ks_pend[kResolve];  // query-code mode: the entries' code sums in flight
    auto issue_ids = [&](int64_t cbase) {
#pragma unroll
        for (int u = 0; u < kResolve; ++u) {
            const int j = gtid + u * kGaThreads;
            const int64_t e = cbase + j;
            id[u] = (j < CHUNK && e < e_end) ? (ids ? (int64_t)__ldg(ids + e) : e) : INT64_MIN;
        }
    };
    auto resolve_rows = [&]() {
        int row[kResolve];
#pragma unroll
        for (int u = 0; u < kResolve; ++u) {
            row[u] = -1;
            if (id[u] != INT64_MIN) {
                if (id[u] >= p.shard_lo && id[u] < p.shard_hi) row[u] = (int)(id[u] - p.shard_lo);
                else if (p.window == WS_CSA_IDX_ALL) atomicExch(p.status, kDevBadIndex);   // skipped, and reported
            }
        }
#pragma unroll
        for (int u = 0; u < kResolve; ++u) {
            sc_pend[u] = row[u] >= 0 ? (KV_I8 ? __ldg(p.kv_scales + kv_seq + row[u]) : 1.f) : 0.f;
            if (QM) ks_pend[u] = row[u] >= 0 ? __ldg(p.kv_sums + kv_seq + row[u]) : 0;
            const int j = gtid + u * kGaThreads;
            if (j < CHUNK) s_crow[j] = row[u];
        }
    };
    auto finish_scales = [&]() {
        float mx = 0.f;
#pragma unroll
        for (int u = 0; u < kResolve; ++u) {
            const int j = gtid + u * kGaThreads;
            if (j < CHUNK) {
                s_csc[j] = sc_pend[u];
                if (QM) s_cks[j] = ks_pend[u];
                mx = fmaxf(mx, sc_pend[u]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) s_wmax[warp - kSmWarps] = mx;
    };
    auto resolve_chunk = [&](int64_t cbase) {
        issue_ids(cbase);
        resolve_rows();
        finish_scales();
    };
    // the first chunk's ids are requested before anything else: every later step of the gather waits on them
    if (warp >= kSmWarps && warp < kMmaWarp && ntiles > 0) issue_ids(e_begin);

    // ---- the query rows (softmax warps, QTPR threads per row, QDPT dims each): every 16-byte load is
    //      issued at once and lands, unconverted, in the 16-byte slot its converted form takes (an fp32
    //      chunk of 8 dims: its two halves in the hi and the lo slot); rows past nrows are zero
    constexpr int QTPR = 32 * kSmWarps / NQ, QDPT = HD / QTPR;   // 2 x 256 dims (bf16 q), 4 x 128 (fp32 q)
    constexpr int QES = QM ? 1 : (QSPLIT ? 4 : 2);               // bytes per query element as loaded
    constexpr int QL = QDPT * QES / 16;                          // 16-byte loads per thread (32; 16 for codes)
    static_assert(QDPT % 32 == 0 && QDPT * QTPR == HD, "query split");
    const int qr = tid / QTPR, qpart = tid - qr * QTPR;          // meaningful for the softmax warps
    auto qslot = [&](int c, int half) {   // 8-dim chunk c of this thread's share; half: lo part (fp32 q)
        const int c8 = qpart * (QDPT / 8) + c;
        return sm + C::OFF_Q + (half * 8 + (c8 >> 3)) * C::QBOX + swz(qr, c8 & 7);
    };
    uint4 qraw[QL];
    if (warp < kSmWarps) {   // requested now; stored once the CTA-wide setup below is done
        const bool ok = qr < nrows;
        const int64_t qoff = ((int64_t)seq * p.nq + row0 + (ok ? qr : 0)) * HD + qpart * QDPT;
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.q) + qoff * QES);
#pragma unroll
        for (int j = 0; j < QL; ++j) qraw[j] = ok ? __ldg(src + j) : make_uint4(0, 0, 0, 0);
    }
    uint32_t qmax_bits = 0;   // largest |q| of this thread's share, as float bits (fp16 products only)
    auto store_q = [&]() {
        if (QM) {   // 16 u8 codes -> two 8-dim fp16 chunks: byte b -> fp16 bits 0x6400 | b = 1024 + b, minus 1024
            const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
#pragma unroll
            for (int j = 0; j < QL; ++j) {
                const uint32_t src[4] = {qraw[j].x, qraw[j].y, qraw[j].z, qraw[j].w};
                uint32_t w[8];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t lo = __byte_perm(src[u], 0x64646464u, 0x4140);
                    const uint32_t hi = __byte_perm(src[u], 0x64646464u, 0x4342);
                    const __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&lo), k1024);
                    const __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&hi), k1024);
                    w[2 * u] = *reinterpret_cast<const uint32_t*>(&a);
                    w[2 * u + 1] = *reinterpret_cast<const uint32_t*>(&b);
                }
                *reinterpret_cast<uint4*>(qslot(2 * j, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4*>(qslot(2 * j + 1, 0)) = make_uint4(w[4], w[5], w[6], w[7]);
            }
            return;
        }
#pragma unroll
        for (int j = 0; j < QL; ++j) {
            if (KV_I8) {   // magnitudes by integer max: non-negative floats order as their bits
                const uint32_t w[4] = {qraw[j].x, qraw[j].y, qraw[j].z, qraw[j].w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    qmax_bits = QSPLIT ? max(qmax_bits, w[u] & 0x7fffffffu) : __vmaxu2(qmax_bits, w[u] & 0x7fff7fffu);
            }
            *reinterpret_cast<uint4*>(QSPLIT ? qslot(j >> 1, j & 1) : qslot(j, 0)) = qraw[j];
        }
        if (!QSPLIT) qmax_bits = max(qmax_bits & 0xffffu, qmax_bits >> 16) << 16;   // bf16 -> float bits
    };

    const uint32_t kbase = smem_u32(sm + C::OFF_K), qbase = smem_u32(sm + C::OFF_Q), pbase = smem_u32(sm + C::OFF_P);
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(BAR(B_KFULL + i), kGaThreads);
            mbar_init(BAR(B_KEMPTY + i), 1);
            mbar_init(BAR(B_SFULL + i), 1);
            mbar_init(BAR(B_SEMPTY + i), kSmWarps);
            mbar_init(BAR(B_PFULL + i), kSmWarps);
            mbar_init(BAR(B_PEMPTY + i), 1);
        }
        *s_abort = 0;
        s_qexp[0] = 0;   // largest |q| of the group (float bits), for the fp16 query scale
        fence_mbar_init();
    }
    if (warp == kMmaWarp) tmem_alloc(smem_u32(s_tmem), C::TMEM_COLS);
    __syncthreads();
    pdl_launch_dependents();   // the merge grid may be scheduled now; it waits for this grid's completion

    const uint32_t tbase = *s_tmem;
    // S = Q . K^T and O^T += K^T . P^T
    constexpr uint32_t id1 = KV_I8 ? idesc_f16_f32(64, TT, false, false) : idesc_bf16_f32(64, TT, false, false);
    constexpr uint32_t id2 = P_F16 ? idesc_f16_f32(128, NQ, true, false) : idesc_bf16_f32(128, NQ, true, false);
    // QM = 2: the codes tile (first product) always sits in ring slot 0 and the values tile (second product)
    // in slot 1; otherwise tile t uses slot t & 1 for both
    auto k_slot = [&](int t) { return QM == 2 ? 0 : (t & 1); };
    auto v_slot = [&](int t) { return QM == 2 ? 1 : (t & 1); };

    float m_final = -INFINITY, l_final = 0.f;   // softmax threads: this head's running max and sum
    int eref_final = 0;                          // and the value-scale exponent O was accumulated in
    if (warp >= kSmWarps && warp < kMmaWarp) {
        // ================================================================ gather
        // the first chunk's rows are resolved (and its first tile's loads issued) while the softmax
        // warps convert the query tile
        if (ntiles > 0) {
            resolve_rows();
            named_bar_sync(BAR_GATHER, kGaThreads);   // the first chunk's rows
        }
        // score factor per unit value scale: softmax scale * log2(e), times 2^qe for the scaled fp16
        // query; known once the query tile is ready
        float fscale = 0.f;
        bool q_ready = false;
        auto wait_q = [&]() {
            if (q_ready) return;
            named_bar_sync(BAR_Q, kThreads);
            q_ready = true;
            fscale = KV_I8 ? p.scale_log2 * __int_as_float((127 + s_qexp[1]) << 23) : p.scale_log2;
        };
        // publish tile t's per-entry factors (thread gtid < TT owns entry gtid) and signal the MMA warp
        // cor: -128 * the entry's code sum (query-code mode), read with sc before the chunk can change
        auto publish = [&](int t, float sc, int ex, float cor) {   // ex: the chunk's value-scale exponent
            wait_q();
            const int slot = t & 1;
            if (gtid < TT) {
                const bool ok = sc >= 0.f;
                s_f[slot * TT + gtid] = ok ? sc * fscale : 0.f;
                s_bias[slot * TT + gtid] = ok ? 0.f : -INFINITY;
                // bf16 values (QM = 2) are taken as they are: the entry scale is the score's only
                const float pv = QM == 2 ? 1.f : sc * __int_as_float((127 - ex) << 23);
                s_psc[slot * TT + gtid] = ok ? pv : 0.f;
                if (QM) s_cor[slot * TT + gtid] = ok ? cor : 0.f;
            }
            if (gtid == 0) s_texp[slot] = ex;
            fence_proxy_async_smem();
            mbar_arrive(BAR(B_KFULL + slot));
        };
        auto next_chunk = [&](int t) {   // tile t starts a new chunk
            named_bar_sync(BAR_GATHER, kGaThreads);
            resolve_chunk(e_begin + (int64_t)t * TT);
            named_bar_sync(BAR_GATHER, kGaThreads);
        };
        auto chunk_exp = [&]() {   // ceil(log2(largest value scale of the current chunk)), in [-126, 126]
            const float mx = fmaxf(fmaxf(s_wmax[0], s_wmax[1]), s_wmax[2]);
            if (!(mx > 0.f)) return 0;
            const int b = __float_as_int(mx);
            return min(max(((b >> 23) & 0xff) - 127 + ((b & 0x7fffff) != 0), -126), 126);
        };
        auto entry_scale = [&](int t) {  // this thread's entry of tile t: its scale, or -1 when none
            const int off = (t * TT) % CHUNK + gtid;
            return (gtid < TT && s_crow[off] >= 0) ? s_csc[off] : -1.f;
        };
        auto entry_cor = [&](int t) {    // query-code mode: -128 * the code sum of this thread's entry of tile t
            const int off = (t * TT) % CHUNK + gtid;
            return (QM && gtid < TT && s_crow[off] >= 0) ? -128.f * (float)s_cks[off] : 0.f;
        };
        auto wait_slot = [&](int t) {
            if (QM == 2) {   // one tile of each kind: tile t waits for the second product of tile t - 1
                if (t >= 1) wait_bar(BAR(B_KEMPTY + ((t - 1) & 1)), ((t - 1) >> 1) & 1, s_abort, p.status);
            } else if (t >= 2) {
                wait_bar(BAR(B_KEMPTY + (t & 1)), ((t >> 1) + 1) & 1, s_abort, p.status);
            }
        };
        // 16 int8 codes (one lane's 16-byte chunk c of a row) -> 16 fp16 values in the row's 128-byte box
        auto store_codes16 = [&](uint8_t* box, int rr, int c, const int4& r) {
            const __half2 bias2 = __floats2half2_rn(1152.f, 1152.f);   // 1024 + 128
            const uint32_t src[4] = {(uint32_t)r.x, (uint32_t)r.y, (uint32_t)r.z, (uint32_t)r.w};
            uint32_t w[8];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                // byte b -> fp16 bits 0x6400 | (b + 128) = 1024 + b + 128, then subtract 1152: exact b
                const uint32_t x = src[u] ^ 0x80808080u;
                const uint32_t lo = __byte_perm(x, 0x64646464u, 0x4140);
                const uint32_t hi = __byte_perm(x, 0x64646464u, 0x4342);
                const __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&lo), bias2);
                const __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&hi), bias2);
                w[2 * u] = *reinterpret_cast<const uint32_t*>(&a);
                w[2 * u + 1] = *reinterpret_cast<const uint32_t*>(&b);
            }
            *reinterpret_cast<uint4*>(box + swz(rr, (c & 3) * 2)) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(box + swz(rr, (c & 3) * 2 + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
        };
        const int8_t* kv8 = static_cast<const int8_t*>(p.kv);
        // the int8 codes of tile t's rows: lane c holds 16-byte chunk c of rows rb + 3i
        auto load_codes = [&](int4 (&r)[kGaRows], int t) {
            const int off = (t * TT) % CHUNK, rb = warp - kSmWarps;
#pragma unroll
            for (int i = 0; i < kGaRows; ++i) {
                const int rr = rb + kGaWarps * i;
                const int row = rr < TT ? s_crow[off + rr] : -1;
                r[i] = row >= 0 ? __ldg(reinterpret_cast<const int4*>(kv8 + (kv_seq + row) * HD + lane * 16))
                                : make_int4(0, 0, 0, 0);
            }
        };
        if (KV_I8 && QM != 2) {
            const int c = lane, rb = warp - kSmWarps;   // 32 chunks of 16 int8 per row; rows rb + 3i
            auto store = [&](const int4 (&r)[kGaRows], int t, float sc, int ex, float cor) {
                wait_slot(t);
                uint8_t* box = sm + C::OFF_K + (t & 1) * KSLOT + (c >> 2) * KBOX;   // 64 dims per box
#pragma unroll
                for (int i = 0; i < kGaRows; ++i) {
                    const int rr = rb + kGaWarps * i;
                    if (rr < TT) store_codes16(box, rr, c, r[i]);
                }
                publish(t, sc, ex, cor);
            };
            auto load = load_codes;
            // two tiles in flight: the next tile's loads are issued before this tile is converted
            int4 ra[kGaRows], rb2[kGaRows];
            float sca = 0.f, scb = 0.f, cora = 0.f, corb = 0.f;
            int exa = 0, exb = 0;
            if (ntiles > 0) {
                load(ra, 0);   // needs only the rows; the scales arrive meanwhile
                finish_scales();
                named_bar_sync(BAR_GATHER, kGaThreads);
                sca = entry_scale(0);
                cora = entry_cor(0);
                exa = chunk_exp();
            }
            // one call site each for load and store (the code of this loop stays small): the buffers
            // trade places after every tile instead
#pragma unroll 1
            for (int t = 0; t < ntiles; ++t) {
                if (t + 1 < ntiles) {
                    if (((t + 1) * TT) % CHUNK == 0) next_chunk(t + 1);
                    scb = entry_scale(t + 1);
                    corb = entry_cor(t + 1);
                    exb = chunk_exp();
                    load(rb2, t + 1);
                }
                store(ra, t, sca, exa, cora);
#pragma unroll
                for (int i = 0; i < kGaRows; ++i) ra[i] = rb2[i];
                sca = scb;
                cora = corb;
                exa = exb;
            }
        } else if (QM == 2) {
            // the _full operator: codes of tile t -> slot 0 (fp16, first product), its bf16 values -> slot 1
            // (second product).  One tile of each, so tile t is written after the second product of t - 1;
            // the codes and the first half of the value rows are loaded before that wait, the second half
            // after the codes are stored (registers: 22 + 22 sixteen-byte chunks at most).
            const __nv_bfloat16* vals = static_cast<const __nv_bfloat16*>(p.kv_val);
            const int rb = warp - kSmWarps;
            constexpr int kHalf = (kGaRows + 1) / 2;   // value rows per half (11)
            auto load_vals = [&](uint4 (&v)[2 * kHalf], int t, int i0) {
                const int off = (t * TT) % CHUNK;
#pragma unroll
                for (int i = 0; i < kHalf; ++i) {
                    const int rr = rb + kGaWarps * (i0 + i);
                    const int row = (i0 + i < kGaRows && rr < TT) ? s_crow[off + rr] : -1;
                    const __nv_bfloat16* src = vals + (kv_seq + max(row, 0)) * HD;
                    v[2 * i] = row >= 0 ? __ldg(reinterpret_cast<const uint4*>(src + lane * 8)) : make_uint4(0, 0, 0, 0);
                    v[2 * i + 1] = row >= 0 ? __ldg(reinterpret_cast<const uint4*>(src + (lane + 32) * 8))
                                            : make_uint4(0, 0, 0, 0);
                }
            };
            auto store_vals = [&](const uint4 (&v)[2 * kHalf], int i0) {
                uint8_t* slot = sm + C::OFF_K + KSLOT;
#pragma unroll
                for (int i = 0; i < kHalf; ++i) {
                    const int rr = rb + kGaWarps * (i0 + i);
                    if (i0 + i >= kGaRows || rr >= TT) continue;
                    *reinterpret_cast<uint4*>(slot + (lane >> 3) * KBOX + swz(rr, lane & 7)) = v[2 * i];
                    *reinterpret_cast<uint4*>(slot + (4 + (lane >> 3)) * KBOX + swz(rr, lane & 7)) = v[2 * i + 1];
                }
            };
            if (ntiles > 0) {
                finish_scales();
                named_bar_sync(BAR_GATHER, kGaThreads);
            }
#pragma unroll 1
            for (int t = 0; t < ntiles; ++t) {
                if (t > 0 && (t * TT) % CHUNK == 0) next_chunk(t);
                const float sc = entry_scale(t);
                int4 rc[kGaRows];
                uint4 va[2 * kHalf];
                load_codes(rc, t);
                load_vals(va, t, 0);
                wait_slot(t);
                uint8_t* box = sm + C::OFF_K + (lane >> 2) * KBOX;   // slot 0
#pragma unroll
                for (int i = 0; i < kGaRows; ++i) {
                    const int rr = rb + kGaWarps * i;
                    if (rr < TT) store_codes16(box, rr, lane, rc[i]);
                }
                store_vals(va, 0);
                load_vals(va, t, kHalf);
                store_vals(va, kHalf);
                publish(t, sc, 0, entry_cor(t));
            }
        } else {
            const __nv_bfloat16* kv = static_cast<const __nv_bfloat16*>(p.kv);
            const int rb = warp - kSmWarps;   // 64 chunks of 8 bf16 per row: lane and lane + 32; rows rb + 3i
            if (ntiles > 0) {
                finish_scales();
                named_bar_sync(BAR_GATHER, kGaThreads);
            }
            for (int t = 0; t < ntiles; ++t) {
                if (t > 0 && (t * TT) % CHUNK == 0) next_chunk(t);
                const float sc = entry_scale(t);
                const int off = (t * TT) % CHUNK;
                uint4 v[2 * kGaRows];
#pragma unroll
                for (int i = 0; i < kGaRows; ++i) {
                    const int rr = rb + kGaWarps * i;
                    const int row = rr < TT ? s_crow[off + rr] : -1;
                    const __nv_bfloat16* src = kv + (kv_seq + max(row, 0)) * HD;
                    v[2 * i] = row >= 0 ? __ldg(reinterpret_cast<const uint4*>(src + lane * 8)) : make_uint4(0, 0, 0, 0);
                    v[2 * i + 1] = row >= 0 ? __ldg(reinterpret_cast<const uint4*>(src + (lane + 32) * 8))
                                            : make_uint4(0, 0, 0, 0);
                }
                wait_slot(t);
                uint8_t* slot = sm + C::OFF_K + (t & 1) * KSLOT;
#pragma unroll
                for (int i = 0; i < kGaRows; ++i) {
                    const int rr = rb + kGaWarps * i;
                    if (rr >= TT) continue;
                    *reinterpret_cast<uint4*>(slot + (lane >> 3) * KBOX + swz(rr, lane & 7)) = v[2 * i];
                    *reinterpret_cast<uint4*>(slot + (4 + (lane >> 3)) * KBOX + swz(rr, lane & 7)) = v[2 * i + 1];
                }
                publish(t, sc, 0, 0.f);
            }
        }
        wait_q();   // every gather thread takes part in the query barrier once, with or without tiles
    } else if (warp == kMmaWarp) {
        // ================================================================ MMA issue (lane 0)
        // Issue whichever product is ready: the second product of the oldest
        // tile first (it frees a K slot and lets the next P be written), else
        // the first product of the next tile.
        int g1 = 0, g2 = 0;   // next tile for the first / second product
        named_bar_sync(BAR_Q, kThreads);   // the query tile is in shared memory
        tc_fence_after();
        uint64_t t_last = globaltimer_ns();
        while (g2 < ntiles) {
            int choice = 0;
            if (lane == 0) {
                if (*s_abort) {
                    choice = 3;
                } else if (g2 < g1 && mbar_try_wait(BAR(B_PFULL + (g2 & 1)), (g2 >> 1) & 1)) {
                    choice = 2;
                } else if (g1 < ntiles && mbar_try_wait(BAR(B_KFULL + (g1 & 1)), (g1 >> 1) & 1) &&
                           (g1 < 2 || mbar_try_wait(BAR(B_SEMPTY + (g1 & 1)), ((g1 >> 1) + 1) & 1))) {
                    choice = 1;
                } else if (globaltimer_ns() - t_last > 2000000000ull) {
                    *s_abort = 1;
                    atomicExch(p.status, kDevTimeout);
                    choice = 3;
                }
            }
            choice = __shfl_sync(0xffffffffu, choice, 0);
            if (choice == 3) break;
            if (choice == 0) continue;
            tc_fence_after();
            if (lane == 0) {
                t_last = globaltimer_ns();
                // Descriptors are formed once per product; the operand steps are added to the start-address
                // field (address >> 4, 14 bits: every shared address here is below 256 KB, so no carry),
                // which keeps the issue loop at a few instructions per MMA.
                if (choice == 1) {
                    const int slot = g1 & 1;
                    const uint64_t dq = sdesc_sw128(qbase, 16, 1024), dk = sdesc_sw128(kbase + k_slot(g1) * KSLOT, 16, 1024);
                    const uint32_t td = tbase + C::S_COL + slot * TT;
#pragma unroll
                    for (int part = 0; part < (QSPLIT ? 2 : 1); ++part)
#pragma unroll
                        for (int kb = 0; kb < 8; ++kb)
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                umma_bf16(td, dq + (uint64_t)(((part * 8 + kb) * C::QBOX + kk * 32) >> 4),
                                          dk + (uint64_t)((kb * KBOX + kk * 32) >> 4), id1, (part | kb | kk) != 0);
                    umma_commit(BAR(B_SFULL + slot));
                } else {
                    const uint64_t dv = sdesc_sw128(kbase + v_slot(g2) * KSLOT, KBOX, 1024);
                    const uint64_t dp = sdesc_sw128(pbase + (g2 & 1) * C::PBYTES, 16, 1024);
                    const uint32_t acc0 = g2 > 0 ? 1u : 0u;
#pragma unroll
                    for (int mb = 0; mb < 4; ++mb)
#pragma unroll
                        for (int ks = 0; ks < TT / 16; ++ks)
                            umma_bf16(tbase + C::O_COL + mb * NQ, dv + (uint64_t)((2 * mb * KBOX + ks * 2048) >> 4),
                                      dp + (uint64_t)((ks * 32) >> 4), id2, ks > 0 ? 1u : acc0);
                    umma_commit(BAR(B_KEMPTY + (g2 & 1)));
                    umma_commit(BAR(B_PEMPTY + (g2 & 1)));
                }
            }
            if (choice == 1) ++g1; else ++g2;
            __syncwarp();
        }
    } else {
        // ================================================================ query tile (softmax warps)
        store_q();
        {   // the query tile, continued: the group's exponent (fp16 products), then the conversion in place,
            // four chunks at a time (a compact loop: this once-per-CTA code is bound by instruction fetch,
            // and four independent chunks keep a single warp per scheduler busy)
            auto chunk8 = [&](int c, float (&v)[8]) {   // dims [8c, 8c + 8) of this thread's share, unconverted
                const uint4 a = *reinterpret_cast<const uint4*>(qslot(c, 0));
                if (QSPLIT) {
                    const uint4 b = *reinterpret_cast<const uint4*>(qslot(c, 1));
                    v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y);
                    v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
                    v[4] = __uint_as_float(b.x); v[5] = __uint_as_float(b.y);
                    v[6] = __uint_as_float(b.z); v[7] = __uint_as_float(b.w);
                } else {
                    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        v[2 * u] = __uint_as_float(w[u] << 16);
                        v[2 * u + 1] = __uint_as_float(w[u] & 0xffff0000u);
                    }
                }
            };
            float sq = 1.f;
            if (QM) {   // query codes are final as stored (|code| <= 255): no exponent
                if (tid == 0) s_qexp[1] = 0;
            } else if (KV_I8) {   // fp16 products: the group's q * 2^-qe has its largest magnitude in [2^14, 2^15)
                uint32_t mx = qmax_bits;
#pragma unroll
                for (int o = 1; o < QTPR; o <<= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                if (qpart == 0 && mx > 0u) atomicMax(&s_qexp[0], (int)mx);   // non-negative float bits: int order
                named_bar_sync(BAR_SOFTMAX, 32 * kSmWarps);
                const int mb = s_qexp[0];
                const int qe = mb > 0 ? min(max(((mb >> 23) & 0xff) - 127 - 14, -126), 113) : 0;
                sq = __int_as_float((127 - qe) << 23);
                if (tid == 0) s_qexp[1] = qe;
            }
            if ((KV_I8 || QSPLIT) && !QM) {   // a bf16 query for bf16 products is already in its final form
#pragma unroll 1
                for (int c0 = 0; c0 < QDPT / 8; c0 += 4) {
                    float vv[4][8];
#pragma unroll
                    for (int k = 0; k < 4; ++k) chunk8(c0 + k, vv[k]);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                    const int c = c0 + k;
                    const float (&v)[8] = vv[k];
                    uint32_t hi[4], lo[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float a = v[2 * u] * sq, b = v[2 * u + 1] * sq;   // exact: a power of two
                        if (KV_I8) {
                            const __half2 hh = __floats2half2_rn(a, b);
                            hi[u] = *reinterpret_cast<const uint32_t*>(&hh);
                            const float2 hf = __half22float2(hh);
                            const __half2 l2 = __floats2half2_rn(a - hf.x, b - hf.y);
                            lo[u] = *reinterpret_cast<const uint32_t*>(&l2);
                        } else {
                            hi[u] = pack_bf16(a, b);
                            lo[u] = pack_bf16(a - __uint_as_float(hi[u] << 16), b - __uint_as_float(hi[u] & 0xffff0000u));
                        }
                    }
                    *reinterpret_cast<uint4*>(qslot(c, 0)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    if (QSPLIT) *reinterpret_cast<uint4*>(qslot(c, 1)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                }
            }
            fence_proxy_async_smem();   // the tile -> the async proxy (tensor-core operand)
            named_bar_arrive(BAR_Q, kThreads);
        }
        // ================================================================ softmax (thread = head)
        const int h = warp * 16 + lane;
        const bool own = lane < 16 && h < NQ;
        const bool active = own && h < nrows;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        float m = -INFINITY, l = 0.f;
        int eref = 0;   // value-scale exponent O is accumulated in (the largest chunk exponent so far)
        // query-code mode: this head's u8 query scale (the score is ((dot - 128 ksum) * q_scale) * factor)
        const float qsh = (QM && active) ? __ldg(p.q_scales + (int64_t)seq * p.nq + row0 + h) : 1.f;
        for (int t = 0; t < ntiles; ++t) {
            const int sb = t & 1;
            wait_bar(BAR(B_SFULL + sb), (t >> 1) & 1, s_abort, p.status);
            tc_fence_after();
            // this tile's chunk exponent: O and l are rescaled when it grows, P is scaled down when it is smaller
            const int ex = s_texp[sb];
            float alpha = 1.f, g = 1.f;   // alpha: factor on O (and, its max part, on l); g: on P
            int need = 0;
            if (t == 0) {
                eref = ex;
            } else if (ex > eref) {
                alpha = __int_as_float((127 + max(eref - ex, -126)) << 23);
                need = 1;
                eref = ex;
            } else if (ex < eref) {
                g = __int_as_float((127 + max(ex - eref, -126)) << 23);
            }
            float am = 1.f;   // the max part of alpha
            float x[TT];
#pragma unroll
            for (int j = 0; j < TT / 16; ++j) tmem_ld16(tbase + lane_base + C::S_COL + sb * TT + j * 16, x + j * 16);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(BAR(B_SEMPTY + sb));
            if (active) {
                const float4* f4 = reinterpret_cast<const float4*>(s_f + sb * TT);
                const float4* b4 = reinterpret_cast<const float4*>(s_bias + sb * TT);
                float mt0 = -INFINITY, mt1 = -INFINITY;
#pragma unroll
                for (int j = 0; j < TT / 4; ++j) {
                    const float4 f = f4[j], b = b4[j];
                    if (QM) {   // the integer dot (exact in fp32) less 128 * ksum, times the query scale
                        const float4 c = reinterpret_cast<const float4*>(s_cor + sb * TT)[j];
                        x[4 * j] = (x[4 * j] + c.x) * qsh;
                        x[4 * j + 1] = (x[4 * j + 1] + c.y) * qsh;
                        x[4 * j + 2] = (x[4 * j + 2] + c.z) * qsh;
                        x[4 * j + 3] = (x[4 * j + 3] + c.w) * qsh;
                    }
                    x[4 * j] = fmaf(x[4 * j], f.x, b.x);
                    x[4 * j + 1] = fmaf(x[4 * j + 1], f.y, b.y);
                    x[4 * j + 2] = fmaf(x[4 * j + 2], f.z, b.z);
                    x[4 * j + 3] = fmaf(x[4 * j + 3], f.w, b.w);
                    mt0 = fmaxf(mt0, fmaxf(x[4 * j], x[4 * j + 1]));
                    mt1 = fmaxf(mt1, fmaxf(x[4 * j + 2], x[4 * j + 3]));
                }
                const float mt = fmaxf(mt0, mt1);
                const bool grow = mt > m + kLazy;   // also true when m == -inf and mt is finite
                const float mn = grow ? mt : m;
                if (grow) {
                    am = ex2(m - mn);               // 0 when m == -inf
                    need |= m != -INFINITY;
                }
                alpha *= am;
                m = mn;
                const float4* s4 = reinterpret_cast<const float4*>(s_psc + sb * TT);
                const float mneg = mn == -INFINITY ? 0.f : -mn;   // with mn == -inf every x is -inf: p = 0
                float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
                for (int j = 0; j < TT / 4; ++j) {
                    const float4 s = s4[j];
                    const float p0 = ex2(x[4 * j] + mneg), p1 = ex2(x[4 * j + 1] + mneg);
                    const float p2 = ex2(x[4 * j + 2] + mneg), p3 = ex2(x[4 * j + 3] + mneg);
                    ls0 += p0 + p1;
                    ls1 += p2 + p3;
                    x[4 * j] = p0 * s.x;            // the value scale folded into P
                    x[4 * j + 1] = p1 * s.y;
                    x[4 * j + 2] = p2 * s.z;
                    x[4 * j + 3] = p3 * s.w;
                }
                if (g != 1.f) {
#pragma unroll
                    for (int j = 0; j < TT; ++j) x[j] *= g;
                }
                l = l * am + (ls0 + ls1);
            }
            if (own) s_alpha[sb * 64 + h] = alpha;
            need = __any_sync(0xffffffffu, need);
            if (lane == 0) s_need[sb * 4 + warp] = need;
            named_bar_sync(BAR_SOFTMAX, 32 * kSmWarps);
            const int any = s_need[sb * 4] | s_need[sb * 4 + 1] | s_need[sb * 4 + 2] | s_need[sb * 4 + 3];
            // Second product j is the (j >> 1)-th completion of P-empty barrier j & 1.  Each wait below
            // is for a product no older than one this thread already waited for two tiles ago and
            // no newer than the last P it wrote, so the barrier is never two phases from the parity.
            if (t >= 2) {   // second product t - 2 has read P buffer t & 1
                wait_bar(BAR(B_PEMPTY + sb), ((t >> 1) + 1) & 1, s_abort, p.status);
                tc_fence_after();
            }
            if (t > 0 && any) {
                // second product t - 1 has finished: O is stable
                wait_bar(BAR(B_PEMPTY + (sb ^ 1)), ((t - 1) >> 1) & 1, s_abort, p.status);
                tc_fence_after();
                // O *= alpha per head (column); this warp's 32 dims of each 128-dim block.  Rare (lazy
                // rescale), so kept as a compact loop; the 16 factors are read before the TMEM store.
#pragma unroll 1
                for (int it = 0; it < 4 * (NQ / 16); ++it) {
                    const int mb = it / (NQ / 16), cb = it % (NQ / 16);
                    const uint32_t ta = tbase + lane_base + C::O_COL + mb * NQ + cb * 16;
                    float v[16], a[16];
                    tmem_ld16(ta, v);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 x = reinterpret_cast<const float4*>(s_alpha + sb * 64 + cb * 16)[q];
                        a[4 * q] = x.x; a[4 * q + 1] = x.y; a[4 * q + 2] = x.z; a[4 * q + 3] = x.w;
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int u = 0; u < 16; ++u) v[u] *= a[u];
                    tmem_st16(ta, v);
                }
                tmem_wait_st();
            }
            if (own) {   // this head's P row: 64 entries, 8 swizzled 16-byte chunks (zeros when inactive)
                uint8_t* prow = sm + C::OFF_P + sb * C::PBYTES + h * 128;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t w4[4] = {0u, 0u, 0u, 0u};
                    if (active) {
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            if (P_F16) {
                                const __half2 hp = __floats2half2_rn(x[8 * j + 2 * u], x[8 * j + 2 * u + 1]);
                                w4[u] = *reinterpret_cast<const uint32_t*>(&hp);
                            } else {
                                w4[u] = pack_bf16(x[8 * j + 2 * u], x[8 * j + 2 * u + 1]);
                            }
                        }
                    }
                    const uint4 w = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    *reinterpret_cast<uint4*>(prow + ((j ^ (h & 7)) << 4)) = w;
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(BAR(B_PFULL + sb));
        }
        if (ntiles > 0) {   // the last second product has finished: O is final
            wait_bar(BAR(B_PEMPTY + ((ntiles - 1) & 1)), ((ntiles - 1) >> 1) & 1, s_abort, p.status);
            tc_fence_after();
        }
        m_final = m;
        l_final = l;
        eref_final = eref;
    }
#undef BAR
    // ---- epilogue: each head's normaliser and log-sum-exp (softmax threads), then all eight warps
    //      move O^T out of TMEM (warp w reads TMEM lanes 32*(w%4).., dims of blocks 2*(w/4), 2*(w/4)+1)
    const bool have = ntiles > 0 && !*s_abort;
    if (warp < kSmWarps && lane < 16 && warp * 16 + lane < NQ) {
        const int h = warp * 16 + lane;
        const bool ok = have && h < nrows && l_final > 0.f;
        // O^T was accumulated with the value scales times 2^-eref: 2^eref / l normalises it
        s_rinv[h] = ok ? __int_as_float((127 + eref_final) << 23) / l_final : 0.f;
        s_rlse[h] = ok ? m_final * kLn2 + logf(l_final) : -INFINITY;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const int64_t orow0 = (int64_t)seq * p.nq + row0;   // output row of this group's first query row
    const int64_t nrows_all = (int64_t)gridDim.y / p.ngroups * p.nq;   // bs * nq
    const bool partial = splits > 1;
    const bool bf16_out = !partial && !p.out_f32;
    // this group's nrows output rows are contiguous: staged row-major in the (now idle) K ring and
    // written with one bulk copy, or, when the output is not 16-byte aligned, stored directly
    const bool bulk = partial || p.out_aligned;
    uint8_t* dst = partial ? reinterpret_cast<uint8_t*>(p.part_o + ((size_t)split * nrows_all + orow0) * HD)
                           : static_cast<uint8_t*>(p.out) + orow0 * HD * (bf16_out ? 2 : 4);
    // Warp w: TMEM lanes 32*(w%4).. = dims d, 16 heads (columns) at a time.  The 16 factors are read
    // into registers before the stores (shared-memory stores would otherwise order every later factor
    // load behind them); s_rinv is 0 for rows past nrows and for empty heads, where O is 0 too (P was 0),
    // except with no tiles at all, when O was never written: zeros then.  The loops are kept compact and
    // free of branches: this once-per-CTA code is bound by instruction fetch, not arithmetic.
    const int q4 = warp & 3;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const uint32_t stage = smem_u32(sm + C::OFF_K);
    auto o_block = [&](int mb, int cb, float (&v)[16]) {   // v = O[head cb*16 + u][dim] * factor
        float f[16];
        if (have) tmem_ld16(tbase + lane_base + C::O_COL + mb * NQ + cb * 16, v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 x = reinterpret_cast<const float4*>(s_rinv + cb * 16)[q];
            f[4 * q] = x.x; f[4 * q + 1] = x.y; f[4 * q + 2] = x.z; f[4 * q + 3] = x.w;
        }
        if (have) {
            tmem_wait_ld();
        } else {
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = 0.f;
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] *= f[u];
    };
    if (partial) {
        if (have) {   // an empty partial writes only its -inf log-sum-exp
            // 16 rows at a time: staged (fp32, row-major), then one bulk copy, which overlaps the staging
            // of the next 16 rows
            float* po = p.part_o + ((size_t)split * nrows_all + orow0) * HD;
#pragma unroll 1
            for (int cb = 0; cb < NQ / 16 && cb * 16 < nrows; ++cb) {
#pragma unroll 1
                for (int mi = 0; mi < 2; ++mi) {
                    const int mb = (warp >> 2) * 2 + mi, d = mb * 128 + q4 * 32 + lane;
                    float v[16];
                    o_block(mb, cb, v);
#pragma unroll
                    for (int u = 0; u < 16; ++u)
                        asm volatile("st.shared.f32 [%0], %1;" ::"r"(stage + (uint32_t)(((cb * 16 + u) * HD + d) * 4)),
                                     "f"(v[u]) : "memory");
                }
                fence_proxy_async_smem();   // the staged rows -> the async proxy
                __syncthreads();
                if (tid == 0) {
                    bulk_store(po + cb * 16 * HD, stage + (uint32_t)(cb * 16 * HD * 4),
                               (uint32_t)(min(16, nrows - cb * 16) * HD * 4));
                    bulk_commit();
                }
            }
            if (tid == 0) bulk_wait_all();   // complete before the CTA exits (the merge grid reads it)
        }
    } else {
        // the output itself (bf16 or fp32): staged and written with one bulk copy when 16-byte aligned
        const int esz = bf16_out ? 2 : 4;
#pragma unroll 1
        for (int it = 0; it < 2 * (NQ / 16); ++it) {
            const int mb = (warp >> 2) * 2 + it / (NQ / 16), cb = it % (NQ / 16);
            if (cb * 16 >= nrows) continue;   // uniform across the warp
            const int d = mb * 128 + q4 * 32 + lane;
            float v[16];
            o_block(mb, cb, v);
            if (bulk) {
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const uint32_t a = stage + (uint32_t)(((cb * 16 + u) * HD + d) * esz);
                    if (bf16_out) {
                        const __nv_bfloat16 b = __float2bfloat16_rn(v[u]);
                        asm volatile("st.shared.b16 [%0], %1;" ::"r"(a), "h"(*reinterpret_cast<const uint16_t*>(&b))
                                     : "memory");
                    } else {
                        asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v[u]) : "memory");
                    }
                }
            } else {
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int h = cb * 16 + u;
                    if (h >= nrows) break;
                    if (bf16_out) reinterpret_cast<__nv_bfloat16*>(dst)[h * HD + d] = __float2bfloat16_rn(v[u]);
                    else reinterpret_cast<float*>(dst)[h * HD + d] = v[u];
                }
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (bulk && tid == 0) {
            bulk_store(dst, stage, (uint32_t)(nrows * HD * esz));
            bulk_commit();
            bulk_wait_all();
        }
    }
    tc_fence_before();   // every TMEM read is done before the dealloc below
    __syncthreads();
    if (tid < nrows) {
        if (partial) p.part_lse[(size_t)split * nrows_all + orow0 + tid] = s_rlse[tid];
        else if (p.out_lse) p.out_lse[orow0 + tid] = s_rlse[tid];
    }
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tbase, C::TMEM_COLS);
}

// CTAs each (sequence, group) is split over: the most that keep the whole
// grid within one wave of one CTA per SM, at most kMaxSplit, and no more than
// give every CTA one full tile.  `per_seq` bounds the entries of one sequence.
static int split_count(int64_t groups, int64_t per_seq, int nsm) {
    if (groups >= nsm) return 1;
    int64_t s = std::min<int64_t>(nsm / groups, kMaxSplit);
    s = std::min<int64_t>(s, per_seq / TT);
    return (int)std::max<int64_t>(s, 1);
}

template <bool KV_I8, bool QSPLIT, int QM = 0>
static int launch(const Params& p, int groups, int splits, cudaStream_t st) {
    auto kfn = csa_decode_kernel<KV_I8, QSPLIT, QM>;
    static int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg<QSPLIT>::SMEM) !=
            cudaSuccess)
            return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for csa_decode_kernel");
        configured_dev = dev;
    }
    kfn<<<dim3((unsigned)splits, (unsigned)groups, 1), kThreads, Cfg<QSPLIT>::SMEM, st>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace csa

size_t csa_workspace_bytes(int bs, int nq, int q_f32) {
    using namespace csa;
    const int NQ = q_f32 ? Cfg<true>::NQ : Cfg<false>::NQ;
    const int64_t groups = (int64_t)bs * ((nq + NQ - 1) / NQ);
    const int splits = split_count(groups, INT64_MAX, device_sm_count());   // the most any k can use
    // the partials follow the fixed counter header every workspace starts with (left untouched here),
    // so one workspace can serve this kernel and the kernels whose merge tickets live in that header
    const size_t parts = splits > 1 ? (size_t)splits * bs * nq * (HD + 1) * sizeof(float) : 0;
    return kCounterHeaderBytes + parts;
}

int csa_launch(const CsaLaunch& a) {
    using namespace csa;
    if (!a.workspace || a.workspace_bytes < csa_workspace_bytes(a.bs, a.nq, a.q_f32))
        return set_error(WS_ERR_WORKSPACE, "csa_decode: workspace missing or smaller than ws_csa_decode_workspace_size");
    if (reinterpret_cast<uintptr_t>(a.workspace) % 16)
        return set_error(WS_ERR_INVALID_ARG, "csa_decode: workspace must be 16-byte aligned");
    Params p;
    memset(&p, 0, sizeof(p));
    p.q = a.q;
    p.q_f32 = a.q_f32;
    p.nq = a.nq;
    const int NQ = a.q_f32 ? Cfg<true>::NQ : Cfg<false>::NQ;
    p.ngroups = (a.nq + NQ - 1) / NQ;
    if ((int64_t)a.bs * p.ngroups > 65535) return set_error(WS_ERR_UNSUPPORTED, "csa_decode: too many query groups");
    p.kv = a.kv;
    p.kv_i8 = a.kv_i8;
    p.kv_scales = a.kv_scales;
    p.q_scales = a.q_scales;
    p.kv_sums = a.kv_sums;
    p.kv_val = a.kv_val;
    p.idx = a.idx;
    p.k = a.k;
    p.window = a.window;
    p.shard_lo = a.shard_lo;
    p.shard_hi = a.shard_lo + a.nc_local;
    p.dense_begin = std::max(a.dense_begin, p.shard_lo);
    p.dense_end = std::max(p.dense_begin, std::min(a.dense_end, p.shard_hi));
    p.nc_local = a.nc_local;
    p.scale_log2 = a.scale * kLog2e;
    p.out = a.out;
    p.out_f32 = a.out_f32;
    p.out_aligned = reinterpret_cast<uintptr_t>(a.out) % 16 == 0;
    p.out_lse = a.out_lse;
    p.status = device_status_word();
    if (a.bs == 0 || a.nq == 0) return WS_OK;
    // entries one sequence selects (a sharded sorted list selects about k * nc_local / nc; k bounds it)
    const int64_t per_seq = a.idx ? (int64_t)a.k : p.dense_end - p.dense_begin;
    const int groups = a.bs * p.ngroups;
    const int splits = split_count(groups, per_seq, device_sm_count());
    const int64_t rows = (int64_t)a.bs * a.nq;
    if (splits > 1) {
        p.part_o = reinterpret_cast<float*>(static_cast<uint8_t*>(a.workspace) + kCounterHeaderBytes);
        p.part_lse = p.part_o + (size_t)splits * rows * HD;
    }
    cudaStream_t st = static_cast<cudaStream_t>(a.stream);
    int rc;
    if (a.q_u8)
        rc = a.kv_val ? launch<true, false, 2>(p, groups, splits, st) : launch<true, false, 1>(p, groups, splits, st);
    else if (a.kv_i8)
        rc = a.q_f32 ? launch<true, true>(p, groups, splits, st) : launch<true, false>(p, groups, splits, st);
    else
        rc = a.q_f32 ? launch<false, true>(p, groups, splits, st) : launch<false, false>(p, groups, splits, st);
    if (rc != WS_OK || splits == 1) return rc;
    return lse_merge_launch(p.part_o, rows * HD, p.part_lse, rows, splits, rows, HD, a.out,
                            a.out_f32 ? WS_DTYPE_F32 : WS_DTYPE_BF16, a.out_lse, st, /*after_primary=*/true);
}

}  // namespace ws
