// GQA / MLA(non-absorbed) split-KV decode attention for sm_100a.
//
// Replaces the AVX-512 run_kernel<KV_BF16,Q_BF16,Normalize> of the reference
// (kernel/cpu_attn.cpp:193-570) behind fused_cpu_attn (:572-636) and
// fused_cpu_attn_mla (:638-672), and the runtime's two-share
// (physically partitioned) decode + LSE merge (system/mixoffload.py:1263-1268,
// :1456-1464).
//
// One persistent launch.  The KV work is a list of segments (a segment is the
// token range of one KV row -- a (batch, kv-head) pair -- inside one share);
// each segment is cut into 64-token tiles and the flattened tile space is
// split evenly over the CTAs (one CTA per SM).  Per CTA:
//   * warp 4 (one elected lane) streams K and V tiles with 3-D TMA
//     (SWIZZLE_128B boxes of 64 dims x 64 tokens) through an S-stage mbarrier
//     ring;
//   * warps 0-3 each take 16 tokens of every tile and run the decode on the
//     tensor cores with the operands swapped so that the query group is the
//     MMA N dimension:  S^T[16 tok x 8 grp] = K[16 x Dk] . Q^T[Dk x 8]  and
//     O^T[Dv x 8] += V^T[Dv x 16] . P^T[16 x 8]  (mma.sync m16n8k16 bf16,
//     fp32 accumulate; P^T is transposed in registers with movmatrix);
//   * at every segment boundary the four warps' online-softmax states are
//     merged in shared memory into one piece (o, m, l).  A segment that sits
//     inside one CTA is written out directly; otherwise pieces go to the
//     workspace and the CTA that files the last piece of a group (found with
//     an atomic ticket) merges them by log-sum-exp and writes the output.
#include "common.cuh"
#include "ws_internal.h"

namespace ws {

constexpr int kTile = 64;        // tokens per TMA tile
// Ragged shares: every non-empty segment starts with kSegLead empty tiles in the flattened tile space.
// They carry no data (nothing is loaded or computed for them) but count in the even split over the
// CTAs, so a CTA whose range crosses many short segments takes fewer tiles: each segment change costs
// it a segment lookup, a piece and a query reload, about as long as kSegLead tiles of streaming.
constexpr int kSegLead = 6;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxShares = 4;
// Most pieces one group can have: one per CTA plus one per extra share.  The
// host caps the grid at kMaxPieces - kMaxShares CTAs.
constexpr int kMaxPieces = 160;

struct GqaMaps {
    CUtensorMap k[kMaxShares];
    CUtensorMap v[kMaxShares];
};

struct GqaParams {
    const __nv_bfloat16* q;
    int64_t q_row_stride;      // elements between consecutive group-rows of q
    int G, Dk, Dv;
    float scale;
    int varlen;                // 0: dense rows, 1: ragged shares
    int n_rows, L;             // dense
    int B, Hkv, nshare;        // varlen
    const int* cu[kMaxShares]; // varlen, packed share: cumulative token offsets [B+1]
    const int* lens[kMaxShares];  // varlen, padded share: tokens per sequence [B] (rows b*Hkv + h)
    int tok_in_dim2[kMaxShares];
    int has_map[kMaxShares];
    int n_groups;
    int out_mode;
    void* out;
    void* out_max;
    void* out_sum;
    float* out_lse;
    int64_t out_row_stride;    // elements between output group-rows
    int64_t ml_row_stride;     // elements between max/sum/lse group-rows
    float* ws_part;
    int* ws_cnt;
    int* status;
    int defer_merge;           // pieces are merged by gqa_merge_kernel (dense rows over many CTAs; shares)
    int* ws_pre;               // deferred varlen merge: the tile prefix over sequences [B+1], from CTA 0
};

struct Seg {
    int j;        // segment index
    int map;      // share
    int y;        // row coordinate (kv row or kv head)
    int x0;       // first token of the segment in its share
    int len;      // tokens
    int group;    // output group-row
    int t0;       // first tile in the flattened tile space
    int lead;     // empty tiles before the segment's first data tile (ragged shares: kSegLead)
};

template <int DKP, int DVP, int NT, int STAGES>
struct GqaCfg {
    static constexpr int NG = NT * 8;                       // padded query groups
    static constexpr int KBOX = DKP / 64, VBOX = DVP / 64;
    static constexpr int BOX_BYTES = kTile * 128;
    static constexpr int STAGE_BYTES = (KBOX + VBOX) * BOX_BYTES;
    static constexpr int RED_FLOATS = kConsumerWarps * NG * (DVP + 2);
    static constexpr int SLOT_FLOATS = NG * DVP + 2 * NG;
    // merge of a group's pieces: slot list, per-piece (weight, l), group (M, L)
    static constexpr int COMB_BYTES = kMaxPieces * 4 + 2 * kMaxPieces * NG * 4 + 2 * NG * 4;
    static constexpr size_t fixed_smem() {
        return 1024 /*align slack*/ + size_t(STAGES) * STAGE_BYTES + RED_FLOATS * 4 + 2 * STAGES * 8 + 64 +
               COMB_BYTES;
    }
};

// ---------------------------------------------------------------- segments
struct SegTable {
    const GqaParams* p;
    const int* pre;   // varlen: exclusive prefix of tiles per sequence, [B+1] in smem
    int tpr;          // dense: tiles per row

    // Tokens of sequence b in share s: a packed share gives offsets, a padded
    // share (one capacity-sized row per (sequence, kv-head)) gives lengths.
    __device__ __forceinline__ int seq_len(int s, int b) const {
        return p->lens[s] ? __ldg(p->lens[s] + b) : __ldg(p->cu[s] + b + 1) - __ldg(p->cu[s] + b);
    }

    // Tiles of a ragged segment of len tokens in the flattened tile space (its lead-in included).
    __device__ __forceinline__ static int vtiles(int len) { return len > 0 ? (len + kTile - 1) / kTile + kSegLead : 0; }

    __device__ __forceinline__ int64_t total() const {
        return p->varlen ? (int64_t)pre[p->B] : (int64_t)p->n_rows * tpr;
    }

    __device__ Seg of_tile(int64_t t) const {
        Seg s;
        if (!p->varlen) {
            int j = (int)(t / tpr);
            s.j = j; s.map = 0; s.y = j; s.x0 = 0; s.len = p->L; s.group = j; s.t0 = j * tpr; s.lead = 0;
            return s;
        }
        // largest b with pre[b] <= t
        int lo = 0, hi = p->B;   // pre[lo] <= t < pre[hi]
        while (hi - lo > 1) {
            int mid = (lo + hi) >> 1;
            if (pre[mid] <= t) lo = mid; else hi = mid;
        }
        const int b = lo;
        int th = 0;
        for (int sh = 0; sh < p->nshare; ++sh) th += vtiles(seq_len(sh, b));
        int r = (int)(t - pre[b]);
        const int h = r / th;
        r -= h * th;
        int base = pre[b] + h * th;
        int sh = 0;
        for (; sh < p->nshare; ++sh) {
            const int ts = vtiles(seq_len(sh, b));
            if (r < ts) break;
            r -= ts;
            base += ts;
        }
        s.j = (b * p->Hkv + h) * p->nshare + sh;
        s.map = sh;
        if (p->lens[sh]) {
            s.y = b * p->Hkv + h;
            s.x0 = 0;
        } else {
            s.y = h;
            s.x0 = __ldg(p->cu[sh] + b);
        }
        s.len = seq_len(sh, b);
        s.group = b * p->Hkv + h; s.t0 = base; s.lead = kSegLead;
        return s;
    }

    // First tile and tile count of the js-th segment of `group`.
    __device__ __forceinline__ void seg_tiles(int group, int js, int64_t& t0, int64_t& nt) const {
        if (!p->varlen) {
            t0 = (int64_t)group * tpr;
            nt = tpr;
            return;
        }
        const int b = group / p->Hkv, h = group - b * p->Hkv;
        int th = 0, before = 0, mine = 0;
        for (int sh = 0; sh < p->nshare; ++sh) {
            const int ts = vtiles(seq_len(sh, b));
            if (sh < js) before += ts;
            if (sh == js) mine = ts;
            th += ts;
        }
        t0 = pre[b] + (int64_t)h * th + before;
        nt = mine;
    }

    // Number of pieces filed for `group` by all CTAs (0 if the group is empty).
    __device__ int pieces(int group, int64_t total_tiles, int nctas) const {
        const int nseg_g = p->varlen ? p->nshare : 1;
        int n = 0;
        for (int js = 0; js < nseg_g; ++js) {
            int64_t t0, nt;
            seg_tiles(group, js, t0, nt);
            if (nt > 0)
                n += (int)(split_owner(t0 + nt - 1, total_tiles, nctas) - split_owner(t0, total_tiles, nctas) + 1);
        }
        return n;
    }
};

// ------------------------------------------------------------------ output
// m2 is the running max in log2 units (score * scale * log2 e); it is
// reported in natural units (score * scale) like the reference's max.
__device__ __forceinline__ void store_final(const GqaParams& p, int group, int grp, int d, float o_un, float m2,
                                            float l) {
    const float m = m2 * kLn2;
    const bool empty = !(l > 0.f);
    const int64_t oi = (int64_t)group * p.out_row_stride + (int64_t)grp * p.Dv + d;
    if (p.out_mode == WS_OUT_UNNORM_F32) {
        static_cast<float*>(p.out)[oi] = empty ? 0.f : o_un;
    } else {
        const float v = empty ? 0.f : o_un / l;
        if (p.out_mode == WS_OUT_NORM_BF16) static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(v);
        else static_cast<float*>(p.out)[oi] = v;
    }
    if (d == 0) {
        const int64_t mi = (int64_t)group * p.ml_row_stride + grp;
        const float mm = empty ? -INFINITY : m;
        const float ll = empty ? 0.f : l;
        if (p.out_max) {
            if (p.out_mode == WS_OUT_NORM_BF16) {
                static_cast<__nv_bfloat16*>(p.out_max)[mi] = __float2bfloat16_rn(mm);
                static_cast<__nv_bfloat16*>(p.out_sum)[mi] = __float2bfloat16_rn(ll);
            } else {
                static_cast<float*>(p.out_max)[mi] = mm;
                static_cast<float*>(p.out_sum)[mi] = ll;
            }
        }
        if (p.out_lse) p.out_lse[mi] = empty ? -INFINITY : mm + logf(ll);
    }
}

// ------------------------------------------------------------------ kernel
template <int DKP, int DVP, int NT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
gqa_decode_kernel(const __grid_constant__ GqaMaps maps, const __grid_constant__ GqaParams p) {
    using C = GqaCfg<DKP, DVP, NT, STAGES>;
    constexpr int NG = C::NG;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_base = smem;
    float* red = reinterpret_cast<float*>(smem + size_t(STAGES) * C::STAGE_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + C::RED_FLOATS);
    int* flags = reinterpret_cast<int*>(bars + 2 * STAGES);
    int* pslot = flags + 16;                                          // [kMaxPieces]
    float* pw = reinterpret_cast<float*>(pslot + kMaxPieces);         // [kMaxPieces][NG]
    float* pl = pw + kMaxPieces * NG;                                 // [kMaxPieces][NG]
    float* gml = pl + kMaxPieces * NG;                                // [2][NG]
    int* pre = reinterpret_cast<int*>(gml + 2 * NG);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grid_ctas = gridDim.x, cta = blockIdx.x;

    SegTable tab;
    tab.p = &p;
    tab.pre = pre;
    tab.tpr = p.varlen ? 0 : (p.L + kTile - 1) / kTile;

    if (p.varlen) {
        // exclusive prefix over sequences of (tiles per head * Hkv), serial (B is small)
        if (tid == 0) {
            int acc = 0;
            for (int b = 0; b < p.B; ++b) {
                pre[b] = acc;
                int th = 0;
                for (int sh = 0; sh < p.nshare; ++sh) th += SegTable::vtiles(tab.seq_len(sh, b));
                acc += th * p.Hkv;
            }
            pre[p.B] = acc;
            if (p.defer_merge && blockIdx.x == 0)
                for (int b = 0; b <= p.B; ++b) p.ws_pre[b] = pre[b];   // for gqa_merge_kernel's piece lists
        }
    }
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&bars[s]), 1);                        // full: producer arrive + tx
            mbar_init(smem_u32(&bars[STAGES + s]), kConsumerWarps);  // empty: one arrive per warp
        }
        fence_mbar_init();
        flags[0] = 0;   // abort
    }
    __syncthreads();
    pdl_launch_dependents();   // a deferred merge may be scheduled now; it waits for this grid's completion

    const int64_t total = tab.total();
    // Tiles are split over min(grid, total) CTAs so that every working CTA
    // owns at least one tile: the piece bookkeeping counts one piece per CTA
    // between a segment's first and last owner.  Surplus CTAs own nothing.
    const int nctas = total < 1 ? 1 : (total < grid_ctas ? (int)total : grid_ctas);
    const int64_t t_begin = cta < nctas ? split_start(cta, total, nctas) : total;
    const int64_t t_end = cta < nctas ? split_start(cta + 1, total, nctas) : total;
    const uint32_t full0 = smem_u32(&bars[0]), empty0 = smem_u32(&bars[STAGES]);

    if (warp == kConsumerWarps) {
        // ----------------------------------------------------------- producer
        if (lane == 0) {
            for (int s = 0; s < p.nshare; ++s)
                if (p.has_map[s]) {
                    tma_prefetch_desc(&maps.k[s]);
                    tma_prefetch_desc(&maps.v[s]);
                }
            int64_t i = 0;
            Seg sg;
            int64_t seg_end = -1;   // first tile after the current segment
            int stage = 0;
            uint32_t use = 0;
            for (int64_t t = t_begin; t < t_end; ++t, ++i) {
                if (t >= seg_end) {
                    sg = tab.of_tile(t);
                    seg_end = sg.t0 + sg.lead + (sg.len + kTile - 1) / kTile;
                }
                const int r = (int)(t - sg.t0) - sg.lead;
                if (r < 0) continue;   // a segment's lead-in: no data, no stage
                if (use > 0 && !mbar_wait_bounded(empty0 + 8 * stage, (use & 1) ^ 1)) {
                    atomicExch(p.status, kDevTimeout);
                    break;
                }
                const int x = sg.x0 + r * kTile;
                const int c1 = p.tok_in_dim2[sg.map] ? sg.y : x;
                const int c2 = p.tok_in_dim2[sg.map] ? x : sg.y;
                const uint32_t fb = full0 + 8 * stage;
                mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
                const uint32_t dst = smem_u32(stage_base + size_t(stage) * C::STAGE_BYTES);
#pragma unroll
                for (int kb = 0; kb < C::KBOX; ++kb) tma_load_3d(dst + kb * C::BOX_BYTES, &maps.k[sg.map], fb, kb * 64, c1, c2);
#pragma unroll
                for (int vb = 0; vb < C::VBOX; ++vb)
                    tma_load_3d(dst + (C::KBOX + vb) * C::BOX_BYTES, &maps.v[sg.map], fb, vb * 64, c1, c2);
                if (++stage == STAGES) {
                    stage = 0;
                    ++use;
                }
            }
        }
        return;
    }

    // --------------------------------------------------------------- consumers
    const int ctid = tid;   // 0..127
    // Empty groups (no tokens at all): written once, by CTA group % grid.
    for (int g = cta; g < p.n_groups; g += grid_ctas) {
        if (tab.pieces(g, total, nctas) == 0) {
            for (int e = ctid; e < p.G * p.Dv; e += kConsumerWarps * 32)
                store_final(p, g, e / p.Dv, e % p.Dv, 0.f, -INFINITY, 0.f);
        }
    }

    const int gq = lane >> 2, cq = lane & 3;    // mma fragment coordinates
    const int lq = lane >> 3, lr = lane & 7;    // ldmatrix address coordinates
    const float sl2 = p.scale * kLog2e;

    uint32_t qf[DKP / 16][NT][2];
    float o[DVP / 16][NT][4];
    float m_run[NT][2], l_run[NT][2];

    Seg cur;
    cur.j = -1;

    auto reset_state = [&]() {
#pragma unroll
        for (int i = 0; i < DVP / 16; ++i)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[i][nt][e] = 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m_run[nt][0] = m_run[nt][1] = -INFINITY;
            l_run[nt][0] = l_run[nt][1] = 0.f;
        }
    };

    auto load_q = [&](int group) {
        const __nv_bfloat16* qrow = p.q + (int64_t)group * p.q_row_stride;
#pragma unroll
        for (int ks = 0; ks < DKP / 16; ++ks)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int grp = nt * 8 + gq;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int d = ks * 16 + h * 8 + 2 * cq;
                    uint32_t v = 0;
                    if (grp < p.G && d < p.Dk) {   // Dk % 16 == 0, so d + 1 < Dk as well
                        const uint16_t* qe = reinterpret_cast<const uint16_t*>(qrow + (int64_t)grp * p.Dk + d);
                        v = (uint32_t)qe[0] | ((uint32_t)qe[1] << 16);
                    }
                    qf[ks][nt][h] = v;
                }
            }
    };

    // Merge the four warps' states into one piece and file it.
    auto flush = [&](const Seg& sg) {
        float* rm = red;                                   // [4][NG]
        float* rl = red + kConsumerWarps * NG;             // [4][NG]
        float* ro = red + 2 * kConsumerWarps * NG;         // [4][NG][DVP]
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float l = l_run[nt][j];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                if (gq == 0) {
                    rm[warp * NG + nt * 8 + 2 * cq + j] = m_run[nt][j];
                    rl[warp * NG + nt * 8 + 2 * cq + j] = l;
                }
            }
#pragma unroll
        for (int i = 0; i < DVP / 16; ++i)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int grp = nt * 8 + 2 * cq + (e & 1);
                    const int d = i * 16 + gq + ((e >> 1) << 3);
                    ro[(warp * NG + grp) * DVP + d] = o[i][nt][e];
                }
        named_bar_sync(1, kConsumerWarps * 32);

        // pieces of the group: counted from the segment table, except for ragged shares (always merged by
        // gqa_merge_kernel), which only need to know whether this segment is the group's only piece: the
        // group's tiles per head come from the prefix in shared memory, so no global load is waited on
        int np;
        if (p.varlen) {
            const int b = sg.group / p.Hkv;
            const int64_t th = (pre[b + 1] - pre[b]) / p.Hkv;
            const int64_t seg_tiles = SegTable::vtiles(sg.len);
            np = (seg_tiles == th && split_owner(sg.t0, total, nctas) == split_owner(sg.t0 + th - 1, total, nctas))
                     ? 1 : 2;
        } else {
            np = tab.pieces(sg.group, total, nctas);
        }
        const int slot = cta + sg.j;
        float* part = p.ws_part + (int64_t)slot * C::SLOT_FLOATS;
        // the warps' weights per query group, once: thread g < NG turns column g of rm into the weights
        // 2^(m_w - M) and column g of rl into (M, L) -- rl[g] = M, rl[NG + g] = L
        if (ctid < NG) {
            float mw[kConsumerWarps], M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                mw[w] = rm[w * NG + ctid];
                M = fmaxf(M, mw[w]);
            }
            const float Mu = (M == -INFINITY) ? 0.f : M;
            float L = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float wt = ex2(mw[w] - Mu);
                L += wt * rl[w * NG + ctid];
                rm[w * NG + ctid] = wt;
            }
            rl[ctid] = M;
            rl[NG + ctid] = L;
        }
        named_bar_sync(1, kConsumerWarps * 32);
        // the weighted sum, four values per thread and step (every warp's float4 load issued together)
        for (int ch = ctid; ch < NG * DVP / 4; ch += kConsumerWarps * 32) {
            const int e = ch * 4, grp = e / DVP, d = e - grp * DVP;
            float4 v[kConsumerWarps];
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w)
                v[w] = *reinterpret_cast<const float4*>(ro + (w * NG + grp) * DVP + d);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float wt = rm[w * NG + grp];
                acc.x += wt * v[w].x;
                acc.y += wt * v[w].y;
                acc.z += wt * v[w].z;
                acc.w += wt * v[w].w;
            }
            const float M = rl[grp], L = rl[NG + grp];
            if (np == 1) {
                if (grp < p.G) {
                    if (d < p.Dv) store_final(p, sg.group, grp, d, acc.x, M, L);
                    if (d + 1 < p.Dv) store_final(p, sg.group, grp, d + 1, acc.y, M, L);
                    if (d + 2 < p.Dv) store_final(p, sg.group, grp, d + 2, acc.z, M, L);
                    if (d + 3 < p.Dv) store_final(p, sg.group, grp, d + 3, acc.w, M, L);
                }
            } else {
                *reinterpret_cast<float4*>(part + e) = acc;
                if (d == 0) {
                    part[NG * DVP + grp] = M;
                    part[NG * DVP + NG + grp] = L;
                }
            }
        }
        if (np > 1 && !p.defer_merge) {
            __threadfence();
            named_bar_sync(1, kConsumerWarps * 32);
            if (ctid == 0) flags[1] = (atomicAdd(p.ws_cnt + sg.group, 1) == np - 1);
            named_bar_sync(1, kConsumerWarps * 32);
            if (flags[1]) {
                __threadfence();
                // This CTA filed the group's last piece: merge all of them.
                // (1) list the pieces -- for each segment of the group, the CTAs spanning it
                if (ctid == 0) {
                    const int nseg_g = p.varlen ? p.nshare : 1;
                    const int j0 = p.varlen ? sg.group * p.nshare : sg.group;
                    int n = 0;
                    for (int js = 0; js < nseg_g; ++js) {
                        int64_t t0, nt_;
                        tab.seg_tiles(sg.group, js, t0, nt_);
                        if (nt_ == 0) continue;
                        const int64_t c0 = split_owner(t0, total, nctas), c1 = split_owner(t0 + nt_ - 1, total, nctas);
                        for (int64_t c = c0; c <= c1 && n < kMaxPieces; ++c) pslot[n++] = (int)(c + j0 + js);
                    }
                    flags[2] = n;
                }
                named_bar_sync(1, kConsumerWarps * 32);
                const int npc = flags[2];
                // (2) every piece's (m, l) per query group, in parallel
                for (int x = ctid; x < npc * NG; x += kConsumerWarps * 32) {
                    const float* pp = p.ws_part + (int64_t)pslot[x / NG] * C::SLOT_FLOATS + NG * DVP;
                    pw[x] = __ldcg(pp + x % NG);
                    pl[x] = __ldcg(pp + NG + x % NG);
                }
                named_bar_sync(1, kConsumerWarps * 32);
                // (3) per query group: global max, piece weights, total sum
                if (ctid < NG) {
                    float M = -INFINITY;
                    for (int k = 0; k < npc; ++k) M = fmaxf(M, pw[k * NG + ctid]);
                    const float Mu = (M == -INFINITY) ? 0.f : M;
                    float L = 0.f;
                    for (int k = 0; k < npc; ++k) {
                        const float w = ex2(pw[k * NG + ctid] - Mu);
                        pw[k * NG + ctid] = w;
                        L += w * pl[k * NG + ctid];
                    }
                    gml[ctid] = M;
                    gml[NG + ctid] = L;
                }
                named_bar_sync(1, kConsumerWarps * 32);
                // (4) weighted sum of the pieces' o: each thread owns CPT float4 chunks and
                //     keeps KB pieces' loads in flight per chunk (the loads are latency-bound)
                {
                    constexpr int NCH = NG * DVP / 4;
                    constexpr int CPT = (NCH + kConsumerWarps * 32 - 1) / (kConsumerWarps * 32);
                    constexpr int KB = CPT >= 4 ? 8 : 32 / CPT;   // 16 or 32 pieces' loads in flight per chunk
                    float4 acc[CPT];
#pragma unroll
                    for (int c = 0; c < CPT; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int k0 = 0; k0 < npc; k0 += KB) {
                        float4 v[CPT][KB];
#pragma unroll
                        for (int u = 0; u < KB; ++u)
#pragma unroll
                            for (int c = 0; c < CPT; ++c) {
                                const int ch = ctid + c * kConsumerWarps * 32;
                                v[c][u] = (k0 + u < npc && ch < NCH)
                                              ? __ldcg(reinterpret_cast<const float4*>(
                                                    p.ws_part + (int64_t)pslot[k0 + u] * C::SLOT_FLOATS + ch * 4))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
                            }
#pragma unroll
                        for (int u = 0; u < KB; ++u)
#pragma unroll
                            for (int c = 0; c < CPT; ++c) {
                                const int ch = ctid + c * kConsumerWarps * 32;
                                if (k0 + u < npc && ch < NCH) {
                                    const float w = pw[(k0 + u) * NG + (ch * 4) / DVP];
                                    acc[c].x += w * v[c][u].x; acc[c].y += w * v[c][u].y;
                                    acc[c].z += w * v[c][u].z; acc[c].w += w * v[c][u].w;
                                }
                            }
                    }
#pragma unroll
                    for (int c = 0; c < CPT; ++c) {
                        const int ch = ctid + c * kConsumerWarps * 32;
                        if (ch >= NCH) continue;
                        const int e = ch * 4, grp = e / DVP, d = e - grp * DVP;
                        if (grp >= p.G || d >= p.Dv) continue;
                        const float M = gml[grp], L = gml[NG + grp];
                        store_final(p, sg.group, grp, d, acc[c].x, M, L);
                        if (d + 1 < p.Dv) store_final(p, sg.group, grp, d + 1, acc[c].y, M, L);
                        if (d + 2 < p.Dv) store_final(p, sg.group, grp, d + 2, acc[c].z, M, L);
                        if (d + 3 < p.Dv) store_final(p, sg.group, grp, d + 3, acc[c].w, M, L);
                    }
                }
                if (ctid == 0) p.ws_cnt[sg.group] = 0;   // ready for the next launch
            }
        }
        named_bar_sync(1, kConsumerWarps * 32);   // red[] is reused by the next flush
    };

    reset_state();
    int64_t seg_end = -1;   // first tile after the current segment
    int stage = 0;
    uint32_t use = 0;
    for (int64_t t = t_begin; t < t_end; ++t) {
        if (t >= seg_end) {
            const Seg sg = tab.of_tile(t);
            load_q(sg.group);   // its loads land while the previous segment is flushed (qf is free now)
            if (cur.j >= 0) flush(cur);
            cur = sg;
            seg_end = sg.t0 + sg.lead + (sg.len + kTile - 1) / kTile;
            reset_state();
        }
        const Seg& sg = cur;
        const int rt = (int)(t - sg.t0) - sg.lead;   // data tile of the segment
        if (rt < 0) continue;                         // a segment's lead-in: nothing was loaded
        if (!mbar_wait_bounded(full0 + 8 * stage, use & 1)) {
            atomicExch(p.status, kDevTimeout);
            break;
        }
        const int nv = min(kTile, sg.len - rt * kTile) - warp * 16;   // valid tokens of this warp
        if (nv > 0) {
            const uint32_t kbase = smem_u32(stage_base + size_t(stage) * C::STAGE_BYTES);
            const uint32_t vbase = kbase + C::KBOX * C::BOX_BYTES;
            // ---- S^T = K . Q^T  (two accumulators to halve the dependency chain)
            float sa[NT][4], sb[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) sa[nt][e] = sb[nt][e] = 0.f;
#pragma unroll
            for (int ks = 0; ks < DKP / 16; ++ks) {
                const int d0 = ks * 16;
                const int row = warp * 16 + (lq & 1) * 8 + lr;
                const int chunk = ((d0 & 63) >> 3) + (lq >> 1);
                uint32_t a0, a1, a2, a3;
                ldsm_x4(kbase + (d0 >> 6) * C::BOX_BYTES + swz128(row, chunk), a0, a1, a2, a3);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    if (ks & 1) mma_bf16_16816(sb[nt], a0, a1, a2, a3, qf[ks][nt][0], qf[ks][nt][1]);
                    else mma_bf16_16816(sa[nt], a0, a1, a2, a3, qf[ks][nt][0], qf[ks][nt][1]);
                }
            }
            // ---- online softmax over this warp's 16 tokens
            uint32_t pb[NT][2];
            const bool v_top = gq < nv, v_bot = gq + 8 < nv;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float pt[2], pbm[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const float xt = v_top ? (sa[nt][j] + sb[nt][j]) * sl2 : -INFINITY;
                    const float xb = v_bot ? (sa[nt][2 + j] + sb[nt][2 + j]) * sl2 : -INFINITY;
                    float mx = fmaxf(xt, xb);
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    // running max in log2 units
                    const float m_old = m_run[nt][j];
                    const float m_new = fmaxf(m_old, mx);
                    const float mu = (m_new == -INFINITY) ? 0.f : m_new;
                    const float alpha = ex2(m_old - mu);
                    pt[j] = ex2(xt - mu);
                    pbm[j] = ex2(xb - mu);
                    l_run[nt][j] = l_run[nt][j] * alpha + pt[j] + pbm[j];
                    m_run[nt][j] = m_new;
#pragma unroll
                    for (int ii = 0; ii < DVP / 16; ++ii) {
                        o[ii][nt][j] *= alpha;
                        o[ii][nt][2 + j] *= alpha;
                    }
                }
                pb[nt][0] = movmatrix_t(pack_bf16(pt[0], pt[1]));
                pb[nt][1] = movmatrix_t(pack_bf16(pbm[0], pbm[1]));
            }
            // ---- O^T += V^T . P^T
            // Rows past the segment's end may hold anything (unused cache
            // capacity); P is 0 there but 0 * NaN is not, so those V entries are
            // zeroed.  a0/a1 carry tokens 2c, 2c+1 and a2/a3 tokens 2c+8, 2c+9.
            const uint32_t vm01 = (2 * cq < nv ? 0x0000ffffu : 0u) | (2 * cq + 1 < nv ? 0xffff0000u : 0u);
            const uint32_t vm23 = (2 * cq + 8 < nv ? 0x0000ffffu : 0u) | (2 * cq + 9 < nv ? 0xffff0000u : 0u);
#pragma unroll
            for (int ii = 0; ii < DVP / 16; ++ii) {
                const int d0 = ii * 16;
                const int row = warp * 16 + (lq >> 1) * 8 + lr;
                const int chunk = ((d0 & 63) >> 3) + (lq & 1);
                uint32_t a0, a1, a2, a3;
                ldsm_x4_t(vbase + (d0 >> 6) * C::BOX_BYTES + swz128(row, chunk), a0, a1, a2, a3);
                a0 &= vm01; a1 &= vm01; a2 &= vm23; a3 &= vm23;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma_bf16_16816(o[ii][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * stage);
        if (++stage == STAGES) {
            stage = 0;
            ++use;
        }
    }
    if (cur.j >= 0) flush(cur);
}

// --------------------------------------------------------------- deferred merge
// Dense rows whose tiles span many CTAs: each CTA has filed its piece (un-normalised o of the group's
// heads, their max and sum), and the group's pieces are combined here by log-sum-exp.  One single-warp
// CTA per (group, head, 32 value dims), so the reads spread over as many SMs as there are such items:
// lane k takes piece k's (m, l) and lane d accumulates value dim d over the pieces; up to 64 pieces
// are read in one round trip.  A programmatic dependent launch of the decode grid.
constexpr int kMergeBatch = 64;   // pieces merged in one round trip (two lanes' worth of (m, l))
template <int DVP, int NG, bool VARLEN>
__global__ void __launch_bounds__(32) gqa_merge_kernel(const GqaParams p, int tpr, int64_t total, int nctas) {
    constexpr int SLOT_FLOATS = NG * DVP + 2 * NG;
    __shared__ float s_w[kMaxPieces];
    pdl_wait_primary();
    const int lane = threadIdx.x;
    const int nchunk = (p.Dv + 31) / 32;
    const int64_t item = blockIdx.x;
    const int chunk = (int)(item % nchunk);
    const int64_t gg = item / nchunk;
    const int group = (int)(gg / p.G), grp = (int)(gg - (int64_t)group * p.G);
    // The group's pieces as runs of consecutive slots, one run per segment: piece k sits in slot
    // k + off[r] for the run r with k < end[r] (dense rows: one run, slots c0 + group + k).
    int end[kMaxShares], off[kMaxShares];
    int npc = 0;
#pragma unroll
    for (int r = 0; r < kMaxShares; ++r) {
        end[r] = INT_MAX;
        off[r] = 0;
    }
    if constexpr (!VARLEN) {
        const int64_t t0 = (int64_t)group * tpr;
        const int c0 = (int)split_owner(t0, total, nctas);
        npc = (int)split_owner(t0 + tpr - 1, total, nctas) - c0 + 1;
        end[0] = npc;
        off[0] = c0 + group;
    } else {
        // the decode kernel's tile split: pre[] from its CTA 0, over min(grid, total) CTAs
        const int64_t tot = __ldcg(p.ws_pre + p.B);
        const int nct = tot < 1 ? 1 : (int)(tot < nctas ? tot : nctas);
        const int b = group / p.Hkv, h = group - b * p.Hkv;
        SegTable tab;
        tab.p = &p;
        tab.pre = nullptr;
        tab.tpr = 0;
        int ts[kMaxShares], th = 0;
#pragma unroll
        for (int sh = 0; sh < kMaxShares; ++sh) {
            ts[sh] = sh < p.nshare ? SegTable::vtiles(tab.seq_len(sh, b)) : 0;
            th += ts[sh];
        }
        int64_t t0 = __ldcg(p.ws_pre + b) + (int64_t)h * th;
        int r = 0;
#pragma unroll
        for (int sh = 0; sh < kMaxShares; ++sh) {
            if (ts[sh] > 0) {
                const int c0 = (int)split_owner(t0, tot, nct), c1 = (int)split_owner(t0 + ts[sh] - 1, tot, nct);
                off[r] = c0 + group * p.nshare + sh - npc;
                npc += c1 - c0 + 1;
                end[r] = npc;
                ++r;
            }
            t0 += ts[sh];
        }
    }
    if (npc <= 1) return;   // a group in one piece (or none): the decode kernel wrote its output itself
    auto piece = [&](int k) -> const float* {
        const int o = VARLEN ? (k < end[0] ? off[0] : k < end[1] ? off[1] : k < end[2] ? off[2] : off[3]) : off[0];
        return p.ws_part + (int64_t)(k + o) * SLOT_FLOATS;
    };
    const int d = chunk * 32 + lane;
    const bool dv = d < p.Dv;
    const int colo = grp * DVP + (dv ? d : 0);
    float M, L, acc = 0.f;
    if (npc <= kMergeBatch) {
        // one round trip: lane k's (m, l) of pieces k and k + 32 and lane d's value column, all issued together
        float v[kMergeBatch], mk[2], lk[2];
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) v[u] = u < npc ? __ldcg(piece(u) + colo) : 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int k = lane + 32 * r;
            const float* pp = piece(k < npc ? k : 0) + NG * DVP;
            mk[r] = k < npc ? __ldcg(pp + grp) : -INFINITY;
            lk[r] = k < npc ? __ldcg(pp + NG + grp) : 0.f;
        }
        M = fmaxf(mk[0], mk[1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float Mu = (M == -INFINITY) ? 0.f : M;
        float w[2];
        L = 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            w[r] = mk[r] == -INFINITY ? 0.f : ex2(mk[r] - Mu);
            L += w[r] * lk[r];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) acc = fmaf(__shfl_sync(0xffffffffu, w[u >> 5], u & 31), v[u], acc);
    } else {
        M = -INFINITY;
        for (int k = lane; k < npc; k += 32) M = fmaxf(M, __ldcg(piece(k) + NG * DVP + grp));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float Mu = (M == -INFINITY) ? 0.f : M;
        L = 0.f;
        for (int k = lane; k < npc; k += 32) {
            const float* pp = piece(k) + NG * DVP;
            const float w = ex2(__ldcg(pp + grp) - Mu);
            s_w[k] = w;
            L += w * __ldcg(pp + NG + grp);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        __syncwarp();
        for (int k0 = 0; k0 < npc; k0 += kMergeBatch) {
            float v[kMergeBatch];
#pragma unroll
            for (int u = 0; u < kMergeBatch; ++u)
                v[u] = k0 + u < npc ? __ldcg(piece(k0 + u) + colo) : 0.f;
#pragma unroll
            for (int u = 0; u < kMergeBatch; ++u)
                if (k0 + u < npc) acc = fmaf(s_w[k0 + u], v[u], acc);
        }
    }
    if (!dv) return;
    store_final(p, group, grp, d, acc, M, L);
}

template <int DVP, int NG>
static int launch_merge(const GqaParams& p, int tpr, int64_t total, int nctas, cudaStream_t st) {
    const int64_t items = (int64_t)p.n_groups * p.G * ((p.Dv + 31) / 32);
    if (items > INT32_MAX) return set_error(WS_ERR_UNSUPPORTED, "gqa_decode: too many rows for the deferred merge");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)items);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = p.varlen ? cudaLaunchKernelEx(&cfg, gqa_merge_kernel<DVP, NG, true>, p, tpr, total, nctas)
                                   : cudaLaunchKernelEx(&cfg, gqa_merge_kernel<DVP, NG, false>, p, tpr, total, nctas);
    return e == cudaSuccess ? WS_OK : set_error(WS_ERR_CUDA, cudaGetErrorString(e));
}

// -------------------------------------------------------------------- host
template <int DKP, int DVP, int NT, int STAGES>
static int launch_cfg(const GqaMaps& maps, const GqaParams& p, int nctas, size_t extra_smem, cudaStream_t st) {
    using C = GqaCfg<DKP, DVP, NT, STAGES>;
    const size_t smem = C::fixed_smem() + extra_smem;
    auto kfn = gqa_decode_kernel<DKP, DVP, NT, STAGES>;
    static int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
            return set_error(WS_ERR_CUDA, "cudaFuncSetAttribute failed for gqa_decode_kernel");
        configured_dev = dev;
    }
    if (smem > 227 * 1024) return set_error(WS_ERR_UNSUPPORTED, "gqa_decode: shared memory plan exceeds 227 KB");
    kfn<<<nctas, kThreads, smem, st>>>(maps, p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(WS_ERR_CUDA, cudaGetErrorString(e));
    return WS_OK;
}

size_t gqa_slot_bytes(int G, int Dv) {
    const int NT = G <= 8 ? 1 : 2;
    const int DVP = (Dv + 63) / 64 * 64;
    return size_t(NT * 8 * DVP + 2 * NT * 8) * 4;
}

static int dispatch(const GqaMaps& maps, const GqaParams& p, int Dk, int Dv, int nctas, size_t extra_smem,
                    cudaStream_t st) {
    const int DKP = (Dk + 63) / 64 * 64, DVP = (Dv + 63) / 64 * 64;
    const int NT = p.G <= 8 ? 1 : 2;
#define WS_GQA_CASE(dk, dv, nt, stg) \
    if (DKP == dk && DVP == dv && NT == nt) return launch_cfg<dk, dv, nt, stg>(maps, p, nctas, extra_smem, st);
    WS_GQA_CASE(64, 64, 1, 6)
    WS_GQA_CASE(64, 64, 2, 6)
    WS_GQA_CASE(128, 128, 1, 4)
    WS_GQA_CASE(128, 128, 2, 4)
    WS_GQA_CASE(192, 128, 1, 4)
    WS_GQA_CASE(192, 128, 2, 3)
    WS_GQA_CASE(128, 64, 1, 4)
    // the other head sizes the reference accepts (any multiple of 16): dims up to 256, rounded up to 64
    WS_GQA_CASE(64, 128, 1, 6)
    WS_GQA_CASE(64, 128, 2, 5)
    WS_GQA_CASE(192, 192, 1, 3)
    WS_GQA_CASE(192, 192, 2, 3)
    WS_GQA_CASE(256, 256, 1, 2)
    WS_GQA_CASE(256, 256, 2, 2)
#undef WS_GQA_CASE
    return set_error(WS_ERR_UNSUPPORTED, "gqa_decode: unsupported (Dk, Dv, G) combination");
}

int gqa_launch(const GqaLaunch& a) {
    if (a.G < 1 || a.G > 16) return set_error(WS_ERR_UNSUPPORTED, "gqa_decode: groups must be in [1, 16]");
    if (a.Dk < 16 || a.Dk % 16 || a.Dv < 16 || a.Dv % 16)
        return set_error(WS_ERR_INVALID_ARG, "gqa_decode: head dims must be positive multiples of 16");
    if (a.nshare < 1 || a.nshare > kMaxShares) return set_error(WS_ERR_INVALID_ARG, "gqa_decode: 1..4 shares");

    GqaMaps maps;
    memset(&maps, 0, sizeof(maps));
    GqaParams p;
    memset(&p, 0, sizeof(p));
    p.q = static_cast<const __nv_bfloat16*>(a.q);
    p.q_row_stride = a.q_row_stride;
    p.G = a.G; p.Dk = a.Dk; p.Dv = a.Dv; p.scale = a.scale;
    p.varlen = a.varlen;
    p.n_rows = a.n_rows; p.L = a.L;
    p.B = a.B; p.Hkv = a.Hkv; p.nshare = a.nshare;
    p.n_groups = a.varlen ? a.B * a.Hkv : a.n_rows;
    p.out_mode = a.out_mode;
    p.out = a.out; p.out_max = a.out_max; p.out_sum = a.out_sum; p.out_lse = a.out_lse;
    p.out_row_stride = a.out_row_stride; p.ml_row_stride = a.ml_row_stride;
    p.status = a.status;

    for (int s = 0; s < a.nshare; ++s) {
        const KvShare& sh = a.shares[s];
        p.cu[s] = sh.cu_seqlens;
        p.lens[s] = sh.seqlens;
        if (sh.n_tok == 0 || sh.n_rows == 0) continue;   // nothing to map; no tile will reference it
        const int tmk = make_kv_map(&maps.k[s], sh.k, sh.k_stride_tok, sh.k_stride_row, a.Dk, sh.n_tok, sh.n_rows,
                                    kTile, &p.tok_in_dim2[s]);
        if (tmk != WS_OK) return tmk;
        int dummy = 0;
        const int tmv = make_kv_map(&maps.v[s], sh.v, sh.v_stride_tok, sh.v_stride_row, a.Dv, sh.n_tok, sh.n_rows,
                                    kTile, &dummy);
        if (tmv != WS_OK) return tmv;
        if (dummy != p.tok_in_dim2[s])
            return set_error(WS_ERR_UNSUPPORTED, "gqa_decode: K and V must share the same stride order");
        p.has_map[s] = 1;
    }

    const int nsm = std::min(device_sm_count(), kMaxPieces - kMaxShares);
    int64_t total_tiles;
    int nctas;
    if (!a.varlen) {
        total_tiles = (int64_t)a.n_rows * ((a.L + kTile - 1) / kTile);
        nctas = (int)std::min<int64_t>(nsm, std::max<int64_t>(total_tiles, 1));
    } else {
        nctas = nsm;
        total_tiles = -1;
    }
    if (p.n_groups > kMaxGroupsPerLaunch)
        return set_error(WS_ERR_UNSUPPORTED, "gqa_decode: more than 65536 output row groups in one launch");
    const int nseg = a.varlen ? a.B * a.Hkv * a.nshare : a.n_rows;
    const size_t base_need = gqa_workspace_bytes(a.G, a.Dv, nseg, p.n_groups, nctas);
    const size_t need = base_need + (a.varlen ? gqa_varlen_extra_bytes(a.B) : 0);
    if (a.workspace_bytes < need || (need && !a.workspace))
        return set_error(WS_ERR_WORKSPACE, "gqa_decode: workspace too small (see ws_gqa_workspace_size)");
    if (reinterpret_cast<uintptr_t>(a.workspace) % 16)
        return set_error(WS_ERR_WORKSPACE, "gqa_decode: workspace must be 16-byte aligned");
    p.ws_cnt = static_cast<int*>(a.workspace);
    p.ws_part = reinterpret_cast<float*>(static_cast<uint8_t*>(a.workspace) + kCounterHeaderBytes);
    if (a.varlen) {
        // Ragged shares: a CTA's range crosses many short segments, and a ticket merge at each segment end
        // (fence, atomic, the last CTA reading the group's pieces) stalls its tile stream for microseconds
        // each time; the pieces are filed and merged by gqa_merge_kernel instead.
        p.defer_merge = 1;
        p.ws_pre = reinterpret_cast<int*>(static_cast<uint8_t*>(a.workspace) + base_need);
    }
    const size_t extra_smem = a.varlen ? size_t(a.B + 1) * 4 : 0;
    // Dense rows spanning more than 8 CTAs each: the last CTA of a row would read every piece of it alone,
    // so the pieces are merged by gqa_merge_kernel over many SMs instead.
    const int tpr = (a.L + kTile - 1) / kTile;
    if (!a.varlen && a.L > 0 && total_tiles > 0) {
        const int64_t per_cta = (total_tiles + nctas - 1) / nctas;
        p.defer_merge = (tpr + per_cta - 1) / per_cta + 1 > 8;
    }
    cudaStream_t st = static_cast<cudaStream_t>(a.stream);
    const int DVP = (a.Dv + 63) / 64 * 64, NG = (a.G <= 8 ? 1 : 2) * 8;
    if (p.defer_merge && DVP > 256)   // checked before the decode is launched
        return set_error(WS_ERR_UNSUPPORTED, "gqa_decode: unsupported value width for the deferred merge");
    int rc = dispatch(maps, p, a.Dk, a.Dv, nctas, extra_smem, st);
    if (rc != WS_OK || !p.defer_merge) return rc;
#define WS_GQA_MERGE(dvp, ng) \
    if (DVP == dvp && NG == ng) return launch_merge<dvp, ng>(p, tpr, total_tiles, nctas, st);
    WS_GQA_MERGE(64, 8)
    WS_GQA_MERGE(64, 16)
    WS_GQA_MERGE(128, 8)
    WS_GQA_MERGE(128, 16)
    WS_GQA_MERGE(192, 8)
    WS_GQA_MERGE(192, 16)
    WS_GQA_MERGE(256, 8)
    WS_GQA_MERGE(256, 16)
#undef WS_GQA_MERGE
    return set_error(WS_ERR_UNSUPPORTED, "gqa_decode: unsupported value width for the deferred merge");
}

size_t gqa_workspace_bytes(int G, int Dv, int nseg, int n_groups, int nctas) {
    (void)n_groups;
    return kCounterHeaderBytes + size_t(nseg + nctas) * gqa_slot_bytes(G, Dv);
}

size_t gqa_varlen_extra_bytes(int B) { return align_up(size_t(B + 1) * 4, 256); }

}  // namespace ws
