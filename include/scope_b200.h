/*
 * scope_b200.h -- C ABI of the B200 (sm_100a) decode-attention engine for
 * physically partitioned KV caches.
 *
 * Every entry point:
 *   - takes DEVICE pointers (the caller's CUDA allocations on the current
 *     device) and plain sizes / strides (in ELEMENTS unless the name ends in
 *     _bytes), and a cudaStream_t passed as `void* stream` (NULL = the legacy
 *     default stream);
 *   - launches asynchronously on that stream and never synchronises;
 *   - returns WS_OK (0) or a WS_ERR_* code; ws_last_error() then returns a
 *     message (thread-local).
 * No decode entry point allocates device memory (ws_peer_buffer_create is
 * the one allocating entry, for the multi-GPU exchange): callers pass a 16-byte
 * aligned workspace whose size the matching *_workspace_size() returns.  A workspace must be zeroed
 * once when it is allocated (its counters reset themselves after every
 * launch) and must not be shared by launches that may overlap in time.
 * Exception: when ws_status_take() returns WS_ERR_DEVICE, a launch may have
 * given up between taking and returning a merge counter, so every workspace
 * used since the previous ws_status_take() must be zeroed again before its
 * next use.
 *
 * bf16 tensors are passed as their 16-bit storage.  The reference interfaces
 * each entry replaces are cited as path:line of the reference checkout.
 */
#ifndef SCOPE_B200_H
#define SCOPE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes */
#define WS_OK 0
#define WS_ERR_INVALID_ARG 1   /* shape / pointer / alignment rejected on the host */
#define WS_ERR_UNSUPPORTED 2   /* valid request this build has no kernel for     */
#define WS_ERR_CUDA 3          /* a CUDA runtime call failed                      */
#define WS_ERR_WORKSPACE 4     /* workspace missing or too small                  */
#define WS_ERR_DEVICE 5        /* a kernel reported a device-side failure         */

/* ---- element types */
#define WS_DTYPE_BF16 0
#define WS_DTYPE_F32 1
#define WS_DTYPE_I8 2

/* ---- GQA output modes (what the reference wrappers return) */
#define WS_OUT_NORM_BF16 0   /* out bf16 normalised, max/sum bf16: fused_cpu_attn on bf16 (kernel/cpu_attn.cpp:631-634) */
#define WS_OUT_UNNORM_F32 1  /* o fp32 NOT normalised, max/sum fp32: fused_cpu_attn_mla (kernel/cpu_attn.cpp:668-671)   */
#define WS_OUT_NORM_F32 2    /* out fp32 normalised, max/sum fp32: fused_cpu_attn on fp32 (kernel/cpu_attn.cpp:635)     */

const char* ws_last_error(void);
int ws_version(void);

/* Device-side status word: kernels whose bounded waits give up (they never
 * spin forever) record WS_ERR_DEVICE there.  Returns the word for the current
 * device and clears it (synchronises the given stream). */
int ws_status_take(void* stream);

/*
 * GQA / MLA decode over one strided KV share.
 * Replaces fused_cpu_attn (kernel/cpu_attn.cpp:572-636),
 * fused_cpu_attn_mla (kernel/cpu_attn.cpp:638-672) and
 * fused_cpu_attn_fp32 (kernel/cpu_attn.cpp:817-848).
 *   q    [B_kv, G, Dk] contiguous (dtype bf16, or fp32 with dtype WS_DTYPE_F32)
 *   k    element (b, t, d) at k + b*k_stride_b + t*k_stride_t + d   (Dk wide)
 *   v    element (b, t, d) at v + b*v_stride_b + t*v_stride_t + d   (Dv wide)
 *   out  [B_kv, G, Dv]; out_max, out_sum [B_kv, G]  (types per out_mode)
 *   out_lse [B_kv, G] fp32, optional (NULL): max + log(sum)
 * Constraints (bf16): 1 <= G <= 16; Dk, Dv multiples of 16 with
 * (ceil64(Dk), ceil64(Dv)) in {(64,64), (128,128), (128,64), (192,128)};
 * k, v 16-byte aligned, strides multiples of 8 elements.  L == 0 gives
 * out = 0, max = -inf, sum = 0.
 */
int ws_gqa_decode(const void* q, const void* k, const void* v,
                  int64_t k_stride_b, int64_t k_stride_t, int64_t v_stride_b, int64_t v_stride_t,
                  int B_kv, int G, int Dk, int Dv, int L, float scale, int dtype, int out_mode,
                  void* out, void* out_max, void* out_sum, float* out_lse,
                  void* workspace, size_t workspace_bytes, void* stream);
size_t ws_gqa_decode_workspace_size(int B_kv, int G, int Dv, int L);

/*
 * ws_gqa_decode without a workspace argument.  No counterpart in the
 * reference: it is for callers that can pass their inputs and outputs but no
 * other device memory -- e.g. a server whose memory manager has already
 * reserved the GPU's HBM for its KV-cache pool, or a plugin host that passes
 * only tensors -- and for whom cudaMalloc would fail or stall the decode loop.
 * The kernel's scratch is a built-in 4 MiB array per device (see
 * ws_gqa_decode_noalloc_max_scratch), held by every GPU that loads this
 * library until the process exits.  Same arguments and results as
 * ws_gqa_decode with dtype WS_DTYPE_BF16.
 *   - Shapes whose scratch (ws_gqa_decode_workspace_size) exceeds the array
 *     are rejected with WS_ERR_WORKSPACE.
 *   - The first call on a device looks up the array's device address; make it
 *     before any stream capture.
 *   - All calls on a device share the array: calls that may overlap on the
 *     GPU race.  Issue them in order on one stream.
 * Allocates nothing (no cudaMalloc, cudaFree or allocating library call).
 */
int ws_gqa_decode_noalloc(const void* q, const void* k, const void* v,
                          int64_t k_stride_b, int64_t k_stride_t, int64_t v_stride_b, int64_t v_stride_t,
                          int B_kv, int G, int Dk, int Dv, int L, float scale, int out_mode,
                          void* out, void* out_max, void* out_sum, float* out_lse, void* stream);
size_t ws_gqa_decode_noalloc_max_scratch(void);

/*
 * Ragged-batch GQA decode over up to 4 physically separate KV shares of every
 * sequence, with the per-share partials merged by log-sum-exp.  Two launches:
 * the decode files one partial per (CTA, share segment) in the workspace, and
 * a programmatic dependent launch merges each row's partials.  Replaces the runtime's per-share fused_cpu_attn calls plus the
 * Python merge (system/mixoffload.py:1263-1268, :1333-1334, :1456-1464;
 * system/qwenoffload.py:1606-1617).
 *   q        [B, Hkv*G, Dk] bf16 contiguous (head h = kvh*G + g)
 *   share s, one of two layouts (element (t, r, d) at k_s + t*k_stride_t + r*k_stride_h + d):
 *     packed:  cu_seqlens_s [B+1] int32 DEVICE token offsets, seqlens_s = NULL;
 *              r = kv head, sequence b owns tokens [cu[b], cu[b+1]); n_tok = total tokens
 *              (e.g. [n_tok, Hkv, D] token-major or [Hkv, n_tok, D] head-major)
 *     padded:  seqlens_s [B] int32 DEVICE token counts, cu_seqlens_s = NULL;
 *              r = b*Hkv + kv head, tokens [0, seqlens[b]) of a row of capacity n_tok
 *              (the reference's [B*Hkv, max_seq, D] cache, system/qwenoffload.py:59-141)
 *   out      [B, Hkv*G, Dv] bf16 normalised;  out_lse [B, Hkv*G] fp32
 */
typedef struct ws_kv_share {
    const void* k;
    const void* v;
    const int32_t* cu_seqlens;   /* device, [B+1] (packed) or NULL */
    const int32_t* seqlens;      /* device, [B] (padded) or NULL */
    int64_t n_tok;               /* packed: total tokens; padded: row capacity */
    int64_t k_stride_t, k_stride_h, v_stride_t, v_stride_h;
} ws_kv_share;

int ws_gqa_decode_shares(const void* q, int B, int Hkv, int G, int Dk, int Dv, float scale,
                         const ws_kv_share* shares, int n_shares,
                         void* out, float* out_lse, void* workspace, size_t workspace_bytes, void* stream);
size_t ws_gqa_decode_shares_workspace_size(int B, int Hkv, int G, int Dv, int n_shares);

/*
 * Absorbed-MLA decode: many heads over one shared latent KV (V = the latent).
 * Replaces fused_cpu_attn_mla_compressed (kernel/cpu_attn.cpp:852-1022).
 *   q_proj [B*nH, 512], q_pe [B*nH, 64], c_kv [B, S, 512], k_pe [B, S, 64]:
 *   bf16, contiguous, 16-byte aligned.
 *   score(h, t) = scale * (q_proj[h].c_kv[t] + q_pe[h].k_pe[t]);  o[h] = sum_t softmax * c_kv[t]
 *   out_mode WS_OUT_UNNORM_F32: out [B*nH, 512] fp32 NOT normalised + out_max, out_sum
 *     [B*nH] fp32 (the reference's outputs); WS_OUT_NORM_BF16 / _F32: out normalised.
 *   out_lse [B*nH] fp32 optional (NULL).  out_max/out_sum may be NULL.
 * Two launches on the stream: the tcgen05 split-KV kernel and its merge
 * (a programmatic dependent launch).  nH must be a multiple of 16: each group
 * of 16 heads is one tensor-core tile (callers with other head counts pad
 * q_proj / q_pe with zero rows).
 */
int ws_mla_decode(const void* q_proj, const void* q_pe, const void* c_kv, const void* k_pe, int B, int nH, int S,
                  float scale, int out_mode, void* out, float* out_max, float* out_sum, float* out_lse,
                  void* workspace, size_t workspace_bytes, void* stream);
size_t ws_mla_decode_workspace_size(int B, int nH, int S);
/* The same over latent sequences c_batch_stride / pe_batch_stride elements
 * apart (a cache [B, cap, 512] / [B, cap, 64] read for its first S tokens;
 * strides multiples of 8 elements).  Same reference interface as above. */
int ws_mla_decode_strided(const void* q_proj, const void* q_pe, const void* c_kv, int64_t c_batch_stride,
                          const void* k_pe, int64_t pe_batch_stride, int B, int nH, int S, float scale, int out_mode,
                          void* out, float* out_max, float* out_sum, float* out_lse, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Absorbed-MLA decode step with the projections either side of the attention:
 * the decode branch of _mla_compressed_forward (system/deepseek.py:257-265 the
 * absorb, :355-404 the attention over the cache and the merge, :405-407 the
 * up-projection), which the reference runs as torch.bmm + the CPU kernel + bmm:
 *   q_proj = q_nope . W_UK ;  o = softmax(scale (q_proj . c + q_pe . p)) . c ;
 *   out = bf16(o / l) . W_UV^T
 *   q_nope [B, nH, nop] bf16 (nop % 4 == 0, <= 256); q_pe [B*nH, 64], c_kv [B, S, 512],
 *   k_pe [B, S, 64] bf16;
 *   w_uk: head h's [nop, 512] block at w_uk + h * w_uk_head_stride, w_uv: head
 *   h's [vhd, 512] block at w_uv + h * w_uv_head_stride (elements; bf16, 16-byte
 *   aligned).  The reference's kv_b_proj.weight viewed [nH, nop + vhd, 512] is
 *   passed as is: w_uk = weight, w_uv = weight + nop * 512, both head strides
 *   (nop + vhd) * 512;
 *   out [B, nH, vhd] bf16; out_lse [B*nH] fp32 optional (NULL).
 * Four launches: the absorb GEMM (fp32 accumulation, bf16 q_proj kept in the
 * workspace), the split-KV decode and its merge (bf16 o_n in the workspace), and
 * the up-projection GEMM (programmatic dependent launches after the decode).
 * This build supports nH == 16.
 */
int ws_mla_decode_absorbed(const void* q_nope, const void* w_uk, int64_t w_uk_head_stride, const void* q_pe,
                           const void* c_kv, const void* k_pe, const void* w_uv, int64_t w_uv_head_stride, int B,
                           int nH, int S, int nop, int vhd, float scale, void* out, float* out_lse, void* workspace,
                           size_t workspace_bytes, void* stream);
size_t ws_mla_decode_absorbed_workspace_size(int B, int nH, int S);
/* The same step over a latent cache read in place: latent sequences
 * c_batch_stride / pe_batch_stride elements apart (multiples of 8). */
int ws_mla_decode_absorbed_strided(const void* q_nope, const void* w_uk, int64_t w_uk_head_stride, const void* q_pe,
                                   const void* c_kv, int64_t c_batch_stride, const void* k_pe, int64_t pe_batch_stride,
                                   const void* w_uv, int64_t w_uv_head_stride, int B, int nH, int S, int nop, int vhd,
                                   float scale, void* out, float* out_lse, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* ---- CSA index modes (ws_csa_decode with an id list) */
#define WS_CSA_IDX_ALL 0            /* every id must lie in this buffer's range; others are skipped and
                                       reported as WS_ERR_DEVICE by ws_status_take */
#define WS_CSA_IDX_SORTED_SHARD 1   /* ids ascending per sequence; only those in this buffer's range count */
#define WS_CSA_IDX_SHARD 2          /* ids in any order; those outside this buffer's range are skipped */

/*
 * CSA decode: nq query rows per sequence over a shared 512-wide latent KV
 * (K = V), gathered by a top-k id list or over a dense id range.
 * Replaces indexer_attn_cpu (kernel/cpu_attn_ds4_ext/csa_attn.cpp:1819-1883),
 * fused_csa_attn (:200-281) and fused_csa_attn_range (:1587-1656); int8 KV
 * with one fp32 scale per entry is the storage of the int8 family
 * (value = int8 * scale, csa_attn.cpp:1338-1344), attended without quantising q.
 *   q        [bs, nq, 512], q_dtype WS_DTYPE_F32 or WS_DTYPE_BF16, contiguous
 *   kv       [bs, nc, 512], kv_dtype WS_DTYPE_BF16 or WS_DTYPE_I8, contiguous;
 *            row j of sequence b holds entry id shard_lo + j (shard_lo = 0
 *            for an unsharded cache)
 *   kv_scales [bs, nc] fp32 (WS_DTYPE_I8 only)
 *   idx      [bs, k] int32 entry ids (duplicates attend twice, as the
 *            reference does), idx_mode one of WS_CSA_IDX_*; or idx = NULL:
 *            attend ids [kv_begin, kv_end) (clipped to this buffer's range)
 *   score = scale * q . value;  out [bs, nq, 512] normalised in out_dtype
 *   (WS_DTYPE_F32 or WS_DTYPE_BF16), out_lse [bs, nq] fp32 (may be NULL).
 * A row with no entry gives out = 0, lse = -inf (the partial of an empty
 * shard).  One launch; the workspace (ws_csa_decode_workspace_size bytes,
 * 16-byte aligned) carries the partials the CTAs of a sequence exchange,
 * after the counter header, which this entry never touches (so one zeroed
 * workspace can serve it and the GQA / MLA entries in turn).
 */
int ws_csa_decode(const void* q, int q_dtype, int bs, int nq, int hd, const void* kv, int kv_dtype,
                  const float* kv_scales, int64_t nc, int64_t shard_lo, const int32_t* idx, int k, int idx_mode,
                  int64_t kv_begin, int64_t kv_end, float scale, void* out, int out_dtype, float* out_lse,
                  void* workspace, size_t workspace_bytes, void* stream);
size_t ws_csa_decode_workspace_size(int bs, int nq, int q_dtype);

/*
 * CSA decode in the reference's integer-score form: u8 query codes against
 * s8 entry codes.  Replaces fused_csa_attn_bsq_int8_preq
 * (kernel/cpu_attn_ds4_ext/csa_attn.cpp:1235-1357), fused_csa_attn_bsq_int8_full
 * (:1359-1483) and the attention of fused_csa_attn_bsq_int8 (:766-883, after
 * its two quantisers, ws_csa_q_quantize_u8 and ws_csa_kv_quantize_s8):
 *   q_u8 [bs, nq, 512] u8 codes (value + 128), q_scales [bs, nq] fp32
 *   kv_i8 [bs, nc, 512] s8 codes, kv_scales [bs, nc] fp32, kv_sums [bs, nc] int32
 *   score = ((sum_d q_u8 * kv_i8) - 128 * kv_sums) * q_scale * kv_scale * scale
 *   (the integer dot is exact, as the reference's VNNI dot is)
 *   value = kv_i8 * kv_scale, or, with kv_bf16 [bs, nc, 512] non-NULL, the
 *   bf16 entry itself (the _full operator).
 * The id list / dense range, shard arguments, outputs and workspace are those
 * of ws_csa_decode with q_dtype WS_DTYPE_BF16 (64-row query groups).
 */
int ws_csa_decode_qcodes(const uint8_t* q_u8, const float* q_scales, int bs, int nq, int hd, const int8_t* kv_i8,
                         const float* kv_scales, const int32_t* kv_sums, const void* kv_bf16, int64_t nc,
                         int64_t shard_lo, const int32_t* idx, int k, int idx_mode, int64_t kv_begin, int64_t kv_end,
                         float scale, void* out, int out_dtype, float* out_lse, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * Per-row quantisers of the CSA int8 family, bit-exact with the reference:
 * ws_csa_kv_quantize_s8 replaces kv_quantize_bf16_to_int8
 * (kernel/cpu_attn_ds4_ext/csa_attn.cpp:1203-1233) and ws_csa_q_quantize_u8
 * replaces q_quantize_fp32_to_u8 (:1175-1201).
 *   kv [rows, hd] bf16 -> out int8 [rows, hd], scales fp32 [rows], sums int32 [rows]
 *   q  [rows, hd] fp32 -> out uint8 [rows, hd] (value + 128), scales fp32 [rows]
 * hd % 8 == 0; all pointers 16-byte aligned.
 */
int ws_csa_kv_quantize_s8(const void* kv, int64_t rows, int hd, void* out, float* scales, int32_t* sums,
                          void* stream);
int ws_csa_q_quantize_u8(const float* q, int64_t rows, int hd, void* out, float* scales, void* stream);

/*
 * Exchange of sequence-shard partials over NVLink peer memory (root gather):
 * the device-side form of the runtime's share merge (system/qwenoffload.py:1606-1617,
 * system/mixoffload.py:1456-1464) across GPUs of one box.
 * Rank 0 allocates the exchange buffer (ws_peer_buffer_create: the one entry
 * point that allocates device memory; ws_peer_exchange_bytes gives its size)
 * and hands the 64-byte CUDA IPC handle to the other ranks, which map it with
 * ws_peer_buffer_open.  Each rank's partial is o fp32 [rows, dim] normalised,
 * then lse fp32 [rows] (for ws_gqa_decode: out_mode WS_OUT_NORM_F32, out_lse
 * right after the rows x dim floats).  Per step, on every rank in the same order:
 *   - rank 0's decode writes its partial at base + ws_peer_slot_offset(.., 0),
 *     then ws_peer_merge: a bounded wait until every rank's flag reaches this
 *     step, the log-sum-exp merge into out [rows, dim] (bf16 or fp32) and
 *     out_lse [rows], then the step is published as consumed;
 *   - rank r > 0's decode writes its partial to a local, 16-byte aligned block
 *     (rounded up to a multiple of 64 floats), then ws_peer_push: a bounded
 *     wait until rank 0 has consumed the previous step, the copy into rank r's
 *     slot over NVLink, and the release of rank r's flag.  `state` is two
 *     int64 words of rank r's memory, zeroed once (its step count and a ticket).
 * The step counts live on the devices and every pointer is fixed, so the steps
 * can be captured in a CUDA graph.  Both are programmatic dependent launches:
 * they poll the other ranks while the kernel before them drains and read its
 * output only after it completes.  A wait that gives up (2 s from the launch's
 * start) records WS_ERR_DEVICE for ws_status_take; the exchange must then be
 * rebuilt.  world <= 32, dim % 4 == 0.
 */
size_t ws_peer_exchange_bytes(int world, int64_t rows, int dim);
size_t ws_peer_slot_offset(int world, int64_t rows, int dim, int rank);
int ws_peer_buffer_create(size_t bytes, void** dev_ptr, void* ipc_handle);
int ws_peer_buffer_open(const void* ipc_handle, void** dev_ptr);
int ws_peer_buffer_close(void* dev_ptr);
int ws_peer_buffer_free(void* dev_ptr);
int ws_peer_push(const float* block, void* root_base, int world, int64_t rows, int dim, int rank, int64_t* state,
                 void* stream);
int ws_peer_merge(void* root_base, int world, int64_t rows, int dim, void* out, int out_dtype, float* out_lse,
                  void* stream);

/*
 * The same exchange in scatter-merge form, for partials large against the
 * NVLink time of one block: every rank owns the contiguous share of rows
 * [rows*q/world, rows*(q+1)/world) and merges it, so a rank sends and receives
 * (world - 1) / world of one block, and only the merged shares (in the out
 * dtype) travel to rank 0, which returns the whole result.
 * Every rank allocates ws_peer_rs_bytes(world, rows, dim) with
 * ws_peer_buffer_create, the ranks exchange their IPC handles, and each maps
 * every other rank's buffer with ws_peer_buffer_open.  `bases` is a device
 * array of `world` int64 addresses, entry q this rank's address of rank q's
 * buffer (its own at entry `rank`).  Per step, on every rank in the same order:
 * the decode writes this rank's partial into a local 16-byte aligned `block`
 * (o fp32 [rows, dim] normalised, then lse [rows]); ws_peer_rs_scatter (a
 * bounded wait until every peer has read the previous step, the copies, the
 * release of this rank's flag in every peer's buffer); ws_peer_rs_merge (a
 * bounded wait for every flag, the log-sum-exp merge of this rank's share;
 * rank 0 writes out [rows, dim] (bf16 or fp32, the same out_dtype on every
 * rank) and out_lse [rows] (may be NULL), the other ranks ignore out).
 * `state` is two int64 words of this rank's memory, zeroed once.  The step
 * counts live on the devices, so the steps can be captured in a CUDA graph.
 * A wait that gives up (2 s) records WS_ERR_DEVICE; the exchange must then be
 * rebuilt.  world <= 32, dim % 4 == 0.
 */
size_t ws_peer_rs_bytes(int world, int64_t rows, int dim);
int ws_peer_rs_scatter(const float* block, const int64_t* bases, int world, int64_t rows, int dim, int rank,
                       int64_t* state, void* stream);
int ws_peer_rs_merge(const float* block, const int64_t* bases, int world, int64_t rows, int dim, int rank,
                     const int64_t* state, void* out, int out_dtype, float* out_lse, void* stream);

/* ---- indexer top-k orders */
#define WS_TOPK_BY_SCORE 0   /* descending score, ties: lower id first (the reference's partial_sort order) */
#define WS_TOPK_BY_ID 1      /* ascending id: the layout WS_CSA_IDX_SORTED_SHARD wants */

/*
 * Indexer top-k of the CSA path.  Replaces indexer_topk_cpu / indexer_topk_cpu_par
 * (kernel/cpu_attn_ds4_ext/csa_attn.cpp:1658-1817).
 *   q [bs, nH, hd], kv [bs, nc, hd] in dtype (WS_DTYPE_F32 or WS_DTYPE_BF16), w [bs, nH] fp32
 *   score[b, j] = sum_h w[b, h] * relu(q[b, h] . kv[b, j])   (fp32)
 *   out_ids [bs, min(k, nc)] int32 in `order`; out_scores [bs, nc] fp32 (optional: NULL keeps them in the
 *   workspace of ws_indexer_topk_workspace_size bytes, which is then required).  With a workspace of that
 *   size the select also spreads its pass over the scores across several CTAs per sequence; without one
 *   (out_scores given, workspace NULL) it runs one CTA per sequence.
 * nH <= 64, hd % 16 == 0 and <= 256, k <= 4096.  Two launches.
 */
int ws_indexer_topk(const void* q, const void* kv, int dtype, const float* w, int bs, int nH, int hd, int64_t nc,
                    int k, int order, int32_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes,
                    void* stream);
size_t ws_indexer_topk_workspace_size(int bs, int64_t nc);

/*
 * Append n_new tokens to a device-resident KV cache (the write side of the
 * partitioned cache; replaces the host copies of InplaceKVCache.append_4d,
 * system/qwenoffload.py:97-122, and InplaceKVCacheCompressed.append,
 * system/deepseek.py:171-194).  Strides in elements:
 *   dst (row, t0 + i, d) at dst + row*dst_stride_row + (t0+i)*dst_stride_tok + d, t0 + n_new <= capacity
 *   src (row, i, d)      at src + row*src_stride_row + i*src_stride_tok + d
 * for row < rows, i < n_new, d < D; dtype WS_DTYPE_BF16 / F32 / I8.  One launch.
 */
int ws_kv_append(void* dst, int64_t dst_stride_row, int64_t dst_stride_tok, int64_t capacity, const void* src,
                 int64_t src_stride_row, int64_t src_stride_tok, int64_t rows, int64_t n_new, int D, int dtype,
                 int64_t t0, void* stream);

/*
 * Log-sum-exp merge of P partial attention results (the cross-GPU combine of
 * a sequence-sharded KV cache, and the runtime merges it replaces:
 * system/qwenoffload.py:1606-1617 lse form).
 *   o_parts   [P, R, D] fp32 normalised partials;  lse_parts [P, R] fp32
 *   out       [R, D] in out_dtype (WS_DTYPE_BF16 or WS_DTYPE_F32);  out_lse [R] fp32 (optional)
 * Rows whose partials are all -inf give out = 0, lse = -inf.
 */
int ws_lse_merge(const float* o_parts, const float* lse_parts, int P, int64_t R, int D,
                 void* out, int out_dtype, float* out_lse, void* stream);
/* The same with partial p's o rows at o_parts + p * o_part_stride and its lse
 * values at lse_parts + p * lse_part_stride (elements): the layout of one
 * all_gather over per-rank blocks [o (R*D), lse (R)], merged in place. */
int ws_lse_merge_strided(const float* o_parts, int64_t o_part_stride, const float* lse_parts,
                         int64_t lse_part_stride, int P, int64_t R, int D, void* out, int out_dtype,
                         float* out_lse, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SCOPE_B200_H */
