// Host-side internals shared by the .cu files of libscope_b200.so.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <algorithm>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/scope_b200.h"

namespace ws {

int set_error(int code, const char* msg);
int device_sm_count();
int make_kv_map(CUtensorMap* map, const void* base, int64_t stride_tok, int64_t stride_row, int D, int64_t n_tok,
                int64_t n_rows, int box_tok, int* tok_in_dim2);
int* device_status_word();

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Every workspace starts with a fixed header of merge counters (one int per
// output row group, group g at index g) and the partial results follow it.
// Because the header never moves, a workspace can be shared by launches of
// any shapes: counters are touched only by the merge tickets, which return
// them to zero, and partials never land on them.
constexpr size_t kCounterHeaderBytes = size_t(256) << 10;
constexpr int kMaxGroupsPerLaunch = int(kCounterHeaderBytes / 4);
constexpr int kMaxHeadsPerLaunch = 16;   // query heads per kv row one GQA launch takes (two MMA column tiles)

struct KvShare {
    const void* k;
    const void* v;
    const int* cu_seqlens;      // varlen, packed share
    const int* seqlens;         // varlen, padded share
    int64_t n_tok, n_rows;      // TMA extents: tokens, rows (kv rows or kv heads)
    int64_t k_stride_tok, k_stride_row, v_stride_tok, v_stride_row;   // elements
};

struct GqaLaunch {
    const void* q;
    int64_t q_row_stride;
    int G, Dk, Dv;
    float scale;
    int varlen;
    int n_rows, L;              // dense
    int B, Hkv;                 // varlen
    int nshare;
    KvShare shares[4];
    int out_mode;
    void* out;
    void* out_max;
    void* out_sum;
    float* out_lse;
    int64_t out_row_stride, ml_row_stride;
    void* workspace;
    size_t workspace_bytes;
    int* status;
    void* stream;
};

int gqa_launch(const GqaLaunch& a);
size_t gqa_workspace_bytes(int G, int Dv, int nseg, int n_groups, int nctas);
size_t gqa_varlen_extra_bytes(int B);   // ragged shares: the tile prefix for the deferred merge
size_t gqa_slot_bytes(int G, int Dv);

int gqa_f32_launch(const void* q, const void* k, const void* v, int64_t k_sb, int64_t k_st, int64_t v_sb,
                   int64_t v_st, int B_kv, int G, int D, int L, float scale, int out_mode, void* out, void* out_max,
                   void* out_sum, float* out_lse, void* workspace, size_t workspace_bytes, cudaStream_t st);

size_t mla_workspace_bytes(int B, int nH, int S);
// after_primary: the decode grid is a programmatic dependent of the previous launch on the stream (its
// setup overlaps that grid; its producer waits for it before loading q, and with kv_after_primary before
// the first latent load too, for a previous grid that may append to the cache)
// nH: a multiple of 16 (groups of 16 heads share one latent read); c_bstride / pe_bstride: elements between
// latent sequences (-1: contiguous [B, S, *])
int mla_launch(const void* q_proj, const void* q_pe, const void* c_kv, const void* k_pe, int B, int nH, int S,
               float scale, int out_mode, void* out, float* out_max, float* out_sum, float* out_lse, void* workspace,
               size_t workspace_bytes, cudaStream_t st, bool after_primary = false,
               bool kv_after_primary = false, int64_t c_bstride = -1, int64_t pe_bstride = -1);
size_t mla_absorbed_workspace_bytes(int B, int nH, int S);
int mla_absorbed_launch(const void* q_nope, const void* w_uk, int64_t w_uk_head_stride, const void* q_pe,
                        const void* c_kv, const void* k_pe, const void* w_uv, int64_t w_uv_head_stride, int B, int nH,
                        int S, int nop, int vhd, float scale, void* out, float* out_lse, void* workspace,
                        size_t workspace_bytes, cudaStream_t st, int64_t c_bstride = -1, int64_t pe_bstride = -1);

struct CsaLaunch {
    const void* q;
    int q_f32;
    int q_u8;                     // q holds u8 codes with q_scales (query-code mode; kv_i8 set, q_f32 clear)
    const float* q_scales;        // [bs * nq]
    const int32_t* kv_sums;       // [bs, nc_local] code sums of the int8 entries
    const void* kv_val;           // null, or bf16 values [bs, nc_local, 512] (the _full operator)
    int bs, nq;
    const void* kv;
    int kv_i8;
    const float* kv_scales;
    int64_t nc_local, shard_lo;   // the buffer holds entries [shard_lo, shard_lo + nc_local)
    const int* idx;               // [bs, k] or null for the dense range
    int k, window;
    int64_t dense_begin, dense_end;
    float scale;
    void* out;
    int out_f32;
    float* out_lse;
    void* workspace;
    size_t workspace_bytes;
    void* stream;
};

int csa_launch(const CsaLaunch& a);
size_t csa_workspace_bytes(int bs, int nq, int q_f32);
int csa_kv_quantize_launch(const void* kv, int64_t rows, int hd, void* out, float* scales, int32_t* sums,
                           cudaStream_t st);
int csa_q_quantize_launch(const float* q, int64_t rows, int hd, void* out, float* scales, cudaStream_t st);

size_t indexer_workspace_bytes(int bs, int64_t nc);
int indexer_topk_launch(const void* q, const void* kv, int bf16, const float* w, int bs, int nH, int hd, int64_t nc,
                        int k, int by_id, int32_t* out_ids, float* out_scores, void* workspace,
                        size_t workspace_bytes, cudaStream_t st);

int kv_append_launch(void* dst, int64_t dst_row, int64_t dst_tok, const void* src, int64_t src_row, int64_t src_tok,
                     int64_t rows, int64_t n_new, int D, int elem_bytes, int64_t t0, cudaStream_t st);

int lse_merge_launch(const float* o_parts, int64_t o_part_stride, const float* lse_parts, int64_t lse_part_stride,
                     int P, int64_t R, int D, void* out, int out_dtype, float* out_lse, cudaStream_t st,
                     bool after_primary = false);   // true: a programmatic dependent launch of the previous grid

}  // namespace ws
