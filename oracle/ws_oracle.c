/*
 * ws_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference decode-attention operators (the WriteScope
 * artifact's AVX-512 torch extensions).  It is the checker that the CUDA path
 * is compared against; nothing in the shipped library links, calls or loads
 * it.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may use it.
 *
 * Every routine accumulates in float64 (the reference accumulates in fp32
 * with -ffast-math), so it is a strictly tighter reference than the
 * operator it restates.  The two lossy quantisers (bf16->int8 per row,
 * fp32->u8 per row) are restated bit-exactly in fp32, because their rounding
 * is part of the operator's definition.
 *
 * Reference citations (paths relative to the reference checkout):
 *   orc_gqa_decode          kernel/cpu_attn.cpp:193-570  (run_kernel; per-token
 *                           online update :276-288, :336-343; tile merge :533-569)
 *                           wrappers fused_cpu_attn :572-636,
 *                           fused_cpu_attn_mla :638-672, fused_cpu_attn_fp32 :817-848
 *   orc_mla_compressed      kernel/cpu_attn.cpp:852-1022
 *   orc_csa_attend          kernel/cpu_attn_ds4_ext/csa_attn.cpp:200-281
 *                           (fused_csa_attn), :1587-1656 (fused_csa_attn_range),
 *                           :1819-1883 (indexer_attn_cpu, gather by top-k ids)
 *   orc_kv_quantize_s8      csa_attn.cpp:729-764, :1203-1233
 *   orc_q_quantize_u8       csa_attn.cpp:704-727, :1175-1201
 *   orc_csa_int8_preq       csa_attn.cpp:1235-1357
 *   orc_lse_merge           system/qwenoffload.py:1606-1617 (lse form),
 *                           system/mixoffload.py:1456-1464 (max/sum form)
 *   orc_indexer_topk        csa_attn.cpp:1658-1736
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>

static inline double bf16_to_d(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return (double)f;
}

static inline float bf16_to_f(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Element loader: kind 0 = bf16 (uint16 storage), 1 = fp32, 2 = int8. */
static inline double ld(const void* base, int kind, int64_t idx) {
    if (kind == 0) return bf16_to_d(((const uint16_t*)base)[idx]);
    if (kind == 1) return (double)((const float*)base)[idx];
    return (double)((const int8_t*)base)[idx];
}

/*
 * GQA / MLA decode over a strided [B_kv, L, D] KV share.
 *   q   [B_kv, G, Dk] contiguous
 *   k   element (b, i, d) at b*k_sb + i*k_si + d
 *   v   element (b, i, d) at b*v_sb + i*v_si + d
 * Outputs (float64): o_norm [B_kv, G, Dv] (normalised), mx [B_kv, G]
 * (running max of scaled scores), sm [B_kv, G] (sum of exp(s - mx)).
 * Per token:  s = scale * q.k ; nm = max(m, s) ; eo = exp(m - nm) ;
 *             en = exp(s - nm) ; sum = eo*sum + en ; o = eo*o + en*v
 * (kernel/cpu_attn.cpp:336-343).  L == 0 gives mx = -inf, sm = 0, o = 0.
 */
void orc_gqa_decode(const void* q, const void* k, const void* v, int kind,
                    int64_t k_sb, int64_t k_si, int64_t v_sb, int64_t v_si,
                    int B_kv, int G, int Dk, int Dv, int L, double scale,
                    double* o_norm, double* mx, double* sm) {
    #pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B_kv; b++) {
        for (int g = 0; g < G; g++) {
            double* o = o_norm + ((int64_t)b * G + g) * Dv;
            double m = -INFINITY, s_acc = 0.0;
            for (int d = 0; d < Dv; d++) o[d] = 0.0;
            int64_t qoff = ((int64_t)b * G + g) * Dk;
            for (int i = 0; i < L; i++) {
                int64_t ko = (int64_t)b * k_sb + (int64_t)i * k_si;
                int64_t vo = (int64_t)b * v_sb + (int64_t)i * v_si;
                double dot = 0.0;
                for (int d = 0; d < Dk; d++) dot += ld(q, kind, qoff + d) * ld(k, kind, ko + d);
                double sc = dot * scale;
                double nm = sc > m ? sc : m;
                double eo = exp(m - nm), en = exp(sc - nm);
                s_acc = eo * s_acc + en;
                m = nm;
                for (int d = 0; d < Dv; d++) o[d] = eo * o[d] + en * ld(v, kind, vo + d);
            }
            if (L > 0)
                for (int d = 0; d < Dv; d++) o[d] /= s_acc;
            mx[(int64_t)b * G + g] = m;
            sm[(int64_t)b * G + g] = s_acc;
        }
    }
}

/*
 * Absorbed-MLA decode (kernel/cpu_attn.cpp:852-1022).
 *   q_proj [B*nH, clr], q_pe [B*nH, qrd], c_kv [B, S, clr], k_pe [B, S, qrd] (bf16)
 *   score(h, t) = scale * (q_proj[h].c[t] + q_pe[h].p[t]);  V = c (the latent).
 * Outputs o_unnorm [B*nH, clr] (NOT normalised, as the reference returns),
 * mx [B*nH], sm [B*nH].
 */
void orc_mla_compressed(const uint16_t* q_proj, const uint16_t* q_pe,
                        const uint16_t* c_kv, const uint16_t* k_pe,
                        int B, int nH, int S, int clr, int qrd, double scale,
                        double* o_unnorm, double* mx, double* sm) {
    #pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; b++) {
        for (int h = 0; h < nH; h++) {
            int64_t r = (int64_t)b * nH + h;
            double* o = o_unnorm + r * clr;
            double m = -INFINITY, s_acc = 0.0;
            for (int d = 0; d < clr; d++) o[d] = 0.0;
            for (int t = 0; t < S; t++) {
                const uint16_t* c = c_kv + ((int64_t)b * S + t) * clr;
                const uint16_t* p = k_pe + ((int64_t)b * S + t) * qrd;
                double dot = 0.0;
                for (int d = 0; d < clr; d++) dot += bf16_to_d(q_proj[r * clr + d]) * bf16_to_d(c[d]);
                for (int d = 0; d < qrd; d++) dot += bf16_to_d(q_pe[r * qrd + d]) * bf16_to_d(p[d]);
                double sc = dot * scale;
                double nm = sc > m ? sc : m;
                double eo = exp(m - nm), en = exp(sc - nm);
                s_acc = eo * s_acc + en;
                m = nm;
                for (int d = 0; d < clr; d++) o[d] = eo * o[d] + en * bf16_to_d(c[d]);
            }
            mx[r] = m;
            sm[r] = s_acc;
        }
    }
}

/*
 * CSA attention of many query rows over one shared latent KV (K = V), over
 * either a contiguous entry range [kv_s, kv_e) (idx == NULL) or a gathered
 * id list idx[b, 0..n_idx) (indexer_attn_cpu, csa_attn.cpp:1819-1883).
 *   q     [bs, nq, hd]  (nq = n_heads * seqlen rows per sequence), q_kind 0 bf16 / 1 fp32
 *   kv    [bs, nc, hd]  kv_kind 0 bf16, 2 int8 (then kv_scale[bs, nc] fp32
 *                        multiplies each entry: value = int8 * scale, exact)
 * Outputs o [bs, nq, hd] normalised, lse [bs, nq] = m + log(sum).
 * Ids outside [0, nc) are skipped and counted in the return value.
 */
int64_t orc_csa_attend(const void* q, int q_kind, const void* kv, int kv_kind,
                       const float* kv_scale, const int32_t* idx, int n_idx,
                       int kv_s, int kv_e,
                       int bs, int nq, int hd, int nc, double scale,
                       double* o, double* lse) {
    int64_t bad = 0;
    #pragma omp parallel for collapse(2) schedule(static) reduction(+:bad)
    for (int b = 0; b < bs; b++) {
        for (int r = 0; r < nq; r++) {
            int64_t row = (int64_t)b * nq + r;
            double* orow = o + row * hd;
            double m = -INFINITY, s_acc = 0.0;
            for (int d = 0; d < hd; d++) orow[d] = 0.0;
            int n = idx ? n_idx : (kv_e - kv_s);
            for (int i = 0; i < n; i++) {
                int64_t e = idx ? (int64_t)idx[(int64_t)b * n_idx + i] : (int64_t)(kv_s + i);
                if (e < 0 || e >= nc) { bad++; continue; }
                int64_t eo_ = ((int64_t)b * nc + e) * hd;
                double es = (kv_kind == 2) ? (double)kv_scale[(int64_t)b * nc + e] : 1.0;
                double dot = 0.0;
                for (int d = 0; d < hd; d++) dot += ld(q, q_kind, row * hd + d) * ld(kv, kv_kind, eo_ + d);
                double sc = dot * es * scale;
                double nm = sc > m ? sc : m;
                double eo = exp(m - nm), en = exp(sc - nm);
                s_acc = eo * s_acc + en;
                m = nm;
                for (int d = 0; d < hd; d++) orow[d] = eo * orow[d] + en * es * ld(kv, kv_kind, eo_ + d);
            }
            if (s_acc > 0.0)
                for (int d = 0; d < hd; d++) orow[d] /= s_acc;
            lse[row] = m + log(s_acc);
        }
    }
    return bad;
}

/* Round-half-to-even fp32 -> int32 with x86 cvtps2dq semantics for the
 * in-range values these quantisers produce (|x| <= 127.5 + eps). */
static inline int32_t cvt_rne(float x) { return (int32_t)nearbyintf(x); }

static inline int32_t sat(int32_t x, int32_t lo, int32_t hi) { return x < lo ? lo : (x > hi ? hi : x); }

/*
 * Per-row symmetric bf16 -> int8 quantiser (csa_attn.cpp:729-764):
 *   maxv = max(max|x|, 1e-6); scale = maxv*(1/127); inv = 127/maxv;
 *   q = sat_s8(sat_s16(rne(x*inv)));  sum = sum(q).
 */
void orc_kv_quantize_s8(const uint16_t* kv, int64_t rows, int hd,
                        int8_t* out, float* scales, int32_t* sums) {
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const uint16_t* x = kv + r * hd;
        float maxv = 0.0f;
        for (int d = 0; d < hd; d++) { float a = fabsf(bf16_to_f(x[d])); if (a > maxv) maxv = a; }
        if (maxv < 1e-6f) maxv = 1e-6f;
        /* the reference is built with -ffast-math, which turns maxv/127 into
           maxv * (1/127); restated that way so scales match bit for bit */
        scales[r] = maxv * (1.0f / 127.0f);
        float inv = 127.0f / maxv;
        int32_t s = 0;
        for (int d = 0; d < hd; d++) {
            int32_t v = cvt_rne(bf16_to_f(x[d]) * inv);
            v = sat(sat(v, -32768, 32767), -128, 127);
            out[r * hd + d] = (int8_t)v;
            s += v;
        }
        sums[r] = s;
    }
}

/*
 * Per-row fp32 -> u8 quantiser (csa_attn.cpp:704-727):
 *   maxv = max(max|x|, 1e-6); scale = maxv*(1/127); inv = 127/maxv;
 *   u = sat_u8(sat_s16(rne(x*inv) + 128)).
 */
void orc_q_quantize_u8(const float* q, int64_t rows, int hd, uint8_t* out, float* scales) {
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float* x = q + r * hd;
        float maxv = 0.0f;
        for (int d = 0; d < hd; d++) { float a = fabsf(x[d]); if (a > maxv) maxv = a; }
        if (maxv < 1e-6f) maxv = 1e-6f;
        scales[r] = maxv * (1.0f / 127.0f);   /* -ffast-math form, as above */
        float inv = 127.0f / maxv;
        for (int d = 0; d < hd; d++) {
            int32_t v = cvt_rne(x[d] * inv) + 128;
            v = sat(sat(v, -32768, 32767), 0, 255);
            out[r * hd + d] = (uint8_t)v;
        }
    }
}

/*
 * CSA in the reference's integer-score form (csa_attn.cpp:1235-1483, and the
 * attention of :766-883 after its quantisers).  Query rows arrive as u8 codes
 * with one scale each, entries as s8 codes with a scale and a code sum:
 *   dot   = sum_d u8[d] * s8[d] - 128 * ksum                 (int32, exact; :1323-1328)
 *   score = (float)dot * q_scale * k_scale * scale            (fp32, this order; :1329)
 * The value is int8 * k_scale (:1338-1344) or, with kv_bf16 non-NULL, the
 * bf16 entry (:1465-1470).  Entries are all nc (idx NULL) or the ids
 * idx[b, 0..n_idx).  The softmax and the value sums are carried in float64.
 */
void orc_csa_int8_codes(const uint8_t* q_u8, const float* q_scales, const int8_t* kv_i8,
                        const float* kv_scales, const int32_t* kv_sums, const uint16_t* kv_bf16,
                        const int32_t* idx, int n_idx, int bs, int nq, int hd, int nc, float scale,
                        double* o, double* lse) {
    #pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < bs; b++) {
        for (int r = 0; r < nq; r++) {
            int64_t row = (int64_t)b * nq + r;
            double* orow = o + row * hd;
            double m = -INFINITY, s_acc = 0.0;
            for (int d = 0; d < hd; d++) orow[d] = 0.0;
            int n = idx ? n_idx : nc;
            for (int j = 0; j < n; j++) {
                int64_t i = idx ? (int64_t)idx[(int64_t)b * n_idx + j] : (int64_t)j;
                if (i < 0 || i >= nc) continue;
                const int8_t* ki = kv_i8 + ((int64_t)b * nc + i) * hd;
                float ksc = kv_scales[(int64_t)b * nc + i];
                int32_t dot = 0;
                for (int d = 0; d < hd; d++) dot += (int32_t)q_u8[row * hd + d] * (int32_t)ki[d];
                dot -= 128 * kv_sums[(int64_t)b * nc + i];
                float scf = (float)dot * q_scales[row] * ksc * scale;
                double sc = (double)scf;
                double nm = sc > m ? sc : m;
                double eo = exp(m - nm), en = exp(sc - nm);
                s_acc = eo * s_acc + en;
                m = nm;
                if (kv_bf16) {
                    const uint16_t* vb = kv_bf16 + ((int64_t)b * nc + i) * hd;
                    for (int d = 0; d < hd; d++) orow[d] = eo * orow[d] + en * bf16_to_d(vb[d]);
                } else {
                    for (int d = 0; d < hd; d++) orow[d] = eo * orow[d] + en * (double)ksc * (double)ki[d];
                }
            }
            if (s_acc > 0.0)
                for (int d = 0; d < hd; d++) orow[d] /= s_acc;
            lse[row] = m + log(s_acc);
        }
    }
}

/*
 * fused_csa_attn_bsq_int8_preq (csa_attn.cpp:1235-1357): the fp32 query is
 * quantised per row to u8 exactly as the reference does, then scored and
 * summed as orc_csa_int8_codes does with int8 * k_scale values.
 */
void orc_csa_int8_preq(const float* q, const int8_t* kv_i8, const float* kv_scales,
                       const int32_t* kv_sums, int bs, int nq, int hd, int nc,
                       float scale, double* o, double* lse) {
    uint8_t* qu = (uint8_t*)malloc((size_t)bs * nq * hd);
    float* qs = (float*)malloc((size_t)bs * nq * sizeof(float));
    orc_q_quantize_u8(q, (int64_t)bs * nq, hd, qu, qs);
    orc_csa_int8_codes(qu, qs, kv_i8, kv_scales, kv_sums, NULL, NULL, 0, bs, nq, hd, nc, scale, o, lse);
    free(qu);
    free(qs);
}

/*
 * LSE merge of P partials (system/qwenoffload.py:1606-1617):
 *   o_p [P, R, D] normalised, lse_p [P, R]  ->  o [R, D], lse [R]
 *   M = max_p lse_p ; L = M + log(sum_p exp(lse_p - M)) ; o = sum_p exp(lse_p - L) o_p
 * A row whose partials are all -inf gives o = 0, lse = -inf.
 */
void orc_lse_merge(const double* o_p, const double* lse_p, int P, int64_t R, int D,
                   double* o, double* lse) {
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < R; r++) {
        double M = -INFINITY;
        for (int p = 0; p < P; p++) if (lse_p[(int64_t)p * R + r] > M) M = lse_p[(int64_t)p * R + r];
        double* orow = o + r * D;
        for (int d = 0; d < D; d++) orow[d] = 0.0;
        if (M == -INFINITY) { lse[r] = -INFINITY; continue; }
        double s = 0.0;
        for (int p = 0; p < P; p++) s += exp(lse_p[(int64_t)p * R + r] - M);
        double L = M + log(s);
        for (int p = 0; p < P; p++) {
            double w = exp(lse_p[(int64_t)p * R + r] - L);
            if (w == 0.0) continue;
            const double* op = o_p + ((int64_t)p * R + r) * D;
            for (int d = 0; d < D; d++) orow[d] += w * op[d];
        }
        lse[r] = L;
    }
}

/*
 * Indexer top-k (csa_attn.cpp:1658-1736):
 *   score[n] = sum_h relu(q[h].kv[n]) * w[h]  (fp32 inputs, float64 here)
 *   out[b, 0..k) = ids of the k largest scores, largest first; ties broken
 *   by the smaller id (the reference's partial_sort leaves ties unspecified).
 */
static const double* g_sort_scores;
static int cmp_desc(const void* a, const void* b) {
    int ia = *(const int*)a, ib = *(const int*)b;
    double sa = g_sort_scores[ia], sb = g_sort_scores[ib];
    if (sa > sb) return -1;
    if (sa < sb) return 1;
    return ia - ib;
}

void orc_indexer_topk(const float* q_idx, const float* kv_idx, const float* w,
                      int bs, int nH, int hd, int nc, int k, int32_t* out, double* scores_out) {
    if (k > nc) k = nc;
    double* sc = (double*)malloc(sizeof(double) * nc);
    int* ids = (int*)malloc(sizeof(int) * nc);
    for (int b = 0; b < bs; b++) {
        for (int n = 0; n < nc; n++) {
            double s = 0.0;
            for (int h = 0; h < nH; h++) {
                double dot = 0.0;
                for (int d = 0; d < hd; d++)
                    dot += (double)q_idx[((int64_t)b * nH + h) * hd + d] *
                           (double)kv_idx[((int64_t)b * nc + n) * hd + d];
                s += (dot > 0.0 ? dot : 0.0) * (double)w[(int64_t)b * nH + h];
            }
            sc[n] = s;
            ids[n] = n;
            if (scores_out) scores_out[(int64_t)b * nc + n] = s;
        }
        g_sort_scores = sc;
        qsort(ids, nc, sizeof(int), cmp_desc);
        for (int i = 0; i < k; i++) out[(int64_t)b * k + i] = ids[i];
    }
    free(sc);
    free(ids);
}

/*
 * The indexer score in the reference's own fp32 arithmetic
 * (csa_attn.cpp:1706-1724): per head, 16 lane accumulators (lane l takes
 * dims l, l+16, ... with a fused multiply-add each, :1712-1716), reduced as
 * _mm512_reduce_add_ps does (the two 8-lane halves, then the two 4-lane
 * halves, then lanes {0+2, 1+3}, then the last add; :128-130), then
 * s = fma(relu(dot), w[h], s) over the heads in order (:1720-1721; the
 * reference's -O3 -ffast-math build contracts the multiply-add).
 * contract = 0 evaluates the last step as s + relu(dot) * w[h] instead.
 */
void orc_indexer_scores_f32(const float* q_idx, const float* kv_idx, const float* w,
                            int bs, int nH, int hd, int64_t nc, int contract, float* scores) {
    #pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < bs; b++) {
        for (int64_t n = 0; n < nc; n++) {
            const float* kv = kv_idx + ((int64_t)b * nc + n) * hd;
            float s = 0.0f;
            for (int h = 0; h < nH; h++) {
                const float* q = q_idx + ((int64_t)b * nH + h) * hd;
                float a[16];
                for (int l = 0; l < 16; l++) a[l] = 0.0f;
                for (int d = 0; d < hd; d += 16)
                    for (int l = 0; l < 16; l++) a[l] = fmaf(q[d + l], kv[d + l], a[l]);
                float t3[8], t6[4];
                for (int i = 0; i < 8; i++) t3[i] = a[i + 8] + a[i];
                for (int i = 0; i < 4; i++) t6[i] = t3[i + 4] + t3[i];
                float t80 = t6[0] + t6[2], t81 = t6[1] + t6[3];
                float dot = t80 + t81;
                float r = dot > 0.0f ? dot : 0.0f;
                if (contract) {
                    s = fmaf(r, w[(int64_t)b * nH + h], s);
                } else {
                    float pr = r * w[(int64_t)b * nH + h];
                    s = s + pr;
                }
            }
            scores[(int64_t)b * nc + n] = s;
        }
    }
}
