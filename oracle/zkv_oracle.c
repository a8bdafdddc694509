/*
 * zkv_oracle.c -- CPU restatement of the ZoomKV sparse decode-attention hot
 * path (TEST INFRASTRUCTURE ONLY; see zkv_oracle.h for the contract and the
 * reference file:line each routine follows).
 *
 * Build with -ffp-contract=off: several routines reproduce the reference
 * CUDA kernels' fp32 operation order bit for bit, and a fused multiply-add
 * would change the rounding.
 */
#include "zkv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <pthread.h>
#include <string.h>

float orc_bf2f(uint16_t b) {
    uint32_t u = ((uint32_t)b) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t orc_f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest, ties to even */
    return (uint16_t)(u >> 16);
}

/* bf16 binary ops: compute in fp32 and round once.  For bf16 operands the
 * fp32 result rounded to bf16 equals the correctly rounded bf16 result
 * (24 >= 2*8+2), which is what torch's CPU bf16 ops and the CUDA bf16
 * intrinsics both produce. */
static inline uint16_t bsub(uint16_t a, uint16_t b) { return orc_f2bf(orc_bf2f(a) - orc_bf2f(b)); }
static inline uint16_t badd(uint16_t a, uint16_t b) { return orc_f2bf(orc_bf2f(a) + orc_bf2f(b)); }
static inline uint16_t bmul(uint16_t a, uint16_t b) { return orc_f2bf(orc_bf2f(a) * orc_bf2f(b)); }
static inline uint16_t bdiv(uint16_t a, uint16_t b) { return orc_f2bf(orc_bf2f(a) / orc_bf2f(b)); }

uint16_t orc_kivi_scale(uint16_t mn, uint16_t mx) {
    /* __hdiv(__hsub(mx, mn), 15) -- kivi_qk_dot.cu:215-216;
     * (chunk_max - chunk_min) / 15.0 -- quant_pack.py:64 */
    return bdiv(bsub(mx, mn), orc_f2bf(15.0f));
}

/* a*b + c on bf16 operands with ONE rounding to bf16 (round to nearest
 * even), i.e. a bf16 fused multiply-add.  The exact value is formed in
 * double (a*b is exact there), narrowed to binary32 with round-to-odd (so
 * the final rounding sees every discarded bit) and rounded once to bf16. */
uint16_t orc_bfma(uint16_t a, uint16_t b, uint16_t c) {
    const double x = fma((double)orc_bf2f(a), (double)orc_bf2f(b), (double)orc_bf2f(c));
    float f = (float)x;
    if ((double)f != x) {
        uint32_t u;
        memcpy(&u, &f, 4);
        if (fabs((double)f) > fabs(x)) u -= 1u; /* the neighbour toward zero */
        u |= 1u;                                /* sticky: round to odd */
        memcpy(&f, &u, 4);
    }
    return orc_f2bf(f);
}

/* KIVI dequant as the production stage-2 kernel computes it:
 * bf16(code*scale + mn) with one rounding.  kivi_qk_dot.cu:264-275 writes it
 * as __hmul2 then __hadd2, but the kernel the reference builds rounds once
 * (measured bit for bit against that kernel's outputs on a B200:
 * tests/golden/ref_cuda.npz). */
uint16_t orc_dequant_fused(int code, uint16_t scale, uint16_t zero) {
    return orc_bfma(orc_f2bf((float)code), scale, zero);
}

uint16_t orc_dequant(int code, uint16_t scale, uint16_t zero) {
    /* code*scale then +mn, two bf16 ops, no FMA -- kivi_qk_dot.cu:264-275 */
    return badd(bmul(orc_f2bf((float)code), scale), zero);
}

/* code = round_half_even(clamp(bf16(bf16(x - mn) / scale_safe), 0, 15)),
 * scale_safe = bf16(max(scale, 1e-8)) -- _kivi_pack_chunks :2006-2011,
 * quantize_kcache_4bit quant_pack.py:115-121. */
static inline int kivi_code(uint16_t x, uint16_t mn, uint16_t scale) {
    float sc = orc_bf2f(scale);
    uint16_t safe = orc_f2bf(sc > 1e-8f ? sc : 1e-8f);
    float y = orc_bf2f(bdiv(bsub(x, mn), safe));
    if (y < 0.0f) y = 0.0f;
    if (y > 15.0f) y = 15.0f;
    return (int)rintf(y);
}

void orc_kivi_encode_chunk(const uint16_t* keys, int64_t ld, int D, int chunk,
                           uint16_t* mn, uint16_t* mx, uint16_t* centroid,
                           int32_t* packed) {
    int t, d, w, j;
    for (d = 0; d < D; ++d) {
        uint16_t lo = keys[d], hi = keys[d];
        float sum = 0.0f;
        for (t = 0; t < chunk; ++t) {
            uint16_t v = keys[t * ld + d];
            if (orc_bf2f(v) < orc_bf2f(lo)) lo = v;
            if (orc_bf2f(v) > orc_bf2f(hi)) hi = v;
            sum += orc_bf2f(v);
        }
        mn[d] = lo;
        mx[d] = hi;
        /* torch.mean over the chunk axis: fp32 sum then divide, one bf16
         * rounding (_compute_and_store_chunk_minmax :2123) */
        centroid[d] = orc_f2bf(sum / (float)chunk);
    }
    for (w = 0; w < D / 8; ++w) {
        for (t = 0; t < chunk; ++t) {
            uint32_t word = 0;
            for (j = 0; j < 8; ++j) {
                d = 8 * w + j;
                uint16_t sc = orc_kivi_scale(mn[d], mx[d]);
                word |= ((uint32_t)kivi_code(keys[t * ld + d], mn[d], sc)) << (4 * j);
            }
            packed[w * chunk + t] = (int32_t)word;
        }
    }
}

void orc_vquant_token(const uint16_t* v, int D, int group, int32_t* codes,
                      uint16_t* meta) {
    int g, d;
    uint16_t code_of[1024];
    for (g = 0; g < D / group; ++g) {
        uint16_t lo = v[g * group], hi = v[g * group];
        for (d = g * group; d < (g + 1) * group; ++d) {
            if (orc_bf2f(v[d]) < orc_bf2f(lo)) lo = v[d];
            if (orc_bf2f(v[d]) > orc_bf2f(hi)) hi = v[d];
        }
        uint16_t sc = orc_kivi_scale(lo, hi);
        meta[2 * g] = sc;
        meta[2 * g + 1] = lo;
        for (d = g * group; d < (g + 1) * group; ++d)
            code_of[d] = (uint16_t)kivi_code(v[d], lo, sc);
    }
    for (d = 0; d < D / 8; ++d) {
        uint32_t word = 0;
        int j;
        for (j = 0; j < 8; ++j) word |= ((uint32_t)code_of[8 * d + j]) << (4 * j);
        codes[d] = (int32_t)word;
    }
}

/* ---------------- Quest score (quest_chunk_score.cu:31-103) ---------------- */
static float quest_one(const uint16_t* q, const uint16_t* mn, const uint16_t* mx) {
    float s[32];
    int t, off;
    for (t = 0; t < 32; ++t) {
        float acc = 0.0f;
        int j;
        for (j = 0; j < 4; ++j) {
            int d = 4 * t + j;
            float qd = orc_bf2f(q[d]);
            float a = qd * orc_bf2f(mn[d]);
            float b = qd * orc_bf2f(mx[d]);
            float f = fmaxf(a, b);
            acc = (j == 0) ? f : acc + f;
        }
        s[t] = acc;
    }
    for (off = 16; off >= 1; off >>= 1) {
        float n[32];
        for (t = 0; t < 32; ++t) n[t] = s[t] + s[t ^ off];
        memcpy(s, n, sizeof(s));
    }
    return s[0];
}

void orc_quest_score(const uint16_t* q, const uint16_t* mn, const uint16_t* mx,
                     const uint8_t* valid, float* scores, int rows,
                     int n_chunks, int n_max) {
    int r, c;
    for (r = 0; r < rows; ++r)
        for (c = 0; c < n_chunks; ++c) {
            size_t base = ((size_t)r * n_max + c) * 128;
            if (valid && !valid[(size_t)r * n_max + c]) {
                scores[(size_t)r * n_chunks + c] = -INFINITY;
                continue;
            }
            scores[(size_t)r * n_chunks + c] = quest_one(q + (size_t)r * 128, mn + base, mx + base);
        }
}

/* ---------------- deterministic top-k ---------------- */
static inline uint32_t ordered_u32(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

typedef struct { uint32_t key; int32_t idx; } kv_t;

static int cmp_desc(const void* pa, const void* pb) {
    const kv_t* a = (const kv_t*)pa;
    const kv_t* b = (const kv_t*)pb;
    if (a->key != b->key) return a->key > b->key ? -1 : 1;
    return a->idx < b->idx ? -1 : (a->idx > b->idx);
}

static int cmp_i64(const void* pa, const void* pb) {
    int64_t a = *(const int64_t*)pa, b = *(const int64_t*)pb;
    return a < b ? -1 : (a > b);
}

/* select the k largest keys (ties -> lowest index), ascending index order */
static void select_keys(kv_t* buf, int len, int k, int64_t* out) {
    int i;
    if (len <= k) {
        for (i = 0; i < k; ++i) out[i] = i < len ? i : -1;
        return;
    }
    qsort(buf, (size_t)len, sizeof(kv_t), cmp_desc);
    for (i = 0; i < k; ++i) out[i] = buf[i].idx;
    qsort(out, (size_t)k, sizeof(int64_t), cmp_i64);
}

void orc_topk_f32(const float* scores, int rows, int len, int64_t row_stride,
                  int k, int64_t* out) {
    kv_t* buf = (kv_t*)malloc(sizeof(kv_t) * (size_t)(len > 0 ? len : 1));
    int r, i;
    for (r = 0; r < rows; ++r) {
        for (i = 0; i < len; ++i) {
            buf[i].key = ordered_u32(scores[(size_t)r * row_stride + i]);
            buf[i].idx = i;
        }
        select_keys(buf, len, k, out + (size_t)r * k);
    }
    free(buf);
}

/* ---------------- hierarchical Quest ---------------- */
void orc_large_minmax(const uint16_t* mn, const uint16_t* mx, int rows, int n_max, int valid_end, int factor,
                      int n_max_large, uint16_t* lmn, uint16_t* lmx, uint8_t* lvalid) {
    int r, g, b, d;
    for (r = 0; r < rows; ++r)
        for (g = 0; g < n_max_large; ++g) {
            int b_lo = g * factor, b_hi = b_lo + factor;
            size_t o = ((size_t)r * n_max_large + g) * 128;
            if (b_hi > valid_end) b_hi = valid_end;
            if (b_hi > n_max) b_hi = n_max;
            lvalid[(size_t)r * n_max_large + g] = b_hi > b_lo;
            for (d = 0; d < 128; ++d) {
                uint16_t a = 0, z = 0;
                if (b_hi > b_lo) {
                    a = mn[((size_t)r * n_max + b_lo) * 128 + d];
                    z = mx[((size_t)r * n_max + b_lo) * 128 + d];
                    for (b = b_lo + 1; b < b_hi; ++b) {
                        uint16_t u = mn[((size_t)r * n_max + b) * 128 + d];
                        uint16_t v = mx[((size_t)r * n_max + b) * 128 + d];
                        if (orc_bf2f(u) < orc_bf2f(a)) a = u;
                        if (orc_bf2f(v) > orc_bf2f(z)) z = v;
                    }
                }
                lmn[o + d] = a;
                lmx[o + d] = z;
            }
        }
}

void orc_sub_chunk_score(const uint16_t* q, const uint16_t* mn, const uint16_t* mx, const int64_t* large_idx,
                         int rows, int n_max, int n_sel, int factor, float* sub) {
    int r, j, s;
    for (r = 0; r < rows; ++r)
        for (j = 0; j < n_sel; ++j)
            for (s = 0; s < factor; ++s) {
                int64_t c = large_idx[(size_t)r * n_sel + j] * factor + s;
                float* o = sub + (size_t)r * n_sel * factor + (size_t)j * factor + s;
                if (c < 0 || c >= n_max) {
                    *o = -INFINITY;
                    continue;
                }
                *o = quest_one(q + (size_t)r * 128, mn + ((size_t)r * n_max + c) * 128,
                               mx + ((size_t)r * n_max + c) * 128);
            }
}

void orc_map_back(const int64_t* large_idx, const int64_t* sub_pos, int rows, int nk_large, int nk_small,
                  int factor, int n_chunks, int64_t* out) {
    int r, k;
    for (r = 0; r < rows; ++r)
        for (k = 0; k < nk_small; ++k) {
            int64_t p = sub_pos[(size_t)r * nk_small + k];
            int64_t* o = out + (size_t)r * nk_small + k;
            int64_t sel, c;
            if (p < 0 || p >= (int64_t)nk_large * factor) {
                *o = -1;
                continue;
            }
            sel = p / factor;
            c = large_idx[(size_t)r * nk_large + sel] * factor + (p - sel * factor);
            if (c < 0) c = 0;
            if (c >= n_chunks) c = n_chunks - 1;
            *o = c;
        }
}

void orc_hier_select(const uint16_t* q, const uint16_t* mn, const uint16_t* mx, int n_max, const uint16_t* lmn,
                     const uint16_t* lmx, const uint8_t* lvalid, int n_max_large, int rows, int n_chunks,
                     int factor, int nk_large, int nk_small, int64_t* out, int64_t* large_idx_out, float* sub_out) {
    int n_large = n_chunks / factor, r;
    int n_sub = nk_large * factor;
    float* ls = (float*)malloc(sizeof(float) * (size_t)(n_large > 0 ? n_large : 1));
    int64_t* li = (int64_t*)malloc(sizeof(int64_t) * (size_t)(nk_large > 0 ? nk_large : 1));
    float* sub = (float*)malloc(sizeof(float) * (size_t)(n_sub > 0 ? n_sub : 1));
    int64_t* pos = (int64_t*)malloc(sizeof(int64_t) * (size_t)(nk_small > 0 ? nk_small : 1));
    for (r = 0; r < rows; ++r) {
        const uint16_t* qr = q + (size_t)r * 128;
        orc_quest_score(qr, lmn + (size_t)r * n_max_large * 128, lmx + (size_t)r * n_max_large * 128,
                        lvalid ? lvalid + (size_t)r * n_max_large : NULL, ls, 1, n_large, n_max_large);
        orc_topk_f32(ls, 1, n_large, n_large, nk_large, li);
        orc_sub_chunk_score(qr, mn + (size_t)r * n_max * 128, mx + (size_t)r * n_max * 128, li, 1, n_max,
                            nk_large, factor, sub);
        orc_topk_f32(sub, 1, n_sub, n_sub, nk_small, pos);
        orc_map_back(li, pos, 1, nk_large, nk_small, factor, n_chunks, out + (size_t)r * nk_small);
        if (large_idx_out) memcpy(large_idx_out + (size_t)r * nk_large, li, sizeof(int64_t) * (size_t)nk_large);
        if (sub_out) memcpy(sub_out + (size_t)r * n_sub, sub, sizeof(float) * (size_t)n_sub);
    }
    free(ls);
    free(li);
    free(sub);
    free(pos);
}

void orc_topk_i32(const int32_t* vals, int rows, int len, int64_t row_stride,
                  int k, int64_t* out) {
    kv_t* buf = (kv_t*)malloc(sizeof(kv_t) * (size_t)(len > 0 ? len : 1));
    int r, i;
    for (r = 0; r < rows; ++r) {
        for (i = 0; i < len; ++i) {
            buf[i].key = ((uint32_t)vals[(size_t)r * row_stride + i]) ^ 0x80000000u;
            buf[i].idx = i;
        }
        select_keys(buf, len, k, out + (size_t)r * k);
    }
    free(buf);
}

/* ---------------- CDS density + mask ---------------- */
void orc_chunk_density(const int64_t* chunk_ids, const uint16_t* centroid,
                       const uint16_t* raw_q, float* out, int rows, int nk,
                       int n_chunks, int n_max) {
    int r, s, d, stride;
    float buf[128];
    for (r = 0; r < rows; ++r)
        for (s = 0; s < nk; ++s) {
            int64_t c = chunk_ids[(size_t)r * nk + s];
            if (c < 0 || c >= n_chunks) {
                out[(size_t)r * nk + s] = -1e30f;
                continue;
            }
            const uint16_t* cent = centroid + ((size_t)r * n_max + (size_t)c) * 128;
            for (d = 0; d < 128; ++d) buf[d] = orc_bf2f(cent[d]) * orc_bf2f(raw_q[(size_t)r * 128 + d]);
            for (stride = 64; stride > 0; stride >>= 1)
                for (d = 0; d < stride; ++d) buf[d] = buf[d] + buf[d + stride];
            out[(size_t)r * nk + s] = buf[0];
        }
}

void orc_mask_from_topk(const int64_t* positions, uint8_t* mask, int rows,
                        int n_dense, int nk) {
    int r, j;
    for (r = 0; r < rows; ++r) {
        memset(mask + (size_t)r * nk, 0, (size_t)nk);
        for (j = 0; j < n_dense; ++j) {
            int64_t p = positions[(size_t)r * n_dense + j];
            if (p >= 0 && p < nk) mask[(size_t)r * nk + p] = 1;
        }
    }
}

/* ---------------- KIVI stage-2 ---------------- */
void orc_kivi_qk(const int64_t* chunk_ids, const uint8_t* dense_mask,
                 const int32_t* packed, int n_pk, const uint16_t* mn,
                 const uint16_t* mx, int n_max, const uint16_t* raw_q,
                 int rows, int nk, int chunk, int dense_topk, int sparse_topk,
                 float* out_scores, int64_t* out_idx) {
    const int D = 128, NP = D / 8;
    int r, s, t, i, j;
    for (r = 0; r < rows; ++r)
        for (s = 0; s < nk; ++s) {
            int64_t cid = chunk_ids[(size_t)r * nk + s];
            int dense = dense_mask[(size_t)r * nk + s] != 0;
            int in_range = cid >= 0 && cid < n_pk;
            kv_t lane[32];
            float sc_of[32];
            for (t = 0; t < chunk; ++t) {
                float acc = -1e30f;
                if (in_range) {
                    const uint16_t* cmn = mn + ((size_t)r * n_max + (size_t)cid) * D;
                    const uint16_t* cmx = mx + ((size_t)r * n_max + (size_t)cid) * D;
                    const int32_t* pk = packed + ((size_t)r * n_pk + (size_t)cid) * NP * chunk;
                    acc = 0.0f;
                    for (i = 0; i < NP; ++i) {
                        uint32_t word = (uint32_t)pk[i * chunk + t];
                        for (j = 0; j < 8; ++j) {
                            int d = 8 * i + j;
                            uint16_t kd = orc_dequant_fused((int)((word >> (4 * j)) & 15u),
                                                            orc_kivi_scale(cmn[d], cmx[d]), cmn[d]);
                            uint16_t prod = bmul(kd, raw_q[(size_t)r * D + d]);
                            acc += orc_bf2f(prod);
                        }
                    }
                }
                sc_of[t] = acc;
                lane[t].key = ordered_u32(acc);
                lane[t].idx = (int32_t)(cid * chunk + t);
            }
            (void)sc_of;
            qsort(lane, (size_t)chunk, sizeof(kv_t), cmp_desc);
            int eff = dense ? dense_topk : sparse_topk;
            for (t = 0; t < chunk; ++t) {
                size_t o = (size_t)r * nk * chunk + (size_t)s * chunk + t;
                if (t < eff) {
                    uint32_t k = lane[t].key;
                    uint32_t bits = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
                    float f;
                    memcpy(&f, &bits, 4);
                    out_scores[o] = f;
                    out_idx[o] = lane[t].idx;
                } else {
                    out_scores[o] = -1e30f;
                    out_idx[o] = 0;
                }
            }
        }
}

/* ---------------- global top-k + gather + concat ---------------- */
void orc_topk_gather_concat(const float* scores, const int64_t* lut,
                            const int64_t* skipped, int64_t* out, int rows,
                            int L, int k, int sk, int64_t out_ld) {
    int64_t* pos = (int64_t*)malloc(sizeof(int64_t) * (size_t)(k > 0 ? k : 1));
    int r, i;
    for (r = 0; r < rows; ++r) {
        int64_t* o = out + (size_t)r * out_ld;
        for (i = 0; i < k; ++i) o[i] = 0;
        for (i = 0; i < sk; ++i) o[k + i] = skipped[(size_t)r * sk + i];
        if (L <= k) {
            for (i = 0; i < k; ++i) o[i] = i < L ? lut[(size_t)r * L + i] : 0;
            continue;
        }
        orc_topk_f32(scores + (size_t)r * L, 1, L, L, k, pos);
        for (i = 0; i < k; ++i) o[i] = lut[(size_t)r * L + pos[i]];
    }
    free(pos);
}

/* ---------------- attention ---------------- */
void orc_attn_dense(const float* q, const float* K, const float* V, int n,
                    int G, int D, float scale, float* out, float* lse) {
    double* s = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    int g, i, d;
    for (g = 0; g < G; ++g) {
        double m = -INFINITY, l = 0.0;
        for (i = 0; i < n; ++i) {
            double acc = 0.0;
            for (d = 0; d < D; ++d) acc += (double)q[g * D + d] * (double)K[(size_t)i * D + d];
            s[i] = acc * (double)scale;
            if (s[i] > m) m = s[i];
        }
        for (d = 0; d < D; ++d) out[g * D + d] = 0.0f;
        if (n == 0) {
            lse[g] = -INFINITY;
            continue;
        }
        for (i = 0; i < n; ++i) {
            s[i] = exp(s[i] - m);
            l += s[i];
        }
        for (d = 0; d < D; ++d) {
            double acc = 0.0;
            for (i = 0; i < n; ++i) acc += s[i] * (double)V[(size_t)i * D + d];
            out[g * D + d] = (float)(acc / l);
        }
        lse[g] = (float)(m + log(l));
    }
    free(s);
}

static void page_row(const uint16_t* q, const uint16_t* mn, const uint16_t* mx,
                     const uint8_t* valid, const int32_t* kcodes,
                     const int32_t* vcodes, const uint16_t* vmeta,
                     const uint16_t* nearK, const uint16_t* nearV, int G,
                     int n_max, int n_c, int nk, int n_near, float scale,
                     uint16_t* out, float* lse, int64_t* sel) {
    const int D = 128, C = 16, NP = D / 8, NG = D / 32;
    uint16_t raw_q[128];
    int d, g, i, t;
    /* GQA-mean query, compute() :1622-1626 (bf16 mean over the group) */
    for (d = 0; d < D; ++d) {
        float acc = 0.0f;
        for (g = 0; g < G; ++g) acc += orc_bf2f(q[g * D + d]);
        raw_q[d] = orc_f2bf(acc / (float)G);
    }
    float* scores = (float*)malloc(sizeof(float) * (size_t)n_c);
    orc_quest_score(raw_q, mn, mx, valid, scores, 1, n_c, n_max);
    int64_t* chosen = (int64_t*)malloc(sizeof(int64_t) * (size_t)nk);
    orc_topk_f32(scores, 1, n_c, n_c, nk, chosen);
    if (sel) memcpy(sel, chosen, sizeof(int64_t) * (size_t)nk);
    int n = nk * C + n_near;
    float* K = (float*)malloc(sizeof(float) * (size_t)n * D);
    float* V = (float*)malloc(sizeof(float) * (size_t)n * D);
    int row = 0;
    for (i = 0; i < nk; ++i) {
        int64_t c = chosen[i];
        if (c < 0) c = 0; /* clamp, _quest_pick_coarse_indices :2239 */
        const uint16_t* cmn = mn + (size_t)c * D;
        const uint16_t* cmx = mx + (size_t)c * D;
        const int32_t* kc = kcodes + (size_t)c * NP * C;
        const int32_t* vc = vcodes + (size_t)c * D * 2;
        const uint16_t* vm = vmeta + (size_t)c * 2 * NG * C;
        for (t = 0; t < C; ++t, ++row) {
            for (d = 0; d < D; ++d) {
                uint32_t kw = (uint32_t)kc[(d / 8) * C + t];
                int kcode = (int)((kw >> (4 * (d % 8))) & 15u);
                K[(size_t)row * D + d] = orc_bf2f(orc_dequant(kcode, orc_kivi_scale(cmn[d], cmx[d]), cmn[d]));
                uint32_t vw = (uint32_t)vc[d * 2 + (t >> 3)];
                int vcode = (int)((vw >> (4 * (t & 7))) & 15u);
                uint16_t vs = vm[(0 * NG + d / 32) * C + t];
                uint16_t vz = vm[(1 * NG + d / 32) * C + t];
                V[(size_t)row * D + d] = orc_bf2f(orc_dequant(vcode, vs, vz));
            }
        }
    }
    for (t = 0; t < n_near; ++t, ++row)
        for (d = 0; d < D; ++d) {
            K[(size_t)row * D + d] = orc_bf2f(nearK[(size_t)t * D + d]);
            V[(size_t)row * D + d] = orc_bf2f(nearV[(size_t)t * D + d]);
        }
    float qf[8 * 128];
    float of[8 * 128];
    for (i = 0; i < G * D; ++i) qf[i] = orc_bf2f(q[i]);
    orc_attn_dense(qf, K, V, n, G, D, scale, of, lse);
    for (i = 0; i < G * D; ++i) out[i] = orc_f2bf(of[i]);
    free(scores);
    free(chosen);
    free(K);
    free(V);
}

typedef struct {
    const uint16_t *q, *mn, *mx;
    const uint8_t* valid;
    const int32_t *kcodes, *vcodes;
    const uint16_t *vmeta, *nearK, *nearV;
    int rows, G, n_max, n_c, nk, near_ld, n_near, tid, nthreads;
    float scale;
    uint16_t* out;
    float* lse;
    int64_t* sel;
} page_job_t;

static void* page_worker(void* arg) {
    const page_job_t* j = (const page_job_t*)arg;
    const int D = 128;
    int r;
    for (r = j->tid; r < j->rows; r += j->nthreads)
        page_row(j->q + (size_t)r * j->G * D, j->mn + (size_t)r * j->n_max * D,
                 j->mx + (size_t)r * j->n_max * D,
                 j->valid ? j->valid + (size_t)r * j->n_max : NULL,
                 j->kcodes + (size_t)r * j->n_max * D / 8 * 16,
                 j->vcodes + (size_t)r * j->n_max * D * 2,
                 j->vmeta + (size_t)r * j->n_max * 2 * (D / 32) * 16,
                 j->nearK + (size_t)r * j->near_ld * D, j->nearV + (size_t)r * j->near_ld * D,
                 j->G, j->n_max, j->n_c, j->nk, j->n_near, j->scale,
                 j->out + (size_t)r * j->G * D, j->lse + (size_t)r * j->G,
                 j->sel ? j->sel + (size_t)r * j->nk : NULL);
    return NULL;
}

void orc_page_decode(const uint16_t* q, const uint16_t* mn, const uint16_t* mx,
                     const uint8_t* valid, const int32_t* kcodes,
                     const int32_t* vcodes, const uint16_t* vmeta,
                     const uint16_t* nearK, const uint16_t* nearV,
                     int rows, int G, int n_max, int n_c, int nk,
                     int near_ld, int n_near, float scale, uint16_t* out,
                     float* lse, int64_t* sel, int threads) {
    page_job_t jobs[256];
    pthread_t tids[256];
    int t;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > rows) threads = rows > 0 ? rows : 1;
    for (t = 0; t < threads; ++t) {
        page_job_t j = {q, mn, mx, valid, kcodes, vcodes, vmeta, nearK, nearV,
                        rows, G, n_max, n_c, nk, near_ld, n_near, t, threads,
                        scale, out, lse, sel};
        jobs[t] = j;
    }
    for (t = 1; t < threads; ++t) pthread_create(&tids[t], NULL, page_worker, &jobs[t]);
    page_worker(&jobs[0]);
    for (t = 1; t < threads; ++t) pthread_join(tids[t], NULL);
}

/* ---------------- page mode over raw rows ---------------- */
static void raw_row(const uint16_t* q, const uint16_t* mn, const uint16_t* mx,
                    const uint8_t* valid, const uint16_t* keys, const uint16_t* values,
                    int64_t page_base, int G, int n_max, int n_c, int nk, int n_sink,
                    int near_start, int n_near, float scale, uint16_t* out, float* lse,
                    int64_t* sel) {
    const int D = 128, C = 16;
    uint16_t raw_q[128];
    int d, g, i, t;
    for (d = 0; d < D; ++d) {
        float acc = 0.0f;
        for (g = 0; g < G; ++g) acc += orc_bf2f(q[g * D + d]);
        raw_q[d] = orc_f2bf(acc / (float)G);
    }
    const int nsel = n_c > 0 ? nk : 0;
    int64_t* chosen = (int64_t*)malloc(sizeof(int64_t) * (size_t)(nsel > 0 ? nsel : 1));
    if (nsel > 0 && nsel < n_c) {
        float* scores = (float*)malloc(sizeof(float) * (size_t)n_c);
        orc_quest_score(raw_q, mn, mx, valid, scores, 1, n_c, n_max);
        orc_topk_f32(scores, 1, n_c, n_c, nsel, chosen);
        free(scores);
    } else {
        for (i = 0; i < nsel; ++i) chosen[i] = i;
    }
    if (sel) memcpy(sel, chosen, sizeof(int64_t) * (size_t)nsel);
    const int n = nsel * C + n_sink + n_near;
    float* K = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * D);
    float* V = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * D);
    int row = 0;
    for (t = 0; t < n_sink; ++t, ++row)
        for (d = 0; d < D; ++d) {
            K[(size_t)row * D + d] = orc_bf2f(keys[(size_t)t * D + d]);
            V[(size_t)row * D + d] = orc_bf2f(values[(size_t)t * D + d]);
        }
    for (i = 0; i < nsel; ++i)
        for (t = 0; t < C; ++t, ++row) {
            const size_t tok = (size_t)(page_base + chosen[i] * C + t);
            for (d = 0; d < D; ++d) {
                K[(size_t)row * D + d] = orc_bf2f(keys[tok * D + d]);
                V[(size_t)row * D + d] = orc_bf2f(values[tok * D + d]);
            }
        }
    for (t = 0; t < n_near; ++t, ++row)
        for (d = 0; d < D; ++d) {
            const size_t tok = (size_t)(near_start + t);
            K[(size_t)row * D + d] = orc_bf2f(keys[tok * D + d]);
            V[(size_t)row * D + d] = orc_bf2f(values[tok * D + d]);
        }
    float qf[8 * 128];
    float of[8 * 128];
    for (i = 0; i < G * D; ++i) qf[i] = orc_bf2f(q[i]);
    orc_attn_dense(qf, K, V, n, G, D, scale, of, lse);
    for (i = 0; i < G * D; ++i) out[i] = orc_f2bf(of[i]);
    free(chosen);
    free(K);
    free(V);
}

typedef struct {
    const uint16_t *q, *mn, *mx;
    const uint8_t* valid;
    const uint16_t *keys, *values;
    int64_t cap, page_base;
    int rows, G, n_max, n_c, nk, n_sink, near_start, n_near, tid, nthreads;
    float scale;
    uint16_t* out;
    float* lse;
    int64_t* sel;
} raw_job_t;

static void* raw_worker(void* arg) {
    const raw_job_t* j = (const raw_job_t*)arg;
    const int D = 128;
    const int nsel = j->n_c > 0 ? j->nk : 0;
    int r;
    for (r = j->tid; r < j->rows; r += j->nthreads)
        raw_row(j->q + (size_t)r * j->G * D, j->mn + (size_t)r * j->n_max * D, j->mx + (size_t)r * j->n_max * D,
                j->valid ? j->valid + (size_t)r * j->n_max : NULL, j->keys + (size_t)r * j->cap * D,
                j->values + (size_t)r * j->cap * D, j->page_base, j->G, j->n_max, j->n_c, j->nk, j->n_sink,
                j->near_start, j->n_near, j->scale, j->out + (size_t)r * j->G * D, j->lse + (size_t)r * j->G,
                j->sel ? j->sel + (size_t)r * nsel : NULL);
    return NULL;
}

void orc_page_decode_raw(const uint16_t* q, const uint16_t* mn, const uint16_t* mx,
                         const uint8_t* valid, const uint16_t* keys,
                         const uint16_t* values, int64_t cap, int64_t page_base,
                         int rows, int G, int n_max, int n_c, int nk, int n_sink,
                         int near_start, int n_near, float scale, uint16_t* out,
                         float* lse, int64_t* sel, int threads) {
    raw_job_t jobs[256];
    pthread_t tids[256];
    int t;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > rows) threads = rows > 0 ? rows : 1;
    for (t = 0; t < threads; ++t) {
        raw_job_t j = {q, mn, mx, valid, keys, values, cap, page_base, rows, G, n_max, n_c, nk,
                       n_sink, near_start, n_near, t, threads, scale, out, lse, sel};
        jobs[t] = j;
    }
    for (t = 1; t < threads; ++t) pthread_create(&tids[t], NULL, raw_worker, &jobs[t]);
    raw_worker(&jobs[0]);
    for (t = 1; t < threads; ++t) pthread_join(tids[t], NULL);
}

/* ---------------- LSE merge ---------------- */
void orc_lse_merge(const float* a, const float* la, const float* b,
                   const float* lb, float* out, float* lse_out, int rows,
                   int dim) {
    int r, d;
    for (r = 0; r < rows; ++r) {
        float m = fmaxf(la[r], lb[r]);
        float wa = expf(la[r] - m), wb = expf(lb[r] - m);
        float den = wa + wb;
        for (d = 0; d < dim; ++d)
            out[(size_t)r * dim + d] = (wa * a[(size_t)r * dim + d] + wb * b[(size_t)r * dim + d]) / den;
        if (lse_out) lse_out[r] = m + logf(den);
    }
}

/* Batch helpers (rows of contiguous tokens). */
void orc_kivi_encode_rows(const uint16_t* keys, int rows, int T, int D, int chunk,
                          uint16_t* mn, uint16_t* mx, uint16_t* centroid, int32_t* packed) {
    int r, c, nc = T / chunk;
    for (r = 0; r < rows; ++r)
        for (c = 0; c < nc; ++c) {
            size_t o = (size_t)r * nc + c;
            orc_kivi_encode_chunk(keys + ((size_t)r * T + (size_t)c * chunk) * D, D, D, chunk, mn + o * D,
                                  mx + o * D, centroid + o * D, packed + o * (D / 8) * chunk);
        }
}

void orc_vquant_rows(const uint16_t* v, int64_t n_tokens, int D, int group, int32_t* codes, uint16_t* meta) {
    int64_t i;
    for (i = 0; i < n_tokens; ++i)
        orc_vquant_token(v + i * D, D, group, codes + i * (D / 8), meta + i * (D / group) * 2);
}
