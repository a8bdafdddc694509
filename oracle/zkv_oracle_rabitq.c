/*
 * zkv_oracle_rabitq.c -- CPU restatement of the ParisKV / RaBitQ retrieval
 * path (polar-ANN collision counting, 4-bit RaBitQ rerank, popcount scores).
 * TEST INFRASTRUCTURE ONLY (see zkv_oracle.h).
 *
 * Layouts are token-major ("[rows][cap][...]"), the layout of this build's
 * cache; tests transpose the reference's block-major tensors
 * ([bs, H, B, len(, m/2)]) into it before calling.
 *
 * Reduction orders (fp32) are fixed and mirrored by the CUDA kernels:
 *   128-dim sums: per 4-dim lane ((d0+d1)+(d2+d3)), then a halving tree over
 *   the 32 lanes (lane i + lane i+16, ...);  8-dim block sums:
 *   ((d0+d1)+(d2+d3)) + ((d4+d5)+(d6+d7)).  torch's bf16-rounded results
 *   agree with these orders on the reference fixtures.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "zkv_oracle.h"

#define RQ_D 128
#define RQ_B 16
#define RQ_M 8
#define RQ_K 256

static inline float bf(uint16_t b) { return orc_bf2f(b); }
static inline uint16_t rb(float f) { return orc_f2bf(f); }

/* 128-dim fp32 sum in the lane-tree order. */
static float sum128(const float* v) {
    float lane[32];
    for (int l = 0; l < 32; ++l) lane[l] = (v[4 * l] + v[4 * l + 1]) + (v[4 * l + 2] + v[4 * l + 3]);
    for (int h = 16; h >= 1; h >>= 1)
        for (int l = 0; l < h; ++l) lane[l] = lane[l] + lane[l + h];
    return lane[0];
}

static float sum8(const float* v) { return ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7])); }

/* Magnitude decision thresholds and reconstruction centres as bf16
 * (cache_hub/polar_cache.py:267-270). */
static const float kThr[7] = {0.0843f, 0.1698f, 0.2578f, 0.3499f, 0.4487f, 0.5585f, 0.6901f};
static const float kCen[8] = {0.0420f, 0.1266f, 0.2130f, 0.3025f, 0.3973f, 0.5001f, 0.6169f, 0.7633f};

void orc_rq_mag_tables(uint16_t* thr7, uint16_t* cen8) {
    for (int i = 0; i < 7; ++i) thr7[i] = rb(kThr[i]);
    for (int i = 0; i < 8; ++i) cen8[i] = rb(kCen[i]);
}

/* Normalise, sign-flip and Walsh-Hadamard-rotate one 128-dim bf16 vector:
 *   n = bf16(||x||) clamped to bf16(1e-8); y = bf16(x / n) * s;
 *   FWHT in fp32 with the butterfly order of hadamard_fallback.py:10-24
 *   (strides 1, 2, ..., 64; (a+b, a-b)); times fp32(1/sqrt(128)); bf16.
 * ParisKV batch_encode steps 1-2 (cache_hub/polar_cache.py:1143-1151) and
 * _encode_query_blocks (:1108-1127). Returns n (bf16). */
static uint16_t rotate128(const uint16_t* x, const uint16_t* signs, uint16_t* out) {
    float v[RQ_D], sq[RQ_D];
    for (int d = 0; d < RQ_D; ++d) {
        v[d] = bf(x[d]);
        sq[d] = v[d] * v[d];
    }
    uint16_t n = rb(sqrtf(sum128(sq)));
    float nf = bf(n);
    const float eps = bf(rb(1e-8f));
    if (nf < eps) nf = eps;
    for (int d = 0; d < RQ_D; ++d) v[d] = bf(rb(v[d] / nf)) * bf(signs[d]);
    for (int h = 1; h < RQ_D; h <<= 1)
        for (int base = 0; base < RQ_D; base += 2 * h)
            for (int i = base; i < base + h; ++i) {
                const float a = v[i], b = v[i + h];
                v[i] = a + b;
                v[i + h] = a - b;
            }
    const float scale = (float)(1.0 / sqrt((double)RQ_D));
    for (int d = 0; d < RQ_D; ++d) out[d] = rb(v[d] * scale);
    return n;
}

/* ParisKV batch_encode (cache_hub/polar_cache.py:1130-1198) for one key:
 *   codes[b]   = bitpack(y_b >= 0), bit j = dim 8b+j          (:1157-1160)
 *   r_b        = bf16(||y_b||); u = bf16(y_b / max(r_b, 1e-8)) (:1170-1174)
 *   t_j        = bucketize(|u_j|, thr) = #{thr < |u_j|}        (:1179)
 *   alpha_b    = max(sum_j fp32(bf16(cen[t_j] * |u_j|)), 1e-6) (:1183-1191)
 *   weight_b   = bf16(fp32(r_b / alpha_b) * n)                  (:1193-1194)
 *   packed     = byte i of block b = (v_{2i+1} << 4) | v_{2i}, v = sign<<3|t
 *                (_pack_4bit_codes :1067-1083)
 * plus this build's popcount-estimator factor (RaBitQ, Gao & Long 2024):
 *   factor = n / max(<xbar, o'>, 1e-6), <xbar, o'> = (sum_j |y_j|) / sqrt(128). */
void orc_rq_encode_key(const uint16_t* key, const uint16_t* signs, uint8_t* codes, uint8_t* packed,
                       uint16_t* weight, float* factor) {
    uint16_t y[RQ_D];
    const uint16_t n = rotate128(key, signs, y);
    float yf[RQ_D], ay[RQ_D];
    for (int d = 0; d < RQ_D; ++d) {
        yf[d] = bf(y[d]);
        ay[d] = fabsf(yf[d]);
    }
    const float eps8 = bf(rb(1e-8f));
    for (int b = 0; b < RQ_B; ++b) {
        const float* yb = yf + RQ_M * b;
        uint8_t c = 0;
        float sq[RQ_M];
        for (int j = 0; j < RQ_M; ++j) {
            if (yb[j] >= 0.0f) c |= (uint8_t)(1u << j);
            sq[j] = yb[j] * yb[j];
        }
        codes[b] = c;
        const uint16_t r = rb(sqrtf(sum8(sq)));
        float rf = bf(r);
        if (rf < eps8) rf = eps8;
        float prod[RQ_M];
        uint8_t v4[RQ_M];
        for (int j = 0; j < RQ_M; ++j) {
            const float u = fabsf(bf(rb(yb[j] / rf)));
            int t = 0;
            while (t < 7 && bf(rb(kThr[t])) < u) ++t;
            prod[j] = bf(rb(bf(rb(kCen[t])) * u));
            v4[j] = (uint8_t)((((c >> j) & 1u) << 3) | (unsigned)t);
        }
        float alpha = sum8(prod);
        if (alpha < 1e-6f) alpha = 1e-6f;
        weight[b] = rb((bf(r) / alpha) * bf(n));
        for (int i = 0; i < RQ_M / 2; ++i) packed[4 * b + i] = (uint8_t)((v4[2 * i + 1] << 4) | v4[2 * i]);
    }
    float ip = sum128(ay) * (float)(1.0 / sqrt((double)RQ_D));
    if (ip < 1e-6f) ip = 1e-6f;
    *factor = bf(n) / ip;
}

/* Encode tokens [tok_start, tok_start + n_tok) of every row and add them to
 * the per-(row, block) bucket histogram hist[rows][16][256]
 * (_count_cluster_keys, cache_hub/polar_cache.py:1203-1226). */
void orc_rq_encode_rows(const uint16_t* keys, int64_t ld_row, int rows, int n_tok, int tok_start, int64_t cap,
                        const uint16_t* signs, uint8_t* codes, uint8_t* packed, uint16_t* weight, float* factor,
                        int32_t* hist) {
    for (int r = 0; r < rows; ++r)
        for (int t = 0; t < n_tok; ++t) {
            const int64_t k = tok_start + t;
            const int64_t o = (int64_t)r * cap + k;
            orc_rq_encode_key(keys + (int64_t)r * ld_row + (int64_t)t * RQ_D, signs, codes + o * RQ_B,
                              packed + o * 64, weight + o * RQ_B, factor + o);
            if (hist)
                for (int b = 0; b < RQ_B; ++b) hist[((int64_t)r * RQ_B + b) * RQ_K + codes[o * RQ_B + b]] += 1;
        }
}

/* Query side: GQA mean over G heads (fp32 sum in head order, / G, bf16;
 * polar_cache.compute :1262-1265), then rotate128.  q [rows][G][128];
 * q_blocks [rows][128] (= [rows][16][8]); q_norm [rows]. */
void orc_rq_query(const uint16_t* q, int rows, int G, const uint16_t* signs, uint16_t* q_blocks, uint16_t* q_norm,
                  uint16_t* q_mean) {
    for (int r = 0; r < rows; ++r) {
        uint16_t m[RQ_D];
        for (int d = 0; d < RQ_D; ++d) {
            float s = 0.0f;
            for (int g = 0; g < G; ++g) s += bf(q[((int64_t)r * G + g) * RQ_D + d]);
            m[d] = rb(s / (float)G);
        }
        if (q_mean) memcpy(q_mean + (int64_t)r * RQ_D, m, sizeof(m));
        q_norm[r] = rotate128(m, signs, q_blocks + (int64_t)r * RQ_D);
    }
}

/* Bucket score of cluster c in block b: q_b . V[c] with V[c]_j = +1 if bit j
 * of c else -1 (the codebook file codebook_d128_m8_Kr1_Kw256_rabitq_sign.json
 * holds exactly these 256 LSB-first sign patterns), fp32 in dim order,
 * rounded to bf16 (torch.matmul of bf16 operands, polar_cache.py:1704). */
static float bucket_score(const uint16_t* qb, int c) {
    float s = 0.0f;
    for (int j = 0; j < RQ_M; ++j) s += ((c >> j) & 1) ? bf(qb[j]) : -bf(qb[j]);
    return bf(rb(s));
}

/* Per-(row, block) hit weight of every bucket (get_cache_cnt_fused,
 * polar_cache.py:1688-1728 + collision.cu convert_to_bits :72-153):
 * buckets sorted by score descending (ties: lower bucket id first -- the
 * reference's argsort leaves ties unspecified), before[r] = exclusive prefix
 * of hist over that order, weight = #{t : before[rank] < target[t]}. */
void orc_collision_weights(const uint16_t* q_blocks, const int32_t* hist, int rows, const int64_t* targets,
                           int n_tiers, uint8_t* table) {
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < RQ_B; ++b) {
            const uint16_t* qb = q_blocks + (int64_t)r * RQ_D + RQ_M * b;
            float sc[RQ_K];
            int order[RQ_K];
            for (int c = 0; c < RQ_K; ++c) {
                sc[c] = bucket_score(qb, c);
                order[c] = c;
            }
            /* stable insertion sort, descending */
            for (int i = 1; i < RQ_K; ++i) {
                const int x = order[i];
                int j = i - 1;
                while (j >= 0 && sc[order[j]] < sc[x]) {
                    order[j + 1] = order[j];
                    --j;
                }
                order[j + 1] = x;
            }
            const int32_t* h = hist + ((int64_t)r * RQ_B + b) * RQ_K;
            uint8_t* w = table + ((int64_t)r * RQ_B + b) * RQ_K;
            int64_t before = 0;
            for (int p = 0; p < RQ_K; ++p) {
                const int c = order[p];
                int hit = 0;
                for (int t = 0; t < n_tiers; ++t) hit += before < targets[t];
                w[c] = (uint8_t)hit;
                before += h[c];
            }
        }
}

/* cnt[r][k] = sum_b table[r][b][codes[r][k][b]]  (update_cache_cnt_kernel,
 * collision.cu:161-245). codes token-major [rows][cap][16]. */
void orc_collision_count(const uint8_t* table, const uint8_t* codes, int64_t cap, int rows, int kv_len, int32_t* cnt) {
    for (int r = 0; r < rows; ++r)
        for (int k = 0; k < kv_len; ++k) {
            int s = 0;
            for (int b = 0; b < RQ_B; ++b)
                s += table[((int64_t)r * RQ_B + b) * RQ_K + codes[((int64_t)r * cap + k) * RQ_B + b]];
            cnt[(int64_t)r * kv_len + k] = s;
        }
}

/* update_cache_cnt_overall_ref (collision_fused/collision_test.py:89-121)
 * with the reference's own sorted bucket ids, block-major codes
 * [rows][B][kv_len] (u8 or int32 given as int32), any bucket count K. */
void orc_update_cache_cnt_sorted(const int64_t* sorted_ids, const int32_t* hist, const int32_t* codes, int rows,
                                 int B, int K, int kv_len, const int64_t* targets, int n_tiers, int32_t* cnt) {
    uint8_t* w = (uint8_t*)malloc((size_t)K);
    memset(cnt, 0, sizeof(int32_t) * (size_t)rows * (size_t)kv_len);
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < B; ++b) {
            const int64_t* ids = sorted_ids + ((int64_t)r * B + b) * K;
            const int32_t* h = hist + ((int64_t)r * B + b) * K;
            int64_t before = 0;
            for (int p = 0; p < K; ++p) {
                int hit = 0;
                for (int t = 0; t < n_tiers; ++t) hit += before < targets[t];
                w[ids[p]] = (uint8_t)hit;
                before += h[ids[p]];
            }
            const int32_t* cb = codes + ((int64_t)r * B + b) * kv_len;
            for (int k = 0; k < kv_len; ++k) cnt[(int64_t)r * kv_len + k] += w[cb[k]];
        }
    free(w);
}

/* 4-bit RaBitQ rerank score of candidate key idx as the production kernel
 * computes it (rerank.cu:52-143): sequential bf16 fused multiply-adds
 *   dot_b = fma(v7, q7, ... fma(v1, q1, fma(v0, q0, 0)))   one rounding each
 *   res   = fma(dot_b, w_b, res)                          one rounding
 *   score = res * |q|                                     rounded
 * v_j = +-cen[t_j] (sign bit 3 of the nibble; even dim in the low nibble).
 * The source writes `temp += k * q` and `res += temp * w` on bf16 values;
 * the kernel the reference builds fuses each into one rounding (measured bit
 * for bit on a B200: tests/golden/ref_cuda.npz), whereas the Python check
 * (test_rerank_topk.py python_rabitq_scores:60-111) rounds the product and
 * the sum separately. */
void orc_rerank4(const int64_t* cand, int C, const uint8_t* packed, const uint16_t* weight, int64_t cap,
                 const uint16_t* q_blocks, const uint16_t* q_norm, const uint16_t* cen8, int rows,
                 uint16_t* scores) {
    for (int r = 0; r < rows; ++r)
        for (int i = 0; i < C; ++i) {
            const int64_t k = cand[(int64_t)r * C + i];
            const uint8_t* p = packed + ((int64_t)r * cap + k) * 64;
            const uint16_t* w = weight + ((int64_t)r * cap + k) * RQ_B;
            uint16_t res = 0;
            for (int b = 0; b < RQ_B; ++b) {
                uint16_t dot = 0;
                for (int j = 0; j < RQ_M; ++j) {
                    const unsigned nib = (p[4 * b + j / 2] >> (4 * (j & 1))) & 0xFu;
                    uint16_t v = cen8[nib & 7u];
                    if (!(nib & 8u)) v ^= 0x8000u;
                    dot = orc_bfma(v, q_blocks[(int64_t)r * RQ_D + RQ_M * b + j], dot);
                }
                res = orc_bfma(dot, w[b], res);
            }
            scores[(int64_t)r * C + i] = rb(bf(res) * bf(q_norm[r]));
        }
}

/* coarse_2bit_score (rerank/coarse_2bit_score.cu:86-156) by brute force over
 * dims: v_q . v_k = (1 - 2 xs)(1 + m_q + m_k + m_q m_k) summed over the 128
 * dims, xs = q_sign ^ k_sign, m = magnitude-high bit (bit 2 of the nibble),
 * k_sign = bit 3.  q_signs/q_mags [rows][16] bytes, bit j = dim 8b+j. */
void orc_coarse2bit(const uint8_t* packed, int64_t cap, const uint8_t* q_signs, const uint8_t* q_mags, int rows,
                    int kv_len, int32_t* out) {
    for (int r = 0; r < rows; ++r)
        for (int k = 0; k < kv_len; ++k) {
            const uint8_t* p = packed + ((int64_t)r * cap + k) * 64;
            int s = 0;
            for (int b = 0; b < RQ_B; ++b)
                for (int j = 0; j < RQ_M; ++j) {
                    const unsigned nib = (p[4 * b + j / 2] >> (4 * (j & 1))) & 0xFu;
                    const int ks = (nib >> 3) & 1, km = (nib >> 2) & 1;
                    const int qs = (q_signs[r * RQ_B + b] >> j) & 1, qm = (q_mags[r * RQ_B + b] >> j) & 1;
                    const int xs = qs ^ ks;
                    s += (1 - 2 * xs) * (1 + qm + km + qm * km);
                }
            out[(int64_t)r * kv_len + k] = s;
        }
}

/* 4-bit scalar quantisation of the rotated query for the popcount estimator
 * (RaBitQ, Gao & Long, SIGMOD 2024, sec. 3.3, deterministic rounding):
 *   lo = min q_j, delta = (max q_j - lo) / 15 (1 if 0),
 *   qbar_j = clamp(rint((q_j - lo) / delta), 0, 15).
 * planes [rows][4][16]: byte b of plane p has bit j = bit p of qbar_{8b+j}.
 * qparams [rows][4] = {lo, delta, sum qbar, |q|}. */
void orc_rq_query_4bit(const uint16_t* q_blocks, const uint16_t* q_norm, int rows, uint8_t* planes, float* qparams) {
    for (int r = 0; r < rows; ++r) {
        const uint16_t* qb = q_blocks + (int64_t)r * RQ_D;
        float lo = bf(qb[0]), hi = bf(qb[0]);
        for (int d = 1; d < RQ_D; ++d) {
            const float v = bf(qb[d]);
            lo = v < lo ? v : lo;
            hi = v > hi ? v : hi;
        }
        float delta = (hi - lo) / 15.0f;
        if (!(delta > 0.0f)) delta = 1.0f;
        uint8_t* pl = planes + (int64_t)r * 64;
        memset(pl, 0, 64);
        int sum = 0;
        for (int d = 0; d < RQ_D; ++d) {
            int qb4 = (int)rintf((bf(qb[d]) - lo) / delta);
            qb4 = qb4 < 0 ? 0 : (qb4 > 15 ? 15 : qb4);
            sum += qb4;
            for (int p = 0; p < 4; ++p)
                if ((qb4 >> p) & 1) pl[p * RQ_B + d / RQ_M] |= (uint8_t)(1u << (d % RQ_M));
        }
        qparams[4 * r + 0] = lo;
        qparams[4 * r + 1] = delta;
        qparams[4 * r + 2] = (float)sum;
        qparams[4 * r + 3] = bf(q_norm[r]);
    }
}

/* Popcount estimate of <k, q> for candidate keys from their 1-bit codes:
 *   I = sum_p 2^p popc(x & plane_p), P = popc(x)            (integers)
 *   <xbar, q'> ~ (2 delta I + 2 lo P - delta S - D lo) / sqrt(D)
 *   est = (<xbar, q'> * factor_k) * |q|
 * fp32, in exactly this operation order (the kernel uses _rn intrinsics). */
void orc_popcount_est(const int64_t* cand, int C, const uint8_t* codes, const float* factor, int64_t cap,
                      const uint8_t* planes, const float* qparams, int rows, float* est, int32_t* ints) {
    const float inv_sqrt_d = (float)(1.0 / sqrt((double)RQ_D));
    for (int r = 0; r < rows; ++r) {
        const uint8_t* pl = planes + (int64_t)r * 64;
        const float lo = qparams[4 * r], delta = qparams[4 * r + 1], S = qparams[4 * r + 2], qn = qparams[4 * r + 3];
        const float c0 = delta * S + (float)RQ_D * lo;
        for (int i = 0; i < C; ++i) {
            const int64_t k = cand ? cand[(int64_t)r * C + i] : i;
            const uint8_t* x = codes + ((int64_t)r * cap + k) * RQ_B;
            int I = 0, P = 0;
            for (int b = 0; b < RQ_B; ++b) {
                P += __builtin_popcount(x[b]);
                for (int p = 0; p < 4; ++p) I += __builtin_popcount(x[b] & pl[p * RQ_B + b]) << p;
            }
            if (ints) {
                ints[2 * ((int64_t)r * C + i)] = I;
                ints[2 * ((int64_t)r * C + i) + 1] = P;
            }
            const float num = ((2.0f * delta) * (float)I + (2.0f * lo) * (float)P) - c0;
            est[(int64_t)r * C + i] = ((num * inv_sqrt_d) * factor[(int64_t)r * cap + k]) * qn;
        }
    }
}

/* Exact inner products of candidate raw keys with the (GQA-mean) query:
 * fp32 products of bf16 operands summed in the 128-dim lane-tree order. */
void orc_exact_ip(const int64_t* idx, int n, const uint16_t* keys, int64_t ld_row, const uint16_t* q, int rows,
                  float* out) {
    for (int r = 0; r < rows; ++r)
        for (int i = 0; i < n; ++i) {
            const uint16_t* k = keys + (int64_t)r * ld_row + idx[(int64_t)r * n + i] * RQ_D;
            float p[RQ_D];
            for (int d = 0; d < RQ_D; ++d) p[d] = bf(k[d]) * bf(q[(int64_t)r * RQ_D + d]);
            out[(int64_t)r * n + i] = sum128(p);
        }
}
