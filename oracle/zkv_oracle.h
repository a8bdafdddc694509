/*
 * zkv_oracle.h -- CPU restatement of the ZoomKV sparse decode-attention hot
 * path.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and the
 * CPU-baseline leg of bench.py call this library as the checker.  The product
 * (zoomkv_revision_b200) never links or calls it.
 *
 * Every routine restates one reference function; the file:line it follows is
 * given beside each declaration (paths relative to the ZoomKV runtime root
 * runtime/zoomkv_urania_runtime_20261011/).  Where the reference's PyTorch
 * and CUDA semantics differ, the CUDA-kernel arithmetic (what production ran)
 * is restated and the difference is noted.
 *
 * bf16 values travel as uint16_t bit patterns.  Rows are (batch, kv_head)
 * pairs flattened to one index; all arrays are dense row-major unless a
 * stride argument says otherwise.
 */
#ifndef ZKV_ORACLE_H
#define ZKV_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float orc_bf2f(uint16_t b);
uint16_t orc_f2bf(float f);

/* Per-chunk raw-key metadata + KIVI 4-bit pack for ONE full chunk of
 * `chunk` tokens (a1 + a2).
 *   _compute_and_store_chunk_minmax  cache_hub/polar_cache_quest_density_single_layer_kivi.py:2119-2130
 *   _kivi_pack_chunks                same file :1965-2020
 *   _pack_along_last_dim             cache_hub/kivi/quant_pack.py:124-141
 * keys: chunk rows of D bf16, row stride `ld` elements.
 * packed: chunk-major [D/8][chunk] int32 (A-1 layout).                   */
void orc_kivi_encode_chunk(const uint16_t* keys, int64_t ld, int D, int chunk,
                           uint16_t* mn, uint16_t* mx, uint16_t* centroid,
                           int32_t* packed);

/* Per-token value quantisation (a16; no counterpart in the reference, whose
 * values stay bf16): groups of `group` dims, scale=(max-min)/15, zero=min,
 * same bf16 arithmetic ladder as the KIVI keys.
 * codes: [D/8] int32 (nibble j of word w = dim 8w+j); meta: [D/group][2]
 * (scale, zero) bf16.                                                     */
void orc_vquant_token(const uint16_t* v, int D, int group,
                      int32_t* codes, uint16_t* meta);

/* bf16 fused multiply-add a*b + c, one rounding (see zkv_oracle.c).      */
uint16_t orc_bfma(uint16_t a, uint16_t b, uint16_t c);
/* KIVI dequant of the production stage-2 kernel: bf16(code*scale + mn),
 * one rounding (kivi_qk_dot.cu:264-275 as built).                         */
uint16_t orc_dequant_fused(int code, uint16_t scale, uint16_t zero);
/* bf16 dequant ladder bf16(bf16(code*scale) + zero); kivi_qk_dot.cu:264-280 */
uint16_t orc_dequant(int code, uint16_t scale, uint16_t zero);
/* KIVI key scale bf16(bf16(mx-mn)/15); kivi_qk_dot.cu:213-217 */
uint16_t orc_kivi_scale(uint16_t mn, uint16_t mx);

/* Quest upper-bound score; quest/quest_chunk_score.cu:31-103 (fp32 products
 * of bf16 inputs, 4-dim per-thread partials, xor-tree over 32 lanes).
 * q [rows][128]; mn/mx [rows][n_max][128]; valid [rows][n_max] or NULL;
 * scores [rows][n_chunks] (-inf where !valid).                           */
void orc_quest_score(const uint16_t* q, const uint16_t* mn, const uint16_t* mx,
                     const uint8_t* valid, float* scores, int rows,
                     int n_chunks, int n_max);

/* Deterministic top-k over fp32 rows (float_topk_3d,
 * topk/float_topk.cu:51-271): the k largest by the order-preserving u32 key,
 * ties broken by lowest index, written in ascending index order.
 * len <= k: out[i] = i < len ? i : -1 (naive path, float_topk.cu:35-40). */
void orc_topk_f32(const float* scores, int rows, int len, int64_t row_stride,
                  int k, int64_t* out);

/* Hierarchical Quest (cache_hub/polar_cache_kivi_quest_density_seperate_
 * kernel.py; off in the single-layer KIVI cache, on by default in the
 * separate-kernel one, :210-237).
 * orc_large_minmax: _update_large_chunk_minmax (:1762-1798) over every
 * group: group g covers chunks [g*factor, min(g*factor + factor, valid_end));
 * its min/max are the element-wise bf16 min/max of those chunks' min/max
 * and it is valid when non-empty (empty groups: zero bits, invalid).
 * mn/mx [rows][n_max][128]; lmn/lmx [rows][n_max_large][128];
 * lvalid [rows][n_max_large].                                             */
void orc_large_minmax(const uint16_t* mn, const uint16_t* mx, int rows, int n_max, int valid_end, int factor,
                      int n_max_large, uint16_t* lmn, uint16_t* lmx, uint8_t* lvalid);
/* quest_sub_chunk_score (quest/quest_chunk_score.cu:263-360): for each of
 * the n_sel selected large chunks of a row, the Quest scores of its factor
 * small chunks, position j*factor + s; a chunk id outside [0, n_max) scores
 * -inf.  large_idx [rows][n_sel]; sub [rows][n_sel*factor].              */
void orc_sub_chunk_score(const uint16_t* q, const uint16_t* mn, const uint16_t* mx, const int64_t* large_idx,
                         int rows, int n_max, int n_sel, int factor, float* sub);
/* quest_map_back (quest/quest_chunk_score.cu:363-416): position p of the
 * sub-chunk top-k -> large_idx[p / factor] * factor + p % factor, clamped to
 * [0, n_chunks); p outside [0, nk_large*factor) -> -1.                    */
void orc_map_back(const int64_t* large_idx, const int64_t* sub_pos, int rows, int nk_large, int nk_small,
                  int factor, int n_chunks, int64_t* out);
/* _quest_pick_coarse_indices_hierarchical (:1852-1940) for one layer:
 * Quest over the n_chunks / factor large chunks (lvalid applied), their top
 * nk_large, the sub-chunk scores of the selected ones, their top nk_small,
 * mapped back to chunk ids.  Top-k as orc_topk_f32 (ties to the lowest
 * index, ascending).  large_idx_out [rows][nk_large] and sub_out
 * [rows][nk_large*factor] may be NULL.                                    */
void orc_hier_select(const uint16_t* q, const uint16_t* mn, const uint16_t* mx, int n_max, const uint16_t* lmn,
                     const uint16_t* lmx, const uint8_t* lvalid, int n_max_large, int rows, int n_chunks,
                     int factor, int nk_large, int nk_small, int64_t* out, int64_t* large_idx_out, float* sub_out);

/* Same selection over int32 rows (radix_topk_3d, topk/radix_topk.cu:157-240).*/
void orc_topk_i32(const int32_t* vals, int rows, int len, int64_t row_stride,
                  int k, int64_t* out);

/* CDS density centroid[chunk]·q; rerank/rerank_topk.cu:560-624 (fp32,
 * 128-thread shared-memory tree).  Invalid id -> -1e30.                   */
void orc_chunk_density(const int64_t* chunk_ids, const uint16_t* centroid,
                       const uint16_t* raw_q, float* out, int rows, int nk,
                       int n_chunks, int n_max);

/* mask_from_topk; rerank/rerank_topk.cu:926-954 */
void orc_mask_from_topk(const int64_t* positions, uint8_t* mask, int rows,
                        int n_dense, int nk);

/* KIVI stage-2 dense/sparse per-chunk top-k; kivi/kivi_qk_dot.cu:108-320.
 * packed [rows][n_pk][D/8][chunk]; mn/mx [rows][n_max][D];
 * out_scores/out_idx [rows][nk*chunk].  Per-chunk order: score desc, token
 * id asc (the reference's bitonic network leaves exact ties unordered).   */
void orc_kivi_qk(const int64_t* chunk_ids, const uint8_t* dense_mask,
                 const int32_t* packed, int n_pk, const uint16_t* mn,
                 const uint16_t* mx, int n_max, const uint16_t* raw_q,
                 int rows, int nk, int chunk, int dense_topk, int sparse_topk,
                 float* out_scores, int64_t* out_idx);

/* Fused global top-k + LUT gather + skipped-tail concat;
 * topk/float_topk_gather_concat.cu:65-300.  out row stride out_ld.       */
void orc_topk_gather_concat(const float* scores, const int64_t* lut,
                            const int64_t* skipped, int64_t* out, int rows,
                            int L, int k, int sk, int64_t out_ld);

/* GQA softmax attention of G query heads over n tokens (fp64 accumulation;
 * the flash_attn_with_kvcache call at
 * cache_hub/polar_cache_quest_density_single_layer_kivi.py:1763-1768).
 * q [G][D] fp32; K,V [n][D] fp32; out [G][D]; lse [G] natural log.       */
void orc_attn_dense(const float* q, const float* K, const float* V, int n,
                    int G, int D, float scale, float* out, float* lse);

/* Page-mode decode for rows (b, kv_head): Quest score -> top nk chunks ->
 * attention over [selected pages (KIVI K + 4-bit V) | near rows (bf16)].
 *   q     [rows][G][D] bf16          mn/mx [rows][n_max][D] bf16
 *   valid [rows][n_max] or NULL      kcodes [rows][n_max][D/8][16] i32
 *   vcodes [rows][n_max][D][2] i32 (dim d, word w = tokens 8w..8w+7)
 *   vmeta [rows][n_max][2][D/32][16] bf16 ([scale|zero][group][token])
 *   nearK/nearV [rows][near_ld][D]   out [rows][G][D] bf16, lse [rows][G]
 *   sel [rows][nk] selected chunk ids (ascending) or NULL.
 * threads > 1 parallelises over rows (pthreads).                            */
void orc_page_decode(const uint16_t* q, const uint16_t* mn, const uint16_t* mx,
                     const uint8_t* valid, const int32_t* kcodes,
                     const int32_t* vcodes, const uint16_t* vmeta,
                     const uint16_t* nearK, const uint16_t* nearV,
                     int rows, int G, int n_max, int n_c, int nk,
                     int near_ld, int n_near, float scale, uint16_t* out,
                     float* lse, int64_t* sel, int threads);

/* Page-mode decode over RAW bf16 rows, the reference's page mode
 * (polar_cache.compute with dense_topk = sparse_topk = 16 and final_topk =
 * budget: cache_hub/polar_cache_quest_density_single_layer_kivi.py:1589-1775;
 * the selected chunks' raw rows are gathered and attended with the sink and
 * near rows at :1734-1750).  Per row: GQA-mean query (:1622-1626) -> Quest
 * scores (quest_chunk_score.cu:75-98 order) -> top nk chunks (lowest index
 * on ties; nk == n_c keeps every chunk) -> fp64 softmax attention over the
 * 16 raw rows of each selected chunk (token page_base + 16 c + t), the sink
 * rows [0, n_sink) and the near rows [near_start, near_start + n_near).
 *   keys/values: row r, token t at base + (r*cap + t)*D (bf16)
 *   out [rows][G][D] bf16, lse [rows][G] natural log, sel [rows][nk] or NULL */
void orc_page_decode_raw(const uint16_t* q, const uint16_t* mn, const uint16_t* mx,
                         const uint8_t* valid, const uint16_t* keys,
                         const uint16_t* values, int64_t cap, int64_t page_base,
                         int rows, int G, int n_max, int n_c, int nk, int n_sink,
                         int near_start, int n_near, float scale, uint16_t* out,
                         float* lse, int64_t* sel, int threads);

/* Batch forms: keys [rows][T][D] (T % chunk == 0) -> mn/mx/centroid
 * [rows][T/chunk][D], packed [rows][T/chunk][D/8][chunk];
 * values [n_tokens][D] -> codes [n_tokens][D/8], meta [n_tokens][D/group][2]. */
void orc_kivi_encode_rows(const uint16_t* keys, int rows, int T, int D, int chunk,
                          uint16_t* mn, uint16_t* mx, uint16_t* centroid, int32_t* packed);
void orc_vquant_rows(const uint16_t* v, int64_t n_tokens, int D, int group,
                     int32_t* codes, uint16_t* meta);

/* Merge two attention partials by log-sum-exp;
 * lse_merge/lse_merge.py:79-119 (fp32).  a,b,out [rows][dim] fp32.      */
void orc_lse_merge(const float* a, const float* la, const float* b,
                   const float* lb, float* out, float* lse_out, int rows,
                   int dim);

/* ---- ParisKV / RaBitQ retrieval (zkv_oracle_rabitq.c); token-major layouts:
 * codes [rows][cap][16] u8, packed [rows][cap][16][4] u8, weight
 * [rows][cap][16] bf16, factor [rows][cap] f32, hist [rows][16][256] i32. */
void orc_rq_mag_tables(uint16_t* thr7, uint16_t* cen8);
/* batch_encode, cache_hub/polar_cache.py:1130-1198 (one key).            */
void orc_rq_encode_key(const uint16_t* key, const uint16_t* signs, uint8_t* codes, uint8_t* packed,
                       uint16_t* weight, float* factor);
void orc_rq_encode_rows(const uint16_t* keys, int64_t ld_row, int rows, int n_tok, int tok_start, int64_t cap,
                        const uint16_t* signs, uint8_t* codes, uint8_t* packed, uint16_t* weight, float* factor,
                        int32_t* hist);
/* GQA mean + _encode_query_blocks, cache_hub/polar_cache.py:1108-1127.    */
void orc_rq_query(const uint16_t* q, int rows, int G, const uint16_t* signs, uint16_t* q_blocks, uint16_t* q_norm,
                  uint16_t* q_mean);
/* get_cache_cnt_fused, cache_hub/polar_cache.py:1688-1728 (weights).     */
void orc_collision_weights(const uint16_t* q_blocks, const int32_t* hist, int rows, const int64_t* targets,
                           int n_tiers, uint8_t* table);
/* update_cache_cnt_kernel, collision_fused/collision.cu:161-245.         */
void orc_collision_count(const uint8_t* table, const uint8_t* codes, int64_t cap, int rows, int kv_len, int32_t* cnt);
/* update_cache_cnt_overall_ref, collision_fused/collision_test.py:89-121. */
void orc_update_cache_cnt_sorted(const int64_t* sorted_ids, const int32_t* hist, const int32_t* codes, int rows,
                                 int B, int K, int kv_len, const int64_t* targets, int n_tiers, int32_t* cnt);
/* partial_rerank_kernel, rerank/rerank.cu:52-143.                        */
void orc_rerank4(const int64_t* cand, int C, const uint8_t* packed, const uint16_t* weight, int64_t cap,
                 const uint16_t* q_blocks, const uint16_t* q_norm, const uint16_t* cen8, int rows,
                 uint16_t* scores);
/* coarse_2bit_score_kernel, rerank/coarse_2bit_score.cu:86-156.          */
void orc_coarse2bit(const uint8_t* packed, int64_t cap, const uint8_t* q_signs, const uint8_t* q_mags, int rows,
                    int kv_len, int32_t* out);
/* 1-bit x 4-bit popcount estimator (RaBitQ paper; no reference code).    */
void orc_rq_query_4bit(const uint16_t* q_blocks, const uint16_t* q_norm, int rows, uint8_t* planes, float* qparams);
void orc_popcount_est(const int64_t* cand, int C, const uint8_t* codes, const float* factor, int64_t cap,
                      const uint8_t* planes, const float* qparams, int rows, float* est, int32_t* ints);
void orc_exact_ip(const int64_t* idx, int n, const uint16_t* keys, int64_t ld_row, const uint16_t* q, int rows,
                  float* out);

#ifdef __cplusplus
}
#endif
#endif
