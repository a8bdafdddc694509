/*
 * zkv.h -- C ABI of libzkv.so, the B200 (sm_100a) kernels of the ZoomKV
 * sparse decode-attention hot path.
 *
 * Conventions
 *   - bf16 tensors are passed as `const void*` (raw bfloat16 storage).
 *   - "rows" = batch * kv_heads, flattened row-major (row = b * H + h).
 *   - Every tensor is dense row-major in the shape given beside it unless a
 *     stride argument is named; strides are in elements.
 *   - head_dim is 128 and the Quest chunk (= KIVI key group = page) is 16
 *     tokens, as in the production ZoomKV configuration.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).
 *   - Every entry point returns ZKV_OK (0) or a ZKV_ERR_* code; launches are
 *     asynchronous, so a device-side failure (bounded wait expired) is
 *     reported through the optional `status` word the caller passes.
 *
 * Each declaration names the reference interface it replaces (paths relative
 * to runtime/zoomkv_urania_runtime_20261011/ of amy-77/zoomkv_revision).
 */
#ifndef ZKV_H
#define ZKV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZKV_OK 0
#define ZKV_ERR_ARG 1         /* bad shape / argument                          */
#define ZKV_ERR_ALIGN 2       /* pointer or stride not 16-byte aligned         */
#define ZKV_ERR_CAPACITY 3    /* size beyond a compiled limit                  */
#define ZKV_ERR_LAUNCH 4      /* CUDA launch / attribute error                 */
#define ZKV_ERR_UNSUPPORTED 5 /* unsupported configuration                     */
#define ZKV_ERR_TIMEOUT 6     /* device-side bounded wait expired (status word) */

const char* zkv_status_string(int status);
/* Library version (major*10000 + minor*100 + patch). */
int zkv_version(void);

/* ---------------------------------------------------------------- encode */

/* Chunk metadata + KIVI 4-bit key pack for `n_chunks` full chunks per row,
 * written at chunk indices [chunk_start, chunk_start + n_chunks).
 * Replaces polar_cache._compute_and_store_chunk_minmax (aligned part) +
 * polar_cache._kivi_pack_chunks
 * (cache_hub/polar_cache_quest_density_single_layer_kivi.py:2119-2141,
 * :1965-2020) and cache_hub/kivi/quant_pack.py:pack_kcache_4bit.
 *   keys      row r, token t at keys + r*keys_ld_row + t*128 (bf16)
 *   chunk_min, chunk_max, centroid  [rows][n_max][128] bf16 (centroid may be NULL)
 *   valid     [rows][n_max] uint8 (may be NULL; set to 1)
 *   packed    [rows][n_max][16][16] int32 (chunk-major A-1 layout)      */
int zkv_kivi_encode(const void* keys, int64_t keys_ld_row, int rows,
                    int n_chunks, int chunk_start, int n_max, void* chunk_min,
                    void* chunk_max, void* centroid, uint8_t* valid,
                    int32_t* packed, void* stream);

/* Per-token 4-bit value quantisation (group 32 along head_dim), written for
 * tokens [tok_start, tok_start + n_tokens) of each row in the page layout the
 * page-mode attention reads.  No counterpart in the reference (its values
 * stay bf16); same scale/zero arithmetic ladder as the KIVI keys.
 *   values    row r, token t at values + r*values_ld_row + t*128 (bf16)
 *   vcodes_t  [rows][n_pages][128][2] int32: dim d of page p, word w holds
 *             the 4-bit codes of tokens 8w..8w+7 (nibble j = token 8w+j)
 *   vmeta     [rows][n_pages][2][4][16] bf16: [scale|zero][group][token]  */
int zkv_vquant_encode(const void* values, int64_t values_ld_row, int rows,
                      int n_tokens, int tok_start, int n_pages,
                      int32_t* vcodes_t, void* vmeta, void* stream);

/* ------------------------------------------------------------ selection */

/* Quest upper-bound chunk scores.
 * Replaces quest_chunk_score (cache_hub/quest/quest_chunk_score.cu:106-154):
 * score = sum_d max(q_d*min_d, q_d*max_d) with the reference kernel's fp32
 * operation order (bit-identical); !valid -> -inf.
 *   raw_q [rows][128] bf16; chunk_min/max [rows][n_max][128] bf16;
 *   valid [rows][n_max] or NULL; scores [rows][n_chunks] fp32            */
int zkv_quest_score(const void* raw_q, const void* chunk_min,
                    const void* chunk_max, const uint8_t* valid, float* scores,
                    int rows, int n_chunks, int n_max, void* stream);

/* Top-k over fp32 rows.  Replaces float_topk_3d
 * (cache_hub/topk/float_topk.cu:280-346).  Selects the k largest by the
 * order-preserving u32 key, ties to the lowest index, and writes them in
 * ascending index order (the reference's order is unspecified).
 * len <= k: out[i] = i < len ? i : -1.   scores row stride row_stride.  */
int zkv_topk_f32(const float* scores, int rows, int len, int64_t row_stride,
                 int k, int64_t* out, void* stream);

/* Same for int32 rows.  Replaces radix_topk_3d
 * (cache_hub/topk/radix_topk.cu:157-240, used by polar_cache.py:1744).    */
int zkv_topk_i32(const int32_t* vals, int rows, int len, int64_t row_stride,
                 int k, int64_t* out, void* stream);

/* CDS density centroid[chunk_id]·raw_q, fp32, invalid id -> -1e30.
 * Replaces partial_chunk_density_scores (cache_hub/rerank/rerank_topk.cu:
 * 560-700; operation order bit-identical).
 *   chunk_ids [rows][nk]; centroid [rows][n_max][128]; raw_q [rows][128];
 *   out [rows][nk]; ids outside [0, n_chunks) are invalid.                */
int zkv_chunk_density(const int64_t* chunk_ids, const void* centroid,
                      const void* raw_q, float* out, int rows, int nk,
                      int n_chunks, int n_max, void* stream);

/* mask[r][:] = 0, then mask[r][positions[r][j]] = 1 for in-range positions.
 * Replaces mask_from_topk (cache_hub/rerank/rerank_topk.cu:926-999).     */
int zkv_mask_from_topk(const int64_t* positions, uint8_t* mask, int rows,
                       int n_dense, int nk, void* stream);

/* KIVI stage-2: per selected chunk, dequantise the 16 tokens' 4-bit keys
 * (bf16(bf16(code*scale)+min)), dot with raw_q (fp32 in dim order), sort
 * the 16 lanes (score desc, token asc) and keep dense_topk / sparse_topk.
 * Replaces partial_chunk_kivi_qk_dense_sparse
 * (cache_hub/kivi/kivi_qk_dot.cu:325-460).
 *   chunk_ids [rows][nk]; dense_mask [rows][nk];
 *   packed row r, chunk c at packed + (r*pk_ld + c)*256 int32 (chunk-major
 *   [16][16]); ids outside [0, n_pk) score -1e30;
 *   chunk_min/max [rows][n_max][128];
 *   raw_q [rows][128]; out_scores/out_idx row r at r*out_ld, nk*16 entries */
int zkv_kivi_qk(const int64_t* chunk_ids, const uint8_t* dense_mask,
                const int32_t* packed, int n_pk, int pk_ld, const void* chunk_min,
                const void* chunk_max, int n_max, const void* raw_q, int rows,
                int nk, int dense_topk, int sparse_topk, float* out_scores,
                int64_t* out_idx, int64_t out_ld, void* stream);

/* out[r][0:k] = lut[r][top_k(scores[r])] (ascending position order),
 * out[r][k:k+sk] = skipped[r][0:sk]; L <= k -> out[i] = i < L ? lut[i] : 0.
 * Replaces float_topk_gather_concat_3d
 * (cache_hub/topk/float_topk_gather_concat.cu:306-377).
 *   scores/lut [rows][L]; skipped row r at skipped + r*sk_ld;
 *   out row stride out_ld                                                  */
int zkv_topk_gather_concat(const float* scores, const int64_t* lut,
                           const int64_t* skipped, int64_t sk_ld, int64_t* out,
                           int rows, int L, int k, int sk, int64_t out_ld,
                           void* stream);

/* ------------------------------------------------------------ attention */

/* GQA decode attention over raw bf16 K/V rows gathered by index, fused with
 * the gather (no K/V copy is materialised).  Per row (b, kv_head) the token
 * set is [seg0_lo, seg0_hi) U {sel[r][j] + sel_offset : j < n_sel}
 * U [seg1_lo, seg1_hi) -- the sink / selected / near zones of the unified
 * cache.  Replaces the h2d_gather_kv + torch.cat + flash_attn_with_kvcache
 * sequence of polar_cache.compute
 * (cache_hub/polar_cache_quest_density_single_layer_kivi.py:1710-1768,
 * cache_hub/gather_trans/trans_h2d.cu:83-205).
 *   q       [rows / H][H*G][128] bf16 == [rows][G][128]
 *   keys, values  row r, token t at base + r*kv_ld_row + t*128 (bf16)
 *   sel     [rows][sel_ld] int64 (may be NULL when n_sel == 0)
 *   out     [rows][G][128] bf16; lse [rows][G] fp32 natural-log (may be NULL)
 *   split   CTAs per row (1, 2, 4 or 8; 0 = automatic)                  */
int zkv_attn_rows(const void* q, const void* keys, const void* values,
                  int64_t kv_ld_row, int rows, int G, int seg0_lo,
                  int seg0_hi, const int64_t* sel, int n_sel, int64_t sel_ld,
                  int64_t sel_offset, int seg1_lo, int seg1_hi, float scale,
                  void* out, float* lse, int split, int32_t* status,
                  void* stream);

/* Per-layer tensors of the page-mode cache (all [rows][...] row-major). */
typedef struct zkv_page_layer {
    const void* chunk_min;  /* [rows][n_max][128] bf16                      */
    const void* chunk_max;  /* [rows][n_max][128] bf16                      */
    const uint8_t* valid;   /* [rows][n_max] or NULL                        */
    const int32_t* kcodes;  /* [rows][n_max][16][16] int32 (A-1 layout)     */
    const int32_t* vcodes_t;/* [rows][n_max][128][2] int32                   */
    const void* vmeta;      /* [rows][n_max][2][4][16] bf16                 */
    const void* near_k;     /* [rows][near_ld][128] bf16 raw rows (sink +   */
    const void* near_v;     /*   residual window), row r at r*near_ld*128   */
    int64_t near_ld;        /* token capacity of the near buffers            */
} zkv_page_layer;

/* One fused launch per layer: GQA-mean query -> Quest scores over n_c
 * chunks -> top nk chunks (ties to the lowest id) -> attention of the G
 * query heads over [selected pages (4-bit K and V, dequantised in registers)
 * U the raw bf16 rows [0, n_sink) U [near_start, near_start + n_near) of the
 * near buffers] -> (out, lse).  A cluster of `cluster`
 * CTAs shares one row: scores and partial softmax states move through
 * distributed shared memory.  This is the HBM-resident form of
 * polar_cache.compute's retrieval branch with page selection
 * (cache_hub/polar_cache_quest_density_single_layer_kivi.py:1589-1775,
 * quest_chunk_score.cu, float_topk.cu, flash_attn_compat.py:44-99).
 *   q [rows][G][128] bf16; out [rows][G][128] bf16; lse [rows][G] or NULL;
 *   sel_out [rows][nk] selected chunk ids (ascending) or NULL;
 *   status: device int32 set to ZKV_ERR_TIMEOUT if a bounded wait expires
 *   (may be NULL); cluster in {1, 2, 4, 8} (0 = automatic).              */
int zkv_page_decode(const void* q, const zkv_page_layer* layer, int rows,
                    int G, int n_max, int n_c, int nk, int n_sink,
                    int near_start, int n_near, float scale, void* out,
                    float* lse, int64_t* sel_out, int32_t* status, int cluster,
                    void* stream);

/* Merge two attention partials by log-sum-exp (fp32 math, bf16 out).
 * Replaces lse_merge_cuda (cache_hub/lse_merge/lse_merge.cu:44-101).
 *   a, b, out [rows][dim] bf16; la, lb [rows] fp32; lse_out [rows] or NULL */
int zkv_lse_merge(const void* a, const float* la, const void* b,
                  const float* lb, void* out, float* lse_out, int rows,
                  int dim, void* stream);

/* N-way merge of fp32 partials [n][rows][dim] with lse [n][rows] (the
 * sequence-split combine step) -> out [rows][dim] bf16, lse_out [rows].   */
int zkv_lse_merge_n(const float* parts, const float* lses, int n, int rows,
                    int dim, void* out, float* lse_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ZKV_H */
