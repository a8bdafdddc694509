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

#include <stddef.h>
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
#define ZKV_ERR_RANGE 7       /* device-side index outside its range (status word) */

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
 *   packed    [rows][n_max][16][16] int32 (chunk-major A-1 layout)
 *   kscale    [rows][n_max][128] bf16 KIVI scale bf16(bf16(max-min)/15) per
 *             chunk and dim (may be NULL; the page-mode attention reads it) */
int zkv_kivi_encode(const void* keys, int64_t keys_ld_row, int rows,
                    int n_chunks, int chunk_start, int n_max, void* chunk_min,
                    void* chunk_max, void* centroid, uint8_t* valid,
                    int32_t* packed, void* kscale, void* stream);

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

/* zkv_quest_score with the GQA mean folded in: q [rows][G][128] bf16
 * (16-byte aligned); raw_q = bf16(fp32 sum of the G heads in head order /
 * G) is formed per CTA (polar_cache compute() :1622-1626 + the Quest score
 * of quest_chunk_score.cu).                                              */
int zkv_quest_score_gqa(const void* q, int G, const void* chunk_min,
                        const void* chunk_max, const uint8_t* valid,
                        float* scores, int rows, int n_chunks, int n_max,
                        void* stream);

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

/* ------------------------------------------------- reference-mode chain */

/* Chunk index of one layer for the reference-mode chain; every tensor is
 * [rows][n_max][...]: chunk_min/max/centroid [..][128] bf16, valid u8 (or
 * NULL), packed [..][16][16] int32 (chunk-major KIVI keys).              */
typedef struct zkv_ref_layer {
    const void* chunk_min;
    const void* chunk_max;
    const void* centroid;
    const uint8_t* valid;
    const int32_t* packed;
} zkv_ref_layer;

/* raw_q [rows][128] = bf16(fp32 sum of the G query heads in head order / G)
 * of q [rows][G][128] bf16: the GQA-mean query of polar_cache.compute
 * (cache_hub/polar_cache_quest_density_single_layer_kivi.py:1622-1625),
 * computed exactly as zkv_page_decode and zkv_reference_select do.       */
int zkv_gqa_mean(const void* q, int rows, int G, void* raw_q, void* stream);

/* Bytes of workspace zkv_reference_select needs (0 on bad arguments).    */
size_t zkv_reference_select_ws_bytes(int rows, int n_chunks, int nk,
                                     int n_dense);

/* The retrieval chain of polar_cache.compute for one layer as one call on
 * one stream (cache_hub/polar_cache_quest_density_single_layer_kivi.py:
 * 1589-1775 minus the attention): raw_q = GQA mean of q [rows][G][128]
 * bf16; Quest scores of chunks [0, n_chunks); top-nk chunks; CDS density
 * and top-n_dense dense mask; KIVI stage 2 over packed chunks
 * [0, n_valid_chunks); global top-k token ids + skipped tail into
 * final_out [rows][final_ld] (same results as the single-op entry points
 * above, called in that order).  Intermediates live in `workspace`
 * (256-byte aligned, >= zkv_reference_select_ws_bytes bytes; every byte
 * read is written first by the same call).  raw_q_out [rows][128] bf16 may
 * be NULL.  dense_topk, sparse_topk in [1, 16].                           */
int zkv_reference_select(const void* q, int G, const zkv_ref_layer* layer,
                         int rows, int n_max, int n_chunks,
                         int n_valid_chunks, int nk, int n_dense,
                         int dense_topk, int sparse_topk, int k,
                         const int64_t* skipped, int64_t sk_ld, int sk,
                         int64_t* final_out, int64_t final_ld,
                         void* raw_q_out, void* workspace, size_t ws_bytes,
                         void* stream);

/* Capacity of the library-owned buffer of zkv_reference_select_noalloc.  */
#define ZKV_REFERENCE_SELECT_NOALLOC_MAX_BYTES (16u << 20)

/* zkv_reference_select with the intermediates in a library-owned device
 * buffer (a static device array, one per device) instead of a caller
 * workspace; allocates nothing.  No reference counterpart: the reference
 * allocates its intermediates through torch.  For callers that cannot
 * allocate device memory: hosts that bind only this C ABI and own no device
 * allocator (cgo, JNI, plain C), and decode loops that must not call
 * cudaMalloc, which can synchronise the device.
 *   Limit: zkv_reference_select_ws_bytes(rows, n_chunks, nk, n_dense) <=
 *   ZKV_REFERENCE_SELECT_NOALLOC_MAX_BYTES (16 MiB), else ZKV_ERR_CAPACITY
 *   (e.g. 64 rows x 2048 chunks with nk = 816, n_dense = 244 needs ~12 MB).
 *   Setup: every call looks the buffer's address up (cudaGetSymbolAddress
 *   on the current device, which must be the stream's device); the first
 *   call on a device also loads the module there, so make it before any
 *   stream capture.
 *   Calls that overlap on one device (concurrent streams or host threads)
 *   race on the one buffer: serialise them.  Nothing needs clearing: every
 *   byte the chain reads is written first by the same call.               */
int zkv_reference_select_noalloc(const void* q, int G,
                                 const zkv_ref_layer* layer, int rows,
                                 int n_max, int n_chunks, int n_valid_chunks,
                                 int nk, int n_dense, int dense_topk,
                                 int sparse_topk, int k,
                                 const int64_t* skipped, int64_t sk_ld,
                                 int sk, int64_t* final_out, int64_t final_ld,
                                 void* raw_q_out, void* stream);

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
    const void* kscale;     /* [rows][n_max][128] bf16 KIVI scales           */
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

/* Long-context form of zkv_page_decode for few rows (same selection; the
 * output can differ by fp32 rounding): the Quest scores of all n_c chunks
 * are computed by a kernel that spreads over every SM
 * (zkv_quest_score_gqa) into `workspace`; then the fused kernel, with up to
 * 4 clusters per row that each attend a share of the selected pages, merged
 * by zkv_lse_merge_n; the fused kernel reads the scores, selects in two
 * levels (each cluster CTA's top nk, then the top nk of those) and attends.
 * Falls back to zkv_page_decode where the fused kernel selects in one level
 * (n_c <= 2048, cluster 1, nk >= n_c).  workspace: device, 256-byte
 * aligned, ws_bytes >= zkv_page_decode_split_ws_bytes(rows, n_c).        */
size_t zkv_page_decode_split_ws_bytes(int rows, int n_c);
int zkv_page_decode_split(const void* q, const zkv_page_layer* layer, int rows,
                          int G, int n_max, int n_c, int nk, int n_sink,
                          int near_start, int n_near, float scale, void* out,
                          float* lse, int64_t* sel_out, int32_t* status,
                          int cluster, void* workspace, size_t ws_bytes,
                          void* stream);

/* Per-layer tensors of the raw-page cache: Quest metadata + the raw bf16
 * K/V rows at absolute token positions (the reference's unified cache). */
typedef struct zkv_raw_layer {
    const void* chunk_min;  /* [rows][n_max][128] bf16                      */
    const void* chunk_max;  /* [rows][n_max][128] bf16                      */
    const uint8_t* valid;   /* [rows][n_max] or NULL                        */
    const void* keys;       /* raw rows: row r, token t at                  */
    const void* values;     /*   base + r*kv_ld_row + t*128 (bf16)          */
    int64_t kv_ld_row;      /* elements per row, a multiple of 128          */
    int64_t page_base;      /* token position of chunk 0 (the sink size)    */
} zkv_raw_layer;

/* Bytes of workspace zkv_page_decode_raw needs.                          */
size_t zkv_page_decode_raw_ws_bytes(int rows, int n_c, int nk, int n_sink,
                                    int n_near);

/* Page-mode decode over the RAW bf16 rows of the selected pages:
 * GQA-mean query -> Quest scores of chunks [0, n_c) ->
 * top nk chunks (ties to the lowest id, ascending) -> attention of the G
 * query heads over [selected chunks' 16 raw rows each, at token
 * page_base + 16 c] U [0, n_sink) U [near_start, near_start + n_near) ->
 * (out, lse).  This is polar_cache.compute's retrieval branch in page mode
 * (dense_topk = sparse_topk = 16, final_topk = budget): the reference
 * attends the raw rows of the selected chunks
 * (cache_hub/polar_cache_quest_density_single_layer_kivi.py:1589-1775,
 * :1734-1750; quest_chunk_score.cu:106-154; float_topk.cu:280-346;
 * attn_hub/flash_attn_compat.py:44-99).  Four launches chained by
 * programmatic dependent launch: Quest scores, per-row select, attention
 * (pages by 2-D TMA tensor copies) into per-CTA partials, per-row merge.
 * nk <= n_c (nk == n_c: every chunk, no scores or select, two launches).
 *   q [rows][G][128] bf16; out [rows][G][128] bf16; lse [rows][G] fp32
 *   natural log (may be NULL); sel_out [rows][nk] int64 or NULL;
 *   status: device int32 set to ZKV_ERR_TIMEOUT if a bounded wait expires;
 *   workspace: device, 256-byte aligned, >= zkv_page_decode_raw_ws_bytes
 *   (scratch only: no state carries between calls, no zero fill needed);
 *   calls sharing a workspace must not overlap on the GPU.
 *   Limits: n_c <= 16384, (n_sink + n_near) / 16 + nk <= 16384,
 *   rows * kv_ld_row / 128 < 2^31 (else ZKV_ERR_CAPACITY).               */
int zkv_page_decode_raw(const void* q, const zkv_raw_layer* layer, int rows,
                        int G, int n_max, int n_c, int nk, int n_sink,
                        int near_start, int n_near, float scale, void* out,
                        float* lse, int64_t* sel_out, int32_t* status,
                        void* workspace, size_t ws_bytes, void* stream);

/* Hierarchical Quest inputs: per-large-chunk min / max (bf16,
 * [rows][n_max_large][128]) and validity ([rows][n_max_large]).            */
typedef struct zkv_quest_large {
    const void* large_min;
    const void* large_max;
    const uint8_t* large_valid;
    int n_max_large;
} zkv_quest_large;

/* Large-chunk min / max of groups [g_lo, g_hi): group g covers chunks
 * [g*factor, min(g*factor + factor, valid_end)); its min / max are the
 * element-wise bf16 min / max of those chunks' min / max and it becomes
 * valid; empty groups are left untouched.  Replaces
 * _update_large_chunk_minmax (cache_hub/polar_cache_kivi_quest_density_
 * seperate_kernel.py:1762-1798).  chunk_min/max [rows][n_max][128] bf16.   */
int zkv_quest_large_minmax(const void* chunk_min, const void* chunk_max, int rows, int n_max, int valid_end,
                           int factor, int g_lo, int g_hi, void* large_min, void* large_max, uint8_t* large_valid,
                           int n_max_large, void* stream);

/* Bytes of workspace zkv_page_decode_raw_hier needs.                     */
size_t zkv_page_decode_raw_hier_ws_bytes(int rows, int n_c, int factor, int nk_large, int nk_small, int n_sink,
                                         int n_near);

/* zkv_page_decode_raw with the hierarchical Quest pick
 * (_quest_pick_coarse_indices_hierarchical, :1852-1940, with
 * quest_chunk_score / quest_sub_chunk_score / quest_map_back of
 * cache_hub/quest/quest_chunk_score.cu and float_topk_3d): Quest over the
 * n_c / factor large chunks (large_valid applied), their top nk_large, the
 * Quest scores of those large chunks' factor sub-chunks each, the top
 * nk_small sub-chunks mapped back to chunk ids (ascending) -> attention
 * over those pages' raw rows + sink + near rows, as zkv_page_decode_raw.
 * Six launches chained by programmatic dependent launch.  factor <= 16;
 * 1 <= nk_large <= n_c / factor; 1 <= nk_small <= nk_large * factor.      */
int zkv_page_decode_raw_hier(const void* q, const zkv_raw_layer* layer, const zkv_quest_large* large, int rows,
                             int G, int n_max, int n_c, int factor, int nk_large, int nk_small, int n_sink,
                             int near_start, int n_near, float scale, void* out, float* lse, int64_t* sel_out,
                             int32_t* status, void* workspace, size_t ws_bytes, void* stream);

/* Sequence split of zkv_page_decode_raw over `world` ranks, one process per
 * GPU (the benchmark's config 3; the reference has no multi-GPU form of
 * compute(), whose single-device steps this splits).  Rank q holds the
 * pages [q per, min(n_c, q per + per)) of every row, per = ceil(n_c / world)
 * rounded up to 16 (zkv_raw_split_range), as its local pages 0, 1, ...;
 * rank 0 also holds the sink and near rows.  Each rank owns one exchange
 * buffer of zkv_raw_split_buffer_bytes, allocated zeroed with
 * zkv_peer_alloc and mapped into every other rank with zkv_peer_open.   */
typedef struct zkv_raw_split {
    void* const* peer_base;  /* [world] every rank's exchange buffer as
                                mapped in this process ([rank]: its own) */
    size_t bytes;            /* size of each buffer (the same on every
                                rank); a call whose shape needs more
                                returns ZKV_ERR_CAPACITY                 */
    int rank, world;         /* world <= 8                               */
} zkv_raw_split;

int zkv_raw_split_range(int n_c, int world, int rank, int* lo, int* hi);
size_t zkv_raw_split_buffer_bytes(int rows, int G, int n_c, int world);
size_t zkv_page_decode_raw_split_ws_bytes(int rows, int n_c, int world, int rank, int nk, int n_sink,
                                          int n_near);

/* One rank's share of a layer: Quest scores of its pages, stored straight
 * into every rank's score row (peer stores over NVLink of 64-bit words
 * {score, epoch of the call}) -> on every rank the top nk of the whole row
 * (a bounded wait until every word carries the call's epoch, then the
 * select of zkv_page_decode_raw: the same ids, ascending, on every rank) ->
 * attention over the selected pages this rank holds (+ sink / near on rank
 * 0) -> each (row, head)'s partial stored into every rank as tagged words,
 * a bounded wait, and the world partials combined in rank order: out /
 * lse, identical on every rank.  Four launches chained by programmatic
 * dependent launch; no fence, flag, collective library or multicast.
 * `layer` holds this rank's pages (chunk_min / chunk_max / valid
 * [rows][n_max >= own pages], page j's rows at token page_base + 16 j);
 * n_c / nk count the whole row's pages; 1 <= nk < n_c <= 16384, every rank
 * holds a page.  sel_out [rows][nk]: the whole selection (global ids).
 * Every rank makes the same sequence of calls with a buffer; a wait that
 * expires (zkv_peer_set_wait_ms) sets ZKV_ERR_TIMEOUT in `status`, after
 * which the group's buffers must be re-created.  Workspace as
 * zkv_page_decode_raw (its own size).                                    */
int zkv_page_decode_raw_split(const void* q, const zkv_raw_layer* layer, const zkv_raw_split* split, int rows,
                              int G, int n_max, int n_c, int nk, int n_sink, int near_start, int n_near,
                              float scale, void* out, float* lse, int64_t* sel_out, int32_t* status,
                              void* workspace, size_t ws_bytes, void* stream);

/* Decode-loop caller kernels (the benchmark's config 4; no reference
 * counterpart of their own: the reference's model code calls flashinfer's
 * rmsnorm / apply_rope_with_cos_sin_cache_inplace / silu_and_mul for these
 * steps, model_hub/qwen.py:481-612).  bf16 in and out, fp32 inside.
 * zkv_rmsnorm: y = x * rsqrt(mean(x^2) + eps) * w per row of dim.
 * zkv_qk_norm_rope: qkv [rows][(hq + 2 hkv) * 128] -> q [rows][hq][128],
 *   k / v [rows][hkv][128]; q and k heads get RMSNorm over the head (q_norm,
 *   k_norm [128]) then the rotate-half RoPE at position *pos (device int64;
 *   cos_t / sin_t fp32 [max_pos][64]).
 * zkv_silu_mul: out [rows][ffn] = silu(gu[:, :ffn]) * gu[:, ffn:].        */
int zkv_rmsnorm(const void* x, const void* w, void* y, int rows, int dim, float eps, void* stream);
int zkv_qk_norm_rope(const void* qkv, const void* q_norm, const void* k_norm, const float* cos_t,
                     const float* sin_t, const int64_t* pos, int rows, int hq, int hkv, float eps, void* q,
                     void* k, void* v, void* stream);
int zkv_silu_mul(const void* gu, void* out, int rows, int ffn, void* stream);

/* Attention over externally selected pages (the sequence-split step):
 * the layer buffer holds pages [sel_lo, sel_hi) of the sequence as its
 * pages 0..; of the global page ids sel [rows][n_sel] (-1 = none) those in
 * [sel_lo, sel_hi) are attended, plus the n_sink / n_near raw rows as in
 * zkv_page_decode (pass 0 on ranks that own none).  Writes the normalised
 * partial to out (bf16) or out_f32 (fp32, [rows][G][128]) and lse [rows][G]
 * (natural log; -inf when a row attended nothing) for an LSE merge.
 * n_sel <= 4096.  Same kernel and numerics as zkv_page_decode's phase 3-4. */
int zkv_page_attend(const void* q, const zkv_page_layer* layer, int rows,
                    int G, int n_max, const int64_t* sel, int n_sel,
                    int64_t sel_lo, int64_t sel_hi, int n_sink,
                    int near_start, int n_near, float scale, void* out,
                    float* out_f32, float* lse, int32_t* status, int cluster,
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

/* ------------------------------------------------- ParisKV / RaBitQ path */
/* Per-key retrieval codes of ParisKV (cache_hub/polar_cache.py), D = 128
 * split into 16 blocks of 8 dims.  Every tensor is addressed as
 * base + row*X_row + block*X_blk + token*X_tok (units in the comments), so
 * both this build's token-major layout (blk 1, tok 16) and the reference's
 * block-major layout (blk cap, tok 1) can be passed.
 *   codes   1-bit sign codes, one byte per block (bit j = dim 8b+j >= 0)
 *   packed  4-bit codes, one 4-byte word per block, byte i = v_{2i+1}<<4 | v_{2i},
 *           v = sign<<3 | magnitude  (units: 4-byte words)
 *   weight  bf16 per block (r_b / alpha_b) * |k|
 *   factor  fp32 per key |k| / <xbar, o'> for the popcount estimator (may be NULL)
 *   hist    [rows][16][256] int32 bucket sizes (cluster_key_counts; may be NULL) */
typedef struct zkv_rq_layout {
    uint8_t* codes;
    int64_t codes_row, codes_blk, codes_tok;
    uint32_t* packed;
    int64_t packed_row, packed_blk, packed_tok;
    void* weight;
    int64_t weight_row, weight_blk, weight_tok;
    float* factor;
    int64_t factor_row;
    int32_t* hist;
} zkv_rq_layout;

/* Encode keys [tok_start, tok_start+n_tok) of every row (raw bf16 rows at
 * keys + r*keys_ld_row + t*128) into `lay`, adding them to lay->hist.
 * signs [128] bf16 (+-1, the SRHT diagonal).  Replaces batch_encode +
 * _count_cluster_keys (cache_hub/polar_cache.py:1130-1198, :1203-1226).  */
int zkv_rq_encode(const void* keys, int64_t keys_ld_row, int rows, int n_tok,
                  int tok_start, const void* signs, const zkv_rq_layout* lay,
                  void* stream);

/* Query side: GQA mean of q [rows][G][128] bf16, then normalise + SRHT:
 * q_blocks [rows][128] bf16, q_norm [rows] bf16, q_mean [rows][128] bf16
 * (may be NULL).  Replaces _encode_query_blocks (polar_cache.py:1108-1127).
 * When planes != NULL also the 4-bit query of the popcount estimator:
 * planes [rows][4][16] u8, qparams [rows][4] fp32 {lo, delta, sum, |q|}. */
int zkv_rq_query(const void* q, int rows, int G, const void* signs,
                 void* q_blocks, void* q_norm, void* q_mean, uint8_t* planes,
                 float* qparams, void* stream);

/* Fused collision count + coarse top-C (get_cache_cnt_fused +
 * _coarse_filter_truncate, polar_cache.py:1688-1747; collision.cu:72-245;
 * radix_topk.cu:157-240).  Per (row, block) the 256 buckets are ordered by
 * bf16 score q_b . V[c] (descending, ties to the lower bucket), a key's
 * count is the number of tiers t whose prefix (before[rank] < targets[t])
 * holds its bucket, summed over the 16 blocks.  idx_out [rows][C] receives
 * the C keys of highest count (ties to the lower index) in ascending index
 * order; cnt_out [rows][kv_len] int32 (may be NULL) the counts.  With
 * idx_out NULL only the counts are produced (update_cache_cnt).
 * 1 <= C <= kv_len; n_tiers <= 8; reads lay->codes and lay->hist.        */
int zkv_collision_topk(const void* q_blocks, const zkv_rq_layout* lay,
                       int rows, int kv_len, const int64_t* targets,
                       int n_tiers, int C, int64_t* idx_out, int32_t* cnt_out,
                       void* stream);

/* 4-bit RaBitQ rerank of candidate keys cand [rows][C] (rerank.cu:52-143,
 * sequential bf16 as python_rabitq_scores) -> scores [rows][C] bf16 (may be
 * NULL) and, when F > 0, the F best candidates' key ids (ties to the lower
 * candidate position, ascending position order) in final [rows][F]
 * (polar_cache.py:1750-1832 topk + gather).  centers [8] bf16.           */
int zkv_rq_rerank4(const int64_t* cand, int C, const zkv_rq_layout* lay,
                   const void* q_blocks, const void* q_norm,
                   const void* centers, int rows, void* scores, int F,
                   int64_t* final_out, void* stream);

/* 2-bit-plane popcount coarse score (coarse_2bit_score.cu:86-156):
 * out [rows][kv_len] int32 from lay->packed and the query's sign /
 * magnitude-high bit planes q_signs, q_mags [rows][16] u8.               */
int zkv_coarse2bit(const zkv_rq_layout* lay, const uint8_t* q_signs,
                   const uint8_t* q_mags, int rows, int kv_len, int32_t* out,
                   void* stream);

/* 1-bit x 4-bit popcount estimator rerank (RaBitQ; no reference kernel):
 * estimates <k, q> for cand [rows][C] (NULL = keys 0..C-1) from lay->codes
 * and lay->factor with the 4-bit query (planes, qparams), keeps the K best
 * (ties to the lower position) in sel_out [rows][K] (key ids, ascending),
 * est_out [rows][C] fp32 (may be NULL); when keys != NULL also the exact
 * fp32 inner products of the selected raw bf16 keys with q_mean
 * [rows][128] in ip_out [rows][K].                                        */
int zkv_rq_popcount_topk(const int64_t* cand, int C, const zkv_rq_layout* lay,
                         const uint8_t* planes, const float* qparams,
                         int rows, int K, int64_t* sel_out, float* est_out,
                         const void* keys, int64_t keys_ld_row,
                         const void* q_mean, float* ip_out, void* stream);

/* ------------------------------------------------------------ offload tier */

/* Gather of selected K/V rows from host-pinned memory into device memory,
 * read by the SMs over the host link (zero-copy through the unified address
 * space).  Replaces h2d_gather_kv (cache_hub/gather_trans/trans_h2d.py:65-105,
 * trans_h2d.cu:83-205).  Per row r (= b * kv_heads + h) and j < n_sel:
 *   dst[r][dst_off + j][:] = src[r][idx[r*idx_ld + j] + src_off][:]
 *   src_k, src_v  host-pinned [rows][src_len][128] bf16 (cudaHostAlloc or
 *                 cudaHostRegister memory; anything else -> ZKV_ERR_ARG)
 *   idx           device [rows][idx_ld] int64 (idx_ld 0: one list for all rows)
 *   dst_k, dst_v  device [rows][dst_len][128] bf16, dst_off + n_sel <= dst_len
 * The reference's call is dst_off = 0, src_off = 0, n_sel = idx_ld = topk.
 * An index outside [0, src_len) is not dereferenced: its row is skipped and
 * ZKV_ERR_RANGE is written to `status` (may be NULL).                      */
int zkv_h2d_gather_kv(const void* src_k, const void* src_v, int rows,
                      int64_t src_len, const int64_t* idx, int64_t idx_ld,
                      int n_sel, int64_t src_off, void* dst_k, void* dst_v,
                      int64_t dst_len, int64_t dst_off, int32_t* status,
                      void* stream);

/* Variable-K form writing into a flash-attention varlen packed buffer.
 * Replaces h2d_gather_kv_packed (trans_h2d.py:108-161,
 * trans_h2d.cu:228-283).  For vh < rows and slot < global_k with
 * slot < cu_topk[vh+1] - cu_topk[vh]:
 *   dst[cu_k[vh] + sl_end + slot][:] = src[vh][idx[cu_topk[vh] + slot]][:]
 *   idx      device [total_topk] int64;  cu_topk, cu_k  device [rows+1] int32
 *   dst_k, dst_v  device [n_dst][128] bf16
 * Rows [cu_k[vh], cu_k[vh] + sl_end) of every segment are not written.  A
 * source index or destination row out of range is skipped and reported as
 * ZKV_ERR_RANGE in `status`.  global_k <= 0 copies nothing.               */
int zkv_h2d_gather_kv_packed(const void* src_k, const void* src_v, int rows,
                             int64_t src_len, const int64_t* idx,
                             const int32_t* cu_topk, const int32_t* cu_k,
                             int sl_end, int global_k, void* dst_k,
                             void* dst_v, int64_t n_dst, int32_t* status,
                             void* stream);

/* The select + attend step of the sequence split, fused: the top nk of a
 * precomputed score row (scores [rows][sc_ld], n_c entries: the whole
 * sequence's chunk scores, -inf past its end) by the cluster two-level
 * select, then attention over the selected pages in [own_lo, own_hi) --
 * held by this layer buffer as pages id - own_lo -- plus n_sink / n_near
 * raw rows, spread over `parts` clusters per row (1..4).  Writes per-part
 * normalised partials out_f32 [parts][rows][G][128] and lse
 * [parts][rows][G] (natural log; -inf for a part with nothing to attend),
 * to be merged with zkv_lse_merge_n together with the other ranks'.
 * sel_out (may be NULL): the global selection [rows][nk].  Requires
 * nk < n_c and a cluster of 2..8 CTAs.  Replaces the float_topk_3d +
 * page attention pair of the split step (no reference counterpart: the
 * reference runs on one device).                                          */
int zkv_page_decode_scored(const void* q, const zkv_page_layer* layer,
                           int rows, int G, int n_max, const float* scores,
                           int64_t sc_ld, int n_c, int nk, int64_t own_lo,
                           int64_t own_hi, int n_sink, int near_start,
                           int n_near, float scale, int parts, float* out_f32,
                           float* lse, int64_t* sel_out, int32_t* status,
                           int cluster, void* stream);

/* ------------------------------------------------------------ peer exchange */

/* The exchange steps of the sequence-split decode over peer memory (NVLink
 * P2P stores), replacing the NCCL all-gathers of the score rows and of the
 * partial (out, lse) (no reference counterpart: the reference runs on one
 * device).  One buffer per rank, shared through CUDA IPC:
 *   zkv_peer_alloc   cudaMalloc'd, zeroed buffer + its IPC handle
 *                    (zkv_peer_handle_bytes() bytes, to be sent to peers);
 *   zkv_peer_open    a peer's handle -> device pointer in this process;
 *   zkv_peer_close / zkv_peer_free  release a mapping / the own buffer.   */
int zkv_peer_handle_bytes(void);
int zkv_peer_alloc(size_t bytes, void** ptr, void* handle);
int zkv_peer_open(const void* handle, void** ptr);
int zkv_peer_close(void* ptr);
int zkv_peer_free(void* ptr);

/* One strided segment of a put: `rows` rows of `row_bytes` from
 * src + r*src_ld_bytes to peer_base + dst_off_bytes + r*dst_ld_bytes (all
 * multiples of 4).                                                        */
typedef struct zkv_peer_seg {
    const void* src;
    int64_t src_ld_bytes;
    int64_t dst_off_bytes;
    int64_t dst_ld_bytes;
    int64_t row_bytes;
    int32_t rows;
    int32_t pad;
} zkv_peer_seg;

/* Copy 1-2 segments into every peer's buffer (peer_base[p], p < world, a
 * host array of device pointers; peer_base[rank] is this rank's own
 * buffer), then raise the flag word `rank` of the uint32 flag array at
 * byte offset flag_off of every peer buffer to *epoch + 1 (release, system
 * scope) once all stores are done.  `epoch`, `done`: device words of this
 * rank (done = 0 initially; the kernel returns it to 0).  chunks: CTAs per
 * peer (0 = automatic: 8 up to 2 ranks, 2 beyond).                        */
int zkv_peer_put(const zkv_peer_seg* segs, int n_seg, void* const* peer_base,
                 int64_t flag_off, int rank, int world, uint32_t* epoch,
                 uint32_t* done, int chunks, void* stream);

/* zkv_peer_put followed by the wait of the same phase in one launch: the
 * CTA that raises the flags then polls this rank's flag array (at flag_off
 * in peer_base[rank]) until all ranks reach *epoch + 1 and advances *epoch;
 * bounded like zkv_peer_wait (ZKV_ERR_TIMEOUT in `status`).               */
int zkv_peer_exchange(const zkv_peer_seg* segs, int n_seg,
                      void* const* peer_base, int64_t flag_off, int rank,
                      int world, uint32_t* epoch, uint32_t* done, int chunks,
                      int32_t* status, void* stream);

/* Wait until flags[0..world) (this rank's flag array) all reach *epoch + 1
 * (acquire, system scope), then advance *epoch.  The wait is bounded: on
 * expiry ZKV_ERR_TIMEOUT is written to `status` and the kernel returns.    */
int zkv_peer_wait(const uint32_t* flags, uint32_t* epoch, int world,
                  int32_t* status, void* stream);

/* Time limit of the peer waits (zkv_peer_wait, zkv_peer_exchange) in ms on
 * the GPU's global timer, 1..600000 (default 5000), for launches enqueued
 * after the call.  On expiry the wait records ZKV_ERR_TIMEOUT in `status`
 * and returns; the ranks' epochs then disagree, so the peer buffers must be
 * re-created (a new peer group).  No reference counterpart: the reference
 * exchanges nothing between GPUs on this path.                            */
int zkv_peer_set_wait_ms(int ms);

#ifdef __cplusplus
}
#endif
#endif /* ZKV_H */
