// zkv_pipeline.cu -- multi-kernel entry points: the reference-mode
// retrieval chain of one layer issued as one C call on one stream, its
// intermediates in a caller-provided workspace.
#include "zkv_common.cuh"

namespace zkv {

// raw_q[r] = bf16(fp32 sum over the G query heads of row r, in head order, / G)
// (the GQA mean of polar_cache.compute, REF:1622-1625).  One warp per row.
__global__ void __launch_bounds__(256) gqa_mean_kernel(const uint16_t* __restrict__ q, int rows, int G,
                                                       uint16_t* __restrict__ raw_q) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < G; ++g) {
        const uint2 v = *reinterpret_cast<const uint2*>(q + ((int64_t)row * G + g) * kHeadDim + 4 * lane);
        s[0] = __fadd_rn(s[0], bfbits2f((uint16_t)(v.x & 0xffffu)));
        s[1] = __fadd_rn(s[1], bfbits2f((uint16_t)(v.x >> 16)));
        s[2] = __fadd_rn(s[2], bfbits2f((uint16_t)(v.y & 0xffffu)));
        s[3] = __fadd_rn(s[3], bfbits2f((uint16_t)(v.y >> 16)));
    }
    uint16_t m[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = f2bfbits(__fdiv_rn(s[i], (float)G));
    *reinterpret_cast<uint2*>(raw_q + (int64_t)row * kHeadDim + 4 * lane) =
        make_uint2((uint32_t)m[0] | ((uint32_t)m[1] << 16), (uint32_t)m[2] | ((uint32_t)m[3] << 16));
}

}  // namespace zkv

using namespace zkv;

namespace {

constexpr size_t kAlign = 256;
inline size_t up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Workspace sections (section-major, each 256-byte aligned).
struct RefWs {
    size_t raw_q, scores, sel32, chunk_ids, density, dense_pos, mask, kscores, kidx, total;
};

inline RefWs ref_ws_layout(int rows, int n_chunks, int nk, int n_dense) {
    RefWs w;
    size_t o = 0;
    const size_t R = (size_t)rows;
    w.raw_q = o;     o += up(R * kHeadDim * 2);
    w.scores = o;    o += up(R * (size_t)((n_chunks + 31) & ~31) * 4);   // rows padded to 32 scores
    w.sel32 = o;     o += up(R * (size_t)nk * 4);
    w.chunk_ids = o; o += up(R * (size_t)nk * 8);
    w.density = o;   o += up(R * (size_t)nk * 4);
    w.dense_pos = o; o += up(R * (size_t)n_dense * 8);
    w.mask = o;      o += up(R * (size_t)nk);
    w.kscores = o;   o += up(R * (size_t)nk * kChunk * 4);
    w.kidx = o;      o += up(R * (size_t)nk * kChunk * 8);
    w.total = o;
    return w;
}

}  // namespace

extern "C" int zkv_gqa_mean(const void* q, int rows, int G, void* raw_q, void* stream) {
    if (!q || !raw_q || rows < 0 || G < 1) return ZKV_ERR_ARG;
    if (((uintptr_t)q & 7) || ((uintptr_t)raw_q & 7)) return ZKV_ERR_ALIGN;
    if (rows == 0) return ZKV_OK;
    return launch_pdl_kernel(gqa_mean_kernel, dim3((rows + 7) / 8), dim3(256), 0, (cudaStream_t)stream,
                             (const uint16_t*)q, rows, G, (uint16_t*)raw_q);
}

extern "C" size_t zkv_reference_select_ws_bytes(int rows, int n_chunks, int nk, int n_dense) {
    if (rows < 0 || n_chunks < 0 || nk < 0 || n_dense < 0) return 0;
    return ref_ws_layout(rows, n_chunks, nk, n_dense).total;
}

extern "C" int zkv_reference_select(const void* q, int G, const zkv_ref_layer* L, int rows, int n_max, int n_chunks,
                                    int n_valid_chunks, int nk, int n_dense, int dense_topk, int sparse_topk, int k,
                                    const int64_t* skipped, int64_t sk_ld, int sk, int64_t* final_out,
                                    int64_t final_ld, void* raw_q_out, void* workspace, size_t ws_bytes,
                                    void* stream) {
    if (!q || !L || !final_out || !workspace || rows < 0 || G < 1 || n_chunks < 1 || n_chunks > n_max || nk < 1 ||
        nk > n_chunks || n_dense < 1 || n_dense > nk || n_valid_chunks < 1 || n_valid_chunks > n_max || k < 1 ||
        k > nk * kChunk || sk < 0 || final_ld < k + sk || (sk > 0 && !skipped))
        return ZKV_ERR_ARG;
    if (!L->chunk_min || !L->chunk_max || !L->centroid || !L->packed) return ZKV_ERR_ARG;
    if (((uintptr_t)q & 7) || ((uintptr_t)workspace & (kAlign - 1))) return ZKV_ERR_ALIGN;
    if (rows == 0) return ZKV_OK;
    const RefWs w = ref_ws_layout(rows, n_chunks, nk, n_dense);
    if (ws_bytes < w.total) return ZKV_ERR_CAPACITY;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint16_t* raw_q = reinterpret_cast<uint16_t*>(ws + w.raw_q);
    float* scores = reinterpret_cast<float*>(ws + w.scores);
    int64_t* ids = reinterpret_cast<int64_t*>(ws + w.chunk_ids);
    float* dens = reinterpret_cast<float*>(ws + w.density);
    int64_t* pos = reinterpret_cast<int64_t*>(ws + w.dense_pos);
    uint8_t* mask = ws + w.mask;
    float* ksc = reinterpret_cast<float*>(ws + w.kscores);
    int64_t* kix = reinterpret_cast<int64_t*>(ws + w.kidx);
    cudaStream_t st = (cudaStream_t)stream;
    int s;
    // Stage 1: the GQA-mean query (recorded for stage 2), the Quest upper
    // bounds over the retrieval chunks and the top-nk chunks: the raw page
    // decode's score and select kernels up to 16384 chunks, else the Quest
    // launch with the GQA mean folded in and the float top-k
    if (n_chunks <= 16384 && G <= 8 && ((uintptr_t)q & 3) == 0 && ((uintptr_t)L->chunk_min & 15) == 0 &&
        ((uintptr_t)L->chunk_max & 15) == 0) {
        if ((s = raw_quest_topk(q, G, L->chunk_min, L->chunk_max, L->valid, rows, n_max, n_chunks, nk, scores,
                                (n_chunks + 31) & ~31, reinterpret_cast<int32_t*>(ws + w.sel32), ids, raw_q, st)))
            return s;
    } else {
        if (((uintptr_t)q & 15) == 0) {
            if ((s = quest_score_gqa_into(q, G, L->chunk_min, L->chunk_max, L->valid, scores, raw_q, rows, n_chunks,
                                          n_max, st)))
                return s;
        } else {
            if ((s = launch_pdl_kernel(gqa_mean_kernel, dim3((rows + 7) / 8), dim3(256), 0, st, (const uint16_t*)q,
                                       rows, G, raw_q)))
                return s;
            if ((s = zkv_quest_score(raw_q, L->chunk_min, L->chunk_max, L->valid, scores, rows, n_chunks, n_max,
                                     stream)))
                return s;
        }
        if ((s = zkv_topk_f32(scores, rows, n_chunks, n_chunks, nk, ids, stream))) return s;
    }
    // Stage 2 (CDS): centroid density, top-n_dense -> dense mask, KIVI qk per chunk.  (A one-CTA-per-row
    // fusion of the first three measured slower: one row's density loads need the whole grid in flight.)
    if ((s = zkv_chunk_density(ids, L->centroid, raw_q, dens, rows, nk, n_chunks, n_max, stream))) return s;
    if (nk <= 4096) {  // top-n_dense written straight as the mask
        if ((s = topk_mask_launch(dens, rows, nk, n_dense, mask, st))) return s;
    } else {
        if ((s = zkv_topk_f32(dens, rows, nk, nk, n_dense, pos, stream))) return s;
        if ((s = zkv_mask_from_topk(pos, mask, rows, n_dense, nk, stream))) return s;
    }
    if ((s = zkv_kivi_qk(ids, mask, L->packed, n_valid_chunks, n_max, L->chunk_min, L->chunk_max, n_max, raw_q, rows,
                         nk, dense_topk, sparse_topk, ksc, kix, (int64_t)nk * kChunk, stream)))
        return s;
    // global top-k token ids + the live skipped tail
    if ((s = zkv_topk_gather_concat(ksc, kix, skipped, sk_ld, final_out, rows, nk * kChunk, k, sk, final_ld, stream)))
        return s;
    if (raw_q_out &&
        cudaMemcpyAsync(raw_q_out, raw_q, (size_t)rows * kHeadDim * 2, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return ZKV_ERR_LAUNCH;
    return ZKV_OK;
}

// ---------------------------------------------------------------- no-allocation form
// The reference-mode chain with its intermediates in this library-owned
// device buffer, for callers that cannot allocate device memory: hosts that
// bind only the C ABI and own no device allocator (cgo, JNI, plain C), and
// decode loops that must not call cudaMalloc (it can synchronise the device).
static __device__ __align__(256) uint8_t g_ref_select_ws[ZKV_REFERENCE_SELECT_NOALLOC_MAX_BYTES];

namespace {
// Address of g_ref_select_ws on the current device (cudaGetSymbolAddress with
// that device current), looked up on every call: after cudaDeviceReset or a
// re-created primary context the module instance and its address change, so
// a cached address could point at memory that no longer exists.  NULL on
// failure.
void* noalloc_workspace() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_ref_select_ws) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}
}  // namespace

extern "C" int zkv_reference_select_noalloc(const void* q, int G, const zkv_ref_layer* L, int rows, int n_max,
                                            int n_chunks, int n_valid_chunks, int nk, int n_dense, int dense_topk,
                                            int sparse_topk, int k, const int64_t* skipped, int64_t sk_ld, int sk,
                                            int64_t* final_out, int64_t final_ld, void* raw_q_out, void* stream) {
    void* ws = noalloc_workspace();
    if (!ws) return ZKV_ERR_LAUNCH;
    // sizes beyond the buffer come back as ZKV_ERR_CAPACITY from the chain
    return zkv_reference_select(q, G, L, rows, n_max, n_chunks, n_valid_chunks, nk, n_dense, dense_topk, sparse_topk,
                                k, skipped, sk_ld, sk, final_out, final_ld, raw_q_out, ws,
                                ZKV_REFERENCE_SELECT_NOALLOC_MAX_BYTES, stream);
}
