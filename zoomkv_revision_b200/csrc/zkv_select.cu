// zkv_select.cu -- the selection stages of the reference-mode decode path:
// Quest chunk scoring, deterministic radix top-k, CDS density + dense mask,
// KIVI stage-2 per-chunk rerank and the fused global top-k/gather/concat.
#include "zkv_common.cuh"

namespace zkv {

template <int UNROLL>
__global__ void __launch_bounds__(256) quest_score_kernel(const uint16_t* __restrict__ raw_q,
                                                          const uint16_t* __restrict__ cmin,
                                                          const uint16_t* __restrict__ cmax,
                                                          const uint8_t* __restrict__ valid,
                                                          float* __restrict__ scores, int n_chunks, int n_max,
                                                          const uint16_t* __restrict__ q = nullptr, int G = 0,
                                                          uint16_t* __restrict__ raw_q_out = nullptr) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    const int r = blockIdx.y;
    const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
    const int warp = threadIdx.x >> 5;
    uint4 qv;
    if (q) {  // GQA mean of the row's G query heads (fp32 sum in head order, / G, bf16)
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int g = 0; g < G; ++g) {
            const uint4 v = *reinterpret_cast<const uint4*>(q + ((int64_t)r * G + g) * kHeadDim + 8 * hl);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[2 * j] = __fadd_rn(acc[2 * j], bfbits2f((uint16_t)(w[j] & 0xffffu)));
                acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], bfbits2f((uint16_t)(w[j] >> 16)));
            }
        }
        uint32_t m[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            m[j] = (uint32_t)f2bfbits(__fdiv_rn(acc[2 * j], (float)G)) |
                   ((uint32_t)f2bfbits(__fdiv_rn(acc[2 * j + 1], (float)G)) << 16);
        qv = make_uint4(m[0], m[1], m[2], m[3]);
        if (raw_q_out && blockIdx.x == 0 && warp == 0 && half == 0)  // one CTA per row records it
            *reinterpret_cast<uint4*>(raw_q_out + (int64_t)r * kHeadDim + 8 * hl) = qv;
    } else {
        qv = *reinterpret_cast<const uint4*>(raw_q + (int64_t)r * kHeadDim + 8 * hl);
    }
    const int base = (blockIdx.x * 8 + warp) * (2 * UNROLL);
    uint4 mn[UNROLL], mx[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        const int c = base + 2 * u + half;
        if (c < n_chunks) {
            const int64_t off = ((int64_t)r * n_max + c) * kHeadDim + 8 * hl;
            mn[u] = __ldcs(reinterpret_cast<const uint4*>(cmin + off));
            mx[u] = __ldcs(reinterpret_cast<const uint4*>(cmax + off));
        } else {
            mn[u] = make_uint4(0, 0, 0, 0);
            mx[u] = mn[u];
        }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        const int c = base + 2 * u + half;
        const float s = quest_half(qv, mn[u], mx[u]);
        if (hl == 0 && c < n_chunks) {
            const bool ok = !valid || valid[(int64_t)r * n_max + c];
            scores[(int64_t)r * n_chunks + c] = ok ? s : -INFINITY;
        }
    }
}

// ----------------------------------------------------------- top-k
constexpr int kTopkThreads = 256;
constexpr int kTopkSmall = 16 * kTopkThreads;  // float rows up to this length take the small-n select

// Stages a float row into shared memory and returns its (min finite, max)
// ordered keys (CTA-wide; ends with a barrier).
__device__ __forceinline__ void stage_row(const float* __restrict__ src, int len, float* sc, uint32_t* lohi,
                                          uint32_t& lo, uint32_t& hi) {
    if (threadIdx.x == 0) {
        lohi[0] = 0xffffffffu;
        lohi[1] = 0u;
    }
    uint32_t l = 0xffffffffu, h = 0u;
    for (int i = threadIdx.x; i < len; i += kTopkThreads) {
        const float v = src[i];
        sc[i] = v;
        const uint32_t kk = ordered_u32(v);
        if (kk > kOrderedNegInf) l = min(l, kk);
        h = max(h, kk);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        l = min(l, __shfl_xor_sync(0xffffffffu, l, o));
        h = max(h, __shfl_xor_sync(0xffffffffu, h, o));
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        atomicMin(&lohi[0], l);
        atomicMax(&lohi[1], h);
    }
    __syncthreads();
    lo = lohi[0];
    hi = lohi[1];
}

template <typename KeyOf>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(KeyOf keyof, int len, int64_t row_stride, int k,
                                                            int64_t* __restrict__ out) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    __shared__ int hist[512];
    __shared__ int misc[8];
    __shared__ int scan[2 * kTopkThreads];
    __shared__ __align__(16) float sc[KeyOf::kFloat ? kTopkSmall : 4];
    __shared__ uint32_t lohi[2];
    const int r = blockIdx.x;
    int64_t* o = out + (int64_t)r * k;
    if (len <= k) {
        for (int i = threadIdx.x; i < k; i += kTopkThreads) o[i] = i < len ? i : -1;
        return;
    }
    if constexpr (KeyOf::kFloat) {
        if (len <= kTopkSmall) {  // same set and order as the general select, fewer barrier phases
            uint32_t lo, hi;
            stage_row(keyof.p + (int64_t)r * row_stride, len, sc, lohi, lo, hi);
            block_topk_small<kTopkThreads>(sc, len, k, lo, hi, hist, misc, scan, [&](int pos, int i) { o[pos] = i; });
            return;
        }
    }
    auto key = [&](int i) { return keyof(r, (int64_t)r * row_stride + i); };
    block_topk<kTopkThreads, KeyOf::kFloat>(key, len, k, hist, misc, scan, [&](int pos, int i) { o[pos] = i; });
}

// The top n_dense positions of one row of density scores written straight as
// the dense mask (mask[r][p] = 1 for the selected p, 0 elsewhere): top-k +
// mask_from_topk in one launch, same selection as topk_kernel.
__global__ void __launch_bounds__(kTopkThreads) topk_mask_kernel(const float* __restrict__ dens, int nk, int n_dense,
                                                                 uint8_t* __restrict__ mask) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    __shared__ int hist[512];
    __shared__ int misc[8];
    __shared__ int scan[2 * kTopkThreads];
    __shared__ __align__(16) float sc[kTopkSmall];
    __shared__ uint32_t lohi[2];
    const int r = blockIdx.x;
    uint8_t* m = mask + (int64_t)r * nk;
    for (int i = threadIdx.x; i < nk; i += kTopkThreads) m[i] = n_dense >= nk ? 1 : 0;
    if (n_dense >= nk) return;
    uint32_t lo, hi;
    stage_row(dens + (int64_t)r * nk, nk, sc, lohi, lo, hi);  // its barriers order the zeroing first
    block_topk_small<kTopkThreads>(sc, nk, n_dense, lo, hi, hist, misc, scan, [&](int, int i) { m[i] = 1; });
}

struct F32Key {
    static constexpr bool kFloat = true;
    const float* p;
    __device__ uint32_t operator()(int, int64_t i) const { return ordered_u32(p[i]); }
};
struct I32Key {
    static constexpr bool kFloat = false;
    const int32_t* p;
    __device__ uint32_t operator()(int, int64_t i) const { return ((uint32_t)p[i]) ^ 0x80000000u; }
};

// ----------------------------------------------------------- density + mask
// One warp per slot; lane l holds dims l, l+32, l+64, l+96 -- the reference's
// 128-thread tree (strides 64, 32 in-lane; 16..1 as xor shuffles) in order.
__global__ void __launch_bounds__(256) density_kernel(const int64_t* __restrict__ ids,
                                                      const uint16_t* __restrict__ cent,
                                                      const uint16_t* __restrict__ raw_q, float* __restrict__ out,
                                                      int rows, int nk, int n_chunks, int n_max) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    const int lane = threadIdx.x & 31;
    const int64_t job = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (job >= (int64_t)rows * nk) return;
    const int r = (int)(job / nk);
    const int64_t cid = ids[job];
    const bool ok = cid >= 0 && cid < n_chunks;
    float p[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
        const uint16_t* c = cent + ((int64_t)r * n_max + cid) * kHeadDim;
        const uint16_t* q = raw_q + (int64_t)r * kHeadDim;
#pragma unroll
        for (int j = 0; j < 4; ++j) p[j] = __fmul_rn(bfbits2f(c[lane + 32 * j]), bfbits2f(q[lane + 32 * j]));
    }
    float b0 = __fadd_rn(p[0], p[2]);  // t and t+64
    float b1 = __fadd_rn(p[1], p[3]);  // t+32 and t+96
    float v = __fadd_rn(b0, b1);       // stride 32
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) out[job] = ok ? v : -1e30f;
}

__global__ void mask_kernel(const int64_t* __restrict__ pos, uint8_t* __restrict__ mask, int n_dense, int nk) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    const int r = blockIdx.x;
    uint8_t* m = mask + (int64_t)r * nk;
    for (int i = threadIdx.x; i < nk; i += blockDim.x) m[i] = 0;
    __syncthreads();
    for (int j = threadIdx.x; j < n_dense; j += blockDim.x) {
        const int64_t p = pos[(int64_t)r * n_dense + j];
        if (p >= 0 && p < nk) m[p] = 1;
    }
}

// ----------------------------------------------------------- KIVI stage-2
// Half-warp per selected chunk, lane = token (as the reference kernel).  The
// dot product runs over dims 0..127 in order: the dequant code*scale + min as
// one bf16 fused multiply-add (one rounding), the product with q rounded to
// bf16, the sum in fp32 -- bit-identical to the kernel the reference builds
// from kivi_qk_dot.cu (checked against its outputs, tests/golden/ref_cuda.npz;
// its source spells the dequant as __hmul2 + __hadd2, which its build fuses).
// The 16 lanes are then sorted by (score desc, token asc) with a bitonic
// network.
__global__ void __launch_bounds__(128) kivi_qk_kernel(const int64_t* __restrict__ ids,
                                                      const uint8_t* __restrict__ dense,
                                                      const int32_t* __restrict__ packed, int n_pk, int pk_ld,
                                                      const uint16_t* __restrict__ cmin,
                                                      const uint16_t* __restrict__ cmax, int n_max,
                                                      const uint16_t* __restrict__ raw_q, int nk, int dense_topk,
                                                      int sparse_topk, float* __restrict__ out_s,
                                                      int64_t* __restrict__ out_i, int64_t out_ld) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    __shared__ __align__(16) uint16_t s_q[kHeadDim];
    __shared__ __align__(16) uint32_t s_mn[8][kHeadDim / 2];
    __shared__ __align__(16) uint32_t s_sc[8][kHeadDim / 2];
    const int r = blockIdx.y;
    const int lane = threadIdx.x & 31, t = lane & 15, sub = lane >> 4, warp = threadIdx.x >> 5;
    const int local = warp * 2 + sub;
    const int slot = blockIdx.x * 8 + local;
    for (int i = threadIdx.x; i < kHeadDim; i += blockDim.x) s_q[i] = raw_q[(int64_t)r * kHeadDim + i];
    const bool valid_slot = slot < nk;
    int64_t cid = 0;
    bool is_dense = false;
    if (valid_slot) {
        cid = ids[(int64_t)r * nk + slot];
        is_dense = dense[(int64_t)r * nk + slot] != 0;
    }
    const bool in_range = valid_slot && cid >= 0 && cid < n_pk;
    if (in_range) {
        // lane t prepares dims [8t, 8t+8): min and scale as bf16 pairs
        const uint16_t* mn = cmin + ((int64_t)r * n_max + cid) * kHeadDim + 8 * t;
        const uint16_t* mx = cmax + ((int64_t)r * n_max + cid) * kHeadDim + 8 * t;
        const uint4 a = *reinterpret_cast<const uint4*>(mn);
        const uint4 b = *reinterpret_cast<const uint4*>(mx);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint16_t s0 = kivi_scale_bits((uint16_t)(aw[j] & 0xffff), (uint16_t)(bw[j] & 0xffff));
            const uint16_t s1 = kivi_scale_bits((uint16_t)(aw[j] >> 16), (uint16_t)(bw[j] >> 16));
            s_mn[local][4 * t + j] = aw[j];
            s_sc[local][4 * t + j] = (uint32_t)s0 | ((uint32_t)s1 << 16);
        }
    }
    __syncthreads();
    float score = -1e30f;
    if (in_range) {
        const int32_t* pk = packed + ((int64_t)r * pk_ld + cid) * (kWords * kChunk) + t;
        const uint32_t* q2 = reinterpret_cast<const uint32_t*>(s_q);
        float acc = 0.0f;
#pragma unroll 4
        for (int i = 0; i < kWords; ++i) {
            const uint32_t w = (uint32_t)__ldg(pk + i * kChunk);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const __nv_bfloat162 c2 = codes2_to_bf162(w >> (8 * p), w >> (8 * p + 4));
                const __nv_bfloat162 k2 =
                    __hfma2(c2, bits_bf162(s_sc[local][4 * i + p]), bits_bf162(s_mn[local][4 * i + p]));
                const __nv_bfloat162 pr = __hmul2_rn(k2, bits_bf162(q2[4 * i + p]));
                acc = __fadd_rn(acc, __low2float(pr));
                acc = __fadd_rn(acc, __high2float(pr));
            }
        }
        score = acc;
    }
    int tok = (int)cid * kChunk + t;
    // bitonic sort over 16 lanes: descending by score, ascending by token on ties
#pragma unroll
    for (int kk = 2; kk <= kChunk; kk <<= 1) {
#pragma unroll
        for (int j = kk >> 1; j >= 1; j >>= 1) {
            const float os = __shfl_xor_sync(0xffffffffu, score, j);
            const int ot = __shfl_xor_sync(0xffffffffu, tok, j);
            const bool desc = (t & kk) == 0;
            const bool lower = (t & j) == 0;
            const bool other_first = (os > score) || (os == score && ot < tok);
            const bool want_first = (desc == lower);
            if (want_first ? other_first : !other_first && !(os == score && ot == tok)) {
                score = os;
                tok = ot;
            }
        }
    }
    if (valid_slot) {
        const int eff = is_dense ? dense_topk : sparse_topk;
        const int64_t o = (int64_t)r * out_ld + (int64_t)slot * kChunk + t;
        out_s[o] = t < eff ? score : -1e30f;
        out_i[o] = t < eff ? (int64_t)tok : 0;
    }
}

// ----------------------------------------------------------- global top-k + gather + concat
__global__ void __launch_bounds__(kTopkThreads) topk_gather_concat_kernel(const float* __restrict__ scores,
                                                                          const int64_t* __restrict__ lut,
                                                                          const int64_t* __restrict__ skipped,
                                                                          int64_t sk_ld,
                                                                          int64_t* __restrict__ out, int L, int k,
                                                                          int sk, int64_t out_ld) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    __shared__ int hist[512];
    __shared__ int misc[8];
    __shared__ int scan[2 * kTopkThreads];
    __shared__ __align__(16) float sc[kTopkSmall];
    __shared__ int pos_s[kTopkSmall];
    __shared__ uint32_t lohi[2];
    const int r = blockIdx.x;
    int64_t* o = out + (int64_t)r * out_ld;
    const int64_t* lu = lut + (int64_t)r * L;
    for (int i = threadIdx.x; i < sk; i += kTopkThreads) o[k + i] = skipped[(int64_t)r * sk_ld + i];
    if (L <= k) {
        for (int i = threadIdx.x; i < k; i += kTopkThreads) o[i] = i < L ? lu[i] : 0;
        return;
    }
    const float* s = scores + (int64_t)r * L;
    if (L <= kTopkSmall) {
        uint32_t lo, hi;
        stage_row(s, L, sc, lohi, lo, hi);
        block_topk_small<kTopkThreads>(sc, L, k, lo, hi, hist, misc, scan, [&](int pos, int i) { pos_s[pos] = i; });
        // the selected positions, then the ids as independent loads
        for (int p = threadIdx.x; p < k; p += kTopkThreads) o[p] = lu[pos_s[p]];
        return;
    }
    auto key = [&](int i) { return ordered_u32(s[i]); };
    block_topk<kTopkThreads, true>(key, L, k, hist, misc, scan, [&](int pos, int i) { o[pos] = lu[i]; });
}

}  // namespace zkv

using namespace zkv;


extern "C" int zkv_quest_score(const void* raw_q, const void* chunk_min, const void* chunk_max, const uint8_t* valid,
                               float* scores, int rows, int n_chunks, int n_max, void* stream) {
    if (rows < 0 || n_chunks < 0 || n_chunks > n_max || rows > 65535) return ZKV_ERR_ARG;
    if (rows == 0 || n_chunks == 0) return ZKV_OK;
    if (((uintptr_t)raw_q & 15) || ((uintptr_t)chunk_min & 15) || ((uintptr_t)chunk_max & 15)) return ZKV_ERR_ALIGN;
    constexpr int U = 4;
    dim3 grid((n_chunks + 8 * 2 * U - 1) / (8 * 2 * U), rows);
    return launch_pdl_kernel(quest_score_kernel<U>, dim3(grid), dim3(256), 0, (cudaStream_t)stream,
                             (const uint16_t*)raw_q, (const uint16_t*)chunk_min,
                             (const uint16_t*)chunk_max, valid, scores, n_chunks,
                             n_max, (const uint16_t*)nullptr, 0, (uint16_t*)nullptr);
}

int quest_score_gqa_into(const void* q, int G, const void* chunk_min, const void* chunk_max, const uint8_t* valid,
                         float* scores, void* raw_q_out, int rows, int n_chunks, int n_max, cudaStream_t stream) {
    if (!q || G < 1 || G > 64 || rows < 0 || n_chunks < 0 || n_chunks > n_max || rows > 65535) return ZKV_ERR_ARG;
    if (rows == 0 || n_chunks == 0) return ZKV_OK;
    if (((uintptr_t)q & 15) || ((uintptr_t)chunk_min & 15) || ((uintptr_t)chunk_max & 15) ||
        ((uintptr_t)raw_q_out & 15))
        return ZKV_ERR_ALIGN;
    constexpr int U = 4;
    dim3 grid((n_chunks + 8 * 2 * U - 1) / (8 * 2 * U), rows);
    return launch_pdl_kernel(quest_score_kernel<U>, dim3(grid), dim3(256), 0, stream,
                             nullptr, (const uint16_t*)chunk_min, (const uint16_t*)chunk_max,
                             valid, scores, n_chunks, n_max, (const uint16_t*)q, G,
                             (uint16_t*)raw_q_out);
}

extern "C" int zkv_quest_score_gqa(const void* q, int G, const void* chunk_min, const void* chunk_max,
                                   const uint8_t* valid, float* scores, int rows, int n_chunks, int n_max,
                                   void* stream) {
    return quest_score_gqa_into(q, G, chunk_min, chunk_max, valid, scores, nullptr, rows, n_chunks, n_max,
                                (cudaStream_t)stream);
}

extern "C" int zkv_topk_f32(const float* scores, int rows, int len, int64_t row_stride, int k, int64_t* out,
                            void* stream) {
    if (rows < 0 || len < 0 || k <= 0 || row_stride < len) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    return launch_pdl_kernel(topk_kernel<F32Key>, dim3(rows), dim3(kTopkThreads), 0, (cudaStream_t)stream,
                             F32Key{scores}, len, row_stride, k, out);
}

extern "C" int zkv_topk_i32(const int32_t* vals, int rows, int len, int64_t row_stride, int k, int64_t* out,
                            void* stream) {
    if (rows < 0 || len < 0 || k <= 0 || row_stride < len) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    return launch_pdl_kernel(topk_kernel<I32Key>, dim3(rows), dim3(kTopkThreads), 0, (cudaStream_t)stream,
                             I32Key{vals}, len, row_stride, k, out);
}

extern "C" int zkv_chunk_density(const int64_t* chunk_ids, const void* centroid, const void* raw_q, float* out,
                                 int rows, int nk, int n_chunks, int n_max, void* stream) {
    if (rows < 0 || nk < 0 || n_chunks > n_max) return ZKV_ERR_ARG;
    if (rows == 0 || nk == 0) return ZKV_OK;
    const int64_t jobs = (int64_t)rows * nk;
    return launch_pdl_kernel(density_kernel, dim3((unsigned)((jobs + 7) / 8)), dim3(256), 0, (cudaStream_t)stream,
                             chunk_ids, (const uint16_t*)centroid, (const uint16_t*)raw_q, out, rows, nk, n_chunks, n_max);
}

int topk_mask_launch(const float* dens, int rows, int nk, int n_dense, uint8_t* mask, cudaStream_t stream) {
    if (rows < 0 || nk < 1 || n_dense < 1 || nk > kTopkSmall) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    return launch_pdl_kernel(topk_mask_kernel, dim3(rows), dim3(kTopkThreads), 0, stream, dens, nk, n_dense, mask);
}

extern "C" int zkv_mask_from_topk(const int64_t* positions, uint8_t* mask, int rows, int n_dense, int nk,
                                  void* stream) {
    if (rows < 0 || n_dense < 0 || nk < 0) return ZKV_ERR_ARG;
    if (rows == 0 || nk == 0) return ZKV_OK;
    return launch_pdl_kernel(mask_kernel, dim3(rows), dim3(256), 0, (cudaStream_t)stream, positions, mask, n_dense, nk);
}

extern "C" int zkv_kivi_qk(const int64_t* chunk_ids, const uint8_t* dense_mask, const int32_t* packed, int n_pk,
                           int pk_ld, const void* chunk_min, const void* chunk_max, int n_max, const void* raw_q, int rows,
                           int nk, int dense_topk, int sparse_topk, float* out_scores, int64_t* out_idx,
                           int64_t out_ld, void* stream) {
    if (rows < 0 || nk < 0 || n_pk > n_max || n_pk > pk_ld || rows > 65535) return ZKV_ERR_ARG;
    if (dense_topk < 1 || dense_topk > kChunk || sparse_topk < 1 || sparse_topk > kChunk) return ZKV_ERR_ARG;
    if (out_ld < (int64_t)nk * kChunk) return ZKV_ERR_ARG;
    if (rows == 0 || nk == 0) return ZKV_OK;
    if (((uintptr_t)chunk_min & 15) || ((uintptr_t)chunk_max & 15) || ((uintptr_t)raw_q & 15)) return ZKV_ERR_ALIGN;
    dim3 grid((nk + 7) / 8, rows);
    return launch_pdl_kernel(kivi_qk_kernel, dim3(grid), dim3(128), 0, (cudaStream_t)stream,
                             chunk_ids, dense_mask, packed, n_pk, pk_ld,
                             (const uint16_t*)chunk_min, (const uint16_t*)chunk_max,
                             n_max, (const uint16_t*)raw_q, nk, dense_topk, sparse_topk,
                             out_scores, out_idx, out_ld);
}

extern "C" int zkv_topk_gather_concat(const float* scores, const int64_t* lut, const int64_t* skipped,
                                      int64_t sk_ld, int64_t* out, int rows, int L, int k, int sk, int64_t out_ld,
                                      void* stream) {
    if (rows < 0 || L < 0 || k <= 0 || sk < 0 || out_ld < (int64_t)k + sk || (sk > 0 && sk_ld < sk)) return ZKV_ERR_ARG;
    if (sk > 0 && !skipped) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    return launch_pdl_kernel(topk_gather_concat_kernel, dim3(rows), dim3(kTopkThreads), 0, (cudaStream_t)stream,
                             scores, lut, skipped, sk_ld, out, L,
                             k, sk, out_ld);
}
