// zkv_encode.cu -- prefill / flush encoders.
//
// zkv_kivi_encode: per full chunk of 16 post-RoPE keys, the per-channel
// min / max / mean (Quest metadata) and the KIVI 4-bit codes packed 8 per
// int32 along head_dim, stored chunk-major [chunk][word][token] (the
// reference's A-1 layout).  Restates polar_cache._compute_and_store_chunk_minmax
// + _kivi_pack_chunks (cache_hub/polar_cache_quest_density_single_layer_kivi.py
// :2119-2141, :1965-2020) bit for bit.
//
// zkv_vquant_encode: per-token 4-bit values, group 32 along head_dim, in the
// page-transposed layout the page-mode attention reads.
#include "zkv_common.cuh"

namespace zkv {

// One warp per (row, chunk); lane l owns dims [4l, 4l+4).  Chunks per block
// = 8 warps; grid-stride over chunks.
__global__ void __launch_bounds__(256) kivi_encode_kernel(const uint16_t* __restrict__ keys, int64_t ld_row,
                                                          int rows, int n_chunks, int chunk_start, int n_max,
                                                          uint16_t* __restrict__ cmin, uint16_t* __restrict__ cmax,
                                                          uint16_t* __restrict__ cent, uint8_t* __restrict__ valid,
                                                          int32_t* __restrict__ packed, uint16_t* __restrict__ kscale) {
    const int lane = threadIdx.x & 31;
    const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int n_warps = gridDim.x * (blockDim.x >> 5);
    const int64_t total = (int64_t)rows * n_chunks;
    for (int64_t job = warp_global; job < total; job += n_warps) {
        const int r = (int)(job / n_chunks);
        const int c = (int)(job % n_chunks);
        const uint16_t* src = keys + (int64_t)r * ld_row + (int64_t)c * kChunk * kHeadDim + 4 * lane;
        uint16_t v[kChunk][4];
#pragma unroll
        for (int t = 0; t < kChunk; ++t) {
            uint2 u = *reinterpret_cast<const uint2*>(src + (int64_t)t * kHeadDim);
            v[t][0] = (uint16_t)(u.x & 0xffff);
            v[t][1] = (uint16_t)(u.x >> 16);
            v[t][2] = (uint16_t)(u.y & 0xffff);
            v[t][3] = (uint16_t)(u.y >> 16);
        }
        uint16_t mn[4], mx[4], ce[4], sc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint16_t lo = v[0][j], hi = v[0][j];
            float sum = 0.0f;
#pragma unroll
            for (int t = 0; t < kChunk; ++t) {
                if (bfbits2f(v[t][j]) < bfbits2f(lo)) lo = v[t][j];
                if (bfbits2f(v[t][j]) > bfbits2f(hi)) hi = v[t][j];
                sum = __fadd_rn(sum, bfbits2f(v[t][j]));
            }
            mn[j] = lo;
            mx[j] = hi;
            ce[j] = f2bfbits(__fdiv_rn(sum, (float)kChunk));
            sc[j] = kivi_scale_bits(lo, hi);
        }
        const int64_t mrow = ((int64_t)r * n_max + chunk_start + c) * kHeadDim + 4 * lane;
        *reinterpret_cast<uint2*>(cmin + mrow) =
            make_uint2((uint32_t)mn[0] | ((uint32_t)mn[1] << 16), (uint32_t)mn[2] | ((uint32_t)mn[3] << 16));
        *reinterpret_cast<uint2*>(cmax + mrow) =
            make_uint2((uint32_t)mx[0] | ((uint32_t)mx[1] << 16), (uint32_t)mx[2] | ((uint32_t)mx[3] << 16));
        if (cent)
            *reinterpret_cast<uint2*>(cent + mrow) =
                make_uint2((uint32_t)ce[0] | ((uint32_t)ce[1] << 16), (uint32_t)ce[2] | ((uint32_t)ce[3] << 16));
        if (kscale)
            *reinterpret_cast<uint2*>(kscale + mrow) =
                make_uint2((uint32_t)sc[0] | ((uint32_t)sc[1] << 16), (uint32_t)sc[2] | ((uint32_t)sc[3] << 16));
        // codes: lane holds 4 dims = half a word; pair lanes (2w, 2w+1) form word w.
        int32_t* pk = packed + ((int64_t)r * n_max + chunk_start + c) * (kWords * kChunk);
#pragma unroll
        for (int t = 0; t < kChunk; ++t) {
            uint32_t half = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) half |= kivi_code(v[t][j], mn[j], sc[j]) << (4 * j);
            uint32_t other = __shfl_xor_sync(0xffffffffu, half, 1);
            if ((lane & 1) == 0) pk[(lane >> 1) * kChunk + t] = (int32_t)(half | (other << 16));
        }
        if (valid && lane == 0) valid[(int64_t)r * n_max + chunk_start + c] = 1;
    }
}

// One warp per (row, token); lane l owns dims [4l, 4l+4); a 32-dim group is
// 8 lanes.  Output page layout: vcodes_t[page][dim][2] (word w = tokens
// 8w..8w+7 of that dim), vmeta[page][scale|zero][group][token].
__global__ void __launch_bounds__(256) vquant_kernel(const uint16_t* __restrict__ values, int64_t ld_row, int rows,
                                                     int n_tokens, int tok_start, int n_pages,
                                                     int32_t* __restrict__ vcodes_t, uint16_t* __restrict__ vmeta) {
    const int lane = threadIdx.x & 31;
    const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int n_warps = gridDim.x * (blockDim.x >> 5);
    const int64_t total = (int64_t)rows * n_tokens;
    for (int64_t job = warp_global; job < total; job += n_warps) {
        const int r = (int)(job / n_tokens);
        const int tk = tok_start + (int)(job % n_tokens);
        const uint16_t* src = values + (int64_t)r * ld_row + (int64_t)(job % n_tokens) * kHeadDim + 4 * lane;
        uint2 u = *reinterpret_cast<const uint2*>(src);
        uint16_t v[4] = {(uint16_t)(u.x & 0xffff), (uint16_t)(u.x >> 16), (uint16_t)(u.y & 0xffff),
                         (uint16_t)(u.y >> 16)};
        uint16_t lo = v[0], hi = v[0];
#pragma unroll
        for (int j = 1; j < 4; ++j) {
            if (bfbits2f(v[j]) < bfbits2f(lo)) lo = v[j];
            if (bfbits2f(v[j]) > bfbits2f(hi)) hi = v[j];
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
            uint16_t olo = (uint16_t)__shfl_xor_sync(0xffffffffu, (uint32_t)lo, off);
            uint16_t ohi = (uint16_t)__shfl_xor_sync(0xffffffffu, (uint32_t)hi, off);
            if (bfbits2f(olo) < bfbits2f(lo)) lo = olo;
            if (bfbits2f(ohi) > bfbits2f(hi)) hi = ohi;
        }
        const uint16_t sc = kivi_scale_bits(lo, hi);
        const int page = tk / kChunk, t = tk % kChunk;
        const int64_t pbase = (int64_t)r * n_pages + page;
        int32_t* vc = vcodes_t + pbase * (kHeadDim * 2);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int d = 4 * lane + j;
            const uint32_t code = kivi_code(v[j], lo, sc);
            // nibble (t & 7) of word (t >> 3) of dim d; tokens of one page are
            // encoded by different warps, so merge with atomicOr after the
            // word was cleared by the page's first token.
            atomicOr(reinterpret_cast<unsigned int*>(vc + d * 2 + (t >> 3)), code << (4 * (t & 7)));
        }
        if ((lane & 7) == 0) {
            const int g = lane >> 3;
            uint16_t* vm = vmeta + pbase * (2 * kVGroups * kChunk);
            vm[(0 * kVGroups + g) * kChunk + t] = sc;
            vm[(1 * kVGroups + g) * kChunk + t] = lo;
        }
    }
}

__global__ void clear_pages_kernel(int32_t* __restrict__ vcodes_t, int rows, int n_pages, int page_lo, int page_hi) {
    const int per = (page_hi - page_lo) * kHeadDim * 2;
    const int64_t total = (int64_t)rows * per;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / per);
        const int o = (int)(i % per);
        vcodes_t[((int64_t)r * n_pages + page_lo) * kHeadDim * 2 + o] = 0;
    }
}

static int grid_for(int64_t jobs, int per_block) {
    int64_t g = (jobs + per_block - 1) / per_block;
    if (g > 148 * 16) g = 148 * 16;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace zkv

using namespace zkv;

extern "C" int zkv_kivi_encode(const void* keys, int64_t keys_ld_row, int rows, int n_chunks, int chunk_start,
                               int n_max, void* chunk_min, void* chunk_max, void* centroid, uint8_t* valid,
                               int32_t* packed, void* kscale, void* stream) {
    if (rows < 0 || n_chunks < 0 || chunk_start < 0 || chunk_start + n_chunks > n_max) return ZKV_ERR_ARG;
    if (rows == 0 || n_chunks == 0) return ZKV_OK;
    if (!keys || !chunk_min || !chunk_max || !packed) return ZKV_ERR_ARG;
    if (((uintptr_t)keys & 7) || (keys_ld_row & 3) || ((uintptr_t)chunk_min & 7) || ((uintptr_t)chunk_max & 7) ||
        (centroid && ((uintptr_t)centroid & 7)) || (kscale && ((uintptr_t)kscale & 7)) || ((uintptr_t)packed & 3))
        return ZKV_ERR_ALIGN;
    const int64_t jobs = (int64_t)rows * n_chunks;
    kivi_encode_kernel<<<grid_for(jobs, 8), 256, 0, (cudaStream_t)stream>>>(
        (const uint16_t*)keys, keys_ld_row, rows, n_chunks, chunk_start, n_max, (uint16_t*)chunk_min,
        (uint16_t*)chunk_max, (uint16_t*)centroid, valid, packed, (uint16_t*)kscale);
    return cudaGetLastError() == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH;
}

extern "C" int zkv_vquant_encode(const void* values, int64_t values_ld_row, int rows, int n_tokens, int tok_start,
                                 int n_pages, int32_t* vcodes_t, void* vmeta, void* stream) {
    if (rows < 0 || n_tokens < 0 || tok_start < 0 || tok_start + n_tokens > n_pages * kChunk) return ZKV_ERR_ARG;
    if (rows == 0 || n_tokens == 0) return ZKV_OK;
    if (!values || !vcodes_t || !vmeta) return ZKV_ERR_ARG;
    if (((uintptr_t)values & 7) || (values_ld_row & 3) || ((uintptr_t)vcodes_t & 3) || ((uintptr_t)vmeta & 1))
        return ZKV_ERR_ALIGN;
    cudaStream_t s = (cudaStream_t)stream;
    // Pages whose first token is being written start from cleared words.
    const int first_new_page = (tok_start + kChunk - 1) / kChunk;
    const int last_page = (tok_start + n_tokens - 1) / kChunk + 1;
    if (tok_start % kChunk == 0 || first_new_page < last_page) {
        const int lo = (tok_start % kChunk == 0) ? tok_start / kChunk : first_new_page;
        if (lo < last_page) {
            const int64_t n = (int64_t)rows * (last_page - lo) * kHeadDim * 2;
            clear_pages_kernel<<<grid_for(n, 256), 256, 0, s>>>(vcodes_t, rows, n_pages, lo, last_page);
        }
    }
    const int64_t jobs = (int64_t)rows * n_tokens;
    vquant_kernel<<<grid_for(jobs, 8), 256, 0, s>>>((const uint16_t*)values, values_ld_row, rows, n_tokens, tok_start,
                                                   n_pages, vcodes_t, (uint16_t*)vmeta);
    return cudaGetLastError() == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH;
}
