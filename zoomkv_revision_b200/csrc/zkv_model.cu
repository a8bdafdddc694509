// zkv_model.cu -- element-wise kernels of the decode-loop caller (the
// benchmark's config 4), so that a Qwen3 decoder layer between two attention
// calls is 8 launches: RMSNorm, the QKV GEMM, per-head q/k RMSNorm + RoPE
// (this file), the o_proj GEMM with the residual in its epilogue, RMSNorm,
// the gate/up GEMM, SiLU-and-multiply (this file), the down GEMM with the
// residual.  The GEMMs are library calls made by the caller.
//
// The reference runs the same steps through flashinfer (rmsnorm,
// apply_rope_with_cos_sin_cache_inplace, silu_and_mul; model_hub/qwen.py:
// 481-612); these are this package's own kernels with fp32 arithmetic.
#include <algorithm>

#include "zkv_common.cuh"

namespace zkv {
namespace model {

constexpr int kNormThreads = 256;

// One CTA per row: y = bf16(x * rsqrt(mean(x^2) + eps) * w), fp32 inside.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const uint16_t* __restrict__ x,
                                                               const uint16_t* __restrict__ w,
                                                               uint16_t* __restrict__ y, int dim, float eps) {
    const int r = blockIdx.x;
    const uint16_t* xr = x + (int64_t)r * dim;
    uint16_t* yr = y + (int64_t)r * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += kNormThreads) {
        const float v = bfbits2f(xr[i]);
        ss += v * v;
    }
    __shared__ float red[kNormThreads / 32];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
    const float inv = rsqrtf(tot / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += kNormThreads)
        yr[i] = f2bfbits(bfbits2f(xr[i]) * inv * bfbits2f(w[i]));
}

// One warp per (row, head) of qkv [rows][(hq + 2 hkv) * 128]: q and k heads
// get RMSNorm over the head (weights qw / kw) and the rotate-half RoPE at
// position *pos (cos / sin tables [max_pos][64]); v heads are copied.
// Lane l holds dims l, l + 32 (first half) and l + 64, l + 96 (their
// rotation partners).
__global__ void qk_norm_rope_kernel(const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ qw,
                                    const uint16_t* __restrict__ kw, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, const int64_t* __restrict__ pos, int hq,
                                    int hkv, float eps, uint16_t* __restrict__ q, uint16_t* __restrict__ k,
                                    uint16_t* __restrict__ v, int rows) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nh = hq + 2 * hkv;
    if (warp >= rows * nh) return;
    const int r = warp / nh, h = warp % nh;
    const uint16_t* src = qkv + ((int64_t)r * nh + h) * kHeadDim;
    float a[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) a[j] = bfbits2f(src[lane + 32 * j]);
    if (h >= hq + hkv) {  // value head: copy
        uint16_t* dst = v + ((int64_t)r * hkv + (h - hq - hkv)) * kHeadDim;
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = src[lane + 32 * j];
        return;
    }
    const bool isq = h < hq;
    const uint16_t* wt = isq ? qw : kw;
    float ss = a[0] * a[0] + a[1] * a[1] + a[2] * a[2] + a[3] * a[3];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss / (float)kHeadDim + eps);
#pragma unroll
    for (int j = 0; j < 4; ++j) a[j] = bfbits2f(f2bfbits(a[j] * inv * bfbits2f(wt[lane + 32 * j])));
    const int64_t p = *pos;
    float out[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int d = lane + 32 * j;  // first-half dim; partner d + 64
        const float c = cos_t[p * (kHeadDim / 2) + d], s = sin_t[p * (kHeadDim / 2) + d];
        out[j] = a[j] * c - a[j + 2] * s;
        out[j + 2] = a[j + 2] * c + a[j] * s;
    }
    uint16_t* dst = isq ? q + ((int64_t)r * hq + h) * kHeadDim : k + ((int64_t)r * hkv + (h - hq)) * kHeadDim;
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = f2bfbits(out[j]);
}

// out[r][i] = bf16(silu(g) * u), g = gu[r][i], u = gu[r][ffn + i], fp32 inside.
__global__ void silu_mul_kernel(const uint16_t* __restrict__ gu, uint16_t* __restrict__ out, int rows, int ffn) {
    const int64_t n = (int64_t)rows * ffn;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / ffn, c = i - r * ffn;
        const float g = bfbits2f(gu[r * 2 * ffn + c]), u = bfbits2f(gu[r * 2 * ffn + ffn + c]);
        out[i] = f2bfbits(g / (1.f + __expf(-g)) * u);
    }
}

}  // namespace model
}  // namespace zkv

using namespace zkv;

extern "C" int zkv_rmsnorm(const void* x, const void* w, void* y, int rows, int dim, float eps, void* stream) {
    if (!x || !w || !y || rows < 0 || dim < 1) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    model::rmsnorm_kernel<<<rows, model::kNormThreads, 0, (cudaStream_t)stream>>>(
        (const uint16_t*)x, (const uint16_t*)w, (uint16_t*)y, dim, eps);
    return launch_status();
}

extern "C" int zkv_qk_norm_rope(const void* qkv, const void* q_norm, const void* k_norm, const float* cos_t,
                                const float* sin_t, const int64_t* pos, int rows, int hq, int hkv, float eps,
                                void* q, void* k, void* v, void* stream) {
    if (!qkv || !q_norm || !k_norm || !cos_t || !sin_t || !pos || !q || !k || !v || rows < 0 || hq < 1 || hkv < 1)
        return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    const int64_t warps = (int64_t)rows * (hq + 2 * hkv);
    const int threads = 256;
    model::qk_norm_rope_kernel<<<(unsigned)((warps * 32 + threads - 1) / threads), threads, 0,
                                  (cudaStream_t)stream>>>((const uint16_t*)qkv, (const uint16_t*)q_norm,
                                                          (const uint16_t*)k_norm, cos_t, sin_t, pos, hq, hkv, eps,
                                                          (uint16_t*)q, (uint16_t*)k, (uint16_t*)v, rows);
    return launch_status();
}

extern "C" int zkv_silu_mul(const void* gu, void* out, int rows, int ffn, void* stream) {
    if (!gu || !out || rows < 0 || ffn < 1) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    const int threads = 256;
    const int64_t n = (int64_t)rows * ffn;
    const unsigned blocks = (unsigned)std::min<int64_t>((n + threads - 1) / threads, 148 * 16);
    model::silu_mul_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>((const uint16_t*)gu, (uint16_t*)out, rows,
                                                                          ffn);
    return launch_status();
}
