// zkv_rabitq.cu -- ParisKV / RaBitQ retrieval kernels (sm_100a).
//
//  * rq_encode_kernel      one warp per key: norm, SRHT (sign flip + fp32
//                          Walsh-Hadamard butterflies in the reference
//                          fallback's order), 1-bit sign codes, 3-bit
//                          magnitudes, block weights, the popcount factor and
//                          a shared-memory bucket histogram per CTA.
//  * rq_query_kernel       one warp per row: GQA mean + the same rotation,
//                          plus the 4-bit query of the popcount estimator.
//  * collision_topk_kernel a cluster of CTAs per row: every CTA orders the
//                          256 buckets of each of the 16 blocks (warp bitonic
//                          sort), turns bucket ranks into tier-hit weights,
//                          counts its key range into shared memory and the
//                          cluster agrees on the top-C threshold through
//                          distributed shared memory; ordered compaction.
//  * rerank4_kernel        RaBitQ 4-bit scores as chains of bf16 fused
//                          multiply-adds (the production rerank.cu as
//                          built), then block top-F.
//  * coarse2bit_kernel     six popcounts per block per key.
//  * popcount_topk_kernel  1-bit x 4-bit popcount estimates, block top-K,
//                          then exact fp32 inner products of the K winners.
// All fp32 arithmetic that must match the CPU restatement uses the _rn
// intrinsics (no contraction) in the restatement's order.
#include "zkv_common.cuh"

namespace zkv {
namespace rq {

constexpr int kB = 16, kM = 8, kK = 256;
constexpr float kInvSqrtD = 0.0883883461356163f;  // (float)(1 / sqrt(128))
constexpr int kMaxTiers = 8;
constexpr int kCntBins = 16 * kMaxTiers + 1;

// bf16 magnitude thresholds / centres of ParisKV (polar_cache.py:267-270)
__constant__ uint32_t c_thr_bits[7] = {0x3DAD0000u, 0x3E2E0000u, 0x3E840000u, 0x3EB30000u,
                                       0x3EE60000u, 0x3F0F0000u, 0x3F310000u};
__constant__ uint32_t c_cen_bits[8] = {0x3D2C0000u, 0x3E020000u, 0x3E5A0000u, 0x3E9B0000u,
                                       0x3ECB0000u, 0x3F000000u, 0x3F1E0000u, 0x3F430000u};

__device__ __forceinline__ float rbf(float x) { return bfbits2f(f2bfbits(x)); }

// (min finite, max) ordered key of sc[0..n) into range[0..1] (CTA-wide;
// ends with a barrier).
template <int NT>
__device__ __forceinline__ void block_key_range(const float* sc, int n, uint32_t* range) {
    uint32_t lo = 0xffffffffu, hi = 0u;
    for (int i = threadIdx.x; i < n; i += NT) {
        const uint32_t k = ordered_u32(sc[i]);
        if (k > kOrderedNegInf) lo = min(lo, k);
        hi = max(hi, k);
    }
    if (threadIdx.x == 0) {
        range[0] = 0xffffffffu;
        range[1] = 0u;
    }
    __syncthreads();
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMin(range, lo);
        atomicMax(range + 1, hi);
    }
    __syncthreads();
}

// Folds every thread's (min, max) ordered key into rank 0's lohi[0..1]
// (one remote atomic pair per warp).
__device__ __forceinline__ void cluster_fold_range(cg::cluster_group& cluster, uint32_t* lohi, uint32_t lo,
                                                   uint32_t hi) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if ((threadIdx.x & 31) == 0) {
        uint32_t* r = cluster.map_shared_rank(lohi, 0);
        atomicMin(r, lo);
        atomicMax(r + 1, hi);
    }
}

__device__ __forceinline__ int warp_excl_scan(int v) {
    const int lane = threadIdx.x & 31;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
    }
    return x - v;
}

__device__ __forceinline__ float warp_sum_tree(float v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

__device__ __forceinline__ float sum4(float a, float b, float c, float d) { return __fadd_rn(__fadd_rn(a, b), __fadd_rn(c, d)); }

// Normalise (bf16 norm, bf16 division), flip by the SRHT signs and apply the
// 128-point Walsh-Hadamard transform in fp32 (butterfly strides 1..64, lane l
// owns dims 4l..4l+3), times 1/sqrt(128), rounded to bf16.  Returns the bf16
// norm bits; y[] receives the rotated bf16 values (as floats).
__device__ __forceinline__ uint16_t rotate128(const float (&x)[4], const float (&sg)[4], float (&y)[4]) {
    const int lane = threadIdx.x & 31;
    float s = sum4(__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1]), __fmul_rn(x[2], x[2]), __fmul_rn(x[3], x[3]));
    s = warp_sum_tree(s);
    const uint16_t nb = f2bfbits(__fsqrt_rn(s));
    const float nf = fmaxf(bfbits2f(nb), rbf(1e-8f));
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(rbf(__fdiv_rn(x[i], nf)), sg[i]);
    {   // stride 1
        const float a0 = v[0], b0 = v[1], a1 = v[2], b1 = v[3];
        v[0] = __fadd_rn(a0, b0); v[1] = __fsub_rn(a0, b0);
        v[2] = __fadd_rn(a1, b1); v[3] = __fsub_rn(a1, b1);
    }
    {   // stride 2
        const float a0 = v[0], b0 = v[2], a1 = v[1], b1 = v[3];
        v[0] = __fadd_rn(a0, b0); v[2] = __fsub_rn(a0, b0);
        v[1] = __fadd_rn(a1, b1); v[3] = __fsub_rn(a1, b1);
    }
#pragma unroll
    for (int m = 1; m <= 16; m <<= 1) {   // strides 4..64 across lanes
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float p = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = (lane & m) ? __fsub_rn(p, v[i]) : __fadd_rn(v[i], p);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = rbf(__fmul_rn(v[i], kInvSqrtD));
    return nb;
}

__device__ __forceinline__ void load_bf16x4(const uint16_t* p, float (&x)[4]) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    x[0] = bfbits2f((uint16_t)(r.x & 0xffffu));
    x[1] = bfbits2f((uint16_t)(r.x >> 16));
    x[2] = bfbits2f((uint16_t)(r.y & 0xffffu));
    x[3] = bfbits2f((uint16_t)(r.y >> 16));
}

// ------------------------------------------------------------------ encode
constexpr int kEncTok = 512;  // keys per CTA (64 per warp)

__global__ void __launch_bounds__(256) rq_encode_kernel(const uint16_t* __restrict__ keys, int64_t ld_row, int n_tok,
                                                        int tok_start, const uint16_t* __restrict__ signs,
                                                        const zkv_rq_layout L) {
    __shared__ int hist_s[kB * kK];
    const int row = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool do_hist = L.hist != nullptr;
    if (do_hist)
        for (int i = threadIdx.x; i < kB * kK; i += 256) hist_s[i] = 0;
    __syncthreads();
    float sg[4];
    load_bf16x4(signs + 4 * lane, sg);
    float thr[7], cen[8];
#pragma unroll
    for (int i = 0; i < 7; ++i) thr[i] = __uint_as_float(c_thr_bits[i]);
#pragma unroll
    for (int i = 0; i < 8; ++i) cen[i] = __uint_as_float(c_cen_bits[i]);
    const float eps8 = rbf(1e-8f);
    const int t_end = min(n_tok, (int)(blockIdx.x + 1) * kEncTok);
    for (int t = blockIdx.x * kEncTok + warp; t < t_end; t += 8) {
        float x[4], y[4];
        load_bf16x4(keys + row * ld_row + (int64_t)t * kHeadDim + 4 * lane, x);
        const uint16_t nb = rotate128(x, sg, y);
        // sign code of this lane's 4 dims; block b = lanes 2b (low nibble), 2b+1
        uint32_t bits4 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) bits4 |= (y[i] >= 0.0f ? 1u : 0u) << i;
        const uint32_t pbits = __shfl_xor_sync(0xffffffffu, bits4, 1);
        const uint32_t code = (lane & 1) ? (pbits | (bits4 << 4)) : (bits4 | (pbits << 4));
        // block radius over 8 dims: ((d0+d1)+(d2+d3)) + ((d4+d5)+(d6+d7))
        const float sq = sum4(__fmul_rn(y[0], y[0]), __fmul_rn(y[1], y[1]), __fmul_rn(y[2], y[2]), __fmul_rn(y[3], y[3]));
        const float psq = __shfl_xor_sync(0xffffffffu, sq, 1);
        const float rs = (lane & 1) ? __fadd_rn(psq, sq) : __fadd_rn(sq, psq);
        const uint16_t rbits = f2bfbits(__fsqrt_rn(rs));
        const float rf = fmaxf(bfbits2f(rbits), eps8);
        float prod[4];
        uint32_t nib16 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float u = fabsf(rbf(__fdiv_rn(y[i], rf)));
            int tq = 0;
            float cv = cen[0];
#pragma unroll
            for (int j = 0; j < 7; ++j)
                if (thr[j] < u) {  // thresholds ascend: the last hit selects cen[tq]
                    tq = j + 1;
                    cv = cen[j + 1];
                }
            prod[i] = rbf(__fmul_rn(cv, u));
            nib16 |= ((((bits4 >> i) & 1u) << 3) | (uint32_t)tq) << (4 * i);
        }
        const float ap = sum4(prod[0], prod[1], prod[2], prod[3]);
        const float pap = __shfl_xor_sync(0xffffffffu, ap, 1);
        const float alpha = fmaxf((lane & 1) ? __fadd_rn(pap, ap) : __fadd_rn(ap, pap), 1e-6f);
        const uint16_t wbits = f2bfbits(__fmul_rn(__fdiv_rn(bfbits2f(rbits), alpha), bfbits2f(nb)));
        const uint32_t pnib = __shfl_xor_sync(0xffffffffu, nib16, 1);
        // popcount-estimator factor |k| / (sum |y| / sqrt(128))
        const float as = warp_sum_tree(sum4(fabsf(y[0]), fabsf(y[1]), fabsf(y[2]), fabsf(y[3])));
        const float ip = fmaxf(__fmul_rn(as, kInvSqrtD), 1e-6f);
        const int64_t k = (int64_t)tok_start + t;
        if (!(lane & 1)) {
            const int b = lane >> 1;
            if (L.codes) L.codes[row * L.codes_row + b * L.codes_blk + k * L.codes_tok] = (uint8_t)code;
            if (L.packed) L.packed[row * L.packed_row + b * L.packed_blk + k * L.packed_tok] = nib16 | (pnib << 16);
            if (L.weight)
                reinterpret_cast<uint16_t*>(L.weight)[row * L.weight_row + b * L.weight_blk + k * L.weight_tok] = wbits;
            if (do_hist) atomicAdd(&hist_s[b * kK + (int)code], 1);
        }
        if (lane == 0 && L.factor) L.factor[row * L.factor_row + k] = __fdiv_rn(bfbits2f(nb), ip);
    }
    if (do_hist) {
        __syncthreads();
        int32_t* gh = L.hist + (int64_t)row * kB * kK;
        for (int i = threadIdx.x; i < kB * kK; i += 256)
            if (hist_s[i]) atomicAdd(&gh[i], hist_s[i]);
    }
}

// ------------------------------------------------------------------ query
__global__ void __launch_bounds__(256) rq_query_kernel(const uint16_t* __restrict__ q, int rows, int G,
                                                       const uint16_t* __restrict__ signs, uint16_t* q_blocks,
                                                       uint16_t* q_norm, uint16_t* q_mean, uint8_t* planes,
                                                       float* qparams) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= rows) return;
    float sg[4];
    load_bf16x4(signs + 4 * lane, sg);
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < G; ++g) {
        float x[4];
        load_bf16x4(q + ((int64_t)row * G + g) * kHeadDim + 4 * lane, x);
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i] = __fadd_rn(s[i], x[i]);
    }
    float m[4];
    uint16_t mb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        mb[i] = f2bfbits(__fdiv_rn(s[i], (float)G));
        m[i] = bfbits2f(mb[i]);
    }
    if (q_mean)
        *reinterpret_cast<uint2*>(q_mean + (int64_t)row * kHeadDim + 4 * lane) =
            make_uint2((uint32_t)mb[0] | ((uint32_t)mb[1] << 16), (uint32_t)mb[2] | ((uint32_t)mb[3] << 16));
    float y[4];
    const uint16_t nb = rotate128(m, sg, y);
    uint16_t yb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) yb[i] = f2bfbits(y[i]);
    *reinterpret_cast<uint2*>(q_blocks + (int64_t)row * kHeadDim + 4 * lane) =
        make_uint2((uint32_t)yb[0] | ((uint32_t)yb[1] << 16), (uint32_t)yb[2] | ((uint32_t)yb[3] << 16));
    if (lane == 0) q_norm[row] = nb;
    if (!planes) return;
    float lo = fminf(fminf(y[0], y[1]), fminf(y[2], y[3]));
    float hi = fmaxf(fmaxf(y[0], y[1]), fmaxf(y[2], y[3]));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    float delta = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
    if (!(delta > 0.0f)) delta = 1.0f;
    int qb4[4], sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        qb4[i] = min(15, max(0, __float2int_rn(__fdiv_rn(__fsub_rn(y[i], lo), delta))));
        sum += qb4[i];
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        uint32_t nib = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) nib |= (uint32_t)((qb4[i] >> p) & 1) << i;
        const uint32_t pn = __shfl_xor_sync(0xffffffffu, nib, 1);
        if (!(lane & 1)) planes[(int64_t)row * 64 + p * kB + (lane >> 1)] = (uint8_t)(nib | (pn << 4));
    }
    if (lane == 0) {
        float* qp = qparams + (int64_t)row * 4;
        qp[0] = lo;
        qp[1] = delta;
        qp[2] = (float)sum;
        qp[3] = bfbits2f(nb);
    }
}

// ------------------------------------------------------------------ block scan
// Exclusive prefix of v over the CTA's threads (thread order); *total gets
// the sum.  scratch >= 33 ints; contains three __syncthreads (the first
// keeps back-to-back calls from overwriting totals still being read).
template <int NT>
__device__ __forceinline__ int block_excl_scan(int v, int* scratch, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) scratch[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < NT / 32 ? scratch[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < NT / 32) scratch[lane] = wi - w;
        if (lane == 31) scratch[32] = wi;
    }
    __syncthreads();
    const int r = scratch[warp] + incl - v;
    *total = scratch[32];
    return r;
}

// ------------------------------------------------------------------ collision + coarse top-C
struct CollArgs {
    const uint16_t* qb;  // [rows][128] bf16
    zkv_rq_layout L;
    int kv_len, C, n_tiers, per;
    int64_t tgt[kMaxTiers];
    int64_t* idx_out;
    int32_t* cnt_out;
};

// Tier-hit weight of every bucket of block b (one warp): bucket scores,
// bitonic sort of (desc score, bucket id), prefix of bucket sizes in that
// order, weight = #tiers whose target exceeds the prefix.
__device__ __forceinline__ void collision_table(const CollArgs& a, int row, int b, uint8_t* table, int* hs) {
    const int lane = threadIdx.x & 31;
    const int32_t* h = a.L.hist + ((int64_t)row * kB + b) * kK;
    int hpre[8];  // bucket sizes in bucket order, loaded alongside the query block
    {
        const int4 h0 = *reinterpret_cast<const int4*>(h + 8 * lane);
        const int4 h1 = *reinterpret_cast<const int4*>(h + 8 * lane + 4);
        hpre[0] = h0.x; hpre[1] = h0.y; hpre[2] = h0.z; hpre[3] = h0.w;
        hpre[4] = h1.x; hpre[5] = h1.y; hpre[6] = h1.z; hpre[7] = h1.w;
    }
    float q[kM];
    {
        const uint4 r = *reinterpret_cast<const uint4*>(a.qb + (int64_t)row * kHeadDim + kM * b);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            q[2 * j] = bfbits2f((uint16_t)(w[j] & 0xffffu));
            q[2 * j + 1] = bfbits2f((uint16_t)(w[j] >> 16));
        }
    }
    uint32_t key[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int c = lane * 8 + r;
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < kM; ++j) s = __fadd_rn(s, ((c >> j) & 1) ? q[j] : -q[j]);
        uint32_t u = f2bfbits(s);
        if (u == 0x8000u) u = 0u;  // -0 == +0
        const uint32_t ou = (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u);
        key[r] = ((~ou & 0xffffu) << 8) | (uint32_t)c;  // ascending key = descending score, then id
    }
#pragma unroll
    for (int k = 2; k <= 256; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 8) {
                const int lm = j >> 3;
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const uint32_t other = __shfl_xor_sync(0xffffffffu, key[r], lm);
                    const int e = lane * 8 + r;
                    const bool up = (e & k) == 0, lower = (e & j) == 0;
                    key[r] = (lower == up) ? min(key[r], other) : max(key[r], other);
                }
            } else {
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    if (r & j) continue;
                    const int r2 = r | j;
                    const int e = lane * 8 + r;
                    const bool up = (e & k) == 0;
                    if ((key[r] > key[r2]) == up) {
                        const uint32_t t = key[r];
                        key[r] = key[r2];
                        key[r2] = t;
                    }
                }
            }
        }
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < 8; ++r) hs[8 * lane + r] = hpre[r];
    __syncwarp();
    int hv[8];
    long long lsum = 0;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        hv[r] = hs[key[r] & 0xffu];
        lsum += hv[r];
    }
    long long incl = lsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    long long before = incl - lsum;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        int w = 0;
        for (int t = 0; t < a.n_tiers; ++t) w += before < a.tgt[t];
        table[b * kK + (key[r] & 0xffu)] = (uint8_t)w;
        before += hv[r];
    }
}

// Sum of the 16 per-block tier weights of one token's codes (one byte per
// block, block b at byte b of the 16-byte record).
__device__ __forceinline__ int count16(const uint8_t* table, const uint4 w) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    int c = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t x = ws[j];
        const uint8_t* t = table + 4 * j * kK;
        c += (int)t[x & 0xffu] + (int)t[kK + __byte_perm(x, 0u, 0x4441u)] +
             (int)t[2 * kK + __byte_perm(x, 0u, 0x4442u)] + (int)t[3 * kK + (x >> 24)];
    }
    return c;
}

// Exclusive prefix, in place, of v[0..nv) over the CTA (thread t owns a
// contiguous run of entries); returns the total.
__device__ __forceinline__ int block_excl_scan_array(int* v, int nv, int* scratch) {
    const int E = (nv + 255) / 256;
    const int e0 = min(nv, (int)threadIdx.x * E), e1 = min(nv, e0 + E);
    int s = 0;
    for (int e = e0; e < e1; ++e) s += v[e];
    int tot;
    int run = block_excl_scan<256>(s, scratch, &tot);
    for (int e = e0; e < e1; ++e) {
        const int x = v[e];
        v[e] = run;
        run += x;
    }
    __syncthreads();
    return tot;
}

// Bit j of gm / qm: key i+j (j < 16, i+j < n) has count > vstar / == vstar.
__device__ __forceinline__ void chunk_masks(const uint8_t* cnts, int i, int n, int vstar, uint32_t& gm,
                                            uint32_t& qm) {
    const uint4 w = *reinterpret_cast<const uint4*>(cnts + i);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    gm = 0u;
    qm = 0u;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int c = (int)((ws[j >> 2] >> (8 * (j & 3))) & 0xffu);
        const bool in = i + j < n;
        gm |= (in && c > vstar) ? (1u << j) : 0u;
        qm |= (in && c == vstar) ? (1u << j) : 0u;
    }
}

// One cluster of CS CTAs per row, CTA r counting keys [r*per, (r+1)*per).
// The 16 per-block weight tables are built once per cluster (block b by CTA
// b % CS) and pushed to every peer through distributed shared memory.
__global__ void __launch_bounds__(256, 4) collision_topk_kernel(const CollArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* table = smem;                                     // [16][256]
    int* hist = reinterpret_cast<int*>(smem + kB * kK);        // [kCntBins] (pad 136)
    int* gh = hist + 136;                                      // global histogram [136]
    int* scratch = gh + 136;                                   // 40
    int* misc = scratch + 40;                                  // 24: vstar, n_gt, eq_r[8], gt_r[8]
    int* hs = misc + 24;                                       // [8 warps][256] bucket sizes (table build)
    int* ghall = hs + 8 * kK;                                  // [CS][136] every CTA's histogram
    uint8_t* cnts = reinterpret_cast<uint8_t*>(ghall + 8 * 136);  // [per] (padded to 512)
    cg::cluster_group cluster = cg::this_cluster();
    const int CS = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
    const int row = blockIdx.x / CS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int k0 = rank * a.per;
    const int n = max(0, min(a.kv_len, k0 + a.per) - k0);
    const int nch = (n + 511) / 512;                           // 512-key chunks
    int* gtc = reinterpret_cast<int*>(cnts + ((a.per + 511) & ~511));  // [nch] counts > vstar
    int* eqn = gtc + nch;                                      // [nch] counts == vstar
    int* eqb = eqn + nch;                                      // [nch] exclusive prefix of eqn
    int* selb = eqb + nch;                                     // [nch] exclusive prefix of selected

    cluster.barrier_arrive();  // peers are running before the first remote store
    for (int b = rank + CS * warp; b < kB; b += CS * 8) collision_table(a, row, b, table, hs + warp * kK);
    for (int i = tid; i < 136; i += 256) hist[i] = 0;
    if (tid < 24) misc[tid] = 0;
    cluster.barrier_wait();
    for (int b = rank + CS * warp; b < kB; b += CS * 8) {
        __syncwarp();
        const uint4* src = reinterpret_cast<const uint4*>(table + b * kK);
        for (int t = lane; t < 16 * CS; t += 32) {
            const int p = t >> 4;
            if (p != rank) reinterpret_cast<uint4*>(cluster.map_shared_rank(table, p) + b * kK)[t & 15] = src[t & 15];
        }
    }
    cluster.sync();  // every table is complete in every CTA

    const bool tokmajor = a.L.codes_blk == 1 && a.L.codes_tok == 16;
    const uint8_t* cb = a.L.codes + row * a.L.codes_row;
    if (tokmajor) {
        constexpr int U = 4;  // tokens per thread in flight
        const uint4* c4 = reinterpret_cast<const uint4*>(cb) + k0;
        for (int base = 0; base < n; base += 256 * U) {
            uint4 w[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = base + u * 256 + tid;
                w[u] = i < n ? __ldcs(c4 + i) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = base + u * 256 + tid;
                if (i < n) {
                    const int c = count16(table, w[u]);
                    cnts[i] = (uint8_t)c;
                    atomicAdd(&hist[c], 1);
                    if (a.cnt_out) a.cnt_out[(int64_t)row * a.kv_len + k0 + i] = c;
                }
            }
        }
    } else {
        for (int i = tid; i < n; i += 256) {
            const int64_t k = k0 + i;
            int c = 0;
#pragma unroll
            for (int b = 0; b < kB; ++b) c += table[b * kK + cb[b * a.L.codes_blk + k * a.L.codes_tok]];
            cnts[i] = (uint8_t)c;
            atomicAdd(&hist[c], 1);
            if (a.cnt_out) a.cnt_out[(int64_t)row * a.kv_len + k] = c;
        }
    }
    if (!a.idx_out) return;  // counts only (uniform over the cluster)
    __syncthreads();
    // push this CTA's histogram into slot `rank` of every CTA; after the
    // barrier all reads are local and no remote access follows
    for (int i = tid; i < CS * kCntBins; i += 256) {
        const int p = i / kCntBins, v = i - p * kCntBins;
        cluster.map_shared_rank(ghall, p)[rank * 136 + v] = hist[v];
    }
    cluster.sync();
    for (int v = tid; v < kCntBins; v += 256) {
        int s = 0;
        for (int r = 0; r < CS; ++r) s += ghall[r * 136 + v];
        gh[v] = s;
    }
    __syncthreads();
    if (warp == 0) {  // threshold value: largest v with #(cnt >= v) >= C
        constexpr int PL = (kCntBins + 31) / 32;  // 5 bins per lane
        int local[PL];
        int tot = 0;
#pragma unroll
        for (int j = PL - 1; j >= 0; --j) {
            const int v = PL * lane + j;
            tot += v < kCntBins ? gh[v] : 0;
            local[j] = tot;
        }
        int incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_down_sync(0xffffffffu, incl, o);
            if (lane + o < 32) incl += t;
        }
        const int above = incl - tot;
#pragma unroll
        for (int j = 0; j < PL; ++j) {
            const int v = PL * lane + j;
            if (v < kCntBins) {
                const int ge = above + local[j], gt = ge - gh[v];
                if (gt < a.C && ge >= a.C) {
                    misc[0] = v;
                    misc[1] = gt;
                }
            }
        }
    }
    __syncthreads();
    const int vstar = misc[0];
    if (warp < CS) {  // per-rank (> vstar, == vstar) counts
        const int* hr = ghall + warp * 136;
        int gt = 0, eq = 0;
        for (int v = lane; v < kCntBins; v += 32) {
            const int x = hr[v];
            gt += v > vstar ? x : 0;
            eq += v == vstar ? x : 0;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            gt += __shfl_xor_sync(0xffffffffu, gt, o);
            eq += __shfl_xor_sync(0xffffffffu, eq, o);
        }
        if (lane == 0) {
            misc[8 + warp] = eq;
            misc[16 + warp] = gt;
        }
    }
    __syncthreads();

    int need_eq = a.C - misc[1], off = 0, take_eq = 0;
    for (int r = 0; r <= rank; ++r) {
        const int t = max(0, min(misc[8 + r], need_eq));
        if (r == rank) {
            take_eq = t;
        } else {
            off += misc[16 + r] + t;
        }
        need_eq -= t;
    }
    // ordered compaction of this CTA's keys in 512-key chunks (lane l owns
    // keys 16l..16l+15 of a chunk, one 16-byte shared load): per-chunk
    // (> vstar, == vstar) counts, a scan of the equal counts (ties go to the
    // lowest keys), a scan of the selected counts, then the writes
    for (int e = warp; e < nch; e += 8) {
        const int i = 512 * e + 16 * lane;
        uint32_t gm, qm;
        chunk_masks(cnts, i, n, vstar, gm, qm);
        const int g = __reduce_add_sync(0xffffffffu, __popc(gm));
        const int q = __reduce_add_sync(0xffffffffu, __popc(qm));
        if (lane == 0) {
            gtc[e] = g;
            eqn[e] = q;
            eqb[e] = q;
        }
    }
    __syncthreads();
    block_excl_scan_array(eqb, nch, scratch);
    for (int e = tid; e < nch; e += 256) selb[e] = gtc[e] + max(0, min(eqn[e], take_eq - eqb[e]));
    __syncthreads();
    block_excl_scan_array(selb, nch, scratch);
    int64_t* out = a.idx_out + (int64_t)row * a.C + off;
    for (int e = warp; e < nch; e += 8) {
        const int i = 512 * e + 16 * lane;
        uint32_t gm, qm;
        chunk_masks(cnts, i, n, vstar, gm, qm);
        int qr = eqb[e] + warp_excl_scan((int)__popc(qm));
        uint32_t sm = gm;
        for (uint32_t r = qm; r; r &= r - 1u) {  // equal keys in order, while ties remain
            if (qr++ < take_eq) sm |= r & (0u - r);
        }
        int p = selb[e] + warp_excl_scan((int)__popc(sm));
        for (uint32_t r = sm; r; r &= r - 1u) out[p++] = k0 + i + (__ffs(r) - 1);
    }
}

// ------------------------------------------------------------------ 4-bit rerank
struct Rerank4Args {
    const int64_t* cand;
    int C, F;
    zkv_rq_layout L;
    const uint16_t* qb;
    const uint16_t* qn;
    const uint16_t* cen;
    uint16_t* scores;
    int64_t* final_out;
};

// A cluster of CS CTAs per row: every CTA scores a contiguous slice of the
// candidates and pushes its fp32 scores into rank 0's shared array (DSMEM);
// rank 0 then selects the top F.
__global__ void __launch_bounds__(256, 4) rerank4_kernel(const Rerank4Args a) {
    extern __shared__ __align__(16) uint8_t smem[];
    float* lut = reinterpret_cast<float*>(smem);           // q row [128] bf16, then the 16 nibble values bf16
    int* hist = reinterpret_cast<int*>(lut + 128 * 16);    // 512
    int* misc = hist + 512;                                // 8
    int* scan = misc + 8;                                  // 512
    uint32_t* lohi = reinterpret_cast<uint32_t*>(scan + 512);  // 4: min / max ordered score (rank 0)
    float* sc = reinterpret_cast<float*>(lohi + 4);        // [C] (rank 0)
    int* sel = reinterpret_cast<int*>(sc + ((a.C + 3) & ~3));  // [F] selected positions (rank 0)
    int* ck = sel + ((a.F + 3) & ~3);                      // [perC] key ids of this CTA's slice
    cg::cluster_group cluster = cg::this_cluster();
    const int CS = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
    const int row = blockIdx.x / CS, tid = threadIdx.x;
    cluster.barrier_arrive();  // peers are running before the first remote store
    const int per = (a.C + CS - 1) / CS;
    const int i0 = rank * per, i1 = min(a.C, i0 + per);
    const int64_t* cr = a.cand + (int64_t)row * a.C;
    for (int i = i0 + tid; i < i1; i += 256) ck[i - i0] = (int)cr[i];
    const uint16_t* qb = a.qb + (int64_t)row * kHeadDim;
    __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(lut);  // [128]
    __nv_bfloat16* v_s = q_s + 128;                              // [16]: nibble -> +-cen
    for (int i = tid; i < 128; i += 256) q_s[i] = bits_bf16(qb[i]);
    if (tid < 16) v_s[tid] = bits_bf16((tid & 8) ? a.cen[tid & 7] : (uint16_t)(a.cen[tid & 7] ^ 0x8000u));
    __syncthreads();
    cluster.barrier_wait();
    float* sc0 = cluster.map_shared_rank(sc, 0);
    const float qn = bfbits2f(a.qn[row]);
    const bool tokmajor = a.L.packed_blk == 1 && a.L.packed_tok == 16 && a.L.weight_blk == 1 && a.L.weight_tok == 16;
    const uint32_t* pk = a.L.packed + row * a.L.packed_row;
    const uint16_t* wt = reinterpret_cast<const uint16_t*>(a.L.weight) + row * a.L.weight_row;
    for (int i = i0 + tid; i < i1; i += 256) {
        const int64_t k = ck[i - i0];
        uint32_t pw[kB];
        uint16_t wv[kB];
        if (tokmajor) {
            const uint4* p4 = reinterpret_cast<const uint4*>(pk + k * 16);
            const uint4* w4 = reinterpret_cast<const uint4*>(wt + k * 16);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint4 v = p4[j];
                pw[4 * j] = v.x; pw[4 * j + 1] = v.y; pw[4 * j + 2] = v.z; pw[4 * j + 3] = v.w;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint4 v = w4[j];
                const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    wv[8 * j + 2 * e] = (uint16_t)(ws[e] & 0xffffu);
                    wv[8 * j + 2 * e + 1] = (uint16_t)(ws[e] >> 16);
                }
            }
        } else {
#pragma unroll
            for (int b = 0; b < kB; ++b) {
                pw[b] = pk[b * a.L.packed_blk + k * a.L.packed_tok];
                wv[b] = wt[b * a.L.weight_blk + k * a.L.weight_tok];
            }
        }
        // rerank.cu:118-129 as built: temp = fma(k_j, q_j, temp) and res =
        // fma(temp, w_b, res), each rounded once to bf16; then res * |q|
        __nv_bfloat16 res = bits_bf16(0);
#pragma unroll
        for (int b = 0; b < kB; ++b) {
            __nv_bfloat16 dot = bits_bf16(0);
#pragma unroll
            for (int j = 0; j < kM; ++j) dot = __hfma(v_s[(pw[b] >> (4 * j)) & 0xfu], q_s[kM * b + j], dot);
            res = __hfma(dot, bits_bf16(wv[b]), res);
        }
        const uint16_t s = bf16_bits(__hmul(res, bits_bf16(f2bfbits(qn))));
        if (a.scores) a.scores[(int64_t)row * a.C + i] = s;
        sc0[i] = __fadd_rn(bfbits2f(s), 0.0f);  // -0 -> +0 for the selection
    }
    cluster.sync();  // every slice is in rank 0's array
    if (rank != 0 || a.F <= 0) return;
    int64_t* fo = a.final_out + (int64_t)row * a.F;
    if (a.F >= a.C) {
        for (int i = tid; i < a.F; i += 256) fo[i] = i < a.C ? cr[i] : -1;
        return;
    }
    if (a.C <= 16 * 256) {
        block_key_range<256>(sc, a.C, lohi);
        block_topk_small<256>(sc, a.C, a.F, lohi[0], lohi[1], hist, misc, scan, [&](int pos, int i) { sel[pos] = i; });
    } else
        block_topk<256, true>([&](int i) { return ordered_u32(sc[i]); }, a.C, a.F, hist, misc, scan,
                              [&](int pos, int i) { sel[pos] = i; });
    __syncthreads();
    for (int pos = tid; pos < a.F; pos += 256) fo[pos] = cr[sel[pos]];
}

// ------------------------------------------------------------------ 2-bit coarse score
__global__ void __launch_bounds__(256) coarse2bit_kernel(zkv_rq_layout L, const uint8_t* __restrict__ q_signs,
                                                         const uint8_t* __restrict__ q_mags, int kv_len,
                                                         int32_t* __restrict__ out) {
    const int row = blockIdx.y;
    const int64_t k = (int64_t)blockIdx.x * 256 + threadIdx.x;
    if (k >= kv_len) return;
    const uint32_t* pk = L.packed + row * L.packed_row;
    int pc_qm = 0, pc_x = 0, pc_qmx = 0, pc_kmx = 0, pc_qkx = 0, pc_km = 0, pc_qk = 0;
#pragma unroll
    for (int b = 0; b < kB; ++b) {
        const uint32_t w = pk[b * L.packed_blk + k * L.packed_tok];
        // sign bit 3 / magnitude-high bit 2 of each nibble -> one byte each
        uint32_t ks = 0, km = 0;
#pragma unroll
        for (int j = 0; j < kM; ++j) {
            ks |= ((w >> (4 * j + 3)) & 1u) << j;
            km |= ((w >> (4 * j + 2)) & 1u) << j;
        }
        const uint32_t s = q_signs[row * kB + b], m = q_mags[row * kB + b];
        const uint32_t xs = s ^ ks;
        pc_qm += __popc(m);
        pc_x += __popc(xs);
        pc_qmx += __popc(m & xs);
        pc_kmx += __popc(km & xs);
        pc_qkx += __popc(m & km & xs);
        pc_km += __popc(km);
        pc_qk += __popc(m & km);
    }
    out[(int64_t)row * kv_len + k] = (kHeadDim + pc_qm + pc_km + pc_qk) - 2 * (pc_x + pc_qmx + pc_kmx + pc_qkx);
}

// ------------------------------------------------------------------ popcount estimator + exact IP
struct PopArgs {
    const int64_t* cand;
    int C, K;
    zkv_rq_layout L;
    const uint8_t* planes;
    const float* qparams;
    int64_t* sel_out;
    float* est_out;
    const uint16_t* keys;
    int64_t keys_ld;
    const uint16_t* q_mean;
    float* ip_out;
};

// Popcount estimate of one candidate from its 16 code bytes.
__device__ __forceinline__ float popcount_est(const uint32_t (&x)[4], const uint32_t (&pl)[4][4], float d2, float l2,
                                              float c0, float factor, float qn) {
    int I = 0, P = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        P += __popc(x[j]);
#pragma unroll
        for (int p = 0; p < 4; ++p) I += __popc(x[j] & pl[p][j]) << p;
    }
    const float num = __fsub_rn(__fadd_rn(__fmul_rn(d2, (float)I), __fmul_rn(l2, (float)P)), c0);
    return __fmul_rn(__fmul_rn(__fmul_rn(num, kInvSqrtD), factor), qn);
}

// A cluster of CS CTAs per row.  Every CTA estimates a contiguous slice of
// the candidates and pushes the estimates into rank 0's shared array; rank 0
// selects the top K, writes their key ids and pushes each id to the CTA that
// owns output slot pos (slots split into CS contiguous runs); every CTA then
// takes the exact inner products of its run.
__global__ void __launch_bounds__(256, 4) popcount_topk_kernel(const PopArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    int* hist = reinterpret_cast<int*>(smem);   // 512
    int* misc = hist + 512;                     // 8
    int* scan = misc + 8;                       // 512
    uint32_t* lohi = reinterpret_cast<uint32_t*>(scan + 512);   // 4: min / max ordered estimate (rank 0)
    float* sc = reinterpret_cast<float*>(lohi + 4);              // [C] (rank 0)
    int* sel = reinterpret_cast<int*>(sc + ((a.C + 3) & ~3));    // [K] selected positions (rank 0)
    int* selk = sel + ((a.K + 3) & ~3);                          // [perK]: key ids of this CTA's run
    cg::cluster_group cluster = cg::this_cluster();
    const int CS = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
    const int row = blockIdx.x / CS, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (rank == 0 && tid == 0) {
        lohi[0] = 0xffffffffu;
        lohi[1] = 0u;
    }
    cluster.barrier_arrive();  // peers are running (and rank 0's lohi set) before the first remote op
    uint32_t pl[4][4];
    {
        const uint4* p = reinterpret_cast<const uint4*>(a.planes + (int64_t)row * 64);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 v = p[j];
            pl[j][0] = v.x; pl[j][1] = v.y; pl[j][2] = v.z; pl[j][3] = v.w;
        }
    }
    const float lo = a.qparams[row * 4], delta = a.qparams[row * 4 + 1], S = a.qparams[row * 4 + 2],
                qn = a.qparams[row * 4 + 3];
    const float c0 = __fadd_rn(__fmul_rn(delta, S), __fmul_rn((float)kHeadDim, lo));
    const float d2 = __fmul_rn(2.0f, delta), l2 = __fmul_rn(2.0f, lo);
    const bool tokmajor = a.L.codes_blk == 1 && a.L.codes_tok == 16;
    const uint8_t* cb = a.L.codes + row * a.L.codes_row;
    const float* fr = a.L.factor + row * a.L.factor_row;
    const int64_t* cr = a.cand ? a.cand + (int64_t)row * a.C : nullptr;
    const int perC = (a.C + CS - 1) / CS;
    const int c_lo = rank * perC, c_hi = min(a.C, c_lo + perC);
    cluster.barrier_wait();
    float* sc0 = cluster.map_shared_rank(sc, 0);
    uint32_t klo = 0xffffffffu, khi = 0u;
    if (tokmajor) {
        constexpr int U = 4;  // candidates per thread in flight
        for (int base = c_lo; base < c_hi; base += 256 * U) {
            int64_t kx[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = base + u * 256 + tid;
                kx[u] = i < c_hi ? (cr ? cr[i] : i) : -1;
            }
            uint4 v[U];
            float f[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                v[u] = make_uint4(0u, 0u, 0u, 0u);
                f[u] = 0.0f;
                if (kx[u] >= 0) {
                    v[u] = *reinterpret_cast<const uint4*>(cb + kx[u] * 16);
                    f[u] = fr[kx[u]];
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = base + u * 256 + tid;
                if (i < c_hi) {
                    const uint32_t x[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                    const float er = popcount_est(x, pl, d2, l2, c0, f[u], qn);
                    if (a.est_out) a.est_out[(int64_t)row * a.C + i] = er;
                    const float e = __fadd_rn(er, 0.0f);  // -0 -> +0 for the selection
                    sc0[i] = e;
                    klo = min(klo, ordered_u32(e));
                    khi = max(khi, ordered_u32(e));
                }
            }
        }
    } else {
        for (int i = c_lo + tid; i < c_hi; i += 256) {
            const int64_t k = cr ? cr[i] : i;
            uint32_t x[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t w = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) w |= (uint32_t)cb[(4 * j + e) * a.L.codes_blk + k * a.L.codes_tok] << (8 * e);
                x[j] = w;
            }
            const float er = popcount_est(x, pl, d2, l2, c0, fr[k], qn);
            if (a.est_out) a.est_out[(int64_t)row * a.C + i] = er;
            const float e = __fadd_rn(er, 0.0f);
            sc0[i] = e;
            klo = min(klo, ordered_u32(e));
            khi = max(khi, ordered_u32(e));
        }
    }
    cluster_fold_range(cluster, lohi, klo, khi);
    cluster.sync();  // every estimate (and the key range) is in rank 0's shared memory
    const int kk = min(a.K, a.C);
    const int perK = (kk + CS - 1) / CS;
    if (rank == 0) {
        int64_t* so = a.sel_out + (int64_t)row * a.K;
        if (a.K >= a.C) {
            for (int i = tid; i < a.K; i += 256) {
                if (i < a.C) sel[i] = i;
                else so[i] = -1;
            }
        } else {
            if (a.C <= 16 * 256)
                block_topk_small<256>(sc, a.C, a.K, lohi[0], lohi[1], hist, misc, scan,
                                      [&](int pos, int i) { sel[pos] = i; });
            else
                block_topk<256, true>([&](int i) { return ordered_u32(sc[i]); }, a.C, a.K, hist, misc, scan,
                                      [&](int pos, int i) { sel[pos] = i; });
        }
        __syncthreads();
        // positions -> key ids (independent loads), pushed to the owner of each slot
        for (int pos = tid; pos < kk; pos += 256) {
            const int i = sel[pos];
            const int64_t k = cr ? cr[i] : i;
            so[pos] = k;
            if (a.keys) cluster.map_shared_rank(selk, pos / perK)[pos % perK] = (int)k;
        }
    }
    if (!a.keys) return;  // uniform over the cluster
    cluster.sync();  // every CTA holds the key ids of its run
    float qv[4];
    load_bf16x4(a.q_mean + (int64_t)row * kHeadDim + 4 * lane, qv);
    const int j_lo = rank * perK, j_hi = min(kk, j_lo + perK);
    constexpr int U = 8;  // candidates per warp in flight (one 256-byte row each)
    const uint16_t* kr = a.keys + row * a.keys_ld + 4 * lane;
    for (int j0 = j_lo + warp * U; j0 < j_hi; j0 += 8 * U) {
        uint2 raw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + u;
            raw[u] = make_uint2(0, 0);
            if (j < j_hi) raw[u] = *reinterpret_cast<const uint2*>(kr + (int64_t)selk[j - j_lo] * kHeadDim);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const float k0 = bfbits2f((uint16_t)(raw[u].x & 0xffffu)), k1 = bfbits2f((uint16_t)(raw[u].x >> 16));
            const float k2 = bfbits2f((uint16_t)(raw[u].y & 0xffffu)), k3 = bfbits2f((uint16_t)(raw[u].y >> 16));
            const float s = warp_sum_tree(sum4(__fmul_rn(k0, qv[0]), __fmul_rn(k1, qv[1]), __fmul_rn(k2, qv[2]),
                                               __fmul_rn(k3, qv[3])));
            if (lane == 0 && j0 + u < j_hi) a.ip_out[(int64_t)row * a.K + j0 + u] = s;
        }
    }
}

}  // namespace rq
}  // namespace zkv

using namespace zkv;
using namespace zkv::rq;

static bool lay_ok(const zkv_rq_layout* L) { return L != nullptr; }

// CTAs per row for the candidate kernels: enough to cover ~4 resident CTAs
// on every SM in one wave, at most 8 (portable cluster), at least 256
// candidates per CTA.
static int cluster_size_for(int rows, int C) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int cs = (4 * sms) / (rows > 0 ? rows : 1);
    const int by_c = (C + 255) / 256;
    cs = cs < by_c ? cs : by_c;
    return cs < 1 ? 1 : (cs > 8 ? 8 : cs);
}

extern "C" int zkv_rq_encode(const void* keys, int64_t keys_ld_row, int rows, int n_tok, int tok_start,
                             const void* signs, const zkv_rq_layout* lay, void* stream) {
    if (!keys || !signs || !lay_ok(lay) || rows < 0 || n_tok < 0 || tok_start < 0 || keys_ld_row < kHeadDim)
        return ZKV_ERR_ARG;
    if (((uintptr_t)keys & 7) || (keys_ld_row & 3) || ((uintptr_t)signs & 7)) return ZKV_ERR_ALIGN;
    if (rows == 0 || n_tok == 0) return ZKV_OK;
    if (rows > 65535) return ZKV_ERR_CAPACITY;
    dim3 grid((n_tok + kEncTok - 1) / kEncTok, rows);
    rq_encode_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint16_t*)keys, keys_ld_row, n_tok, tok_start,
                                                             (const uint16_t*)signs, *lay);
    return launch_status();
}

extern "C" int zkv_rq_query(const void* q, int rows, int G, const void* signs, void* q_blocks, void* q_norm,
                            void* q_mean, uint8_t* planes, float* qparams, void* stream) {
    if (!q || !signs || !q_blocks || !q_norm || rows < 0 || G < 1 || (planes && !qparams)) return ZKV_ERR_ARG;
    if (((uintptr_t)q & 7) || ((uintptr_t)q_blocks & 7) || (q_mean && ((uintptr_t)q_mean & 7)) ||
        ((uintptr_t)signs & 7))
        return ZKV_ERR_ALIGN;
    if (rows == 0) return ZKV_OK;
    rq_query_kernel<<<(rows + 7) / 8, 256, 0, (cudaStream_t)stream>>>(
        (const uint16_t*)q, rows, G, (const uint16_t*)signs, (uint16_t*)q_blocks, (uint16_t*)q_norm,
        (uint16_t*)q_mean, planes, qparams);
    return launch_status();
}

extern "C" int zkv_collision_topk(const void* q_blocks, const zkv_rq_layout* lay, int rows, int kv_len,
                                  const int64_t* targets, int n_tiers, int C, int64_t* idx_out, int32_t* cnt_out,
                                  void* stream) {
    if (!q_blocks || !lay_ok(lay) || !lay->codes || !lay->hist || !targets || (!idx_out && !cnt_out) || rows < 0 ||
        kv_len < 1 || n_tiers < 1 || n_tiers > kMaxTiers || (idx_out && (C < 1 || C > kv_len)))
        return ZKV_ERR_ARG;
    if (((uintptr_t)q_blocks & 15)) return ZKV_ERR_ALIGN;
    if (lay->codes_blk == 1 && lay->codes_tok == 16 && (((uintptr_t)lay->codes & 15) || (lay->codes_row & 15)))
        return ZKV_ERR_ALIGN;
    if (rows == 0) return ZKV_OK;
    int CS = cluster_size_for(rows, (kv_len + 3) / 4);  // >= 1024 keys per CTA
    const int need = (kv_len + 131071) / 131072;       // shared-memory bound on keys per CTA
    CS = CS < need ? (need > 8 ? 8 : need) : CS;
    const int per = (kv_len + CS - 1) / CS;
    const size_t nch = ((size_t)per + 511) / 512;
    const size_t smem = (size_t)kB * kK + (136 + 136 + 40 + 24 + 8 * kK + 8 * 136) * sizeof(int) +
                        (((size_t)per + 511) & ~(size_t)511) + nch * 16;
    if (smem > 200 * 1024) return ZKV_ERR_CAPACITY;
    CollArgs a;
    a.qb = (const uint16_t*)q_blocks;
    a.L = *lay;
    a.kv_len = kv_len;
    a.C = C;
    a.n_tiers = n_tiers;
    a.per = per;
    for (int t = 0; t < kMaxTiers; ++t) a.tgt[t] = t < n_tiers ? targets[t] : 0;
    a.idx_out = idx_out;
    a.cnt_out = cnt_out;
    void* args[] = {&a};
    return launch_clustered((const void*)collision_topk_kernel, rows * CS, 256, CS, smem, (cudaStream_t)stream, args);
}

extern "C" int zkv_rq_rerank4(const int64_t* cand, int C, const zkv_rq_layout* lay, const void* q_blocks,
                              const void* q_norm, const void* centers, int rows, void* scores, int F,
                              int64_t* final_out, void* stream) {
    if (!cand || !lay_ok(lay) || !lay->packed || !lay->weight || !q_blocks || !q_norm || !centers || rows < 0 ||
        C < 1 || F < 0 || (F > 0 && !final_out))
        return ZKV_ERR_ARG;
    const bool tok = lay->packed_blk == 1 && lay->packed_tok == 16 && lay->weight_blk == 1 && lay->weight_tok == 16;
    if (tok && (((uintptr_t)lay->packed & 15) || ((uintptr_t)lay->weight & 15) || (lay->packed_row & 3) ||
                (lay->weight_row & 7)))
        return ZKV_ERR_ALIGN;
    if (rows == 0) return ZKV_OK;
    const int CS = cluster_size_for(rows, C);
    const size_t smem = (128 * 16 + 512 + 8 + 512 + 4) * sizeof(float) + (size_t)((C + 3) & ~3) * sizeof(float) +
                        (size_t)((F + 3) & ~3) * sizeof(int) + (size_t)((C + CS - 1) / CS) * sizeof(int);
    if (smem > 200 * 1024) return ZKV_ERR_CAPACITY;
    Rerank4Args a{cand, C, F, *lay, (const uint16_t*)q_blocks, (const uint16_t*)q_norm, (const uint16_t*)centers,
                  (uint16_t*)scores, final_out};
    void* args[] = {&a};
    return launch_clustered((const void*)rerank4_kernel, rows * CS, 256, CS, smem, (cudaStream_t)stream, args);
}

extern "C" int zkv_coarse2bit(const zkv_rq_layout* lay, const uint8_t* q_signs, const uint8_t* q_mags, int rows,
                              int kv_len, int32_t* out, void* stream) {
    if (!lay_ok(lay) || !lay->packed || !q_signs || !q_mags || !out || rows < 0 || kv_len < 0) return ZKV_ERR_ARG;
    if (rows == 0 || kv_len == 0) return ZKV_OK;
    if (rows > 65535) return ZKV_ERR_CAPACITY;
    dim3 grid((kv_len + 255) / 256, rows);
    coarse2bit_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(*lay, q_signs, q_mags, kv_len, out);
    return launch_status();
}

extern "C" int zkv_rq_popcount_topk(const int64_t* cand, int C, const zkv_rq_layout* lay, const uint8_t* planes,
                                    const float* qparams, int rows, int K, int64_t* sel_out, float* est_out,
                                    const void* keys, int64_t keys_ld_row, const void* q_mean, float* ip_out,
                                    void* stream) {
    if (!lay_ok(lay) || !lay->codes || !lay->factor || !planes || !qparams || !sel_out || rows < 0 || C < 1 || K < 1)
        return ZKV_ERR_ARG;
    if (keys && (!q_mean || !ip_out || keys_ld_row < kHeadDim)) return ZKV_ERR_ARG;
    if (((uintptr_t)planes & 15) || (keys && (((uintptr_t)keys & 7) || (keys_ld_row & 3) || ((uintptr_t)q_mean & 7))))
        return ZKV_ERR_ALIGN;
    if (lay->codes_blk == 1 && lay->codes_tok == 16 && (((uintptr_t)lay->codes & 15) || (lay->codes_row & 15)))
        return ZKV_ERR_ALIGN;
    if (rows == 0) return ZKV_OK;
    const int CS = cluster_size_for(rows, C);
    const int kk = K < C ? K : C;
    const size_t smem = (512 + 8 + 512 + 4) * sizeof(int) + (size_t)((C + 3) & ~3) * sizeof(float) +
                        (size_t)((K + 3) & ~3) * sizeof(int) + (size_t)((kk + CS - 1) / CS) * sizeof(int);
    if (smem > 200 * 1024) return ZKV_ERR_CAPACITY;
    PopArgs a{cand, C, K, *lay, planes, qparams, sel_out, est_out, (const uint16_t*)keys, keys_ld_row,
              (const uint16_t*)q_mean, ip_out};
    void* args[] = {&a};
    return launch_clustered((const void*)popcount_topk_kernel, rows * CS, 256, CS, smem, (cudaStream_t)stream, args);
}
