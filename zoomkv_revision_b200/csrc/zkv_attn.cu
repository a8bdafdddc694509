// zkv_attn.cu -- decode attention for the ZoomKV sparse path.
//
//  * zkv_page_decode: one fused launch per layer.  A thread-block cluster of
//    CS CTAs owns one (batch, kv_head) row:
//      phase 1  each CTA streams its share of the Quest min/max metadata with
//               1-D TMA bulk copies (a 2-slot mbarrier ring per warp) and
//               scores chunks;
//      phase 2  scores are exchanged through distributed shared memory and
//               every CTA runs the same deterministic radix top-k;
//      phase 3  each warp double-buffers its pages (4-bit K, 4-bit V, scales)
//               with bulk copies and runs QK^T / PV on mma.sync m16n8k16,
//               dequantising in registers (no bf16 K/V copy is written);
//      phase 4  warp partials merge in shared memory, CTA partials merge
//               through distributed shared memory on cluster rank 0.
//  * zkv_attn_rows: the reference-mode attention over raw bf16 rows gathered
//    by index (sink / selected / near zones), same warp core and merge.
//  * zkv_lse_merge / zkv_lse_merge_n: log-sum-exp combine of partials.
#include "zkv_common.cuh"

namespace zkv {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kRawStride = 136;  // bf16 per padded staged row (272 B, conflict-free B-fragment loads)
constexpr int kSlotBytes = 4608; // per-warp staging slot (2 per warp)
// KIVI page slot: kc [16][16] i32 @0, vc [128][2] i32 @1024, vmeta @2048,
//                 min @2304, KIVI scale @2560 (2816 B)
constexpr int kPageTx = 1024 + 1024 + 256 + 256 + 256;
// RAW8 slot: K rows [8][136] bf16 @0, V rows @2176
constexpr int kRawV = 8 * kRawStride * 2;
constexpr int kRegionBytes = 2 * kAttnWarps * kSlotBytes;  // 36 KB: phase-1 rings / page slots / merge
// page-decode phase 3: 3 slots per warp of 3 KiB (a KIVI page + its computed
// scale, or a RAW4 item of up to 4 raw rows) so each warp keeps 3 items in flight
constexpr int kPSlotBytes = 3072;
constexpr int kPSlots = 3;
constexpr int kRaw4V = 4 * kRawStride * 2;  // V rows of a RAW4 slot
static_assert(kAttnWarps * kPSlots * kPSlotBytes <= kRegionBytes, "page slots exceed the region");

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct WarpAttn {
    float m;          // running max (log2 units) of head g = lane/4
    float l;          // running sum over this lane's tokens
    float o[8][4];    // O^T accumulators, m-tile j = dims 16j..16j+15
    uint32_t qa[8][2];// A fragments of Q (rows = heads), k-step s
};

__device__ __forceinline__ void warp_attn_init(WarpAttn& st, const uint16_t* q_s, int G) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        if (g < G) {
            st.qa[s][0] = *reinterpret_cast<const uint32_t*>(q_s + g * kHeadDim + 16 * s + 2 * tig);
            st.qa[s][1] = *reinterpret_cast<const uint32_t*>(q_s + g * kHeadDim + 16 * s + 8 + 2 * tig);
        } else {
            st.qa[s][0] = 0;
            st.qa[s][1] = 0;
        }
    }
    st.m = -INFINITY;
    st.l = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) st.o[j][e] = 0.f;
}

// Online-softmax update with the 4 scores (tokens 2tig, 2tig+1, 8+2tig,
// 9+2tig) of head g; returns the B fragment of P^T for the PV product.
__device__ __forceinline__ void warp_softmax(WarpAttn& st, float (&x)[4], int G, uint32_t& b0, uint32_t& b1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(st.m, mx);
    const float alpha = (st.m == -INFINITY) ? 0.f : ex2(st.m - mnew);
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = (x[i] == -INFINITY) ? 0.f : ex2(x[i] - mnew);
    st.l = st.l * alpha + ((p[0] + p[1]) + (p[2] + p[3]));
    st.m = mnew;
    const float a0 = __shfl_sync(0xffffffffu, alpha, (2 * tig) * 4);
    const float a1 = __shfl_sync(0xffffffffu, alpha, (2 * tig + 1) * 4);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        st.o[j][0] *= a0;
        st.o[j][1] *= a1;
        st.o[j][2] *= a0;
        st.o[j][3] *= a1;
    }
    if (g < G) {
        b0 = pack_bf162(p[0], p[1]);
        b1 = pack_bf162(p[2], p[3]);
    } else {
        b0 = 0;
        b1 = 0;
    }
}

// KIVI page: 16 tokens, 4-bit K (chunk-major) + 4-bit V (page-transposed).
__device__ __forceinline__ void warp_page_kivi(WarpAttn& st, uint8_t* slot, int G, float sl2) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int32_t* kc = reinterpret_cast<const int32_t*>(slot);
    const uint32_t* mn2 = reinterpret_cast<const uint32_t*>(slot + 2304);
    const uint32_t* sc2 = reinterpret_cast<const uint32_t*>(slot + 2560);  // per-dim KIVI scale
    const uint32_t sel = nib_sel(tig);
    // S = Q K^T over 8 k-steps of 16 dims; the two k-halves accumulate
    // separately (4 independent MMA chains of 4 instead of 2 of 8) and are
    // added at the end.
    float sacc[2][2][4] = {};  // [k-half][token tile][fragment]
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
            const int s = s4 + 4 * kh;
            const __nv_bfloat162 sA = bits_bf162(sc2[8 * s + tig]);
            const __nv_bfloat162 sB = bits_bf162(sc2[8 * s + 4 + tig]);
            const __nv_bfloat162 nA = neg128(sA), nB = neg128(sB);
            const __nv_bfloat162 mA = bits_bf162(mn2[8 * s + tig]);
            const __nv_bfloat162 mB = bits_bf162(mn2[8 * s + 4 + tig]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int n = 8 * h + g;
                const uint32_t w0 = (uint32_t)kc[(2 * s) * kChunk + n];
                const uint32_t w1 = (uint32_t)kc[(2 * s + 1) * kChunk + n];
                const uint32_t b0 = bf162_bits(dequant2_w(w0, sel, sA, nA, mA));
                const uint32_t b1 = bf162_bits(dequant2_w(w1, sel, sB, nB, mB));
                mma_bf16_16816(sacc[kh][h], st.qa[s][0], 0u, st.qa[s][1], 0u, b0, b1);
            }
        }
    }
    float x[4] = {(sacc[0][0][0] + sacc[1][0][0]) * sl2, (sacc[0][0][1] + sacc[1][0][1]) * sl2,
                  (sacc[0][1][0] + sacc[1][1][0]) * sl2, (sacc[0][1][1] + sacc[1][1][1]) * sl2};
    uint32_t pb0, pb1;
    warp_softmax(st, x, G, pb0, pb1);
    const uint2* vc = reinterpret_cast<const uint2*>(slot + 1024);
    const uint32_t* vs = reinterpret_cast<const uint32_t*>(slot + 2048);
    const uint32_t* vz = vs + 32;
#pragma unroll
    for (int gp = 0; gp < kVGroups; ++gp) {
        const __nv_bfloat162 sLo = bits_bf162(vs[gp * 8 + tig]);
        const __nv_bfloat162 sHi = bits_bf162(vs[gp * 8 + 4 + tig]);
        const __nv_bfloat162 nLo = neg128(sLo), nHi = neg128(sHi);
        const __nv_bfloat162 zLo = bits_bf162(vz[gp * 8 + tig]);
        const __nv_bfloat162 zHi = bits_bf162(vz[gp * 8 + 4 + tig]);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int j = 2 * gp + jj;
            const int d = 16 * j + g;
            const uint2 wa = vc[d];
            const uint2 wb = vc[d + 8];
            const uint32_t a0 = bf162_bits(dequant2_w(wa.x, sel, sLo, nLo, zLo));
            const uint32_t a2 = bf162_bits(dequant2_w(wa.y, sel, sHi, nHi, zHi));
            const uint32_t a1 = bf162_bits(dequant2_w(wb.x, sel, sLo, nLo, zLo));
            const uint32_t a3 = bf162_bits(dequant2_w(wb.y, sel, sHi, nHi, zHi));
            mma_bf16_16816(st.o[j], a0, a1, a2, a3, pb0, pb1);
        }
    }
}

// RAW8 item: up to 8 raw bf16 token rows (padded stride); bit t of `present`
// says whether token t is real (absent rows were zero-filled).
__device__ __forceinline__ void warp_page_raw8(WarpAttn& st, const uint8_t* slot, unsigned present, int G, float sl2) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const uint16_t* K = reinterpret_cast<const uint16_t*>(slot);
    const uint16_t* V = reinterpret_cast<const uint16_t*>(slot + kRawV);
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(K + g * kRawStride + 16 * s + 2 * tig);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(K + g * kRawStride + 16 * s + 8 + 2 * tig);
        mma_bf16_16816(sacc, st.qa[s][0], 0u, st.qa[s][1], 0u, b0, b1);
    }
    float x[4] = {((present >> (2 * tig)) & 1u) ? sacc[0] * sl2 : -INFINITY,
                  ((present >> (2 * tig + 1)) & 1u) ? sacc[1] * sl2 : -INFINITY, -INFINITY, -INFINITY};
    uint32_t pb0, pb1;
    warp_softmax(st, x, G, pb0, pb1);
    pb1 = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int d = 16 * j + g;
        const uint32_t a0 = (uint32_t)V[(2 * tig) * kRawStride + d] | ((uint32_t)V[(2 * tig + 1) * kRawStride + d] << 16);
        const uint32_t a1 =
            (uint32_t)V[(2 * tig) * kRawStride + d + 8] | ((uint32_t)V[(2 * tig + 1) * kRawStride + d + 8] << 16);
        mma_bf16_16816(st.o[j], a0, a1, 0u, 0u, pb0, pb1);
    }
}

// RAW4 item: up to 4 raw bf16 token rows (padded stride); bit t of `present`
// says whether token t is real (absent rows were zero-filled).  Tokens 4..7
// of the m16n8k16 tiles are zero operands.
__device__ __forceinline__ void warp_page_raw4(WarpAttn& st, const uint8_t* slot, unsigned present, int G, float sl2) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const uint16_t* K = reinterpret_cast<const uint16_t*>(slot);
    const uint16_t* V = reinterpret_cast<const uint16_t*>(slot + kRaw4V);
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        uint32_t b0 = 0u, b1 = 0u;
        if (g < 4) {
            b0 = *reinterpret_cast<const uint32_t*>(K + g * kRawStride + 16 * s + 2 * tig);
            b1 = *reinterpret_cast<const uint32_t*>(K + g * kRawStride + 16 * s + 8 + 2 * tig);
        }
        mma_bf16_16816(sacc, st.qa[s][0], 0u, st.qa[s][1], 0u, b0, b1);
    }
    const bool lo = tig < 2;
    float x[4] = {(lo && ((present >> (2 * tig)) & 1u)) ? sacc[0] * sl2 : -INFINITY,
                  (lo && ((present >> (2 * tig + 1)) & 1u)) ? sacc[1] * sl2 : -INFINITY, -INFINITY, -INFINITY};
    uint32_t pb0, pb1;
    warp_softmax(st, x, G, pb0, pb1);
    pb1 = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int d = 16 * j + g;
        uint32_t a0 = 0u, a1 = 0u;
        if (lo) {
            a0 = (uint32_t)V[(2 * tig) * kRawStride + d] | ((uint32_t)V[(2 * tig + 1) * kRawStride + d] << 16);
            a1 = (uint32_t)V[(2 * tig) * kRawStride + d + 8] | ((uint32_t)V[(2 * tig + 1) * kRawStride + d + 8] << 16);
        }
        mma_bf16_16816(st.o[j], a0, a1, 0u, 0u, pb0, pb1);
    }
}

// Warp-level issue of up to 4 raw rows into a RAW4 slot: row_of(t) gives the
// token row offset (in tokens) or -1 when token t of the item is absent.
template <typename RowOf>
__device__ __forceinline__ void issue_raw4(uint8_t* slot, uint64_t* bar, const uint16_t* kbase, const uint16_t* vbase,
                                           RowOf row_of) {
    const int lane = threadIdx.x & 31;
    const int t = lane & 3;
    const int64_t tok = row_of(t);
    const unsigned present = __ballot_sync(0xffffffffu, tok >= 0) & 0xfu;
    const int n_present = __popc(present);
    // zero rows of absent tokens (V must be finite: masked p = 0 multiplies it)
    for (int i = lane; i < 4 * 16 * 2; i += 32) {
        const int rowi = (i >> 4) & 3, part = i >> 6, col = i & 15;
        if (!((present >> rowi) & 1u))
            *reinterpret_cast<uint4*>(slot + part * kRaw4V + rowi * kRawStride * 2 + col * 16) = make_uint4(0, 0, 0, 0);
    }
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)n_present * 512u);
    __syncwarp();
    if (tok >= 0) {
        if (lane < 4) bulk_g2s(slot + t * kRawStride * 2, kbase + tok * kHeadDim, 256, bar);
        else if (lane < 8) bulk_g2s(slot + kRaw4V + t * kRawStride * 2, vbase + tok * kHeadDim, 256, bar);
    }
}

// Warp-level issue of a KIVI page into `slot` (lane 0 issues all copies).
__device__ __forceinline__ void issue_kivi_page(uint8_t* slot, uint64_t* bar, const zkv_page_layer& L, int64_t row,
                                                int n_max, int64_t c) {
    if ((threadIdx.x & 31) == 0) {
        mbar_arrive_expect_tx(bar, kPageTx);
        const int64_t pc = row * n_max + c;
        bulk_g2s(slot, L.kcodes + pc * (kWords * kChunk), 1024, bar);
        bulk_g2s(slot + 1024, L.vcodes_t + pc * (kHeadDim * 2), 1024, bar);
        bulk_g2s(slot + 2048, reinterpret_cast<const uint16_t*>(L.vmeta) + pc * (2 * kVGroups * kChunk), 256, bar);
        bulk_g2s(slot + 2304, reinterpret_cast<const uint16_t*>(L.chunk_min) + pc * kHeadDim, 256, bar);
        bulk_g2s(slot + 2560, reinterpret_cast<const uint16_t*>(L.kscale) + pc * kHeadDim, 256, bar);
    }
}

// Warp-level issue of up to 8 raw rows: row_of(t) gives the token row
// pointer offset (in tokens) or -1 when token t of the item is absent.
template <typename RowOf>
__device__ __forceinline__ void issue_raw8(uint8_t* slot, uint64_t* bar, const uint16_t* kbase, const uint16_t* vbase,
                                           RowOf row_of) {
    const int lane = threadIdx.x & 31;
    const int t = lane & 7;
    const int64_t tok = row_of(t);
    const unsigned present = __ballot_sync(0xffffffffu, tok >= 0) & 0xffu;
    const int n_present = __popc(present);
    // zero rows of absent tokens (V must be finite: masked p = 0 multiplies it)
    for (int i = lane; i < 8 * 16 * 2; i += 32) {
        const int rowi = (i >> 4) & 7, part = i >> 7, col = i & 15;
        if (!((present >> rowi) & 1u))
            *reinterpret_cast<uint4*>(slot + part * kRawV + rowi * kRawStride * 2 + col * 16) = make_uint4(0, 0, 0, 0);
    }
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)n_present * 512u);
    __syncwarp();
    if (tok >= 0) {
        if (lane < 8) bulk_g2s(slot + t * kRawStride * 2, kbase + tok * kHeadDim, 256, bar);
        else if (lane < 16) bulk_g2s(slot + kRawV + t * kRawStride * 2, vbase + tok * kHeadDim, 256, bar);
    }
}

// Merge the warps' states into a CTA partial (m, l, o unnormalised) in smem.
// `scratch` >= kAttnWarps * (8 * 128 + 16) floats.  Caller syncs before.
__device__ void cta_merge(const WarpAttn& st, int G, float* scratch, float* cm, float* cl, float* co) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tig = lane & 3;
    float l = st.l;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    float* wm = scratch + warp * (8 * kHeadDim + 16);
    float* wl = wm + 8;
    float* wo = wm + 16;
    if (tig == 0 && g < 8) {
        wm[g] = st.m;
        wl[g] = l;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int d = 16 * j + g;
        const int h0 = 2 * tig, h1 = 2 * tig + 1;
        if (h0 < G) {
            wo[h0 * kHeadDim + d] = st.o[j][0];
            wo[h0 * kHeadDim + d + 8] = st.o[j][2];
        }
        if (h1 < G) {
            wo[h1 * kHeadDim + d] = st.o[j][1];
            wo[h1 * kHeadDim + d + 8] = st.o[j][3];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * kHeadDim; i += kAttnThreads) {
        const int h = i / kHeadDim, d = i % kHeadDim;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, scratch[w * (8 * kHeadDim + 16) + h]);
        float Ls = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            const float* b = scratch + w * (8 * kHeadDim + 16);
            const float wt = (b[h] == -INFINITY) ? 0.f : ex2(b[h] - M);
            Ls += wt * b[8 + h];
            O += wt * b[16 + h * kHeadDim + d];
        }
        co[h * kHeadDim + d] = O;
        if (d == 0) {
            cm[h] = M;
            cl[h] = Ls;
        }
    }
}

// Cluster combine: every CTA pushes its partial (m, l, o) into rank 0's
// receive area with distributed-shared-memory stores (no remote-load latency
// chains), then rank 0 merges locally and writes out / lse.  `recv` is rank
// 0's staging region (free once all CTAs passed the first cluster barrier).
__device__ void cluster_merge(cg::cluster_group& cluster, int CS, int G, const float* cm, const float* cl,
                              const float* co, float* recv, uint16_t* out_row, float* lse_row,
                              float* out_f32_row = nullptr) {
    constexpr int kPart = 16 + 8 * kHeadDim;  // m[8], l[8], o[8][128]
    const int rank = (int)cluster.block_rank();
    cluster.sync();  // every CTA finished phase 3 and its CTA merge
    {
        float* dst = cluster.map_shared_rank(recv, 0) + rank * kPart;
        if (threadIdx.x < 8) {
            dst[threadIdx.x] = cm[threadIdx.x];
            dst[8 + threadIdx.x] = cl[threadIdx.x];
        }
        for (int i = threadIdx.x; i < G * kHeadDim / 4; i += kAttnThreads)
            reinterpret_cast<float4*>(dst + 16)[i] = reinterpret_cast<const float4*>(co)[i];
    }
    cluster.sync();  // partials visible in rank 0
    if (rank != 0) return;
    for (int i = threadIdx.x; i < G * kHeadDim; i += kAttnThreads) {
        const int h = i / kHeadDim;
        float M = -INFINITY;
        for (int r = 0; r < CS; ++r) M = fmaxf(M, recv[r * kPart + h]);
        float Ls = 0.f, O = 0.f;
        for (int r = 0; r < CS; ++r) {
            const float* b = recv + r * kPart;
            const float wt = (b[h] == -INFINITY) ? 0.f : ex2(b[h] - M);
            Ls += wt * b[8 + h];
            O += wt * b[16 + i];
        }
        const float o = Ls > 0.f ? O / Ls : 0.f;
        if (out_f32_row) {
            out_f32_row[i] = o;
        } else {
            out_row[i] = f2bfbits(o);
        }
        if ((i % kHeadDim) == 0 && lse_row)
            lse_row[h] = (Ls > 0.f) ? (M + __log2f(Ls)) * 0.69314718055994531f : -INFINITY;
    }
}

// One copy of each select in the binary for both levels of the two-level
// select (that instantiation stalls on instruction fetch; the one-level one
// keeps its select inline, where a call measured ~1 us slower).  Top k of sc[0..n) (ties to the
// lowest index, ascending index order): out_id[pos] = id_in ? id_in[i] :
// id_base + i, and out_sc[pos] = sc[i] when out_sc != NULL.  sc is 16-byte
// aligned; lo / hi: min finite and max ordered key.
__device__ __noinline__ void select_pairs(const float* sc, int n, int k, uint32_t lo, uint32_t hi, int* hist,
                                          int* misc, int* scan, const int* id_in, int id_base, float* out_sc,
                                          int* out_id) {
    auto emit = [&](int pos, int i) {
        if (out_sc) out_sc[pos] = sc[i];
        out_id[pos] = id_in ? id_in[i] : id_base + i;
    };
    if (n <= 16 * kAttnThreads)
        block_topk_small<kAttnThreads>(sc, n, k, lo, hi, hist, misc, scan, emit);
    else
        block_topk<kAttnThreads, true>([&](int i) { return ordered_u32(sc[i]); }, n, k, hist, misc, scan, emit, true,
                                       lo, hi);
}

// ---------------------------------------------------------------- page decode
struct PageArgs {
    const uint16_t* q;
    zkv_page_layer L;
    int G, n_max, n_c, nk, n_sink, near_start, n_near, n_c_pad, per, pp, pn;
    int n_cand;     // two-level select: CS * nk candidate slots (0 = one-level)
    const float* sc_in;  // two-level only: precomputed chunk scores [rows][sc_ld] (NULL = score here)
    int64_t sc_ld;
    int parts;           // two-level only: clusters per row, each attends 1/parts of the selected
                         // pages; > 1 writes fp32 partials [part][rows] to out_f32 / lse
    float sl2;
    uint16_t* out;
    float* lse;
    int64_t* sel_out;
    int32_t* status;
    // external selection (sequence split): global page ids [rows][nk]; the
    // ids in [sel_lo, sel_hi) are this layer buffer's pages id - sel_lo
    const int64_t* sel_in;
    int64_t sel_lo, sel_hi;
    float* out_f32;  // fp32 partial output instead of bf16 (may be NULL)
    // two-level scored mode of the sequence split: of the selected global
    // page ids, attend those in [own_lo, own_hi), this buffer's pages
    // id - own_lo (own = 0: attend every selected page)
    int own;
    int64_t own_lo, own_hi;
};

// kTwoLevel: the select runs in two levels over a.n_cand candidates (a
// separate instantiation keeps the one-level kernel's code unchanged).
template <bool kTwoLevel>
__global__ void __launch_bounds__(kAttnThreads, 4) page_decode_kernel(const PageArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int CS = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int64_t cid = blockIdx.x / CS;
    const int64_t row = kTwoLevel ? cid / a.parts : cid;
    const int part = kTwoLevel ? (int)(cid % a.parts) : 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    uint8_t* region = smem;
    float* sc_all = reinterpret_cast<float*>(smem + kRegionBytes);
    float* cand_sc = sc_all + a.n_c_pad;                              // [n_cand] two-level candidates
    int* cand_id = reinterpret_cast<int*>(cand_sc + (kTwoLevel ? a.n_cand : 0));
    int* sel_s = cand_id + (kTwoLevel ? a.n_cand : 0);
    uint16_t* q_s = reinterpret_cast<uint16_t*>(sel_s + ((a.nk + 3) & ~3));
    uint16_t* rq_s = q_s + 8 * kHeadDim;
    float* cm = reinterpret_cast<float*>(rq_s + kHeadDim);
    float* cl = cm + 8;
    float* co = cl + 8;
    int* hist = reinterpret_cast<int*>(co + 8 * kHeadDim);
    int* misc = hist + 512;
    int* scan = misc + 8;
    uint64_t* bars = reinterpret_cast<uint64_t*>(scan + 2 * kAttnThreads);  // [warps][2] phase 1, [warps][3] phase 3
    __shared__ int s_failed;
    __shared__ uint32_t s_mm[2 + 2 * 16];  // own (min, max) key; gathered per cluster rank

    if (threadIdx.x == 0) {
        s_failed = 0;
        s_mm[0] = 0xffffffffu;
        s_mm[1] = 0u;
        for (int i = 0; i < (2 + kPSlots) * kAttnWarps; ++i) mbar_init(bars + i, 1);
        mbar_fence_init();
    }
    // Split cluster barrier: arrive now, wait before the first remote
    // shared-memory store, so every peer CTA is known to be running.
    cluster.barrier_arrive();
    grid_dep_wait();  // inputs may come from the previous kernel on the stream
    // query + GQA-mean query (compute() :1622-1626: bf16 mean over the group)
    for (int i = threadIdx.x; i < a.G * kHeadDim; i += kAttnThreads) q_s[i] = a.q[row * a.G * kHeadDim + i];
    __syncthreads();
    for (int d = threadIdx.x; d < kHeadDim; d += kAttnThreads) {
        float acc = 0.f;
        for (int g = 0; g < a.G; ++g) acc = __fadd_rn(acc, bfbits2f(q_s[g * kHeadDim + d]));
        rq_s[d] = f2bfbits(__fdiv_rn(acc, (float)a.G));
    }
    __syncthreads();

    // ------------------------------------------------ phase 1: Quest scores
    // Each warp streams blocks of 8 chunks (2 KiB of min + 2 KiB of max rows)
    // through its own 2-slot ring; warps run independently.
    constexpr int kBlk = 8;
    const int c0 = rank * a.per;
    const int c1 = min(a.n_c, c0 + a.per);
    const int n_my = max(0, c1 - c0);
    const int n_blk = (n_my + kBlk - 1) / kBlk;
    const uint16_t* gmin = reinterpret_cast<const uint16_t*>(a.L.chunk_min) + (row * a.n_max) * kHeadDim;
    const uint16_t* gmax = reinterpret_cast<const uint16_t*>(a.L.chunk_max) + (row * a.n_max) * kHeadDim;
    if (kTwoLevel && a.sc_in) {  // scores from the all-SM scoring kernel
        const float* src = a.sc_in + row * a.sc_ld;
        uint32_t klo = 0xffffffffu, khi = 0u;
        for (int c = c0 + (int)threadIdx.x; c < c1; c += kAttnThreads) {
            const float val = src[c];
            sc_all[c] = val;
            const uint32_t kk = ordered_u32(val);
            if (kk > kOrderedNegInf) klo = min(klo, kk);
            khi = max(khi, kk);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            klo = min(klo, __shfl_xor_sync(0xffffffffu, klo, off));
            khi = max(khi, __shfl_xor_sync(0xffffffffu, khi, off));
        }
        if (lane == 0) {
            atomicMin(&s_mm[0], klo);
            atomicMax(&s_mm[1], khi);
        }
    } else {
        constexpr int R = 2;
        uint8_t* ring = region + warp * (2 * kSlotBytes);
        uint64_t* rbar = bars + R * warp;
        auto issue_blk = [&](int b, int k) {
            if (lane == 0) {
                const int cc = c0 + b * kBlk;
                const int nch = min(kBlk, c1 - cc);
                uint8_t* dst = ring + k * 4096;
                mbar_arrive_expect_tx(rbar + k, (uint32_t)nch * kHeadDim * 2 * 2);
                bulk_g2s(dst, gmin + (int64_t)cc * kHeadDim, nch * kHeadDim * 2, rbar + k);
                bulk_g2s(dst + 2048, gmax + (int64_t)cc * kHeadDim, nch * kHeadDim * 2, rbar + k);
            }
        };
        int mine = 0;
        for (int b = warp; b < n_blk; b += kAttnWarps) ++mine;
        for (int k = 0; k < R && k < mine; ++k) issue_blk(warp + k * kAttnWarps, k);
        const int hl = lane & 15, half = lane >> 4;
        const uint4 qv = *reinterpret_cast<const uint4*>(rq_s + 8 * hl);
        bool ok = true;
        uint32_t klo = 0xffffffffu, khi = 0u;
        for (int i = 0; i < mine; ++i) {
            const int b = warp + i * kAttnWarps;
            const int k = i % R;
            if (!mbar_wait(rbar + k, (uint32_t)((i / R) & 1), a.status)) ok = false;
            const uint8_t* src = ring + k * 4096;
            const int cc = c0 + b * kBlk;
            const int nch = min(kBlk, c1 - cc);
#pragma unroll
            for (int u = 0; u < kBlk / 2; ++u) {
                const int lc = 2 * u + half;
                uint4 mn = make_uint4(0, 0, 0, 0), mx = mn;
                if (lc < nch) {
                    mn = *reinterpret_cast<const uint4*>(src + lc * kHeadDim * 2 + 16 * hl);
                    mx = *reinterpret_cast<const uint4*>(src + 2048 + lc * kHeadDim * 2 + 16 * hl);
                }
                const float sc = quest_half(qv, mn, mx);
                if (hl == 0 && lc < nch) {
                    const int c = cc + lc;
                    const bool v = !a.L.valid || a.L.valid[row * a.n_max + c];
                    const float val = (ok && v) ? sc : -INFINITY;
                    sc_all[c] = val;
                    const uint32_t kk = ordered_u32(val);
                    if (kk > kOrderedNegInf) klo = min(klo, kk);
                    khi = max(khi, kk);
                }
            }
            __syncwarp();
            if (i + R < mine) issue_blk(b + R * kAttnWarps, k);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            klo = min(klo, __shfl_xor_sync(0xffffffffu, klo, off));
            khi = max(khi, __shfl_xor_sync(0xffffffffu, khi, off));
        }
        if (lane == 0) {
            atomicMin(&s_mm[0], klo);
            atomicMax(&s_mm[1], khi);
        }
        if (!ok && lane == 0) atomicOr(&s_failed, 1);
    }
    __syncthreads();
    cluster.barrier_wait();
    if (threadIdx.x < CS) {
        uint32_t* rmm = cluster.map_shared_rank(s_mm, (int)threadIdx.x);
        rmm[2 + 2 * rank] = s_mm[0];
        rmm[3 + 2 * rank] = s_mm[1];
    }
    if (kTwoLevel) {
        // two-level select, level 1: this CTA's top nk (ties to the lowest
        // chunk), as (score, chunk) pairs in chunk order, into slot `rank` of
        // every CTA's candidate list; padding keys order below -inf.  The
        // global top nk is a subset of the union, and the list is in chunk
        // order, so level 2 picks the same set in the same order.
        float* my_sc = cand_sc + rank * a.nk;
        int* my_id = cand_id + rank * a.nk;
        if (n_my > a.nk) {
            select_pairs(sc_all + c0, n_my, a.nk, s_mm[0], s_mm[1], hist, misc, scan, nullptr, c0, my_sc, my_id);
        } else {
            for (int i = threadIdx.x; i < a.nk; i += kAttnThreads) {
                my_sc[i] = i < n_my ? sc_all[c0 + i] : __uint_as_float(0xffffffffu);
                my_id[i] = i < n_my ? c0 + i : 0;
            }
        }
        __syncthreads();
        for (int p = 1; p < CS; ++p) {
            const int dst_rank = (rank + p) % CS;
            float* rs = cluster.map_shared_rank(my_sc, dst_rank);
            int* ri = cluster.map_shared_rank(my_id, dst_rank);
            for (int i = threadIdx.x; i < a.nk; i += kAttnThreads) {
                rs[i] = my_sc[i];
                ri[i] = my_id[i];
            }
        }
    }
    // push this CTA's score range into every peer's score array
    for (int p = 1; p < CS && !kTwoLevel; ++p) {
        const int dst_rank = (rank + p) % CS;
        float* rsc = cluster.map_shared_rank(sc_all, dst_rank);
        for (int i = c0 + 4 * threadIdx.x; i < c1; i += 4 * kAttnThreads) {
            if (i + 4 <= c1) {
                *reinterpret_cast<float4*>(rsc + i) = *reinterpret_cast<const float4*>(sc_all + i);
            } else {
                for (int e = i; e < c1; ++e) rsc[e] = sc_all[e];
            }
        }
    }

    // ------------------------------------------------ phase 2: select
    cluster.sync();
    __shared__ int s_nsel;
    if (a.sel_in) {  // the pages this buffer owns, in list order
        if (warp == 0) {
            const int64_t* sr = a.sel_in + row * a.nk;
            int base = 0;
            for (int j0 = 0; j0 < a.nk; j0 += 32) {
                const int j = j0 + lane;
                const int64_t id = j < a.nk ? sr[j] : -1;
                const bool own = id >= a.sel_lo && id < a.sel_hi && id - a.sel_lo < a.n_max;
                const unsigned bal = __ballot_sync(0xffffffffu, own);
                if (own) sel_s[base + __popc(bal & ((1u << lane) - 1u))] = (int)(id - a.sel_lo);
                base += __popc(bal);
            }
            if (lane == 0) s_nsel = base;
        }
        __syncthreads();
    } else if (a.n_c <= a.nk) {
        for (int i = threadIdx.x; i < a.nk; i += kAttnThreads) sel_s[i] = i < a.n_c ? i : 0;
        __syncthreads();
    } else {
        uint32_t lo = 0xffffffffu, hi = 0u;
        for (int r = 0; r < CS; ++r) {
            lo = min(lo, s_mm[2 + 2 * r]);
            hi = max(hi, s_mm[3 + 2 * r]);
        }
        if (kTwoLevel) {  // level 2 over the CS * nk candidates
            select_pairs(cand_sc, a.n_cand, a.nk, lo, hi, hist, misc, scan, cand_id, 0, nullptr, sel_s);
        } else if (a.n_c <= 16 * kAttnThreads) {  // inline here: a call costs ~1 us at config 1
            block_topk_small<kAttnThreads>(sc_all, a.n_c, a.nk, lo, hi, hist, misc, scan,
                                           [&](int pos, int i) { sel_s[pos] = i; });
        } else {
            block_topk<kAttnThreads, true>([&](int i) { return ordered_u32(sc_all[i]); }, a.n_c, a.nk, hist, misc,
                                           scan, [&](int pos, int i) { sel_s[pos] = i; }, true, lo, hi);
        }
    }
    if (a.sel_out && rank == 0 && part == 0 && !a.sel_in)
        for (int i = threadIdx.x; i < a.nk; i += kAttnThreads) a.sel_out[row * a.nk + i] = sel_s[i];
    if (kTwoLevel && a.own) {  // keep the selected pages this buffer holds, in list order
        __syncthreads();
        if (warp == 0) {
            int base = 0;
            for (int j0 = 0; j0 < a.nk; j0 += 32) {
                const int j = j0 + lane;
                const int id = j < a.nk ? sel_s[j] : -1;
                const bool mine = id >= a.own_lo && id < a.own_hi;
                const unsigned bal = __ballot_sync(0xffffffffu, mine);
                // in place: every write goes below j0 + 32, after the group's reads
                if (mine) sel_s[base + __popc(bal & ((1u << lane) - 1u))] = (int)(id - a.own_lo);
                base += __popc(bal);
            }
            if (lane == 0) s_nsel = base;
        }
        __syncthreads();
    }

    // ------------------------------------------------ phase 3: attention
    WarpAttn st;
    warp_attn_init(st, q_s, a.G);
    const int nsel = (a.sel_in || (kTwoLevel && a.own)) ? s_nsel : a.nk;
    // this cluster's share of the selection list (the whole list unless parts > 1)
    const int part_pp = kTwoLevel ? (nsel + a.parts - 1) / a.parts : nsel;
    const int part_lo = kTwoLevel ? min(nsel, part * part_pp) : 0;
    const int part_hi = kTwoLevel ? min(nsel, part_lo + part_pp) : nsel;
    const int pp = a.sel_in ? (nsel + CS - 1) / CS : (kTwoLevel ? (part_hi - part_lo + CS - 1) / CS : a.pp);
    const int p_lo = part_lo + rank * pp, p_hi = min(part_hi, p_lo + pp);
    const int n_raw_all = part == 0 ? a.n_sink + a.n_near : 0;  // raw rows: part 0 only
    const int n_lo = rank * a.pn, n_hi = min(n_raw_all, n_lo + a.pn);
    const int n_pages = max(0, p_hi - p_lo);
    const int n_raw = max(0, (n_hi - n_lo + 3) / 4);
    const int n_items = n_pages + n_raw;
    const uint16_t* nk_base = reinterpret_cast<const uint16_t*>(a.L.near_k) + row * a.L.near_ld * kHeadDim;
    const uint16_t* nv_base = reinterpret_cast<const uint16_t*>(a.L.near_v) + row * a.L.near_ld * kHeadDim;
    uint8_t* wslot[kPSlots];
#pragma unroll
    for (int k = 0; k < kPSlots; ++k) wslot[k] = region + (kPSlots * warp + k) * kPSlotBytes;
    uint64_t* wbar = bars + 2 * kAttnWarps + kPSlots * warp;
    auto issue_item = [&](int it, int k) {
        if (it < n_pages) {
            issue_kivi_page(wslot[k], wbar + k, a.L, row, a.n_max, sel_s[p_lo + it]);
        } else {
            const int base = n_lo + 4 * (it - n_pages);
            issue_raw4(wslot[k], wbar + k, nk_base, nv_base, [&](int t) -> int64_t {
                const int v = base + t;
                if (v >= n_hi) return -1;
                return v < a.n_sink ? (int64_t)v : (int64_t)(a.near_start + v - a.n_sink);
            });
        }
    };
    {
        int mine = 0;
        for (int it = warp; it < n_items; it += kAttnWarps) ++mine;
#pragma unroll
        for (int k = 0; k < kPSlots; ++k)
            if (k < mine) issue_item(warp + k * kAttnWarps, k);
        bool ok = true;
        for (int i = 0; i < mine; ++i) {
            const int it = warp + i * kAttnWarps;
            const int k = i % kPSlots;
            if (!mbar_wait(wbar + k, (uint32_t)((i / kPSlots) & 1), a.status)) ok = false;
            if (ok) {
                if (it < n_pages) {
                    warp_page_kivi(st, wslot[k], a.G, a.sl2);
                } else {
                    const int base = n_lo + 4 * (it - n_pages);
                    warp_page_raw4(st, wslot[k], (1u << min(4, n_hi - base)) - 1u, a.G, a.sl2);
                }
            }
            __syncwarp();
            if (i + kPSlots < mine) issue_item(it + kPSlots * kAttnWarps, k);
        }
        if (!ok && lane == 0) atomicOr(&s_failed, 1);
    }

    // ------------------------------------------------ phase 4: merge
    grid_dep_launch_next();
    __syncthreads();
    cta_merge(st, a.G, reinterpret_cast<float*>(region), cm, cl, co);
    const int64_t orow = kTwoLevel ? (int64_t)part * (gridDim.x / (CS * a.parts)) + row : row;
    cluster_merge(cluster, CS, a.G, cm, cl, co, reinterpret_cast<float*>(region),
                  a.out ? a.out + orow * a.G * kHeadDim : nullptr, a.lse ? a.lse + orow * a.G : nullptr,
                  a.out_f32 ? a.out_f32 + orow * a.G * kHeadDim : nullptr);
    if (threadIdx.x == 0 && s_failed) set_status(a.status, ZKV_ERR_TIMEOUT);
}

// ---------------------------------------------------------------- raw rows
struct RowsArgs {
    const uint16_t* q;
    const uint16_t* keys;
    const uint16_t* values;
    int64_t kv_ld_row, kv_cap;
    int G;
    int s0_lo, s0_n, n_sel, s1_lo, s1_n;
    const int64_t* sel;
    int64_t sel_ld, sel_off;
    int ipc;  // 8-token items per CTA
    float sl2;
    uint16_t* out;
    float* lse;
    int32_t* status;
};

__global__ void __launch_bounds__(kAttnThreads, 4) attn_rows_kernel(const RowsArgs a) {
    pdl_begin();  // inputs may come from the previous kernel on the stream
    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int CS = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int64_t row = blockIdx.x / CS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* region = smem;
    uint16_t* q_s = reinterpret_cast<uint16_t*>(smem + kRegionBytes);
    float* cm = reinterpret_cast<float*>(q_s + 8 * kHeadDim);
    float* cl = cm + 8;
    float* co = cl + 8;
    uint64_t* bars = reinterpret_cast<uint64_t*>(co + 8 * kHeadDim);
    __shared__ int s_failed;
    if (threadIdx.x == 0) {
        s_failed = 0;
        for (int i = 0; i < 2 * kAttnWarps; ++i) mbar_init(bars + i, 1);
        mbar_fence_init();
    }
    for (int i = threadIdx.x; i < a.G * kHeadDim; i += kAttnThreads) q_s[i] = a.q[row * a.G * kHeadDim + i];
    __syncthreads();
    const int total = a.s0_n + a.n_sel + a.s1_n;
    const int n_items_all = (total + 7) / 8;
    const int it_lo = rank * a.ipc, it_hi = min(n_items_all, it_lo + a.ipc);
    const uint16_t* kb = a.keys + row * a.kv_ld_row;
    const uint16_t* vb = a.values + row * a.kv_ld_row;
    const int64_t* selr = a.sel ? a.sel + row * a.sel_ld : nullptr;
    auto token_row = [&](int i) -> int64_t {
        if (i >= total) return -1;
        int64_t t;
        if (i < a.s0_n) t = a.s0_lo + i;
        else if (i < a.s0_n + a.n_sel) t = selr[i - a.s0_n] + a.sel_off;
        else t = a.s1_lo + (i - a.s0_n - a.n_sel);
        return (t >= 0 && t < a.kv_cap) ? t : -1;
    };
    WarpAttn st;
    warp_attn_init(st, q_s, a.G);
    uint8_t* wslot[2] = {region + (2 * warp) * kSlotBytes, region + (2 * warp + 1) * kSlotBytes};
    uint64_t* wbar = bars + 2 * warp;
    int mine = 0;
    for (int it = it_lo + warp; it < it_hi; it += kAttnWarps) ++mine;
    auto issue_item = [&](int it, int k) {
        issue_raw8(wslot[k], wbar + k, kb, vb, [&](int t) { return token_row(8 * it + t); });
    };
    if (mine > 0) issue_item(it_lo + warp, 0);
    if (mine > 1) issue_item(it_lo + warp + kAttnWarps, 1);
    bool ok = true;
    for (int i = 0; i < mine; ++i) {
        const int it = it_lo + warp + i * kAttnWarps;
        const int k = i & 1;
        if (!mbar_wait(wbar + k, (uint32_t)((i >> 1) & 1), a.status)) ok = false;
        const int64_t tr = token_row(8 * it + (lane & 7));
        const unsigned pres = __ballot_sync(0xffffffffu, tr >= 0) & 0xffu;
        if (ok) warp_page_raw8(st, wslot[k], pres, a.G, a.sl2);
        __syncwarp();
        if (i + 2 < mine) issue_item(it + 2 * kAttnWarps, k);
    }
    if (!ok && lane == 0) atomicOr(&s_failed, 1);
    __syncthreads();
    cta_merge(st, a.G, reinterpret_cast<float*>(region), cm, cl, co);
    cluster_merge(cluster, CS, a.G, cm, cl, co, reinterpret_cast<float*>(region), a.out + row * a.G * kHeadDim,
                  a.lse ? a.lse + row * a.G : nullptr);
    if (threadIdx.x == 0 && s_failed) set_status(a.status, ZKV_ERR_TIMEOUT);
}

// ---------------------------------------------------------------- LSE merge
__global__ void lse_merge_kernel(const uint16_t* __restrict__ a, const float* __restrict__ la,
                                 const uint16_t* __restrict__ b, const float* __restrict__ lb,
                                 uint16_t* __restrict__ out, float* __restrict__ lse_out, int rows, int dim) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * dim) return;
    const int r = (int)(i / dim);
    const float m = fmaxf(la[r], lb[r]);
    const float wa = expf(la[r] - m), wb = expf(lb[r] - m);
    const float den = wa + wb;
    out[i] = f2bfbits((wa * bfbits2f(a[i]) + wb * bfbits2f(b[i])) / den);
    if (lse_out && (i % dim) == 0) lse_out[r] = m + logf(den);
}

__global__ void lse_merge_n_kernel(const float* __restrict__ parts, const float* __restrict__ lses, int n, int rows,
                                   int dim, uint16_t* __restrict__ out, float* __restrict__ lse_out) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * dim) return;
    const int r = (int)(i / dim);
    float m = -INFINITY;
    for (int p = 0; p < n; ++p) m = fmaxf(m, lses[(int64_t)p * rows + r]);
    float den = 0.f, acc = 0.f;
    for (int p = 0; p < n; ++p) {
        const float lp = lses[(int64_t)p * rows + r];
        const float w = (lp == -INFINITY) ? 0.f : expf(lp - m);
        den += w;
        acc += w * parts[(int64_t)p * rows * dim + i];
    }
    out[i] = f2bfbits(den > 0.f ? acc / den : 0.f);
    if (lse_out && (i % dim) == 0) lse_out[r] = den > 0.f ? m + logf(den) : -INFINITY;
}

}  // namespace zkv

using namespace zkv;

static size_t page_smem(const PageArgs& a) {
    return kRegionBytes + (size_t)a.n_c_pad * 4 + (size_t)a.n_cand * 8 + (size_t)((a.nk + 3) & ~3) * 4 +
           9 * kHeadDim * 2 + (16 + 8 * kHeadDim) * 4 + (512 + 8 + 2 * kAttnThreads) * 4 +
           ((2 + kPSlots) * kAttnWarps) * 8 + 16;
}

static int pick_cluster(int requested, int rows) {
    if (requested == 1 || requested == 2 || requested == 4 || requested == 8) return requested;
    (void)rows;
    return 8;
}

static int page_decode_impl(const void* q, const zkv_page_layer* layer, int rows, int G, int n_max, int n_c, int nk,
                            int n_sink, int near_start, int n_near, float scale, void* out, float* lse,
                            int64_t* sel_out, int32_t* status, int cluster, const float* sc_in, int64_t sc_ld,
                            int parts, float* out_f32, void* stream, int64_t own_lo = 0, int64_t own_hi = -1) {
    // own mode (own_hi >= own_lo): n_c counts the score row's entries, which
    // may run past this buffer's pages; the buffer holds [own_lo, own_hi)
    const bool own = own_hi >= own_lo;
    if (!q || !layer || (!out && !out_f32) || rows < 0 || G < 1 || G > 8 || n_c < 0 || nk < 1 ||
        n_near < 0 || n_sink < 0 || near_start < 0 || (!own && n_c > n_max) || (own && own_hi - own_lo > n_max))
        return ZKV_ERR_ARG;
    if (nk > n_c && n_c > 0) return ZKV_ERR_ARG;
    if ((int64_t)near_start + n_near > layer->near_ld || n_sink > layer->near_ld) return ZKV_ERR_ARG;
    if (n_c > 16384 || nk > 2048) return ZKV_ERR_CAPACITY;
    if (rows == 0) return ZKV_OK;
    const zkv_page_layer& L = *layer;
    if (!L.chunk_min || !L.chunk_max || !L.kscale || !L.kcodes || !L.vcodes_t || !L.vmeta ||
        (n_near + n_sink > 0 && (!L.near_k || !L.near_v)))
        return ZKV_ERR_ARG;
    if (((uintptr_t)L.chunk_min & 15) || ((uintptr_t)L.chunk_max & 15) || ((uintptr_t)L.kscale & 15) ||
        ((uintptr_t)L.kcodes & 15) ||
        ((uintptr_t)L.vcodes_t & 15) || ((uintptr_t)L.vmeta & 15) || ((uintptr_t)L.near_k & 15) ||
        ((uintptr_t)L.near_v & 15) || ((uintptr_t)q & 3))
        return ZKV_ERR_ALIGN;
    const int CS = pick_cluster(cluster, rows);
    PageArgs a;
    a.q = (const uint16_t*)q;
    a.L = L;
    a.G = G;
    a.n_max = n_max;
    a.n_c = n_c;
    a.nk = n_c > 0 ? nk : 0;
    a.n_sink = n_sink;
    a.near_start = near_start;
    a.n_near = n_near;
    a.n_c_pad = (n_c + 3) & ~3;
    a.per = ((n_c + CS - 1) / CS + 3) & ~3;
    a.pp = (a.nk + CS - 1) / CS;
    // past 16 keys per thread the one-level select re-reads shared memory
    a.n_cand = (CS > 1 && (n_c > 16 * kAttnThreads || own) && a.nk < n_c) ? ((CS * a.nk + 3) & ~3) : 0;
    if (own && !a.n_cand) return ZKV_ERR_UNSUPPORTED;  // own mode runs the two-level scored path
    a.sc_in = a.n_cand ? sc_in : nullptr;
    a.sc_ld = sc_ld;
    a.parts = a.n_cand ? parts : 1;
    a.pn = ((n_sink + n_near + CS - 1) / CS + 3) & ~3;
    a.sl2 = scale * 1.4426950408889634f;
    a.out = (uint16_t*)out;
    a.lse = lse;
    a.sel_out = sel_out;
    a.status = status;
    a.sel_in = nullptr;
    a.sel_lo = a.sel_hi = 0;
    a.out_f32 = out_f32;
    a.own = own ? 1 : 0;
    a.own_lo = own_lo;
    a.own_hi = own ? own_hi : 0;
    void* args[] = {&a};
    return launch_clustered(a.n_cand ? (const void*)page_decode_kernel<true> : (const void*)page_decode_kernel<false>,
                            rows * a.parts * CS, kAttnThreads, CS, page_smem(a), (cudaStream_t)stream, args,
                            /*pdl=*/true);
}

extern "C" int zkv_page_decode(const void* q, const zkv_page_layer* layer, int rows, int G, int n_max, int n_c,
                               int nk, int n_sink, int near_start, int n_near, float scale, void* out, float* lse,
                               int64_t* sel_out, int32_t* status, int cluster, void* stream) {
    if (!out) return ZKV_ERR_ARG;
    return page_decode_impl(q, layer, rows, G, n_max, n_c, nk, n_sink, near_start, n_near, scale, out, lse, sel_out,
                            status, cluster, nullptr, 0, 1, nullptr, stream);
}

// workspace: scores [rows][n_c] fp32 | part outputs [parts][rows][G][128] fp32 | part lse [parts][rows][G]
// (sized for parts <= kMaxParts, G <= 8)
constexpr int kMaxParts = 4;
static size_t split_ws_scores_bytes(int rows, int n_c) { return ((size_t)rows * n_c * 4 + 255) & ~(size_t)255; }
static size_t split_ws_parts_bytes(int rows) { return ((size_t)kMaxParts * rows * 8 * kHeadDim * 4 + 255) & ~(size_t)255; }

extern "C" size_t zkv_page_decode_split_ws_bytes(int rows, int n_c) {
    if (rows < 0 || n_c < 0) return 0;
    return split_ws_scores_bytes(rows, n_c) + split_ws_parts_bytes(rows) +
           (((size_t)kMaxParts * rows * 8 * 4 + 255) & ~(size_t)255);
}

extern "C" int zkv_page_decode_split(const void* q, const zkv_page_layer* layer, int rows, int G, int n_max, int n_c,
                                     int nk, int n_sink, int near_start, int n_near, float scale, void* out,
                                     float* lse, int64_t* sel_out, int32_t* status, int cluster, void* workspace,
                                     size_t ws_bytes, void* stream) {
    const int CS = pick_cluster(cluster, rows);
    // the split form only pays where the fused kernel takes the two-level select
    if (!(CS > 1 && n_c > 16 * kAttnThreads && nk < n_c) || rows <= 0 || !layer || n_c > n_max || n_c > 16384)
        return zkv_page_decode(q, layer, rows, G, n_max, n_c, nk, n_sink, near_start, n_near, scale, out, lse, sel_out,
                               status, cluster, stream);
    if (!q || !workspace || ws_bytes < zkv_page_decode_split_ws_bytes(rows, n_c) || G < 1 || G > 8)
        return ZKV_ERR_ARG;
    if (((uintptr_t)workspace & 255) || ((uintptr_t)q & 15)) return ZKV_ERR_ALIGN;
    uint8_t* ws = (uint8_t*)workspace;
    float* scores = (float*)ws;
    float* part_out = (float*)(ws + split_ws_scores_bytes(rows, n_c));
    float* part_lse = (float*)(ws + split_ws_scores_bytes(rows, n_c) + split_ws_parts_bytes(rows));
    int rc = zkv_quest_score_gqa(q, G, layer->chunk_min, layer->chunk_max, layer->valid, scores, rows, n_c, n_max,
                                 stream);
    if (rc != ZKV_OK) return rc;
    // clusters per row: spread the attention over about half of the SMs' CTA slots
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int parts = (2 * sms) / (rows * CS);
    parts = parts < 1 ? 1 : (parts > kMaxParts ? kMaxParts : parts);
    if (parts == 1)
        return page_decode_impl(q, layer, rows, G, n_max, n_c, nk, n_sink, near_start, n_near, scale, out, lse,
                                sel_out, status, cluster, scores, n_c, 1, nullptr, stream);
    rc = page_decode_impl(q, layer, rows, G, n_max, n_c, nk, n_sink, near_start, n_near, scale, nullptr, part_lse,
                          sel_out, status, cluster, scores, n_c, parts, part_out, stream);
    if (rc != ZKV_OK) return rc;
    return zkv_lse_merge_n(part_out, part_lse, parts, rows * G, kHeadDim, out, lse, stream);
}

extern "C" int zkv_page_decode_scored(const void* q, const zkv_page_layer* layer, int rows, int G, int n_max,
                                      const float* scores, int64_t sc_ld, int n_c, int nk, int64_t own_lo,
                                      int64_t own_hi, int n_sink, int near_start, int n_near, float scale, int parts,
                                      float* out_f32, float* lse, int64_t* sel_out, int32_t* status, int cluster,
                                      void* stream) {
    if (!scores || !out_f32 || !lse || sc_ld < n_c || parts < 1 || parts > kMaxParts || own_lo < 0 ||
        own_hi < own_lo || nk >= n_c || pick_cluster(cluster, rows) < 2)
        return ZKV_ERR_ARG;
    if ((uintptr_t)scores & 3) return ZKV_ERR_ALIGN;
    return page_decode_impl(q, layer, rows, G, n_max, n_c, nk, n_sink, near_start, n_near, scale, nullptr, lse,
                            sel_out, status, cluster, scores, sc_ld, parts, out_f32, stream, own_lo, own_hi);
}

extern "C" int zkv_page_attend(const void* q, const zkv_page_layer* layer, int rows, int G, int n_max,
                               const int64_t* sel, int n_sel, int64_t sel_lo, int64_t sel_hi, int n_sink,
                               int near_start, int n_near, float scale, void* out, float* out_f32, float* lse,
                               int32_t* status, int cluster, void* stream) {
    if (!q || !layer || (!out && !out_f32) || !sel || rows < 0 || G < 1 || G > 8 || n_sel < 1 || n_near < 0 ||
        n_sink < 0 || near_start < 0 || sel_hi < sel_lo)
        return ZKV_ERR_ARG;
    if ((int64_t)near_start + n_near > layer->near_ld || n_sink > layer->near_ld) return ZKV_ERR_ARG;
    if (n_sel > 4096) return ZKV_ERR_CAPACITY;
    if (rows == 0) return ZKV_OK;
    const zkv_page_layer& L = *layer;
    if (!L.kcodes || !L.vcodes_t || !L.vmeta || !L.chunk_min || !L.chunk_max || !L.kscale ||
        (n_near + n_sink > 0 && (!L.near_k || !L.near_v)))
        return ZKV_ERR_ARG;
    if (((uintptr_t)L.chunk_min & 15) || ((uintptr_t)L.chunk_max & 15) || ((uintptr_t)L.kscale & 15) ||
        ((uintptr_t)L.kcodes & 15) ||
        ((uintptr_t)L.vcodes_t & 15) || ((uintptr_t)L.vmeta & 15) || ((uintptr_t)L.near_k & 15) ||
        ((uintptr_t)L.near_v & 15) || ((uintptr_t)q & 3))
        return ZKV_ERR_ALIGN;
    const int CS = pick_cluster(cluster, rows);
    PageArgs a;
    a.q = (const uint16_t*)q;
    a.L = L;
    a.G = G;
    a.n_max = n_max;
    a.n_c = 0;  // no scoring phase
    a.nk = n_sel;
    a.n_sink = n_sink;
    a.near_start = near_start;
    a.n_near = n_near;
    a.n_c_pad = 0;
    a.per = 0;
    a.pp = (n_sel + CS - 1) / CS;
    a.n_cand = 0;
    a.sc_in = nullptr;
    a.sc_ld = 0;
    a.parts = 1;
    a.pn = ((n_sink + n_near + CS - 1) / CS + 3) & ~3;
    a.sl2 = scale * 1.4426950408889634f;
    a.out = (uint16_t*)out;
    a.lse = lse;
    a.sel_out = nullptr;
    a.status = status;
    a.sel_in = sel;
    a.sel_lo = sel_lo;
    a.sel_hi = sel_hi;
    a.own = 0;
    a.own_lo = a.own_hi = 0;
    a.out_f32 = out_f32;
    void* args[] = {&a};
    return launch_clustered((const void*)page_decode_kernel<false>, rows * CS, kAttnThreads, CS, page_smem(a),
                            (cudaStream_t)stream, args, /*pdl=*/true);
}

extern "C" int zkv_attn_rows(const void* q, const void* keys, const void* values, int64_t kv_ld_row, int rows, int G,
                             int seg0_lo, int seg0_hi, const int64_t* sel, int n_sel, int64_t sel_ld,
                             int64_t sel_offset, int seg1_lo, int seg1_hi, float scale, void* out, float* lse,
                             int split, int32_t* status, void* stream) {
    if (!q || !keys || !values || !out || rows < 0 || G < 1 || G > 8 || kv_ld_row < kHeadDim) return ZKV_ERR_ARG;
    if (seg0_hi < seg0_lo || seg1_hi < seg1_lo || n_sel < 0 || (n_sel > 0 && (!sel || sel_ld < n_sel)))
        return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    if (((uintptr_t)keys & 15) || ((uintptr_t)values & 15) || (kv_ld_row % 8) || ((uintptr_t)q & 3))
        return ZKV_ERR_ALIGN;
    const int CS = pick_cluster(split, rows);
    RowsArgs a;
    a.q = (const uint16_t*)q;
    a.keys = (const uint16_t*)keys;
    a.values = (const uint16_t*)values;
    a.kv_ld_row = kv_ld_row;
    a.kv_cap = kv_ld_row / kHeadDim;
    a.G = G;
    a.s0_lo = seg0_lo;
    a.s0_n = seg0_hi - seg0_lo;
    a.n_sel = n_sel;
    a.s1_lo = seg1_lo;
    a.s1_n = seg1_hi - seg1_lo;
    a.sel = sel;
    a.sel_ld = sel_ld;
    a.sel_off = sel_offset;
    const int total = a.s0_n + a.n_sel + a.s1_n;
    a.ipc = ((total + 7) / 8 + CS - 1) / CS;
    a.sl2 = scale * 1.4426950408889634f;
    a.out = (uint16_t*)out;
    a.lse = lse;
    a.status = status;
    const size_t smem = kRegionBytes + 8 * kHeadDim * 2 + (16 + 8 * kHeadDim) * 4 + 2 * kAttnWarps * 8 + 16;
    void* args[] = {&a};
    return launch_clustered((const void*)attn_rows_kernel, rows * CS, kAttnThreads, CS, smem, (cudaStream_t)stream, args,
                            true);
}

extern "C" int zkv_lse_merge(const void* a, const float* la, const void* b, const float* lb, void* out,
                             float* lse_out, int rows, int dim, void* stream) {
    if (rows < 0 || dim <= 0) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    const int64_t n = (int64_t)rows * dim;
    lse_merge_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint16_t*)a, la, (const uint16_t*)b, lb, (uint16_t*)out, lse_out, rows, dim);
    return cudaGetLastError() == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH;
}

extern "C" int zkv_lse_merge_n(const float* parts, const float* lses, int n, int rows, int dim, void* out,
                               float* lse_out, void* stream) {
    if (rows < 0 || dim <= 0 || n < 1) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    const int64_t tot = (int64_t)rows * dim;
    lse_merge_n_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, (cudaStream_t)stream>>>(parts, lses, n, rows, dim,
                                                                                       (uint16_t*)out, lse_out);
    return cudaGetLastError() == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH;
}
