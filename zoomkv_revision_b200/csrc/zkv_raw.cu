// zkv_raw.cu -- page-mode decode over the RAW bf16 rows of the selected pages:
// four launches per layer chained by programmatic dependent launch.
//
// The reference's page mode (polar_cache.compute with dense_topk = sparse_topk
// = 16 and final_topk = budget, cache_hub/polar_cache_quest_density_single_
// layer_kivi.py:1589-1775) scores every 16-token chunk with Quest, keeps the
// top nk chunks and runs flash-attention over sink + the selected chunks' raw
// K/V rows + the near window (:1734-1750, attn_hub/flash_attn_compat.py:44-99).
// Here, with no bf16 K/V copy:
//
//  * raw_score_kernel: one CTA per (row, 64 chunks).  Bulk copies bring the
//    chunks' Quest min/max (32 KiB) into shared memory; each half-warp scores
//    a chunk with the reference kernel's fp32 operation order and writes the
//    score to the workspace.
//  * raw_select_kernel: one CTA of 1024 threads per row (2, 4 or 8 keys per
//    thread): invalid chunks -> -inf, then the top nk chunk ids (ties to the
//    lowest id, ascending).
//  * raw_attend_kernel: one CTA per (row, EPC entries of 16 tokens) with EPC
//    chosen so that the grid is one wave (3 CTAs per SM): sink and near rows,
//    then selected pages.  Each warp cycles two slots: a page comes in as
//    four 2-D TMA tensor copies with the 128-byte swizzle (K and V, dims 0-63
//    and 64-127), is read with ldmatrix (K, B operand of S = Q K^T) and
//    ldmatrix.trans (V, A operand of O^T = V^T P^T) into mma.sync m16n8k16
//    with an online softmax, and the slot's next copy is issued at once.  The
//    sink and near pages go out before the wait for the select kernel.  The
//    CTA merges its warps and writes one partial (m, l, o).
//  * raw_merge_kernel: one CTA per (row, head): the partials -> out / lse.
//
// Each kernel waits for its predecessor's grid with griddepcontrol.wait and
// releases its successor right after, so a successor's CTAs become resident
// while the predecessor drains: no flags, counters or atomics cross CTAs and
// the workspace carries no state between calls.
#include <cuda.h>

#include <cstring>
#include <algorithm>
#include <mutex>

#include "zkv_common.cuh"

namespace zkv {
namespace rawpg {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kSlotBytes = 8192;                  // one page: K 2 x 2 KiB + V 2 x 2 KiB
constexpr int kSlots = 2;                         // pages per warp of an attend CTA
constexpr int kTileEntries = kWarps * kSlots;     // pages per attend CTA
constexpr int kAttRegion = kTileEntries * kSlotBytes;  // 64 KiB
constexpr int kScoreWarps = 4;                    // warps of a score CTA, 16 chunks each
constexpr int kScoreThreads = kScoreWarps * 32;
constexpr int kScoreTile = kScoreWarps * 16;      // chunks per score CTA (32 KiB of min/max)
constexpr int kScoreRegion = kScoreWarps * kSlotBytes;
constexpr int kPartFloats = 16 + 8 * kHeadDim;    // m[8], l[8], o[8][128]
constexpr int kSelThreads = 1024;                 // threads of a select CTA
constexpr int kMaxChunks = 16384;
constexpr int kMaxTiles = 2048;                   // attend tiles per row
constexpr int kMaxRanks = 8;                      // sequence split: ranks of a group
constexpr int kXPart = 130;                       // exchanged partial of a (row, head): o[128], m, l (tagged)

struct Args {
    CUtensorMap tk;  // raw keys   as [rows * cap][128] bf16, box 64 x 16, 128-B swizzle
    CUtensorMap tv;  // raw values as [rows * cap][128] bf16
    const uint16_t* q;
    const uint16_t* cmin;
    const uint16_t* cmax;
    const uint8_t* valid;
    int64_t cap, page_base;
    int R, G, n_max, n_c, nk, n_sink, near_start, n_near;
    int ST, AT, RS, RN, E, n_c_pad, EPC;
    float sl2;
    uint16_t* out;
    float* lse;
    int64_t* sel_out;
    int32_t* status;
    float* scores;   // [R][n_c_pad]
    int32_t* sel;    // [R][nk]
    float* parts;    // [R][AT][kPartFloats]
    // hierarchical Quest
    const int32_t* group_ids;  // score kernel: warp j scores the small chunks of large chunk group_ids[r][j]
    const int32_t* map_ids;    // select kernel: position p -> map_ids[r][p / factor] * factor + p % factor
    int n_groups, factor, n_chunks_map;
    uint16_t* raw_q_out;       // score kernel: the GQA-mean query, written by each row's first CTA (or NULL)
    // sequence split (the kSplit instantiations): this rank holds the global
    // pages [chunk_lo, chunk_hi) of the row as its local pages 0, 1, ...; the
    // score row and the selection use global page ids
    int rank, world, chunk_lo, chunk_hi, n_total;  // n_total: pages of the whole row (the select's n)
    uint64_t* xrow[kMaxRanks];     // every rank's tagged score row [R][n_c_pad] (as mapped in this process)
    uint64_t* xpart[kMaxRanks];    // every rank's tagged partials [world][R * G][kXPart]
    uint32_t* ep_s;                // own: [R] calls whose score row was complete
    uint32_t* ep_m;                // own: [R * G] calls whose partials were complete
    int32_t* own_range;            // workspace [R][2]: selection positions [a, b) of the own pages
    uint64_t wait_ns;              // limit of each wait on a peer's words
};

// 2-D tiled TMA load (no multicast): box (x .. x+63, y .. y+15) -> dst.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_acq_rel() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

struct WarpState {
    float m;           // running max (log2 units) of head g = lane / 4
    float l;           // running sum over this lane's tokens
    float o[8][4];     // O^T accumulators, m-tile j = dims 16j..16j+15
    uint32_t qa[8][2]; // A fragments of Q (rows = heads), k-step s
};

__device__ __forceinline__ void state_init(WarpState& st, const uint16_t* qrow, int G) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        st.qa[s][0] = g < G ? __ldg(reinterpret_cast<const uint32_t*>(qrow + g * kHeadDim + 16 * s + 2 * tig)) : 0u;
        st.qa[s][1] = g < G ? __ldg(reinterpret_cast<const uint32_t*>(qrow + g * kHeadDim + 16 * s + 8 + 2 * tig)) : 0u;
    }
    st.m = -INFINITY;
    st.l = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) st.o[j][e] = 0.f;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Online-softmax update with scores of tokens 2tig, 2tig+1, 8+2tig, 9+2tig of
// head g; returns the B fragment of P^T for the PV product.
__device__ __forceinline__ void softmax_step(WarpState& st, float (&x)[4], int G, uint32_t& b0, uint32_t& b1) {
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
    b0 = g < G ? pack_bf162(p[0], p[1]) : 0u;
    b1 = g < G ? pack_bf162(p[2], p[3]) : 0u;
}

// One 16-token page in a slot: K boxes at +0 (dims 0-63) and +2048 (dims
// 64-127), V boxes at +4096 and +6144; token t's 16-byte chunk c sits at
// byte 128 t + 16 (c ^ (t & 7)) of its box (the TMA 128-byte swizzle on a
// 1024-byte-aligned box).  Bit t of `present` marks real tokens; absent
// tokens score -inf and their V rows were zeroed.
__device__ __forceinline__ void page_attend(WarpState& st, uint32_t slot, unsigned present, int G, float sl2) {
    const int lane = threadIdx.x & 31, tig = lane & 3;
    const int mtx = lane >> 3;                  // ldmatrix sub-matrix addressed by this lane
    const int t = (lane & 7) + 8 * (mtx >> 1);  // its token row
    const int hi = mtx & 1;                     // second 8-dim chunk of a 16-dim step
    const uint32_t row = slot + 128u * (uint32_t)t;
    float sacc[2][2][4] = {};  // [k-half][token tile][fragment]
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int c = 2 * s + hi;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(row + (uint32_t)((c >> 3) * 2048 + (((c & 7) ^ (t & 7)) << 4)), b0, b1, b2, b3);
        mma_bf16_16816(sacc[s >> 2][0], st.qa[s][0], 0u, st.qa[s][1], 0u, b0, b1);
        mma_bf16_16816(sacc[s >> 2][1], st.qa[s][0], 0u, st.qa[s][1], 0u, b2, b3);
    }
    float x[4] = {(sacc[0][0][0] + sacc[1][0][0]) * sl2, (sacc[0][0][1] + sacc[1][0][1]) * sl2,
                  (sacc[0][1][0] + sacc[1][1][0]) * sl2, (sacc[0][1][1] + sacc[1][1][1]) * sl2};
    if (present != 0xffffu) {
        const int tk[4] = {2 * tig, 2 * tig + 1, 8 + 2 * tig, 9 + 2 * tig};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (!((present >> tk[i]) & 1u)) x[i] = -INFINITY;
    }
    uint32_t pb0, pb1;
    softmax_step(st, x, G, pb0, pb1);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = 2 * j + hi;
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(row + 4096u + (uint32_t)((c >> 3) * 2048 + (((c & 7) ^ (t & 7)) << 4)), a0, a1, a2, a3);
        mma_bf16_16816(st.o[j], a0, a1, a2, a3, pb0, pb1);
    }
}

// Merge the warps' states into (cm, cl, co) in shared memory; scratch >=
// kWarps * (8 * 128 + 16) floats.  Ends with the block synchronised.
__device__ void merge_warps(const WarpState& st, int G, float* scratch, float* cm, float* cl, float* co) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tig = lane & 3;
    float l = st.l;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    float* wm = scratch + warp * (8 * kHeadDim + 16);
    float* wl = wm + 8;
    float* wo = wm + 16;
    if (tig == 0) {
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
    for (int i = threadIdx.x; i < G * kHeadDim; i += kThreads) {
        const int h = i / kHeadDim, d = i % kHeadDim;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, scratch[w * (8 * kHeadDim + 16) + h]);
        float Ls = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
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
    __syncthreads();
}

// Token start and present mask of entry e of a row (sink pseudo-pages, near
// pseudo-pages, then selected pages); the page's chunk id comes from `chunk`.
__device__ __forceinline__ int64_t entry_tokens(const Args& a, int e, int chunk, unsigned& present) {
    if (e < a.RS) {
        const int n = min(16, a.n_sink - 16 * e);
        present = (1u << n) - 1u;
        return 16 * e;
    }
    if (e < a.RS + a.RN) {
        const int k = e - a.RS;
        const int n = min(16, a.n_near - 16 * k);
        present = (1u << n) - 1u;
        return (int64_t)a.near_start + 16 * k;
    }
    present = 0xffffu;
    return a.page_base + 16 * (int64_t)chunk;
}

// ---------------------------------------------------------------- kernel 1: scores
// Sequence-split tail of the score kernel (after the min/max copies and the
// GQA mean): the warp scores its nch chunks (invalid ones -> -inf, the key
// the select gives an invalid chunk, so the select needs no validity) and
// stores each score into every rank's score row at its global id as a
// tagged word {score, this call's epoch} (over NVLink for the peers).  No
// fence or flag: the reader checks each word's epoch.
__device__ __forceinline__ void split_scores(const Args& a, int r, int cc, int nch, const uint8_t* slot,
                                             uint64_t* bar, const uint16_t* rq, float* sb) {
    const int lane = threadIdx.x & 31;
    if (nch <= 0) return;
    const uint32_t tag = __ldcg(a.ep_s + r) + 1u;
    const bool ok = mbar_wait(bar, 0, a.status);
    const int hl = lane & 15, half = lane >> 4;
    const uint4 qv = *reinterpret_cast<const uint4*>(rq + 8 * hl);
    const uint8_t* vrow = a.valid ? a.valid + (int64_t)r * a.n_max + cc : nullptr;
#pragma unroll 4
    for (int u = 0; u < 8; ++u) {
        const int lc = 2 * u + half;
        uint4 mn = make_uint4(0, 0, 0, 0), mx = mn;
        if (ok && lc < nch) {
            mn = *reinterpret_cast<const uint4*>(slot + lc * 256 + 16 * hl);
            mx = *reinterpret_cast<const uint4*>(slot + 4096 + lc * 256 + 16 * hl);
        }
        const float sc = quest_half(qv, mn, mx);
        if (hl == 0 && lc < nch) sb[lc] = (ok && (!vrow || vrow[lc])) ? sc : -INFINITY;
    }
    __syncwarp();
    for (int i = lane; i < 16 * a.world; i += 32) {  // lane i: chunk i % 16 to rank i / 16
        const int q = i >> 4, c = i & 15;
        if (c < nch)
            st_relaxed_sys_u64(a.xrow[q] + (int64_t)r * a.n_c_pad + a.chunk_lo + cc + c,
                               tagged(__float_as_uint(sb[c]), tag));
    }
}

// One CTA per (row, 64 chunks): each warp bulk-copies its 16 chunks' min and
// max (8 KiB) into shared memory and scores them; the scores go to the
// workspace (kSplit: to every rank's score row, split_scores).  Validity is
// applied by the select (kSplit: here).
template <bool kSplit>
__global__ void __launch_bounds__(kScoreThreads) raw_score_kernel(const __grid_constant__ Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* region = smem;                                   // [kScoreWarps][8 KiB]: min 4 KiB, max 4 KiB
    uint16_t* rq = reinterpret_cast<uint16_t*>(smem + kScoreRegion);
    uint64_t* bars = reinterpret_cast<uint64_t*>(rq + kHeadDim);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = blockIdx.x / a.ST, tile = blockIdx.x % a.ST;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kScoreWarps; ++i) mbar_init(bars + i, 1);
        mbar_fence_init();
    }
    __syncthreads();
    grid_dep_wait();          // q is the previous kernel's output; the workspace may still be read by it
    grid_dep_launch_next();   // the select kernel may become resident (it waits for this grid)
    // cc: first score position of this warp; src: first chunk it reads
    int cc, src, nch;
    bool oob = false;
    if (a.group_ids) {  // sub-chunk scores of the row's selected large chunks (quest_chunk_score.cu:263-360)
        const int j = tile * kScoreWarps + warp;
        cc = j * a.factor;
        nch = j < a.n_groups ? a.factor : 0;
        const int lid = nch ? __ldcg(a.group_ids + (int64_t)r * a.n_groups + j) : 0;
        src = lid * a.factor;
        oob = lid < 0 || src + a.factor > a.n_max;  // scored -inf, as the reference's bound check
    } else {
        cc = tile * kScoreTile + 16 * warp;
        src = cc;
        nch = max(0, min(16, a.n_c - cc));
    }
    uint8_t* slot = region + warp * kSlotBytes;
    if (lane == 0 && nch > 0 && !oob) {
        mbar_arrive_expect_tx(bars + warp, (uint32_t)nch * kHeadDim * 2 * 2);
        bulk_g2s(slot, a.cmin + ((int64_t)r * a.n_max + src) * kHeadDim, nch * kHeadDim * 2, bars + warp);
        bulk_g2s(slot + 4096, a.cmax + ((int64_t)r * a.n_max + src) * kHeadDim, nch * kHeadDim * 2, bars + warp);
    }
    {   // GQA-mean query (compute() :1622-1626: fp32 sum in head order / G, bf16)
        const uint16_t* qr = a.q + (int64_t)r * a.G * kHeadDim;
        for (int d = threadIdx.x; d < kHeadDim; d += kScoreThreads) {
            float acc = 0.f;
            for (int g = 0; g < a.G; ++g) acc = __fadd_rn(acc, bfbits2f(__ldg(qr + g * kHeadDim + d)));
            rq[d] = f2bfbits(__fdiv_rn(acc, (float)a.G));
            if (a.raw_q_out && tile == 0) a.raw_q_out[(int64_t)r * kHeadDim + d] = rq[d];
        }
    }
    __syncthreads();
    if constexpr (kSplit) {
        split_scores(a, r, cc, nch, slot, bars + warp, rq, reinterpret_cast<float*>(bars + kScoreWarps) + 16 * warp);
        return;
    }
    if (nch == 0) return;
    float* srow0 = a.scores + (int64_t)r * a.n_c_pad;
    if (oob) {
        if (lane < nch) srow0[cc + lane] = -INFINITY;
        return;
    }
    const bool ok = mbar_wait(bars + warp, 0, a.status);
    const int hl = lane & 15, half = lane >> 4;
    const uint4 qv = *reinterpret_cast<const uint4*>(rq + 8 * hl);
    float* srow = a.scores + (int64_t)r * a.n_c_pad;
#pragma unroll 4
    for (int u = 0; u < 8; ++u) {
        const int lc = 2 * u + half;
        uint4 mn = make_uint4(0, 0, 0, 0), mx = mn;
        if (ok && lc < nch) {
            mn = *reinterpret_cast<const uint4*>(slot + lc * 256 + 16 * hl);
            mx = *reinterpret_cast<const uint4*>(slot + 4096 + lc * 256 + 16 * hl);
        }
        const float sc = quest_half(qv, mn, mx);
        if (hl == 0 && lc < nch) srow[cc + lc] = ok ? sc : -INFINITY;
    }
}

// ---------------------------------------------------------------- kernel 2: select
// One CTA of kSelThreads per row: the row's scores (invalid chunks -> -inf)
// -> top nk chunk ids, ties to the lowest id, ascending (select_spread with
// 2, 4 or 8 keys per thread up to 8 * kSelThreads chunks, the radix select
// over global scores beyond).
using SelShared = SelSharedT<kSelThreads>;

// kSplit: the row is the whole tagged score row in this rank's exchange
// buffer; every thread waits (bounded) until its words carry this call's
// epoch and copies the scores into the workspace row, which the select then
// reads as on one GPU.  The split select does not wait for the score grid
// to complete (that completion includes the flush of the score kernel's
// stores to the peers, about 3 us): it waits on the words themselves, this
// rank's included.  It cannot wait on a producer that is not running: with
// programmatic dependent launch this grid starts only after every score
// CTA has executed its launch_dependents, i.e. every score CTA is resident
// and none of them waits on this grid.  Nothing earlier needs ordering
// here: those score CTAs passed their own dependency wait (the previous
// call's merge, hence its attend, had completed) before the trigger.  The
// CTA also records which selection positions are the pages this rank holds
// (ids ascend, so they are one run [a, b)).
template <bool kSplit>
__global__ void __launch_bounds__(kSelThreads) raw_select_kernel(const __grid_constant__ Args a) {
    __shared__ SelShared S;
    __shared__ int sx[4];  // kSplit: selected ids below the own range, inside it; a wait expired
    const int r = blockIdx.x, tid = threadIdx.x;
    for (int i = tid; i < kSelBins; i += kSelThreads) S.hist[i] = 0;
    if (tid == 0) S.misc[3] = 0;
    if (kSplit && tid < 4) sx[tid] = 0;
    if constexpr (!kSplit) grid_dep_wait();  // the scores of the score kernel
    grid_dep_launch_next();   // the attend kernel may become resident (it waits for this grid)
    if constexpr (kSplit) {
        const uint32_t target = __ldcg(a.ep_s + r) + 1u;
        const uint64_t* xr = a.xrow[a.rank] + (int64_t)r * a.n_c_pad;
        float* plain = a.scores + (int64_t)r * a.n_c_pad;
        bool ok = true;
        for (int i0 = 0; i0 < a.n_total; i0 += 8 * kSelThreads) {  // 8 words of a thread in flight at once
            uint64_t w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + j * kSelThreads + tid;
                w[j] = i < a.n_total ? ld_relaxed_sys_u64(xr + i) : 0ull;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + j * kSelThreads + tid;
                if (i < a.n_total)
                    plain[i] = __uint_as_float((uint32_t)wait_tagged(xr + i, w[j], target, a.wait_ns, ok));
            }
        }
        if (!ok) {
            set_status(a.status, ZKV_ERR_TIMEOUT);
            sx[2] = 1;
        }
        __syncthreads();  // every word read (the epoch below) and the workspace row written
        if (tid == 0) a.ep_s[r] = target;
        if (sx[2]) {  // no pages of this row are attended
            if (tid == 0) {
                a.own_range[2 * r] = 0;
                a.own_range[2 * r + 1] = 0;
            }
            return;
        }
    }
    const int n = kSplit ? a.n_total : a.n_c, k = a.nk;
    const float* srow = a.scores + (int64_t)r * a.n_c_pad;
    const uint8_t* vrow = (!kSplit && a.valid) ? a.valid + (int64_t)r * a.n_max : nullptr;
    int32_t* selr = a.sel + (int64_t)r * a.nk;
    int64_t* selo = a.sel_out ? a.sel_out + (int64_t)r * a.nk : nullptr;
    auto emit = [&](int pos, int i) {
        if (a.map_ids) {  // quest_map_back (quest_chunk_score.cu:363-416)
            const int sel = i / a.factor;
            i = __ldcg(a.map_ids + (int64_t)r * a.n_groups + sel) * a.factor + (i - sel * a.factor);
            i = min(max(i, 0), a.n_chunks_map - 1);
        }
        selr[pos] = i;
        if (selo) selo[pos] = i;
        if constexpr (kSplit) {
            if (i < a.chunk_lo)
                atomicAdd(&sx[0], 1);
            else if (i < a.chunk_hi)
                atomicAdd(&sx[1], 1);
        }
    };
    auto gkey = [&](int i) { return (vrow && !vrow[i]) ? kOrderedNegInf : ordered_u32(__ldcg(srow + i)); };
    if (n <= 2 * kSelThreads) {
        select_spread<kSelThreads, 2>(S, n, k, srow, vrow, emit, gkey);
    } else if (n <= 4 * kSelThreads) {
        select_spread<kSelThreads, 4>(S, n, k, srow, vrow, emit, gkey);
    } else if (n <= 8 * kSelThreads) {
        select_spread<kSelThreads, 8>(S, n, k, srow, vrow, emit, gkey);
    } else {
        __syncthreads();
        block_topk<kSelThreads, true>(gkey, n, k, S.hist, S.misc, S.scan, emit);
    }
    if constexpr (kSplit) {
        __syncthreads();
        if (tid == 0) {
            a.own_range[2 * r] = sx[0];
            a.own_range[2 * r + 1] = sx[0] + sx[1];
        }
    }
}

// ---------------------------------------------------------------- kernel 3: attend
// One CTA per (row, EPC entries of 16 tokens), sized so that the grid is one
// wave; warp w attends entries e0 + w, e0 + w + 4, ... through two TMA slots
// (the next page's copy is issued as soon as a slot's page is consumed) and
// the CTA writes one partial (m, l, o) of the row.  kSplit: the row's
// entries are this rank's raw rows (rank 0: sink and near) and the selected
// pages this rank holds, spread over the row's CTAs once the selection is
// known (no copies are issued before it).
template <bool kSplit>
__global__ void __launch_bounds__(kThreads, 3) raw_attend_kernel(const __grid_constant__ Args a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((base_u32 + 1023u) & ~1023u) - base_u32);  // swizzled boxes: 1024-B aligned
    uint8_t* region = smem;
    float* region_f = reinterpret_cast<float*>(region);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kAttRegion);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = blockIdx.x / a.AT, tile = blockIdx.x % a.AT;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kWarps * kSlots; ++i) mbar_init(bars + i, 1);
        mbar_fence_init();
    }
    __syncthreads();
    int e0 = tile * a.EPC;
    int e1 = min(a.E, e0 + a.EPC);
    int nw = e1 - e0 > warp ? (e1 - e0 - warp + kWarps - 1) / kWarps : 0;  // pages of this warp (<= 32)
    const int pg0 = a.RS + a.RN;
    const uint32_t slot0 = smem_u32(region) + (uint32_t)(warp * kSlots * kSlotBytes);
    auto issue_chunk = [&](int j, int chunk) -> unsigned {  // warp-uniform; returns the page's present mask
        unsigned pr;
        const int64_t y0 = entry_tokens(a, e0 + warp + kWarps * j, chunk, pr);
        if (lane == 0) {
            const int y = (int)((int64_t)r * a.cap + y0);
            const uint32_t dst = slot0 + (uint32_t)((j & 1) * kSlotBytes);
            uint64_t* bar = bars + warp * kSlots + (j & 1);
            mbar_arrive_expect_tx(bar, kSlotBytes);
            tma_load_2d(dst, &a.tk, 0, y, bar);
            tma_load_2d(dst + 2048, &a.tk, 64, y, bar);
            tma_load_2d(dst + 4096, &a.tv, 0, y, bar);
            tma_load_2d(dst + 6144, &a.tv, 64, y, bar);
        }
        return pr;
    };
    // Sink and near pages do not depend on the selection, and the K/V rows
    // and q were written before the score kernel began: their copies and the
    // query fragments are taken before waiting for the select kernel.
    const bool pre0 = !kSplit && nw > 0 && e0 + warp < pg0;
    const bool pre1 = !kSplit && nw > 1 && e0 + warp + kWarps < pg0;
    unsigned pres0 = pre0 ? issue_chunk(0, 0) : 0u;
    unsigned pres1 = pre1 ? issue_chunk(1, 0) : 0u;
    WarpState st;
    state_init(st, a.q + (int64_t)r * a.G * kHeadDim, a.G);
    grid_dep_wait();          // the selection of the select kernel
    grid_dep_launch_next();   // the merge kernel may become resident (it waits for this grid)
    int sel_a = 0;
    if constexpr (kSplit) {  // own pages: selection positions [sel_a, b); entries spread over the AT CTAs
        sel_a = __ldcg(a.own_range + 2 * r);
        const int ed = pg0 + __ldcg(a.own_range + 2 * r + 1) - sel_a;
        const int epc = (ed + a.AT - 1) / a.AT;
        e0 = tile * epc;
        e1 = min(ed, e0 + epc);
        nw = e1 - e0 > warp ? (e1 - e0 - warp + kWarps - 1) / kWarps : 0;
    }
    // lane j reads the chunk id of the warp's j-th entry (all in flight at once)
    int my_chunk = 0;
    if (lane < nw) {
        const int e = e0 + warp + kWarps * lane;
        if (e >= pg0) {
            const int p = e - pg0;
            if constexpr (kSplit) {
                my_chunk = __ldcg(a.sel + (int64_t)r * a.nk + sel_a + p) - a.chunk_lo;  // a local page
            } else {
                my_chunk = a.ST > 0 ? __ldcg(a.sel + (int64_t)r * a.nk + p) : p;
                if (a.ST == 0 && a.sel_out) a.sel_out[(int64_t)r * a.nk + p] = p;  // identity selection
            }
        }
    }
    auto issue = [&](int j) -> unsigned {
        return issue_chunk(j, __shfl_sync(0xffffffffu, my_chunk, j & 31));
    };
    if (nw > 0 && !pre0) pres0 = issue(0);
    if (nw > 1 && !pre1) pres1 = issue(1);
    for (int j = 0; j < nw; ++j) {
        const int sl = j & 1;
        const unsigned pres = sl ? pres1 : pres0;
        if (!mbar_wait(bars + warp * kSlots + sl, (uint32_t)((j >> 1) & 1), a.status)) break;  // status set
        uint8_t* slot = region + (warp * kSlots + sl) * kSlotBytes;
        if (pres != 0xffffu) {  // zero the V rows of absent tokens (p = 0 must meet finite V)
            for (int i = lane; i < 16 * 16; i += 32) {
                const int tkn = i >> 4, box = (i >> 3) & 1, c = i & 7;
                if (!((pres >> tkn) & 1u))
                    *reinterpret_cast<uint4*>(slot + 4096 + box * 2048 + tkn * 128 + c * 16) = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }
        page_attend(st, slot0 + (uint32_t)(sl * kSlotBytes), pres, a.G, a.sl2);
        if (j + 2 < nw) {  // refill the slot: generic reads/writes of it before the async-proxy copy
            fence_proxy_async();
            __syncwarp();
            const unsigned np = issue(j + 2);
            if (sl) pres1 = np; else pres0 = np;
        }
    }
    __syncthreads();
    float* cm = region_f + 4224;  // past the warp scratch (4 x 1040 floats)
    float* cl = cm + 8;
    float* co = cl + 8;
    merge_warps(st, a.G, region_f, cm, cl, co);
    float* part = a.parts + ((int64_t)r * a.AT + tile) * kPartFloats;
    if (threadIdx.x < 8) {
        part[threadIdx.x] = (int)threadIdx.x < a.G ? cm[threadIdx.x] : -INFINITY;
        part[8 + threadIdx.x] = (int)threadIdx.x < a.G ? cl[threadIdx.x] : 0.f;
    }
    for (int i = threadIdx.x; i < a.G * kHeadDim / 4; i += kThreads)
        reinterpret_cast<float4*>(part + 16)[i] = reinterpret_cast<const float4*>(co)[i];
}

// ---------------------------------------------------------------- kernel 4: merge
// One CTA per (row, head), one thread per dim: the row's AT partials of the
// head -> out (bf16) and lse (natural log).  Partials come in batches of
// kMergeBatch with every load of a batch in flight at once; batches combine
// with an online rescale (one batch when AT <= kMergeBatch).
constexpr int kMergeBatch = 32;

// Sequence-split tail of the merge: this rank's (M, L, O) of (row r, head h)
// (M in log2 units, L and O not normalised) goes to slot `rank` of every
// rank's exchange buffer as tagged words {value, this call's epoch}; every
// thread then waits (bounded) for its dim's word and the (M, L) words of
// every rank in its own buffer and combines the world partials in rank
// order, so every rank writes the same out / lse.  No fence or flag.
__device__ __forceinline__ void split_combine(const Args& a, int r, int h, int d, float M, float L, float O) {
    const int64_t rg = (int64_t)a.R * a.G, rh = (int64_t)r * a.G + h;
    const uint32_t tag = __ldcg(a.ep_m + rh) + 1u;
    for (int q = 0; q < a.world; ++q) {
        uint64_t* dst = a.xpart[q] + ((int64_t)a.rank * rg + rh) * kXPart;
        st_relaxed_sys_u64(dst + d, tagged(__float_as_uint(O), tag));
        if (d == 0) {
            st_relaxed_sys_u64(dst + kHeadDim, tagged(__float_as_uint(M), tag));
            st_relaxed_sys_u64(dst + kHeadDim + 1, tagged(__float_as_uint(L), tag));
        }
    }
    const uint64_t* src = a.xpart[a.rank] + rh * kXPart;
    float mq[kMaxRanks], lq[kMaxRanks], oq[kMaxRanks];
    uint64_t wm[kMaxRanks], wl[kMaxRanks], wo[kMaxRanks];
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q) {  // every load in flight before any wait
        if (q < a.world) {
            const uint64_t* pq = src + q * rg * kXPart;
            wo[q] = ld_relaxed_sys_u64(pq + d);
            wm[q] = ld_relaxed_sys_u64(pq + kHeadDim);
            wl[q] = ld_relaxed_sys_u64(pq + kHeadDim + 1);
        }
    }
    bool ok = true;
    float Ms = -INFINITY;
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q) {
        if (q < a.world) {
            const uint64_t* pq = src + q * rg * kXPart;
            oq[q] = __uint_as_float((uint32_t)wait_tagged(pq + d, wo[q], tag, a.wait_ns, ok));
            mq[q] = __uint_as_float((uint32_t)wait_tagged(pq + kHeadDim, wm[q], tag, a.wait_ns, ok));
            lq[q] = __uint_as_float((uint32_t)wait_tagged(pq + kHeadDim + 1, wl[q], tag, a.wait_ns, ok));
            Ms = fmaxf(Ms, mq[q]);
        }
    }
    if (!ok) set_status(a.status, ZKV_ERR_TIMEOUT);
    float Ls = 0.f, Os = 0.f;
    if (Ms != -INFINITY) {
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q) {
            if (q < a.world) {
                const float wt = (mq[q] == -INFINITY) ? 0.f : ex2(mq[q] - Ms);
                Ls += wt * lq[q];
                Os += wt * oq[q];
            }
        }
    }
    if (d == 0 && a.lse) a.lse[rh] = (Ls > 0.f) ? (Ms + __log2f(Ls)) * 0.69314718055994531f : -INFINITY;
    a.out[rh * kHeadDim + d] = f2bfbits(Ls > 0.f ? Os * (1.f / Ls) : 0.f);
    __syncthreads();  // every thread read the epoch above
    if (d == 0) a.ep_m[rh] = tag;
}

template <bool kSplit>
__global__ void __launch_bounds__(kHeadDim) raw_merge_kernel(const __grid_constant__ Args a) {
    const int r = blockIdx.x / a.G, h = blockIdx.x % a.G, d = threadIdx.x;
    grid_dep_wait();          // the partials of the attend kernel
    grid_dep_launch_next();   // the next launch may become resident (it waits for this grid)
    const float* pr = a.parts + (int64_t)r * a.AT * kPartFloats;
    float M = -INFINITY, L = 0.f, O = 0.f;
    for (int t0 = 0; t0 < a.AT; t0 += kMergeBatch) {
        float m[kMergeBatch], l[kMergeBatch], o[kMergeBatch];
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
            const bool in = t0 + u < a.AT;
            const float* pt = pr + (int64_t)(t0 + u) * kPartFloats;
            m[u] = in ? __ldcg(pt + h) : -INFINITY;
            l[u] = in ? __ldcg(pt + 8 + h) : 0.f;
            o[u] = in ? __ldcg(pt + 16 + h * kHeadDim + d) : 0.f;
        }
        float Mb = M;
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) Mb = fmaxf(Mb, m[u]);
        if (Mb == -INFINITY) continue;  // nothing attended so far
        const float sc = (M == -INFINITY) ? 0.f : ex2(M - Mb);
        L *= sc;
        O *= sc;
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
            const float wt = (m[u] == -INFINITY) ? 0.f : ex2(m[u] - Mb);
            L += wt * l[u];
            O += wt * o[u];
        }
        M = Mb;
    }
    if constexpr (kSplit) {
        split_combine(a, r, h, d, M, L, O);
        return;
    }
    if (d == 0 && a.lse) a.lse[(int64_t)r * a.G + h] = (L > 0.f) ? (M + __log2f(L)) * 0.69314718055994531f : -INFINITY;
    a.out[((int64_t)r * a.G + h) * kHeadDim + d] = f2bfbits(L > 0.f ? O * (1.f / L) : 0.f);
}

// ---------------------------------------------------------------- large-chunk min/max
// _update_large_chunk_minmax (polar_cache_kivi_quest_density_seperate_kernel.py:
// 1762-1798): group g of a row covers chunks [g*factor, min(g*factor + factor,
// valid_end)); its min / max are the element-wise bf16 min / max of those
// chunks' min / max and the group becomes valid.  Empty groups are left as
// they are.  One CTA of 64 threads (two dims each) per (group, row).
__global__ void __launch_bounds__(64) large_minmax_kernel(const uint32_t* __restrict__ mn,
                                                          const uint32_t* __restrict__ mx, int n_max, int valid_end,
                                                          int factor, int g_lo, uint32_t* lmn, uint32_t* lmx,
                                                          uint8_t* lvalid, int n_max_large) {
    const int r = blockIdx.y, g = g_lo + blockIdx.x, t = threadIdx.x;
    const int b_lo = g * factor;
    const int b_hi = min(min(b_lo + factor, valid_end), n_max);
    if (b_hi <= b_lo) return;
    const int64_t src = ((int64_t)r * n_max + b_lo) * (kHeadDim / 2) + t;
    uint32_t a = __ldg(mn + src), z = __ldg(mx + src);
    for (int b = 1; b < b_hi - b_lo; ++b) {
        const uint32_t u = __ldg(mn + src + (int64_t)b * (kHeadDim / 2));
        const uint32_t v = __ldg(mx + src + (int64_t)b * (kHeadDim / 2));
        uint32_t lo = a & 0xffffu, hi = a >> 16;
        if (bfbits2f((uint16_t)(u & 0xffffu)) < bfbits2f((uint16_t)lo)) lo = u & 0xffffu;
        if (bfbits2f((uint16_t)(u >> 16)) < bfbits2f((uint16_t)hi)) hi = u >> 16;
        a = lo | (hi << 16);
        lo = z & 0xffffu;
        hi = z >> 16;
        if (bfbits2f((uint16_t)(v & 0xffffu)) > bfbits2f((uint16_t)lo)) lo = v & 0xffffu;
        if (bfbits2f((uint16_t)(v >> 16)) > bfbits2f((uint16_t)hi)) hi = v >> 16;
        z = lo | (hi << 16);
    }
    const int64_t dst = ((int64_t)r * n_max_large + g) * (kHeadDim / 2) + t;
    lmn[dst] = a;
    lmx[dst] = z;
    if (t == 0) lvalid[(int64_t)r * n_max_large + g] = 1;
}

// ---------------------------------------------------------------- host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &qr) ==
                cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// [n_tok][128] bf16 rows, 16-row x 64-dim boxes, 128-byte swizzle, zero fill
static bool encode_rows(CUtensorMap* map, const void* base, int64_t n_tok) {
    EncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)n_tok};
    const cuuint64_t strides[1] = {(cuuint64_t)kHeadDim * 2};
    const cuuint32_t box[2] = {64, 16};
    const cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor maps of recently used (keys, values, rows) triples: encoding two
// maps costs a few microseconds of host time per call, and a decode loop
// calls the same layers over and over.  A map depends only on the base
// address and the row count, both part of the key.
struct MapEntry {
    const void* keys;
    const void* values;
    int64_t n_tok;
    int dev;
    CUtensorMap tk, tv;
};
constexpr int kMapCache = 128;

static bool cached_maps(CUtensorMap* tk, CUtensorMap* tv, const void* keys, const void* values, int64_t n_tok) {
    static MapEntry cache[kMapCache];
    static int used = 0, next = 0;
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (int i = 0; i < used; ++i) {
            const MapEntry& e = cache[i];
            if (e.keys == keys && e.values == values && e.n_tok == n_tok && e.dev == dev) {
                *tk = e.tk;
                *tv = e.tv;
                return true;
            }
        }
    }
    if (!encode_rows(tk, keys, n_tok) || !encode_rows(tv, values, n_tok)) return false;
    std::lock_guard<std::mutex> lock(mu);
    MapEntry& e = cache[next];
    e.keys = keys;
    e.values = values;
    e.n_tok = n_tok;
    e.dev = dev;
    e.tk = *tk;
    e.tv = *tv;
    next = (next + 1) % kMapCache;
    used = used < kMapCache ? used + 1 : used;
    return true;
}

struct Plan {
    int ST, AT, RS, RN, E, n_c_pad, EPC;
    int ST1, n_large, n_large_pad;  // hierarchical: stage-1 score CTAs per row, large chunks scored, row stride
    size_t off_scores, off_sel, off_sel_large, off_parts, bytes;
};

// Hierarchical Quest inputs (zero `factor`: the flat select).
struct Hier {
    const void* lmin;
    const void* lmax;
    const uint8_t* lvalid;
    int n_max_large, factor, nk_large;
};

static size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

// Attend CTAs resident per SM (shared memory: 3 x 66.6 KiB).
constexpr int kAttendPerSm = 3;

static int sm_count() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

// n_c: chunks scored by the flat select, or the small chunks of a
// hierarchical one (h.factor > 0: n_c / factor large chunks are scored, the
// top h.nk_large of them expand to nk_large * factor sub-chunks, of which
// the top nk are attended).
static Plan make_plan(int R, int n_c, int nk, int n_sink, int n_near, const Hier& h) {
    Plan p;
    const int nsel = n_c > 0 ? nk : 0;
    const bool hier = h.factor > 0;
    p.n_large = hier ? n_c / h.factor : 0;
    p.n_large_pad = (p.n_large + 31) & ~31;
    p.ST1 = hier ? (p.n_large + kScoreTile - 1) / kScoreTile : 0;
    if (hier)  // stage 2: one warp per selected large chunk
        p.ST = (h.nk_large + kScoreWarps - 1) / kScoreWarps;
    else       // no scoring when every chunk is selected
        p.ST = nk < n_c ? (n_c + kScoreTile - 1) / kScoreTile : 0;
    const int n_scored = hier ? h.nk_large * h.factor : n_c;
    p.RS = (n_sink + 15) / 16;
    p.RN = (n_near + 15) / 16;
    p.E = p.RS + p.RN + nsel;
    // CTAs per row: one wave of attend CTAs when the rows allow it, at most
    // 128 entries per CTA (a warp's chunk ids in one warp-wide load), at least
    // kTileEntries entries per CTA; a count just above one merge batch is
    // trimmed to it (one round of partial loads in the merge for at most a
    // quarter more entries per CTA)
    {
        const int slots = kAttendPerSm * sm_count();
        int c = R > 0 ? slots / R : 1;
        c = std::max(1, std::min(c, (p.E + kTileEntries - 1) / kTileEntries));
        if (c > kMergeBatch && c <= kMergeBatch + kMergeBatch / 4) c = kMergeBatch;
        c = std::max(c, (p.E + 127) / 128);
        p.EPC = p.E > 0 ? (p.E + c - 1) / c : 1;
        p.AT = p.E > 0 ? (p.E + p.EPC - 1) / p.EPC : 1;
    }
    p.n_c_pad = (n_scored + 31) & ~31;
    const int stride = std::max(p.n_c_pad, p.n_large_pad);
    p.off_scores = 0;
    p.off_sel = p.off_scores + up256((size_t)R * stride * 4);
    p.off_sel_large = p.off_sel + up256((size_t)R * (nk > 0 ? nk : 1) * 4);
    p.off_parts = p.off_sel_large + (hier ? up256((size_t)R * h.nk_large * 4) : 0);
    // partials for the most CTAs per row any device can use (kTileEntries
    // entries each), so the size does not depend on the SM count
    const int max_tiles = p.E > 0 ? (p.E + kTileEntries - 1) / kTileEntries : 1;
    p.bytes = p.off_parts + up256((size_t)R * max_tiles * kPartFloats * 4);
    return p;
}

static size_t score_smem() { return kScoreRegion + kHeadDim * 2 + kScoreWarps * 8; }
static size_t select_smem() { return 0; }
static size_t attend_smem() { return 1024 + kAttRegion + kWarps * kSlots * 8; }

static int launch_pdl(const void* fn, int grid, int threads, size_t smem, cudaStream_t stream, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return ZKV_ERR_LAUNCH;
    return cudaGetLastError() == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH;
}

static int decode_raw(const void* q, const zkv_raw_layer* layer, int rows, int G, int n_max, int n_c, int nk,
                      int n_sink, int near_start, int n_near, float scale, void* out, float* lse, int64_t* sel_out,
                      int32_t* status, void* workspace, size_t ws_bytes, void* stream, const Hier& h) {
    const bool hier = h.factor > 0;
    if (!q || !layer || !out || !workspace || rows < 0 || G < 1 || G > 8 || n_c < 0 || n_c > n_max || nk < 0 ||
        (n_c > 0 && (nk < 1 || nk > n_c)) || n_sink < 0 || n_near < 0 || near_start < 0)
        return ZKV_ERR_ARG;
    if (hier) {
        const int n_large = n_c / h.factor;
        if (h.factor > 16 || !h.lmin || !h.lmax || n_large < 1 || h.n_max_large < n_large || h.nk_large < 1 ||
            h.nk_large > n_large || nk > h.nk_large * h.factor)
            return ZKV_ERR_ARG;
    }
    const zkv_raw_layer& L = *layer;
    if (!L.keys || !L.values || L.kv_ld_row < kHeadDim || (L.kv_ld_row % kHeadDim) || L.page_base < 0 ||
        (n_c > 0 && (!L.chunk_min || !L.chunk_max)))
        return ZKV_ERR_ARG;
    const int64_t cap = L.kv_ld_row / kHeadDim;
    if (L.page_base + 16 * (int64_t)n_c > cap || (int64_t)near_start + n_near > cap || n_sink > cap)
        return ZKV_ERR_ARG;
    if (n_c > kMaxChunks || (int64_t)rows * cap >= (int64_t)1 << 31) return ZKV_ERR_CAPACITY;
    const Plan p = make_plan(rows, n_c, nk, n_sink, n_near, h);
    if (ws_bytes < p.bytes) return ZKV_ERR_ARG;
    if (p.AT > kMaxTiles || (int64_t)rows * (p.ST + p.ST1 + p.AT) >= ((int64_t)1 << 31)) return ZKV_ERR_CAPACITY;
    if (rows == 0) return ZKV_OK;
    if (((uintptr_t)L.keys & 15) || ((uintptr_t)L.values & 15) || ((uintptr_t)L.chunk_min & 15) ||
        ((uintptr_t)L.chunk_max & 15) || ((uintptr_t)q & 3) || ((uintptr_t)workspace & 255) ||
        (hier && (((uintptr_t)h.lmin & 15) || ((uintptr_t)h.lmax & 15))))
        return ZKV_ERR_ALIGN;
    Args a;
    memset(&a, 0, sizeof(a));
    if (!cached_maps(&a.tk, &a.tv, L.keys, L.values, (int64_t)rows * cap)) return ZKV_ERR_LAUNCH;
    a.q = (const uint16_t*)q;
    a.cmin = (const uint16_t*)L.chunk_min;
    a.cmax = (const uint16_t*)L.chunk_max;
    a.valid = L.valid;
    a.cap = cap;
    a.page_base = L.page_base;
    a.R = rows;
    a.G = G;
    a.n_max = n_max;
    a.n_c = n_c;
    a.nk = n_c > 0 ? nk : 0;
    a.n_sink = n_sink;
    a.near_start = near_start;
    a.n_near = n_near;
    a.ST = p.ST;
    a.AT = p.AT;
    a.RS = p.RS;
    a.RN = p.RN;
    a.E = p.E;
    a.n_c_pad = p.n_c_pad;
    a.EPC = p.EPC;
    a.sl2 = scale * 1.4426950408889634f;
    a.out = (uint16_t*)out;
    a.lse = lse;
    a.sel_out = sel_out;
    a.status = status;
    uint8_t* ws = (uint8_t*)workspace;
    a.scores = (float*)(ws + p.off_scores);
    a.sel = (int32_t*)(ws + p.off_sel);
    a.parts = (float*)(ws + p.off_parts);
    Args a1;  // hierarchical stage 1: Quest over the large chunks, top nk_large of them
    if (hier) {
        int32_t* sel_large = (int32_t*)(ws + p.off_sel_large);
        a1 = a;
        a1.cmin = (const uint16_t*)h.lmin;
        a1.cmax = (const uint16_t*)h.lmax;
        a1.valid = h.lvalid;
        a1.n_max = h.n_max_large;
        a1.n_c = p.n_large;
        a1.nk = h.nk_large;
        a1.n_c_pad = p.n_large_pad;
        a1.ST = p.ST1;
        a1.sel = sel_large;
        a1.sel_out = nullptr;
        // stage 2 (in a): the sub-chunks of the selected large chunks, top nk
        a.valid = nullptr;
        a.n_c = h.nk_large * h.factor;
        a.group_ids = sel_large;
        a.map_ids = sel_large;
        a.n_groups = h.nk_large;
        a.factor = h.factor;
        a.n_chunks_map = n_c;
    }

    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ZKV_ERR_LAUNCH;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(raw_score_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)score_smem()) != cudaSuccess ||
            cudaFuncSetAttribute(raw_select_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)select_smem()) != cudaSuccess ||
            cudaFuncSetAttribute(raw_attend_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)attend_smem()) != cudaSuccess)
            return ZKV_ERR_LAUNCH;
        attr_set[dev] = true;
    }
    void* args[] = {&a};
    void* args1[] = {&a1};
    const cudaStream_t st = (cudaStream_t)stream;
    int rc = ZKV_OK;
    if (hier) {
        rc = launch_pdl((const void*)raw_score_kernel<false>, rows * p.ST1, kScoreThreads, score_smem(), st, args1);
        if (rc == ZKV_OK)
            rc = launch_pdl((const void*)raw_select_kernel<false>, rows, kSelThreads, select_smem(), st, args1);
        if (rc != ZKV_OK) return rc;
    }
    if (p.ST > 0) {
        rc = launch_pdl((const void*)raw_score_kernel<false>, rows * p.ST, kScoreThreads, score_smem(), st, args);
        if (rc == ZKV_OK)
            rc = launch_pdl((const void*)raw_select_kernel<false>, rows, kSelThreads, select_smem(), st, args);
    }
    if (rc == ZKV_OK)
        rc = launch_pdl((const void*)raw_attend_kernel<false>, rows * p.AT, kThreads, attend_smem(), st, args);
    if (rc == ZKV_OK) rc = launch_pdl((const void*)raw_merge_kernel<false>, rows * G, kHeadDim, 0, st, args);
    return rc;
}

// ---------------------------------------------------------------- sequence split
// Pages of a row over `world` ranks: rank q holds [q per, min(n_c, q per + per)),
// per = ceil(n_c / world) rounded up to 16 pages.
static void split_range(int n_c, int world, int rank, int* lo, int* hi) {
    int per = (n_c + world - 1) / world;
    per = (per + 15) & ~15;
    *lo = (int)std::min<int64_t>(n_c, (int64_t)rank * per);
    *hi = std::min(n_c, *lo + per);
}

// The exchange buffer of a split group, the same layout on every rank: the
// epochs of the two exchanges [R] and [R * G] (uint32, this rank's own
// count of completed calls), the tagged score row [R][n_c_pad] and the
// tagged partials [world][R * G][kXPart] (64-bit words {value, epoch}).
struct XLayout {
    size_t ep_s, ep_m, row, part, bytes;
    int n_c_pad;
};

static XLayout x_layout(int R, int G, int n_c, int world) {
    XLayout x;
    size_t o = 0;
    const size_t rg = (size_t)R * G;
    x.n_c_pad = (n_c + 31) & ~31;
    x.ep_s = o; o += up256((size_t)R * 4);
    x.ep_m = o; o += up256(rg * 4);
    x.row = o;  o += up256((size_t)R * x.n_c_pad * 8);
    x.part = o; o += up256((size_t)world * rg * kXPart * 8);
    x.bytes = o;
    return x;
}

// Workspace of one rank: the whole row's scores [R][n_c_pad] fp32 (copied
// out of the tagged row by the select), selection [R][nk] int32, own ranges
// [R][2], the attend CTAs' partials.  Entries per row: this rank's raw rows
// (rank 0) and at most min(nk, n_loc) own pages; the attend grid is sized
// for the expected share, nk / world own pages (one wave, one merge batch
// of partials), and a CTA takes more entries when a rank holds more.
static Plan make_split_plan(int R, int n_c, int n_loc, int world, int nk, int n_sink, int n_near) {
    Plan p = make_plan(R, n_loc, std::min(nk, n_loc), n_sink, n_near, Hier{});
    p.ST = (n_loc + kScoreTile - 1) / kScoreTile;
    if (p.E > 0) {
        const int e_exp = p.RS + p.RN + std::min(n_loc, (nk + world - 1) / world);
        int c = R > 0 ? kAttendPerSm * sm_count() / R : 1;
        c = std::max(1, std::min({c, (e_exp + kTileEntries - 1) / kTileEntries, kMergeBatch}));
        c = std::max(c, (p.E + 127) / 128);
        p.AT = c;
        p.EPC = (p.E + c - 1) / c;
    }
    const int max_tiles = p.E > 0 ? (p.E + kTileEntries - 1) / kTileEntries : 1;
    p.off_scores = 0;
    p.off_sel = up256((size_t)R * ((n_c + 31) & ~31) * 4);
    p.off_sel_large = p.off_sel + up256((size_t)R * nk * 4);  // own ranges
    p.off_parts = p.off_sel_large + up256((size_t)R * 2 * 4);
    p.bytes = p.off_parts + up256((size_t)R * std::max(max_tiles, p.AT) * kPartFloats * 4);
    return p;
}

static size_t split_score_smem() { return score_smem() + kScoreWarps * 16 * 4; }

static int decode_raw_split(const void* q, const zkv_raw_layer* layer, const zkv_raw_split* sp, int rows, int G,
                            int n_max, int n_c, int nk, int n_sink, int near_start, int n_near, float scale,
                            void* out, float* lse, int64_t* sel_out, int32_t* status, void* workspace,
                            size_t ws_bytes, void* stream) {
    if (!q || !layer || !sp || !sp->peer_base || !out || !workspace || rows < 0 || G < 1 || G > 8 ||
        sp->world < 1 || sp->world > kMaxRanks || sp->rank < 0 || sp->rank >= sp->world || n_c < 2 || nk < 1 ||
        nk >= n_c || n_sink < 0 || n_near < 0 || near_start < 0)
        return ZKV_ERR_ARG;
    if (n_c > kMaxChunks) return ZKV_ERR_CAPACITY;
    int lo, hi, lo_last, hi_last;
    split_range(n_c, sp->world, sp->rank, &lo, &hi);
    split_range(n_c, sp->world, sp->world - 1, &lo_last, &hi_last);
    if (hi_last <= lo_last) return ZKV_ERR_ARG;  // every rank holds at least one page
    const int n_loc = hi - lo;
    const bool raw_rows = sp->rank == 0;  // the sink and near rows live on rank 0
    const int ns = raw_rows ? n_sink : 0, nn = raw_rows ? n_near : 0;
    const zkv_raw_layer& L = *layer;
    if (!L.keys || !L.values || !L.chunk_min || !L.chunk_max || L.kv_ld_row < kHeadDim || (L.kv_ld_row % kHeadDim) ||
        L.page_base < 0 || n_max < n_loc)
        return ZKV_ERR_ARG;
    const int64_t cap = L.kv_ld_row / kHeadDim;
    if (L.page_base + 16 * (int64_t)n_loc > cap || (int64_t)near_start + nn > cap || ns > cap) return ZKV_ERR_ARG;
    if ((int64_t)rows * cap >= (int64_t)1 << 31) return ZKV_ERR_CAPACITY;
    const Plan p = make_split_plan(rows, n_c, n_loc, sp->world, nk, ns, nn);
    if (ws_bytes < p.bytes) return ZKV_ERR_ARG;
    if (p.AT > kMaxTiles || (int64_t)rows * (p.ST + p.AT) >= ((int64_t)1 << 31) ||
        (int64_t)rows * G * kXPart * sp->world >= ((int64_t)1 << 31))
        return ZKV_ERR_CAPACITY;
    for (int r = 0; r < sp->world; ++r)
        if (!sp->peer_base[r] || ((uintptr_t)sp->peer_base[r] & 255)) return ZKV_ERR_ARG;
    if (rows == 0) return ZKV_OK;
    if (((uintptr_t)L.keys & 15) || ((uintptr_t)L.values & 15) || ((uintptr_t)L.chunk_min & 15) ||
        ((uintptr_t)L.chunk_max & 15) || ((uintptr_t)q & 3) || ((uintptr_t)workspace & 255))
        return ZKV_ERR_ALIGN;
    const XLayout x = x_layout(rows, G, n_c, sp->world);
    if (sp->bytes < x.bytes) return ZKV_ERR_CAPACITY;  // the exchange buffers are too small for this shape
    Args a;
    memset(&a, 0, sizeof(a));
    if (!cached_maps(&a.tk, &a.tv, L.keys, L.values, (int64_t)rows * cap)) return ZKV_ERR_LAUNCH;
    a.q = (const uint16_t*)q;
    a.cmin = (const uint16_t*)L.chunk_min;
    a.cmax = (const uint16_t*)L.chunk_max;
    a.valid = L.valid;
    a.cap = cap;
    a.page_base = L.page_base;
    a.R = rows;
    a.G = G;
    a.n_max = n_max;
    a.n_c = n_loc;
    a.nk = nk;
    a.n_sink = ns;
    a.near_start = near_start;
    a.n_near = nn;
    a.ST = p.ST;
    a.AT = p.AT;
    a.RS = p.RS;
    a.RN = p.RN;
    a.E = p.E;
    a.EPC = p.EPC;
    a.n_c_pad = x.n_c_pad;
    a.sl2 = scale * 1.4426950408889634f;
    a.out = (uint16_t*)out;
    a.lse = lse;
    a.sel_out = sel_out;
    a.status = status;
    a.rank = sp->rank;
    a.world = sp->world;
    a.chunk_lo = lo;
    a.chunk_hi = hi;
    a.n_total = n_c;
    for (int r = 0; r < sp->world; ++r) {
        uint8_t* b = (uint8_t*)sp->peer_base[r];
        a.xrow[r] = (uint64_t*)(b + x.row);
        a.xpart[r] = (uint64_t*)(b + x.part);
    }
    uint8_t* own = (uint8_t*)sp->peer_base[sp->rank];
    a.ep_s = (uint32_t*)(own + x.ep_s);
    a.ep_m = (uint32_t*)(own + x.ep_m);
    uint8_t* ws = (uint8_t*)workspace;
    a.scores = (float*)(ws + p.off_scores);
    a.sel = (int32_t*)(ws + p.off_sel);
    a.own_range = (int32_t*)(ws + p.off_sel_large);
    a.parts = (float*)(ws + p.off_parts);
    a.wait_ns = peer_wait_ns();

    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ZKV_ERR_LAUNCH;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(raw_score_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)split_score_smem()) != cudaSuccess ||
            cudaFuncSetAttribute(raw_attend_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)attend_smem()) != cudaSuccess)
            return ZKV_ERR_LAUNCH;
        attr_set[dev] = true;
    }
    void* args[] = {&a};
    const cudaStream_t st = (cudaStream_t)stream;
    int rc = launch_pdl((const void*)raw_score_kernel<true>, rows * p.ST, kScoreThreads, split_score_smem(), st, args);
    if (rc == ZKV_OK) rc = launch_pdl((const void*)raw_select_kernel<true>, rows, kSelThreads, 0, st, args);
    if (rc == ZKV_OK)
        rc = launch_pdl((const void*)raw_attend_kernel<true>, rows * p.AT, kThreads, attend_smem(), st, args);
    if (rc == ZKV_OK) rc = launch_pdl((const void*)raw_merge_kernel<true>, rows * G, kHeadDim, 0, st, args);
    return rc;
}

}  // namespace rawpg

}  // namespace zkv

using namespace zkv;

int raw_quest_topk(const void* q, int G, const void* cmin, const void* cmax, const uint8_t* valid, int rows,
                   int n_max, int n_c, int nk, float* scores, int n_c_pad, int32_t* sel32, int64_t* ids,
                   uint16_t* raw_q_out, cudaStream_t stream) {
    using namespace rawpg;
    if (!q || !cmin || !cmax || !scores || !sel32 || !ids || rows < 0 || G < 1 || G > 8 || n_c < 1 ||
        n_c > n_max || n_c > kMaxChunks || nk < 1 || nk > n_c || n_c_pad < ((n_c + 31) & ~31))
        return ZKV_ERR_ARG;
    if (((uintptr_t)cmin & 15) || ((uintptr_t)cmax & 15) || ((uintptr_t)q & 3) || ((uintptr_t)scores & 15))
        return ZKV_ERR_ALIGN;
    if (rows == 0) return ZKV_OK;
    Args a;
    memset(&a, 0, sizeof(a));
    a.q = (const uint16_t*)q;
    a.cmin = (const uint16_t*)cmin;
    a.cmax = (const uint16_t*)cmax;
    a.valid = valid;
    a.R = rows;
    a.G = G;
    a.n_max = n_max;
    a.n_c = n_c;
    a.nk = nk;
    a.ST = (n_c + kScoreTile - 1) / kScoreTile;
    a.n_c_pad = n_c_pad;
    a.scores = scores;
    a.sel = sel32;
    a.sel_out = ids;
    a.raw_q_out = raw_q_out;
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ZKV_ERR_LAUNCH;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(raw_score_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)score_smem()) != cudaSuccess)
            return ZKV_ERR_LAUNCH;
        attr_set[dev] = true;
    }
    void* args[] = {&a};
    int rc = launch_pdl((const void*)raw_score_kernel<false>, rows * a.ST, kScoreThreads, score_smem(), stream, args);
    if (rc == ZKV_OK)
        rc = launch_pdl((const void*)raw_select_kernel<false>, rows, kSelThreads, select_smem(), stream, args);
    return rc;
}


extern "C" size_t zkv_page_decode_raw_ws_bytes(int rows, int n_c, int nk, int n_sink, int n_near) {
    if (rows < 0 || n_c < 0 || nk < 0 || n_sink < 0 || n_near < 0) return 0;
    return rawpg::make_plan(rows, n_c, nk, n_sink, n_near, rawpg::Hier{}).bytes;
}

extern "C" int zkv_page_decode_raw(const void* q, const zkv_raw_layer* layer, int rows, int G, int n_max, int n_c,
                                   int nk, int n_sink, int near_start, int n_near, float scale, void* out, float* lse,
                                   int64_t* sel_out, int32_t* status, void* workspace, size_t ws_bytes,
                                   void* stream) {
    return rawpg::decode_raw(q, layer, rows, G, n_max, n_c, nk, n_sink, near_start, n_near, scale, out, lse, sel_out,
                             status, workspace, ws_bytes, stream, rawpg::Hier{});
}

extern "C" size_t zkv_page_decode_raw_hier_ws_bytes(int rows, int n_c, int factor, int nk_large, int nk_small,
                                                    int n_sink, int n_near) {
    if (rows < 0 || n_c < 0 || factor < 1 || nk_large < 1 || nk_small < 0 || n_sink < 0 || n_near < 0) return 0;
    rawpg::Hier h{};
    h.factor = factor;
    h.nk_large = nk_large;
    return rawpg::make_plan(rows, n_c, nk_small, n_sink, n_near, h).bytes;
}

extern "C" int zkv_page_decode_raw_hier(const void* q, const zkv_raw_layer* layer, const zkv_quest_large* large,
                                        int rows, int G, int n_max, int n_c, int factor, int nk_large, int nk_small,
                                        int n_sink, int near_start, int n_near, float scale, void* out, float* lse,
                                        int64_t* sel_out, int32_t* status, void* workspace, size_t ws_bytes,
                                        void* stream) {
    if (!large || factor < 1) return ZKV_ERR_ARG;
    rawpg::Hier h{large->large_min, large->large_max, large->large_valid, large->n_max_large, factor, nk_large};
    return rawpg::decode_raw(q, layer, rows, G, n_max, n_c, nk_small, n_sink, near_start, n_near, scale, out, lse,
                             sel_out, status, workspace, ws_bytes, stream, h);
}

extern "C" int zkv_quest_large_minmax(const void* chunk_min, const void* chunk_max, int rows, int n_max,
                                      int valid_end, int factor, int g_lo, int g_hi, void* large_min,
                                      void* large_max, uint8_t* large_valid, int n_max_large, void* stream) {
    if (!chunk_min || !chunk_max || !large_min || !large_max || !large_valid || rows < 0 || n_max < 0 ||
        factor < 1 || g_lo < 0 || g_hi < g_lo || g_hi > n_max_large || valid_end < 0)
        return ZKV_ERR_ARG;
    if (((uintptr_t)chunk_min & 3) || ((uintptr_t)chunk_max & 3) || ((uintptr_t)large_min & 3) ||
        ((uintptr_t)large_max & 3))
        return ZKV_ERR_ALIGN;
    if (rows == 0 || g_hi == g_lo) return ZKV_OK;
    if (rows > 65535) return ZKV_ERR_CAPACITY;
    rawpg::large_minmax_kernel<<<dim3((unsigned)(g_hi - g_lo), (unsigned)rows), 64, 0, (cudaStream_t)stream>>>(
        (const uint32_t*)chunk_min, (const uint32_t*)chunk_max, n_max, valid_end, factor, g_lo,
        (uint32_t*)large_min, (uint32_t*)large_max, large_valid, n_max_large);
    return launch_status();
}

extern "C" int zkv_raw_split_range(int n_c, int world, int rank, int* lo, int* hi) {
    if (!lo || !hi || n_c < 0 || world < 1 || world > rawpg::kMaxRanks || rank < 0 || rank >= world)
        return ZKV_ERR_ARG;
    rawpg::split_range(n_c, world, rank, lo, hi);
    return ZKV_OK;
}

extern "C" size_t zkv_raw_split_buffer_bytes(int rows, int G, int n_c, int world) {
    if (rows < 0 || G < 1 || n_c < 0 || world < 1 || world > rawpg::kMaxRanks) return 0;
    return rawpg::x_layout(rows, G, n_c, world).bytes;
}

extern "C" size_t zkv_page_decode_raw_split_ws_bytes(int rows, int n_c, int world, int rank, int nk, int n_sink,
                                                     int n_near) {
    if (rows < 0 || n_c < 0 || world < 1 || world > rawpg::kMaxRanks || rank < 0 || rank >= world || nk < 0 ||
        n_sink < 0 || n_near < 0)
        return 0;
    int lo, hi;
    rawpg::split_range(n_c, world, rank, &lo, &hi);
    return rawpg::make_split_plan(rows, n_c, hi - lo, world, nk, rank == 0 ? n_sink : 0, rank == 0 ? n_near : 0)
        .bytes;
}

extern "C" int zkv_page_decode_raw_split(const void* q, const zkv_raw_layer* layer, const zkv_raw_split* split,
                                         int rows, int G, int n_max, int n_c, int nk, int n_sink, int near_start,
                                         int n_near, float scale, void* out, float* lse, int64_t* sel_out,
                                         int32_t* status, void* workspace, size_t ws_bytes, void* stream) {
    return rawpg::decode_raw_split(q, layer, split, rows, G, n_max, n_c, nk, n_sink, near_start, n_near, scale, out,
                                   lse, sel_out, status, workspace, ws_bytes, stream);
}
