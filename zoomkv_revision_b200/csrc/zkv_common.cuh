// zkv_common.cuh -- shared device helpers for the libzkv sm_100a kernels:
// bf16 arithmetic ladders, TMA bulk copies with mbarrier completion and
// bounded waits, thread-block-cluster helpers, mma.sync fragments and a
// deterministic block-wide radix select.
#pragma once

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/zkv.h"

namespace cg = cooperative_groups;

namespace zkv {

constexpr int kHeadDim = 128;
constexpr int kChunk = 16;           // Quest chunk == KIVI key group == page
constexpr int kWords = kHeadDim / 8; // int32 words of 4-bit codes per token
constexpr int kVGroups = kHeadDim / 32;
// Bounded spin: test_wait polls with a short sleep; ~2^20 polls is well
// under a second, after which the kernel records ZKV_ERR_TIMEOUT.
constexpr uint32_t kMaxPolls = 1u << 20;

// ------------------------------------------------------------ bf16 ladder
__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float bfbits2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
__device__ __forceinline__ uint16_t f2bfbits(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
}

// KIVI scale bf16(bf16(mx - mn) / 15): fp32 ops on bf16 operands rounded once
// to bf16 equal the correctly rounded bf16 ops (24 >= 2*8 + 2).  The division
// by 15 is a multiply by fp32(1/15): for a bf16 dividend d, d/15 repeats a
// 4-bit pattern and is never within the multiply's error of a bf16 rounding
// midpoint, so the bf16 result equals the divided one for every finite d
// (checked exhaustively by the CPU tests).
__device__ __forceinline__ uint16_t kivi_scale_bits(uint16_t mn, uint16_t mx) {
    uint16_t diff = f2bfbits(__fsub_rn(bfbits2f(mx), bfbits2f(mn)));
    return f2bfbits(__fmul_rn(bfbits2f(diff), 1.0f / 15.0f));
}

// code = rint(clamp(bf16(bf16(x - mn) / max(scale, 1e-8)), 0, 15))
__device__ __forceinline__ uint32_t kivi_code(uint16_t x, uint16_t mn, uint16_t scale) {
    float sc = bfbits2f(scale);
    float safe = bfbits2f(f2bfbits(sc > 1e-8f ? sc : 1e-8f));
    float d1 = bfbits2f(f2bfbits(__fsub_rn(bfbits2f(x), bfbits2f(mn))));
    float y = bfbits2f(f2bfbits(__fdiv_rn(d1, safe)));
    y = fminf(fmaxf(y, 0.0f), 15.0f);
    return (uint32_t)__float2int_rn(y);
}

__device__ __forceinline__ __nv_bfloat162 bits_bf162_pre(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }

// Two 4-bit codes -> exact bf16x2 (c_lo, c_hi): OR into the mantissa of
// bf16(128) then subtract 128 (exact).
__device__ __forceinline__ __nv_bfloat162 codes2_to_bf162(uint32_t lo, uint32_t hi) {
    uint32_t v = (lo & 0xFu) | ((hi & 0xFu) << 16) | 0x43004300u;
    __nv_bfloat162 r = *reinterpret_cast<__nv_bfloat162*>(&v);
    const uint32_t k128 = 0x43004300u;
    return __hsub2(r, *reinterpret_cast<const __nv_bfloat162*>(&k128));
}

// bf16(bf16(c * s) + z) on a pair: two separately rounded bf16 ops -- the
// dequant of the reference's PyTorch path (qk_dot.py:304) and the documented
// intent of kivi_qk_dot.cu:264-275.  The `_rn` forms stop ptxas from
// contracting the pair into one fma.bf16x2 (plain __hmul2/__hadd2 lower to
// mul/add.bf16x2 without a rounding qualifier, which ptxas may fuse).
__device__ __forceinline__ __nv_bfloat162 dequant2(__nv_bfloat162 c, __nv_bfloat162 s, __nv_bfloat162 z) {
    return __hadd2_rn(__hmul2_rn(c, s), z);
}

// Same ladder from packed nibbles in 5 instructions per pair.  Byte b of w
// holds codes (c_lo, c_hi) = nibbles (2b, 2b+1); one byte-permute of (w,
// w >> 4) with selector nib_sel(b) puts c_lo in the low nibble of byte 0 and
// c_hi in the low nibble of byte 2, and a LOP3 makes bf16x2(128 + c_lo,
// 128 + c_hi).  fma.rn((128 + c), s, -128 s) is bf16(c * s) exactly (one
// rounding of the exact product c*s) and the add rounds once more:
// bf16(bf16(c*s) + z), bit-identical to dequant2.
__device__ __forceinline__ uint32_t nib_sel(int byte) { return (uint32_t)byte | ((uint32_t)(byte + 4) << 8); }
__device__ __forceinline__ __nv_bfloat162 dequant2_w(uint32_t w, uint32_t sel, __nv_bfloat162 s,
                                                      __nv_bfloat162 neg128s, __nv_bfloat162 z) {
    const uint32_t x = __byte_perm(w, w >> 4, sel);
    const uint32_t v = (x & 0x000F000Fu) | 0x43004300u;
    return __hadd2_rn(__hfma2(bits_bf162_pre(v), s, neg128s), z);
}
__device__ __forceinline__ __nv_bfloat162 neg128(__nv_bfloat162 s) {
    const uint32_t m = 0xC300C300u;  // bf16x2(-128, -128)
    return __hmul2_rn(s, bits_bf162_pre(m));
}

__device__ __forceinline__ __nv_bfloat16 bits_bf16(uint16_t v) { return __ushort_as_bfloat16(v); }
__device__ __forceinline__ uint16_t bf16_bits(__nv_bfloat16 v) { return __bfloat16_as_ushort(v); }
__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf162(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }

__device__ __forceinline__ uint32_t ordered_u32(float x) {
    uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ------------------------------------------------------------ dependent launch
// Wait until the kernels this grid depends on have completed and their
// writes are visible (a no-op unless launched with programmatic dependent
// launch); allow the next kernel on the stream to be scheduled.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Start of a kernel that may be launched with programmatic dependent launch:
// wait for the previous grid on the stream (a no-op without the attribute)
// before any memory access.  The next grid is not released early: in the
// reference-mode chain, dependents made resident at a kernel's start took
// slots from its later waves (3,534 tokens/s with the early release, 3,671
// without programmatic launch, 3,951 with the wait alone).
__device__ __forceinline__ void pdl_begin() { grid_dep_wait(); }

// ------------------------------------------------------------ time
// Nanoseconds of the GPU's global timer: bounds waits by time rather than by
// a count of polls (a sleeping poll can return early or late).
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------ status
__device__ __forceinline__ void set_status(int32_t* status, int code) {
    if (status) atomicExch(status, code);
}

// ------------------------------------------------------------ tagged words
// A 32-bit value in the low half and the epoch of the call that wrote it in
// the high half, stored and loaded as one naturally aligned 64-bit access
// (single-copy atomic), so a reader that sees the epoch it waits for also
// sees that call's value: no fence and no separate flag between a producer
// (this GPU or a peer over NVLink) and its readers.
__device__ __forceinline__ uint64_t tagged(uint32_t value, uint32_t tag) {
    return ((uint64_t)tag << 32) | value;
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool tag_reached(uint64_t w, uint32_t tag) {
    return (int32_t)((uint32_t)(w >> 32) - tag) >= 0;
}
// Re-read the tagged word at p (already loaded once as w) until its epoch
// reaches `tag` or `wait_ns` of the global timer pass; ok becomes false on
// expiry, and a caller whose ok is already false does not wait again.
__device__ __forceinline__ uint64_t wait_tagged(const uint64_t* p, uint64_t w, uint32_t tag, uint64_t wait_ns,
                                               bool& ok) {
    if (tag_reached(w, tag) || !ok) return w;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        __nanosleep(32);
        w = ld_relaxed_sys_u64(p);
        if (tag_reached(w, tag)) return w;
        if (globaltimer_ns() - t0 > wait_ns) {
            ok = false;
            return w;
        }
    }
}

// ------------------------------------------------------------ mbarrier / TMA bulk
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; false (and status set) on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* status) {
    if (mbar_test(bar, parity)) return true;
    for (uint32_t it = 0; it < kMaxPolls; ++it) {
        __nanosleep(64);
        if (mbar_test(bar, parity)) return true;
    }
    set_status(status, ZKV_ERR_TIMEOUT);
    return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).  Never a multicast form.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------ mma.sync bf16
// D(16x8 f32) += A(16x16 bf16, row) * B(16x8 bf16, col)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf162(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return bf162_bits(v);
}

// ------------------------------------------------------------ block radix select
// Deterministic top-k over n uint32 keys (larger key = better): after the
// call, *thr_out is the k-th largest key and *take_eq_out how many elements
// equal to it are taken (lowest indices first).  KeyFn(i) returns key i.
// All NT threads call it; scratch hist[256] + misc[4] in shared memory.
template <int NT, typename KeyFn>
__device__ void block_radix_select(KeyFn key, int n, int k, int* hist, int* misc, uint32_t* thr_out,
                                   int* take_eq_out) {
    uint32_t prefix = 0, mask = 0;
    int remaining = k;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += NT) hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += NT) {
            uint32_t kk = key(i);
            if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & 255u], 1);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // lane l owns bins [8l, 8l+8); suffix sums from the top bin down.
            const int lane = threadIdx.x;
            int local[8];
            int tot = 0;
#pragma unroll
            for (int j = 7; j >= 0; --j) {
                tot += hist[8 * lane + j];
                local[j] = tot;  // count of bins >= 8*lane+j within this lane
            }
            // exclusive suffix over higher lanes
            int incl = tot;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                int v = __shfl_down_sync(0xffffffffu, incl, off);
                if (lane + off < 32) incl += v;
            }
            int above = incl - tot;  // count in bins of higher lanes
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                int ge = above + local[j];
                int gt = ge - hist[8 * lane + j];
                if (gt < remaining && ge >= remaining) {
                    misc[0] = 8 * lane + j;
                    misc[1] = gt;
                }
            }
        }
        __syncthreads();
        const uint32_t digit = (uint32_t)misc[0];
        remaining -= misc[1];
        prefix |= digit << shift;
        mask |= 255u << shift;
        __syncthreads();
    }
    *thr_out = prefix;
    *take_eq_out = remaining;
}

// Writes the selected indices (key > thr, plus the first take_eq with
// key == thr) in ascending index order: out(pos, index).  Contiguous
// per-thread ranges + block exclusive scan.  scan scratch: 2*NT ints.
template <int NT, typename KeyFn, typename OutFn>
__device__ void block_select_compact(KeyFn key, int n, uint32_t thr, int take_eq, int* scan, OutFn out) {
    const int per = (n + NT - 1) / NT;
    const int lo = threadIdx.x * per;
    const int hi = min(n, lo + per);
    int gt = 0, eq = 0;
    for (int i = lo; i < hi; ++i) {
        uint32_t kk = key(i);
        gt += kk > thr;
        eq += kk == thr;
    }
    // block exclusive scan of (gt, eq)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int sg = gt, se = eq;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        int a = __shfl_up_sync(0xffffffffu, sg, off);
        int b = __shfl_up_sync(0xffffffffu, se, off);
        if (lane >= off) {
            sg += a;
            se += b;
        }
    }
    if (lane == 31) {
        scan[warp] = sg;
        scan[NT + warp] = se;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int ag = 0, ae = 0;
        for (int w = 0; w < NT / 32; ++w) {
            int tg = scan[w], te = scan[NT + w];
            scan[w] = ag;
            scan[NT + w] = ae;
            ag += tg;
            ae += te;
        }
    }
    __syncthreads();
    int gbefore = scan[warp] + sg - gt;
    int ebefore = scan[NT + warp] + se - eq;
    for (int i = lo; i < hi; ++i) {
        uint32_t kk = key(i);
        if (kk > thr) {
            out(gbefore + min(ebefore, take_eq), i);
            ++gbefore;
        } else if (kk == thr) {
            if (ebefore < take_eq) out(gbefore + ebefore, i);
            ++ebefore;
        }
    }
    __syncthreads();
}

// ------------------------------------------------------------ fast deterministic top-k
__device__ __forceinline__ float float_of_ordered(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
constexpr uint32_t kOrderedNegInf = 0x007fffffu;  // ordered_u32(-inf)

// Writes the k best of n keys (larger key first, ties to the lowest index) in
// ascending index order via out(pos, index).  Precondition 0 < k < n.
//
// Value-bucketed pivot select: (1) min/max of the keys (or the caller's),
// (2) a 256-bin histogram with equal-width bins, monotone in the key: over
// (key - min) >> shift when all keys share a sign (the ordered-u32 key is
// then piecewise linear in the value), else over the float value (fp32 keys
// only; -inf goes to bin 0); (3) the bin b* holding the k-th best; (4) that
// bin's elements ranked exactly -> pivot (T_key, T_idx); (5) one ballot
// compaction of bin > b* || (bin == b* && (key > T_key || (key == T_key &&
// idx <= T_idx))).  Each thread keeps up to 16 keys in registers across the
// passes (n <= 16 * NT); beyond that the passes re-read the keys.  When the
// pivot bin holds more than NT elements (heavy ties) the 4-round radix select
// runs instead; both give the same set.  Passes walk per-warp contiguous
// segments with lane-consecutive indices (conflict-free; ballots keep the
// order).  Scratch: hist[256], misc[8], scan[2*NT].
template <int NT, bool kFloatKeys, typename KeyFn, typename OutFn>
__device__ void block_topk(KeyFn key, int n, int k, int* hist, int* misc, int* scan, OutFn out,
                           bool have_range = false, uint32_t lo_in = 0, uint32_t hi_in = 0) {
    constexpr int NW = NT / 32;
    constexpr int E = 16;  // keys per thread kept in registers
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = ((n + NW - 1) / NW + 31) & ~31;
    const int seg0 = warp * S, seg1 = min(n, seg0 + S);
    const bool in_regs = S <= 32 * E;
    uint32_t kr[E];
    if (in_regs) {
#pragma unroll
        for (int u = 0; u < E; ++u) {
            const int idx = seg0 + 32 * u + lane;
            kr[u] = idx < seg1 ? key(idx) : 0u;
        }
    }
    auto key_at = [&](int u, int j0) -> uint32_t {
        const int idx = j0 + 32 * u + lane;
        return idx < seg1 ? key(idx) : 0u;
    };
    for (int i = tid; i < 256; i += NT) hist[i] = 0;
    if (tid == 0) misc[3] = 0;
    uint32_t lo = lo_in, hi = hi_in;
    if (!have_range) {
        lo = 0xffffffffu;
        hi = 0u;
        for (int j0 = seg0; j0 < seg1; j0 += 32 * E) {
#pragma unroll
            for (int u = 0; u < E; ++u) {
                const uint32_t kk = in_regs ? kr[u] : key_at(u, j0);
                if (j0 + 32 * u + lane < seg1) {
                    if (!kFloatKeys || kk > kOrderedNegInf) lo = min(lo, kk);
                    hi = max(hi, kk);
                }
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, off));
            hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, off));
        }
        if (lane == 0) {
            scan[warp] = (int)lo;
            scan[NW + warp] = (int)hi;
        }
        __syncthreads();
        lo = 0xffffffffu;
        hi = 0u;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            lo = min(lo, (uint32_t)scan[w]);
            hi = max(hi, (uint32_t)scan[NW + w]);
        }
    } else {
        __syncthreads();
    }
    const bool same_sign = !kFloatKeys || ((lo ^ hi) & 0x80000000u) == 0u;
    const uint32_t span = hi > lo ? hi - lo : 0u;
    const int bits = span ? 32 - __clz(span) : 0;
    const int sh = bits > 8 ? bits - 8 : 0;
    const float flo = float_of_ordered(lo), fhi = float_of_ordered(hi);
    const float inv = (hi > lo) ? 256.0f / (fhi - flo) : 0.0f;
    auto bucket = [&](uint32_t kk) -> uint32_t {
        if (same_sign) return kk >= lo ? min((kk - lo) >> sh, 255u) : 0u;
        if (kk <= kOrderedNegInf || hi <= lo) return 0u;
        const float b = (float_of_ordered(kk) - flo) * inv;
        return b >= 255.0f ? 255u : (b > 0.0f ? (uint32_t)b : 0u);
    };
    // pass A: histogram
    for (int j0 = seg0; j0 < seg1; j0 += 32 * E) {
#pragma unroll
        for (int u = 0; u < E; ++u) {
            const uint32_t kk = in_regs ? kr[u] : key_at(u, j0);
            if (j0 + 32 * u + lane < seg1) atomicAdd(&hist[bucket(kk)], 1);
        }
    }
    __syncthreads();
    if (warp == 0) {
        int local[8];
        int tot = 0;
#pragma unroll
        for (int j = 7; j >= 0; --j) {
            tot += hist[8 * lane + j];
            local[j] = tot;
        }
        int incl = tot;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_down_sync(0xffffffffu, incl, off);
            if (lane + off < 32) incl += v;
        }
        const int above = incl - tot;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int ge = above + local[j];
            const int gt = ge - hist[8 * lane + j];
            if (gt < k && ge >= k) {
                misc[0] = 8 * lane + j;
                misc[1] = gt;
                misc[2] = hist[8 * lane + j];
            }
        }
    }
    __syncthreads();
    const uint32_t bstar = (uint32_t)misc[0];
    const int rem = k - misc[1];
    const int m = misc[2];
    if (m > NT - NW) {  // heavy ties (pivot bin too large for the rank step)
        uint32_t tk;
        int take_eq;
        block_radix_select<NT>(key, n, k, hist, misc, &tk, &take_eq);
        block_select_compact<NT>(key, n, tk, take_eq, scan, out);
        return;
    }
    // pass B: gather the pivot bin, count elements of higher bins per warp
    int above_cnt = 0;
    for (int j0 = seg0; j0 < seg1; j0 += 32 * E) {
#pragma unroll
        for (int u = 0; u < E; ++u) {
            const int idx = j0 + 32 * u + lane;
            const uint32_t kk = in_regs ? kr[u] : key_at(u, j0);
            const uint32_t b = idx < seg1 ? bucket(kk) : 0u;
            above_cnt += __popc(__ballot_sync(0xffffffffu, idx < seg1 && b > bstar));
            if (idx < seg1 && b == bstar) {
                const int p = atomicAdd(&misc[3], 1);
                scan[p] = (int)kk;
                scan[NT + p] = idx;
            }
        }
    }
    __syncthreads();
    // rank the pivot bin; each selected pivot-bin element adds to its warp's count
    __shared__ int s_pw[NW];
    if (tid < NW) s_pw[tid] = 0;
    __syncthreads();
    if (tid < m) {
        const uint32_t mk = (uint32_t)scan[tid];
        const int mi = scan[NT + tid];
        int rank = 0;
        for (int j = 0; j < m; ++j) {
            const uint32_t kj = (uint32_t)scan[j];
            const int ij = scan[NT + j];
            rank += (kj > mk) || (kj == mk && ij < mi);
        }
        if (rank < rem) atomicAdd(&s_pw[mi / S], 1);
        if (rank == rem - 1) {
            misc[4] = (int)mk;
            misc[5] = mi;
        }
    }
    if (lane == 0) scan[2 * NT - NW + warp] = above_cnt;  // tail of scan: candidates use < NT - NW slots
    __syncthreads();
    const uint32_t tk = (uint32_t)misc[4];
    const int ti = misc[5];
    int pos = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) pos += (w < warp) ? scan[2 * NT - NW + w] + s_pw[w] : 0;
    // pass C: ordered write
    const unsigned lt = (1u << lane) - 1u;
    for (int j0 = seg0; j0 < seg1; j0 += 32 * E) {
#pragma unroll
        for (int u = 0; u < E; ++u) {
            const int idx = j0 + 32 * u + lane;
            const uint32_t kk = in_regs ? kr[u] : key_at(u, j0);
            const uint32_t b = bucket(kk);
            const bool f = idx < seg1 && (b > bstar || (b == bstar && (kk > tk || (kk == tk && idx <= ti))));
            const unsigned bal = __ballot_sync(0xffffffffu, f);
            if (f) out(pos + __popc(bal & lt), idx);
            pos += __popc(bal);
        }
    }
    __syncthreads();
}


// Small-n form of block_topk over fp32 scores in shared memory (n <= 16 NT):
// each thread keeps 16 contiguous keys in registers (float4 loads), 512-bin
// histogram, rank of the pivot bin, and a per-thread-count + warp-scan
// compaction (no per-element ballots).  Same selected set and output order
// as block_topk.  lo/hi: min finite key and max key (ordered u32).
// Scratch: hist[512], misc[8], scan[2*NT].
template <int NT, typename OutFn>
__device__ void block_topk_small(const float* sc, int n, int k, uint32_t lo, uint32_t hi, int* hist, int* misc,
                                 int* scan, OutFn out) {
    constexpr int NW = NT / 32, E = 16, NB = 512;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int base = tid * E;
    uint32_t kr[E];
#pragma unroll
    for (int v = 0; v < E / 4; ++v) {
        float4 f = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        if (base + 4 * v < n) f = reinterpret_cast<const float4*>(sc + base)[v];
        kr[4 * v + 0] = ordered_u32(f.x);
        kr[4 * v + 1] = ordered_u32(f.y);
        kr[4 * v + 2] = ordered_u32(f.z);
        kr[4 * v + 3] = ordered_u32(f.w);
    }
    for (int i = tid; i < NB; i += NT) hist[i] = 0;
    if (tid == 0) misc[3] = 0;
    const bool same_sign = ((lo ^ hi) & 0x80000000u) == 0u;
    const uint32_t span = hi > lo ? hi - lo : 0u;
    const int bits = span ? 32 - __clz(span) : 0;
    const int sh = bits > 9 ? bits - 9 : 0;
    const float flo = float_of_ordered(lo), fhi = float_of_ordered(hi);
    const float inv = (hi > lo) ? (float)NB / (fhi - flo) : 0.0f;
    // Straight-line bucket loops (one uniform branch): any bucketing that is
    // monotone in the key and shared by all passes gives the exact selection.
    uint32_t bk[E];
    if (same_sign) {
#pragma unroll
        for (int u = 0; u < E; ++u) {
            const uint32_t kk = kr[u];
            bk[u] = kk >= lo ? min((kk - lo) >> sh, (uint32_t)(NB - 1)) : 0u;
        }
    } else {
        // -inf, NaN-patterned keys below it, and every key when hi <= lo
        // (inv == 0) clamp to bucket 0
#pragma unroll
        for (int u = 0; u < E; ++u) {
            const float fb = fminf(fmaxf((float_of_ordered(kr[u]) - flo) * inv, 0.0f), (float)(NB - 1));
            bk[u] = (uint32_t)fb;
        }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < E; ++u)
        if (base + u < n) atomicAdd(&hist[bk[u]], 1);
    __syncthreads();
    {   // bin of the k-th best: suffix counts, every warp scanning NB / NW bins
        constexpr int PL = NB / NT;  // bins per thread
        const int b0 = PL * tid;
        int local[PL];
        int tot = 0;
#pragma unroll
        for (int j = PL - 1; j >= 0; --j) {
            tot += hist[b0 + j];
            local[j] = tot;
        }
        int incl = tot;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_down_sync(0xffffffffu, incl, off);
            if (lane + off < 32) incl += v;
        }
        if (lane == 0) scan[2 * NT - NW + warp] = incl;  // warp totals (scan[] tail is free here)
        __syncthreads();
        int above = incl - tot;
#pragma unroll
        for (int w = 0; w < NW; ++w) above += w > warp ? scan[2 * NT - NW + w] : 0;
#pragma unroll
        for (int j = 0; j < PL; ++j) {
            const int ge = above + local[j];
            const int gt = ge - hist[b0 + j];
            if (gt < k && ge >= k) {
                misc[0] = b0 + j;
                misc[1] = gt;
                misc[2] = hist[b0 + j];
            }
        }
    }
    __syncthreads();
    const uint32_t bstar = (uint32_t)misc[0];
    const int rem = k - misc[1];
    const int m = misc[2];
    if (m > NT) {  // heavy ties: exact radix path over the same keys
        auto key = [&](int i) { return ordered_u32(sc[i]); };
        uint32_t tk;
        int take_eq;
        block_radix_select<NT>(key, n, k, hist, misc, &tk, &take_eq);
        block_select_compact<NT>(key, n, tk, take_eq, scan, out);
        return;
    }
    uint32_t pm = 0u, gm = 0u;  // this thread's pivot-bin keys (few) and keys of higher bins
#pragma unroll
    for (int u = 0; u < E; ++u) {
        pm |= (uint32_t)(base + u < n && bk[u] == bstar) << u;
        gm |= (uint32_t)(base + u < n && bk[u] > bstar) << u;
    }
    const uint32_t pm_all = pm;
    while (pm) {
        const int u = __ffs(pm) - 1;
        pm &= pm - 1u;
        uint32_t kv = 0u;
#pragma unroll
        for (int j = 0; j < E; ++j) kv = j == u ? kr[j] : kv;
        const int p = atomicAdd(&misc[3], 1);
        scan[p] = (int)kv;
        scan[NT + p] = base + u;
    }
    __syncthreads();
    if (tid < m) {
        const uint32_t mk = (uint32_t)scan[tid];
        const int mi = scan[NT + tid];
        int rank = 0;
        for (int j = 0; j < m; ++j) {
            const uint32_t kj = (uint32_t)scan[j];
            const int ij = scan[NT + j];
            rank += (kj > mk) || (kj == mk && ij < mi);
        }
        if (rank == rem - 1) {
            misc[4] = (int)mk;
            misc[5] = mi;
        }
    }
    __syncthreads();
    const uint32_t tk = (uint32_t)misc[4];
    const int ti = misc[5];
    unsigned fl = gm;  // higher bins, plus the pivot-bin keys ranked at or above (tk, ti)
    for (uint32_t r = pm_all; r; r &= r - 1u) {
        const int u = __ffs(r) - 1;
        uint32_t kv = 0u;
#pragma unroll
        for (int j = 0; j < E; ++j) kv = j == u ? kr[j] : kv;
        if (kv > tk || (kv == tk && base + u <= ti)) fl |= 1u << u;
    }
    const int cnt = __popc(fl);
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
    }
    if (lane == 31) scan[warp] = incl;
    __syncthreads();
    int pos = incl - cnt;
#pragma unroll
    for (int w = 0; w < NW; ++w) pos += (w < warp) ? scan[w] : 0;
#pragma unroll
    for (int u = 0; u < E; ++u)
        if ((fl >> u) & 1u) out(pos++, base + u);
    __syncthreads();
}

// ----------------------------------------------------------- spread select
// Top k of one row of n fp32 scores in global memory (srow; validity bytes
// vrow or NULL: invalid -> -inf), ties to the lowest index, emitted as
// emit(position, index) in ascending index order, by a CTA of NT threads
// holding E = 2, 4 or 8 keys each (n <= E * NT).  Every warp holds keys,
// so each thread's dependent chains stay short: one kSelBins-bin histogram
// over the row's [min finite, max] key range (a bucketing monotone in the
// key) gives the bin of the k-th best; a warp ranks that bin's keys exactly
// when it holds at most 32 (else the exact radix select runs over gkey(i));
// an index-order scan of the kept flags emits the ids.
constexpr int kSelBins = 2048;
template <int NT>
struct SelSharedT {
    int hist[kSelBins];
    int scan[2 * NT];  // fallback scratch
    uint32_t wlo[32], whi[32], lohi[2];
    int wsum[32], wcnt[32];
    int misc[8];                // bin, count above it, its count, candidates, pivot key, pivot id
    uint32_t cand_k[32];
    int cand_i[32];
};

template <int NT, int E, typename Emit, typename GKey>
__device__ __forceinline__ void select_spread(SelSharedT<NT>& S, int n, int k, const float* srow, const uint8_t* vrow,
                                             Emit& emit, GKey& gkey) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = NT / 32;
    const int base = tid * E;
    uint32_t kr[E];
    {
        float f[E];
        const bool vec = ((uintptr_t)srow & (E >= 4 ? 15 : 7)) == 0 && base + E <= n;
        if (vec && E >= 4) {
#pragma unroll
            for (int u = 0; u < E / 4; ++u) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(srow + base) + u);
                f[(4 * u) % E] = v.x;
                f[(4 * u + 1) % E] = v.y;
                f[(4 * u + 2) % E] = v.z;
                f[(4 * u + 3) % E] = v.w;
            }
        } else if (vec) {
            const float2 v = __ldcg(reinterpret_cast<const float2*>(srow + base));
            f[0] = v.x;
            f[1 % E] = v.y;
        } else {
#pragma unroll
            for (int e = 0; e < E; ++e) f[e] = base + e < n ? __ldcg(srow + base + e) : 0.f;
        }
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const bool in = base + e < n;
            const bool ok = !vrow || !in || vrow[base + e] != 0;
            kr[e] = in ? (ok ? ordered_u32(f[e]) : kOrderedNegInf) : 0u;
        }
    }
    uint32_t klo = 0xffffffffu, khi = 0u;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        if (base + e < n) {
            if (kr[e] > kOrderedNegInf) klo = min(klo, kr[e]);
            khi = max(khi, kr[e]);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        klo = min(klo, __shfl_xor_sync(0xffffffffu, klo, off));
        khi = max(khi, __shfl_xor_sync(0xffffffffu, khi, off));
    }
    if (lane == 0) {
        S.wlo[warp] = klo;
        S.whi[warp] = khi;
    }
    __syncthreads();
    if (warp == 0) {
        klo = lane < NW ? S.wlo[lane] : 0xffffffffu;
        khi = lane < NW ? S.whi[lane] : 0u;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            klo = min(klo, __shfl_xor_sync(0xffffffffu, klo, off));
            khi = max(khi, __shfl_xor_sync(0xffffffffu, khi, off));
        }
        if (lane == 0) {
            S.lohi[0] = klo;
            S.lohi[1] = khi;
        }
    }
    __syncthreads();
    const uint32_t lo = S.lohi[0], hi = S.lohi[1];
    // bucket: monotone in the key; -inf (and every key when hi <= lo) -> bin 0
    const bool same_sign = ((lo ^ hi) & 0x80000000u) == 0u;
    const uint32_t span = hi > lo ? hi - lo : 0u;
    const int bits = span ? 32 - __clz(span) : 0;
    const int sh = bits > 11 ? bits - 11 : 0;
    const float flo = float_of_ordered(lo), fhi = float_of_ordered(hi);
    const float inv = (hi > lo) ? (float)kSelBins / (fhi - flo) : 0.0f;
    uint32_t bk[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const uint32_t kk = kr[e];
        if (same_sign) {
            bk[e] = kk >= lo ? min((kk - lo) >> sh, (uint32_t)(kSelBins - 1)) : 0u;
        } else {
            const float fb = fminf(fmaxf((float_of_ordered(kk) - flo) * inv, 0.0f), (float)(kSelBins - 1));
            bk[e] = (uint32_t)fb;
        }
        if (base + e < n) atomicAdd(&S.hist[bk[e]], 1);
    }
    __syncthreads();
    {   // suffix counts: thread t owns bins [PL t, PL t + PL)
        constexpr int PL = kSelBins / NT;
        int h[PL], suf[PL];
        int tot = 0;
#pragma unroll
        for (int j = PL - 1; j >= 0; --j) {
            h[j] = S.hist[PL * tid + j];
            tot += h[j];
            suf[j] = tot;
        }
        int incl = tot;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_down_sync(0xffffffffu, incl, off);
            if (lane + off < 32) incl += v;
        }
        if (lane == 0) S.wsum[warp] = incl;
        __syncthreads();
        int above = lane < NW && lane > warp ? S.wsum[lane] : 0;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) above += __shfl_xor_sync(0xffffffffu, above, off);
        above += incl - tot;
#pragma unroll
        for (int j = 0; j < PL; ++j) {
            const int ge = above + suf[j], gt = ge - h[j];
            if (gt < k && ge >= k) {
                S.misc[0] = PL * tid + j;
                S.misc[1] = gt;
                S.misc[2] = h[j];
            }
        }
    }
    __syncthreads();
    const uint32_t bstar = (uint32_t)S.misc[0];
    const int rem = k - S.misc[1], m = S.misc[2];
    uint32_t tk = 0u;
    int ti = 0x7fffffff;  // rem == m: the whole bin is kept
    if (rem < m) {
        if (m > 32) {  // heavy ties or a narrow range: the exact radix select over the same keys
            __syncthreads();
            block_topk<NT, true>(gkey, n, k, S.hist, S.misc, S.scan, emit);
            return;
        }
#pragma unroll
        for (int e = 0; e < E; ++e) {
            if (base + e < n && bk[e] == bstar) {
                const int p = atomicAdd(&S.misc[3], 1);
                S.cand_k[p] = kr[e];
                S.cand_i[p] = base + e;
            }
        }
        __syncthreads();
        if (warp == 0) {  // exact rank of each candidate: key descending, id ascending
            const uint32_t ck = lane < m ? S.cand_k[lane] : 0u;
            const int ci = lane < m ? S.cand_i[lane] : 0x7fffffff;
            int rank = 0;
            for (int j = 0; j < m; ++j) {
                const uint32_t kj = __shfl_sync(0xffffffffu, ck, j);
                const int ij = __shfl_sync(0xffffffffu, ci, j);
                rank += (kj > ck) || (kj == ck && ij < ci);
            }
            if (lane < m && rank == rem - 1) {
                S.misc[4] = (int)ck;
                S.misc[5] = ci;
            }
        }
        __syncthreads();
        tk = (uint32_t)S.misc[4];
        ti = S.misc[5];
    }
    unsigned fl = 0u;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const bool keep = base + e < n &&
                          (bk[e] > bstar || (bk[e] == bstar && (kr[e] > tk || (kr[e] == tk && base + e <= ti))));
        fl |= (unsigned)keep << e;
    }
    const int cnt = __popc(fl);
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
    }
    if (lane == 31) S.wcnt[warp] = incl;
    __syncthreads();
    int pos = lane < NW && lane < warp ? S.wcnt[lane] : 0;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) pos += __shfl_xor_sync(0xffffffffu, pos, off);
    pos += incl - cnt;
#pragma unroll
    for (int e = 0; e < E; ++e)
        if ((fl >> e) & 1u) emit(pos++, base + e);
}


// ----------------------------------------------------------- Quest score
// Half-warp per chunk: lane hl (0..15) loads dims [8hl, 8hl+8) of q, min and
// max as one 16-byte vector each.  The reference kernel's operation order
// (thread t: ((f0+f1)+f2)+f3 over dims 4t..4t+3, then an xor tree with
// offsets 16,8,4,2,1) maps onto two partials per lane and xor offsets
// 8,4,2,1 plus a final in-lane add, so the fp32 result is bit-identical.
__device__ __forceinline__ float quest_half(uint4 qv, uint4 mnv, uint4 mxv) {
    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
    const uint32_t nw[4] = {mnv.x, mnv.y, mnv.z, mnv.w};
    const uint32_t xw[4] = {mxv.x, mxv.y, mxv.z, mxv.w};
    float c[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int wi = 2 * h + (j >> 1);
            const int sh = (j & 1) * 16;
            const float q = __uint_as_float(((qw[wi] >> sh) & 0xffffu) << 16);
            const float a = __fmul_rn(q, __uint_as_float(((nw[wi] >> sh) & 0xffffu) << 16));
            const float b = __fmul_rn(q, __uint_as_float(((xw[wi] >> sh) & 0xffffu) << 16));
            const float f = fmaxf(a, b);
            acc = (j == 0) ? f : __fadd_rn(acc, f);
        }
        c[h] = acc;
    }
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        c[0] = __fadd_rn(c[0], __shfl_xor_sync(0xffffffffu, c[0], off));
        c[1] = __fadd_rn(c[1], __shfl_xor_sync(0xffffffffu, c[1], off));
    }
    return __fadd_rn(c[0], c[1]);
}

}  // namespace zkv

static inline int launch_status() { return cudaGetLastError() == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH; }

// Launch a kernel that begins with pdl_begin() with programmatic dependent
// launch allowed: it may become resident while the previous kernel on the
// stream drains, and waits for it before touching memory.
template <typename... KArgs, typename... Args>
static int launch_pdl_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...) != cudaSuccess) return ZKV_ERR_LAUNCH;
    return launch_status();
}

// Internal launchers shared across translation units (not part of the C ABI).
int quest_score_gqa_into(const void* q, int G, const void* chunk_min, const void* chunk_max, const uint8_t* valid,
                         float* scores, void* raw_q_out, int rows, int n_chunks, int n_max, cudaStream_t stream);
int topk_mask_launch(const float* dens, int rows, int nk, int n_dense, uint8_t* mask, cudaStream_t stream);
// Quest scores + top-nk of the raw page decode's first two kernels (GQA mean
// folded in), for the reference-mode chain: ids [rows][nk] int64 ascending,
// the GQA mean into raw_q_out [rows][128]; scores [rows][n_c_pad] fp32 and
// sel32 [rows][nk] are scratch.  n_c <= 16384.
int raw_quest_topk(const void* q, int G, const void* cmin, const void* cmax, const uint8_t* valid, int rows,
                   int n_max, int n_c, int nk, float* scores, int n_c_pad, int32_t* sel32, int64_t* ids,
                   uint16_t* raw_q_out, cudaStream_t stream);
// Time limit (ns) of the waits on peers for launches enqueued now
// (zkv_peer_set_wait_ms; 5 s by default).
uint64_t peer_wait_ns();

// Launch `nblocks` CTAs of `nthreads` in clusters of CS (cudaLaunchKernelExC),
// raising the kernel's dynamic shared-memory limit once per (kernel, device).
// `pdl`: programmatic dependent launch -- the grid may be scheduled while the
// previous kernel on the stream finishes; the kernel must execute
// griddepcontrol.wait before it reads anything an earlier kernel writes.
static int launch_clustered(const void* fn, int nblocks, int nthreads, int CS, size_t smem, cudaStream_t stream,
                            void** args, bool pdl = false) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)nblocks, 1, 1);
    cfg.blockDim = dim3((unsigned)nthreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    // raise the dynamic shared-memory limit once per (kernel, device, size)
    static thread_local const void* last_fn[8] = {};
    static thread_local size_t last_smem[8] = {};
    static thread_local int last_dev[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
    int dev = 0;
    cudaGetDevice(&dev);
    int slot = -1;
    for (int i = 0; i < 8; ++i)
        if (last_fn[i] == fn && last_dev[i] == dev) slot = i;
    if (slot < 0 || last_smem[slot] < smem) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return ZKV_ERR_LAUNCH;
        if (slot < 0) {
            for (int i = 0; i < 8; ++i)
                if (!last_fn[i]) {
                    slot = i;
                    break;
                }
            if (slot < 0) slot = 0;
        }
        last_fn[slot] = fn;
        last_dev[slot] = dev;
        last_smem[slot] = smem;
    }
    if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return ZKV_ERR_LAUNCH;
    return cudaGetLastError() == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH;
}
