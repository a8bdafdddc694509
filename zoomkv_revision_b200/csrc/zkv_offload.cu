// zkv_offload.cu -- the offload tier: gather of selected K/V rows from
// host-pinned memory into HBM over the host link (PCIe / C2C), read by the
// SMs through the unified address space (zero-copy).
//
// Reference: cache_hub/gather_trans/trans_h2d.cu (h2d_gather_kv,
// h2d_gather_kv_packed) and trans_h2d.py:65-161, which launch one 32-thread
// block per copied row.  Here a warp moves one (K row, V row) pair per item
// -- lanes 0-15 the K row's 16 x 16 B, lanes 16-31 the V row's -- and every
// warp issues the loads of U items before any store, so each lane keeps U
// host reads in flight; the grid is sized to the SM count, not to the row
// count.  Index values are range-checked on the device: an index outside
// the source rows is skipped and reported through the status word, never
// dereferenced.
#include <mutex>
#include <unordered_map>

#include "zkv_common.cuh"

namespace zkv {
namespace {

constexpr int kRowU4 = kHeadDim * 2 / 16;  // 16 B vectors per bf16 row (16)
constexpr int kU = 4;                      // items per warp in flight
constexpr int kWarps = 8;                  // warps per CTA

struct GatherArgs {
    const uint4* src_k;  // device alias of host-pinned [rows][src_len][128] bf16
    const uint4* src_v;
    int64_t src_len;
    uint4* dst_k;  // HBM
    uint4* dst_v;
    // dense form: item = r * n_sel + j, index idx[r*idx_ld + j] + src_off,
    // destination row r*dst_len + dst_off + j
    const int64_t* idx;
    int64_t idx_ld;
    int n_sel;
    int64_t src_off;
    int64_t dst_len;
    int64_t dst_off;
    // packed form (cu_topk != nullptr): item = vh * global_k + slot
    const int32_t* cu_topk;
    const int32_t* cu_k;
    int global_k;
    int sl_end;
    int64_t n_dst;  // rows of the packed destination
    int64_t items;
    int32_t* status;
};

// Resolve item -> (source row, destination row); false when the item copies
// nothing (packed slot beyond its segment) or its index is out of range.
__device__ __forceinline__ bool item_rows(const GatherArgs& a, int64_t it, int64_t& src_row, int64_t& dst_row) {
    if (a.cu_topk) {
        const int vh = (int)(it / a.global_k), slot = (int)(it - (int64_t)vh * a.global_k);
        const int st = __ldg(a.cu_topk + vh), len = __ldg(a.cu_topk + vh + 1) - st;
        if (slot >= len) return false;
        const int64_t key = __ldg(a.idx + st + slot);
        dst_row = (int64_t)__ldg(a.cu_k + vh) + a.sl_end + slot;
        if (key < 0 || key >= a.src_len || dst_row < 0 || dst_row >= a.n_dst) {
            set_status(a.status, ZKV_ERR_RANGE);
            return false;
        }
        src_row = (int64_t)vh * a.src_len + key;
        return true;
    }
    const int64_t r = it / a.n_sel, j = it - r * a.n_sel;
    const int64_t key = __ldg(a.idx + r * a.idx_ld + j) + a.src_off;
    if (key < 0 || key >= a.src_len) {
        set_status(a.status, ZKV_ERR_RANGE);
        return false;
    }
    src_row = r * a.src_len + key;
    dst_row = r * a.dst_len + a.dst_off + j;
    return true;
}

__global__ void __launch_bounds__(kWarps * 32) h2d_gather_kernel(const GatherArgs a) {
    const int lane = threadIdx.x & 31, part = lane & 15;
    const uint4* src = lane < 16 ? a.src_k : a.src_v;
    uint4* dst = lane < 16 ? a.dst_k : a.dst_v;
    const int64_t tw = (int64_t)gridDim.x * kWarps;
    for (int64_t w0 = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); w0 < a.items; w0 += tw * kU) {
        uint4 v[kU];
        int64_t drow[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int64_t it = w0 + u * tw;
            int64_t srow = -1;
            drow[u] = -1;
            if (it < a.items && !item_rows(a, it, srow, drow[u])) drow[u] = -1;
            // ld.global.cv: a host line cached in L2 by an earlier read is
            // re-fetched, so rows written since by the host or a copy engine
            // are seen
            if (drow[u] >= 0) v[u] = __ldcv(src + srow * kRowU4 + part);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (drow[u] >= 0) dst[drow[u] * kRowU4 + part] = v[u];
    }
}

// Host-pinned pointer -> device alias.  Under unified addressing the alias
// equals the host address for cudaHostAlloc'd memory; the lookup is kept so
// registered memory without that property also works, and cached because
// the caches allocate their pinned zones once.
int device_alias(const void* host, const uint4** out) {
    static std::mutex mu;
    static std::unordered_map<const void*, const void*> cache;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(host);
        if (it != cache.end()) {
            *out = reinterpret_cast<const uint4*>(it->second);
            return ZKV_OK;
        }
    }
    void* d = nullptr;
    if (cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0) != cudaSuccess || !d) {
        cudaGetLastError();  // clear the (non-sticky) error of the failed lookup
        return ZKV_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(mu);
    cache.emplace(host, d);
    *out = reinterpret_cast<const uint4*>(d);
    return ZKV_OK;
}

int launch_gather(GatherArgs& a, const void* src_k, const void* src_v, cudaStream_t stream) {
    if ((((uintptr_t)src_k | (uintptr_t)src_v | (uintptr_t)a.dst_k | (uintptr_t)a.dst_v) & 15)) return ZKV_ERR_ALIGN;
    int rc = device_alias(src_k, &a.src_k);
    if (rc == ZKV_OK) rc = device_alias(src_v, &a.src_v);
    if (rc != ZKV_OK) return rc;
    if (a.items == 0) return ZKV_OK;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = (a.items + (int64_t)kWarps * kU - 1) / ((int64_t)kWarps * kU);
    const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
    h2d_gather_kernel<<<grid, kWarps * 32, 0, stream>>>(a);
    return launch_status();
}

}  // namespace
}  // namespace zkv

using namespace zkv;

extern "C" int zkv_h2d_gather_kv(const void* src_k, const void* src_v, int rows, int64_t src_len,
                                 const int64_t* idx, int64_t idx_ld, int n_sel, int64_t src_off, void* dst_k,
                                 void* dst_v, int64_t dst_len, int64_t dst_off, int32_t* status, void* stream) {
    if (!src_k || !src_v || !dst_k || !dst_v || rows < 0 || src_len < 1 || n_sel < 0 || dst_off < 0 ||
        dst_off + n_sel > dst_len || (n_sel > 0 && (!idx || idx_ld < 0 || (idx_ld > 0 && idx_ld < n_sel))))
        return ZKV_ERR_ARG;
    GatherArgs a = {};
    a.src_len = src_len;
    a.dst_k = reinterpret_cast<uint4*>(dst_k);
    a.dst_v = reinterpret_cast<uint4*>(dst_v);
    a.idx = idx;
    a.idx_ld = idx_ld;
    a.n_sel = n_sel;
    a.src_off = src_off;
    a.dst_len = dst_len;
    a.dst_off = dst_off;
    a.items = (int64_t)rows * n_sel;
    a.status = status;
    return launch_gather(a, src_k, src_v, (cudaStream_t)stream);
}

extern "C" int zkv_h2d_gather_kv_packed(const void* src_k, const void* src_v, int rows, int64_t src_len,
                                        const int64_t* idx, const int32_t* cu_topk, const int32_t* cu_k, int sl_end,
                                        int global_k, void* dst_k, void* dst_v, int64_t n_dst, int32_t* status,
                                        void* stream) {
    if (!src_k || !src_v || !dst_k || !dst_v || rows < 0 || src_len < 1 || sl_end < 0 || n_dst < 0)
        return ZKV_ERR_ARG;
    if (global_k <= 0 || rows == 0) return ZKV_OK;  // nothing to copy (as the reference)
    if (!idx || !cu_topk || !cu_k) return ZKV_ERR_ARG;
    GatherArgs a = {};
    a.src_len = src_len;
    a.dst_k = reinterpret_cast<uint4*>(dst_k);
    a.dst_v = reinterpret_cast<uint4*>(dst_v);
    a.idx = idx;
    a.cu_topk = cu_topk;
    a.cu_k = cu_k;
    a.global_k = global_k;
    a.sl_end = sl_end;
    a.n_dst = n_dst;
    a.items = (int64_t)rows * global_k;
    a.status = status;
    return launch_gather(a, src_k, src_v, (cudaStream_t)stream);
}
