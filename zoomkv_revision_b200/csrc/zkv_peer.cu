// zkv_peer.cu -- the exchange steps of the sequence-split decode over peer
// memory (NVLink P2P), without a collective library on the data path.
//
// Every rank allocates one buffer with zkv_peer_alloc and shares its IPC
// handle; each rank opens the others' handles (zkv_peer_open), so every
// rank holds a device pointer into every peer's buffer.  An exchange step
// is then two launches on the rank's stream:
//
//   zkv_peer_put   copies this rank's slice into slot `rank` of every
//                  peer's buffer with plain stores over NVLink, and, once
//                  every CTA's stores are done, raises this rank's flag in
//                  every peer to epoch + 1 (release at system scope);
//   zkv_peer_wait  one warp polls (acquire, system scope) until the flags of
//                  all ranks reach epoch + 1, then advances the local epoch.
//
// zkv_peer_exchange is the two in one launch: the CTA that raises the flags
// then waits for every rank's flags and advances the epoch.
//
// The epoch lives in device memory and only the wait advances it, so a
// captured CUDA graph replays correctly.  Every rank runs the same sequence
// of puts and waits, so epochs agree across ranks.  A wait gives up after a
// time limit on the GPU's global timer (5 s unless zkv_peer_set_wait_ms
// says otherwise; the limit is read when a launch is enqueued, so a
// captured graph keeps the limit of its capture), records ZKV_ERR_TIMEOUT in
// the status word and returns, so a rank that never arrives ends in a
// host-side error, not a hung GPU.  After a timeout the epochs of the ranks
// no longer agree: the peer group must be rebuilt.  No TMA and no multicast
// are used: the copies are 16- or 4-byte thread stores.
#include <atomic>
#include <cstring>

#include "zkv_common.cuh"

namespace zkv {
namespace {

constexpr int kPutThreads = 256;
constexpr int kMaxPeers = 8;
constexpr int kMaxSegs = 2;

struct PutSeg {
    const uint32_t* src;  // [rows][src_ld] words
    int64_t src_ld, dst_ld, dst_off;  // words
    int rows, row_words;
};

struct PutArgs {
    PutSeg seg[kMaxSegs];
    int n_seg;
    uint32_t* dst[kMaxPeers];    // base of every peer's buffer (this rank's mapping)
    uint32_t* flag[kMaxPeers];   // this rank's flag word inside every peer's buffer
    const uint32_t* epoch;       // local
    uint32_t* done;              // local counter of finished CTAs (0 between launches)
    const uint32_t* wait_flags;  // exchange form: this rank's flag array of the phase (NULL: put only)
    uint32_t* epoch_rw;          // exchange form: the epoch the last CTA advances
    int32_t* status;
    int world;
    int chunks;                  // CTAs per peer
    uint64_t wait_ns;            // exchange form: give up waiting after this long
};

std::atomic<uint64_t> g_wait_ns{5000000000ull};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Copy `items` (row, unit) pairs of one segment: item i is unit u0 + i % cnt
// of row i / cnt; every thread issues U loads before its stores.
template <typename T>
__device__ __forceinline__ void put_items(const T* __restrict__ src, T* __restrict__ dst, int64_t src_ld,
                                          int64_t dst_ld, int u0, int cnt, int items) {
    constexpr int U = 4;
    for (int base = threadIdx.x; base < items; base += kPutThreads * U) {
        T v[U];
        int64_t d[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = base + k * kPutThreads;
            d[k] = -1;
            if (i < items) {
                const int r = i / cnt, u = u0 + i - r * cnt;
                v[k] = __ldg(src + r * src_ld + u);
                d[k] = r * dst_ld + u;
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k)
            if (d[k] >= 0) dst[d[k]] = v[k];
    }
}

// CTA (p, c) copies slice c of every row of every segment to peer p (16-byte
// units where the segment's rows are 16-byte aligned, 4-byte ones
// otherwise); the last CTA to finish raises the flags.
__global__ void __launch_bounds__(kPutThreads) peer_put_kernel(const PutArgs a) {
    const int p = blockIdx.x / a.chunks, c = blockIdx.x - p * a.chunks;
    uint32_t* dst = a.dst[p];
    for (int s = 0; s < a.n_seg; ++s) {
        const PutSeg g = a.seg[s];
        const bool vec = ((g.src_ld | g.dst_ld | g.dst_off | g.row_words) & 3) == 0 &&
                         ((uintptr_t)g.src & 15) == 0;
        const int unit = vec ? 4 : 1;
        const int units = g.row_words / unit;
        const int per = (units + a.chunks - 1) / a.chunks;
        const int u0 = min(units, c * per), cnt = min(units, u0 + per) - u0;
        if (cnt <= 0) continue;
        if (vec)
            put_items(reinterpret_cast<const uint4*>(g.src), reinterpret_cast<uint4*>(dst + g.dst_off),
                      g.src_ld / 4, g.dst_ld / 4, u0, cnt, g.rows * cnt);
        else
            put_items(g.src, dst + g.dst_off, g.src_ld, g.dst_ld, u0, cnt, g.rows * cnt);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();  // this CTA's peer stores before its arrival
        const uint32_t prev = atomicAdd(a.done, 1u);
        if (prev == gridDim.x - 1) {  // every CTA's stores are visible system-wide
            __threadfence_system();
            const uint32_t target = *a.epoch + 1u;
            for (int q = 0; q < a.world; ++q) st_release_sys(a.flag[q], target);
            *a.done = 0u;
            if (a.wait_flags) {  // exchange form: this CTA also waits for every rank's put
                bool ok = true;
                const uint64_t t0 = globaltimer_ns();
                for (int q = 0; q < a.world && ok; ++q) {
                    while ((int32_t)(ld_acquire_sys(a.wait_flags + q) - target) < 0) {
                        if (globaltimer_ns() - t0 > a.wait_ns) {
                            ok = false;
                            break;
                        }
                        __nanosleep(128);
                    }
                }
                if (!ok) set_status(a.status, ZKV_ERR_TIMEOUT);
                *a.epoch_rw = target;
            }
        }
    }
}

__global__ void peer_wait_kernel(const uint32_t* flags, uint32_t* epoch, int world, int32_t* status,
                                 uint64_t wait_ns) {
    const int lane = threadIdx.x;
    const uint32_t target = *epoch + 1u;
    bool ok = true;
    if (lane < world) {
        const uint64_t t0 = globaltimer_ns();
        while ((int32_t)(ld_acquire_sys(flags + lane) - target) < 0) {
            if (globaltimer_ns() - t0 > wait_ns) {
                ok = false;
                break;
            }
            __nanosleep(256);
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (lane == 0) {
        if (!ok) set_status(status, ZKV_ERR_TIMEOUT);
        __threadfence();
        *epoch = target;
    }
}

}  // namespace
}  // namespace zkv

using namespace zkv;

uint64_t peer_wait_ns() { return g_wait_ns.load(); }

extern "C" int zkv_peer_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle || bytes == 0) return ZKV_ERR_ARG;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return ZKV_ERR_LAUNCH;
    }
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return ZKV_ERR_LAUNCH;
    }
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return ZKV_OK;
}

extern "C" int zkv_peer_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int zkv_peer_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return ZKV_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return ZKV_ERR_LAUNCH;
    }
    return ZKV_OK;
}

extern "C" int zkv_peer_close(void* ptr) {
    if (!ptr) return ZKV_ERR_ARG;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH;
}

extern "C" int zkv_peer_free(void* ptr) {
    if (!ptr) return ZKV_ERR_ARG;
    return cudaFree(ptr) == cudaSuccess ? ZKV_OK : ZKV_ERR_LAUNCH;
}

static int peer_put_launch(const zkv_peer_seg* segs, int n_seg, void* const* peer_base, int64_t flag_off, int rank,
                           int world, uint32_t* epoch, uint32_t* done, int chunks, bool exchange, int32_t* status,
                           void* stream) {
    if (!segs || n_seg < 1 || n_seg > kMaxSegs || !peer_base || world < 1 || world > kMaxPeers || rank < 0 ||
        rank >= world || !epoch || !done || flag_off < 0 || (flag_off & 3) || chunks < 0)
        return ZKV_ERR_ARG;
    PutArgs a = {};
    for (int s = 0; s < n_seg; ++s) {
        const zkv_peer_seg& g = segs[s];
        if (!g.src || g.rows < 0 || g.row_bytes < 0 || (g.row_bytes & 3) || (g.src_ld_bytes & 3) ||
            (g.dst_ld_bytes & 3) || (g.dst_off_bytes & 3) || ((uintptr_t)g.src & 3) ||
            (g.rows > 1 && (g.src_ld_bytes < g.row_bytes || g.dst_ld_bytes < g.row_bytes)))
            return ZKV_ERR_ARG;
        a.seg[s] = {reinterpret_cast<const uint32_t*>(g.src), g.src_ld_bytes / 4, g.dst_ld_bytes / 4,
                    g.dst_off_bytes / 4, (int)g.rows, (int)(g.row_bytes / 4)};
    }
    a.n_seg = n_seg;
    for (int p = 0; p < world; ++p) {
        if (!peer_base[p] || ((uintptr_t)peer_base[p] & 15)) return ZKV_ERR_ARG;
        a.dst[p] = reinterpret_cast<uint32_t*>(peer_base[p]);
        a.flag[p] = reinterpret_cast<uint32_t*>(static_cast<char*>(peer_base[p]) + flag_off) + rank;
    }
    a.epoch = epoch;
    a.done = done;
    a.wait_flags = exchange ? reinterpret_cast<const uint32_t*>(static_cast<char*>(peer_base[rank]) + flag_off)
                            : nullptr;
    a.epoch_rw = exchange ? epoch : nullptr;
    a.status = status;
    a.world = world;
    a.chunks = chunks > 0 ? chunks : (world <= 2 ? 8 : 2);
    a.wait_ns = g_wait_ns.load();
    peer_put_kernel<<<world * a.chunks, kPutThreads, 0, (cudaStream_t)stream>>>(a);
    return launch_status();
}

extern "C" int zkv_peer_put(const zkv_peer_seg* segs, int n_seg, void* const* peer_base, int64_t flag_off,
                            int rank, int world, uint32_t* epoch, uint32_t* done, int chunks, void* stream) {
    return peer_put_launch(segs, n_seg, peer_base, flag_off, rank, world, epoch, done, chunks, false, nullptr, stream);
}

extern "C" int zkv_peer_exchange(const zkv_peer_seg* segs, int n_seg, void* const* peer_base, int64_t flag_off,
                                 int rank, int world, uint32_t* epoch, uint32_t* done, int chunks, int32_t* status,
                                 void* stream) {
    return peer_put_launch(segs, n_seg, peer_base, flag_off, rank, world, epoch, done, chunks, true, status, stream);
}

extern "C" int zkv_peer_wait(const uint32_t* flags, uint32_t* epoch, int world, int32_t* status, void* stream) {
    if (!flags || !epoch || world < 1 || world > kMaxPeers) return ZKV_ERR_ARG;
    peer_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flags, epoch, world, status, g_wait_ns.load());
    return launch_status();
}

extern "C" int zkv_peer_set_wait_ms(int ms) {
    if (ms < 1 || ms > 600000) return ZKV_ERR_ARG;
    g_wait_ns.store((uint64_t)ms * 1000000ull);
    return ZKV_OK;
}
