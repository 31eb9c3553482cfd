// sm_100a data movers: paged gather/scatter between mapped host DRAM and HBM
// (tmaGather/tmaScatter) and the GPU-fabric WR batch copy.
//
// Bulk path ("TMA"). Persistent grid, one CTA per SM, WARPS independent
// pipelines per CTA. A pipeline is driven by lane 0 of its warp: it keeps
// STAGES bulk loads (cp.async.bulk global->shared, mbarrier complete_tx) in
// flight, turns each landed stage into a bulk store (shared->global,
// bulk_group) and refills a stage as soon as the store reading it has
// drained (wait_group.read 1). The other 31 lanes fetch tile descriptors
// (block index -> addresses) 32 tiles at a time and hand them to lane 0 by
// shuffle, so index loads never sit on the issue path.
//
// Compared with the reference kernel (src/mpcomm_tma_kernels.cu:144-192:
// one load->wait->store->wait per lane, 128 x block_size of shared memory,
// so 64 KiB pages cannot launch), pages are split into STAGE_BYTES tiles,
// shared memory is fixed at WARPS x STAGES x STAGE_BYTES, and every wait
// is bounded.
//
// Vector path ("SM"). One warp per tile, 16-byte loads, 4 in flight per
// lane, 64-bit indexing and no per-element div/mod (reference :259-299 used
// 32-bit indices and a div/mod per 16 bytes).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "kernels/common.cuh"

namespace mpcomm {
namespace kern {

namespace {

std::atomic<uint64_t> g_launches{0};

constexpr int kWarps = 4;
constexpr int kStages = 3;
constexpr uint32_t kStageBytes = 16384;
constexpr size_t kBulkSmem = static_cast<size_t>(kWarps) * kStages * kStageBytes +
                             static_cast<size_t>(kWarps) * kStages * sizeof(uint64_t);
constexpr int kVecWarps = 8;
constexpr uint32_t kVecTileBytes = 65536;

}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }

int sm_count(int dev) {
    static std::mutex mu;
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> g(mu);
    if (!cache[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        cache[dev] = v;
    }
    return cache[dev];
}

uint64_t wait_budget_ns() {
    static const uint64_t v = [] {
        const char *e = std::getenv("MPCOMM_KERNEL_WAIT_BUDGET_MS");
        long long ms = e ? std::atoll(e) : 2000;
        if (ms <= 0) ms = 2000;
        return static_cast<uint64_t>(ms) * 1000000ull;
    }();
    return v;
}

uint32_t *default_status_word(int dev) {
    static std::mutex mu;
    static uint32_t *words[64] = {nullptr};
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> g(mu);
    if (!words[dev]) {
        void *p = nullptr;
        if (cudaMalloc(&p, 256) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, 256);
        words[dev] = static_cast<uint32_t *>(p);
    }
    return words[dev];
}

// ---------------------------------------------------------------------------
// Kernel trace ring (MPCOMM_KERNEL_TRACE=<slots>, 0 = off): per device, a
// device-memory ring of start/end stamps that launches write themselves;
// the host keeps what each slot was used for and reads the ring back only
// when asked (kernel_trace()).
// ---------------------------------------------------------------------------
namespace {

struct TraceMeta {
    uint64_t seq = 0;
    const char *kind = nullptr;
    uint64_t bytes = 0;
};

struct TraceState {
    std::mutex mu;
    size_t slots = 0;
    uint64_t seq = 0;
    KernelStamp *ring[64] = {nullptr};
    std::vector<TraceMeta> meta[64];
};

TraceState &trace_state() {
    static TraceState *t = [] {
        auto *s = new TraceState();
        const char *e = std::getenv("MPCOMM_KERNEL_TRACE");
        long long v = e ? std::atoll(e) : 0;
        s->slots = v > 0 ? static_cast<size_t>(v < 1048576 ? v : 1048576) : 0;
        return s;
    }();
    return *t;
}

}  // namespace

KernelStamp *trace_acquire(const char *kind, uint64_t bytes) {
    TraceState &t = trace_state();
    if (!t.slots) return nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> g(t.mu);
    if (!t.ring[dev]) {
        void *p = nullptr;
        if (cudaMalloc(&p, t.slots * sizeof(KernelStamp)) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        cudaMemset(p, 0, t.slots * sizeof(KernelStamp));
        t.ring[dev] = static_cast<KernelStamp *>(p);
        t.meta[dev].assign(t.slots, TraceMeta{});
    }
    const uint64_t seq = ++t.seq;
    const size_t slot = static_cast<size_t>(seq % t.slots);
    t.meta[dev][slot] = TraceMeta{seq, kind, bytes};
    return t.ring[dev] + slot;
}

int kernel_trace(std::vector<TraceRecord> *out) {
    out->clear();
    TraceState &t = trace_state();
    std::lock_guard<std::mutex> g(t.mu);
    if (!t.slots) return 0;
    std::vector<KernelStamp> host(t.slots);
    for (int dev = 0; dev < 64; ++dev) {
        if (!t.ring[dev]) continue;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(dev);
        cudaError_t e = cudaMemcpy(host.data(), t.ring[dev], t.slots * sizeof(KernelStamp), cudaMemcpyDeviceToHost);
        cudaSetDevice(prev);
        if (e != cudaSuccess) return e;
        for (size_t i = 0; i < t.slots; ++i) {
            const TraceMeta &m = t.meta[dev][i];
            if (!m.seq || !host[i].begin_ns || host[i].end_ns < host[i].begin_ns) continue;
            out->push_back(TraceRecord{m.seq, dev, m.kind, m.bytes, host[i].begin_ns, host[i].end_ns});
        }
    }
    std::sort(out->begin(), out->end(), [](const TraceRecord &a, const TraceRecord &b) { return a.seq < b.seq; });
    return 0;
}

void kernel_trace_reset() {
    TraceState &t = trace_state();
    std::lock_guard<std::mutex> g(t.mu);
    for (int dev = 0; dev < 64; ++dev)
        if (t.ring[dev]) t.meta[dev].assign(t.slots, TraceMeta{});
}

size_t kernel_trace_slots() { return trace_state().slots; }

// ---------------------------------------------------------------------------
// Tile sources
// ---------------------------------------------------------------------------
struct GatherSrc {
    const char *pool;
    const int64_t *idx;
    char *out;
    int64_t n, bs, pool_blocks, tpb;
    uint32_t tile_bytes;
    const uint32_t *gate = nullptr;  // QoS gate: only fabric batches use one
    uint64_t gate_budget = 0;
    __device__ __forceinline__ int64_t count() const { return n * tpb; }
    __device__ __forceinline__ Tile tile(int64_t t) const {
        const int64_t b = t / tpb;
        const int64_t off = (t - b * tpb) * static_cast<int64_t>(tile_bytes);
        const int64_t rem = bs - off;
        const uint32_t len = static_cast<uint32_t>(rem < tile_bytes ? rem : tile_bytes);
        const int64_t p = __ldg(idx + b);
        if (p < 0 || (pool_blocks > 0 && p >= pool_blocks)) return Tile{nullptr, nullptr, len, kBad};
        const char *s = pool + p * bs + off;
        char *d = out + b * bs + off;
        return Tile{s, d, len, tile_kind(s, d, len)};
    }
};

struct ScatterSrc {
    const char *src;
    const int64_t *idx;
    char *pool;
    int64_t n, bs, pool_blocks, tpb;
    uint32_t tile_bytes;
    const uint32_t *gate = nullptr;
    uint64_t gate_budget = 0;
    __device__ __forceinline__ int64_t count() const { return n * tpb; }
    __device__ __forceinline__ Tile tile(int64_t t) const {
        const int64_t b = t / tpb;
        const int64_t off = (t - b * tpb) * static_cast<int64_t>(tile_bytes);
        const int64_t rem = bs - off;
        const uint32_t len = static_cast<uint32_t>(rem < tile_bytes ? rem : tile_bytes);
        const int64_t p = __ldg(idx + b);
        if (p < 0 || (pool_blocks > 0 && p >= pool_blocks)) return Tile{nullptr, nullptr, len, kBad};
        const char *s = src + b * bs + off;
        char *d = pool + p * bs + off;
        return Tile{s, d, len, tile_kind(s, d, len)};
    }
};

struct BatchSrc {
    CopyDesc d[kMaxCopyDescs];
    int64_t start[kMaxCopyDescs + 1];
    int n;
    uint32_t tile_bytes;
    const uint32_t *gate;  // device QoS gate (null = ungated)
    uint64_t gate_budget;  // total pause per pipeline, ns
    __device__ __forceinline__ int64_t count() const { return start[n]; }
    __device__ __forceinline__ Tile tile(int64_t t) const {
        int lo = 0, hi = n;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (start[mid] <= t) lo = mid; else hi = mid;
        }
        const int64_t off = (t - start[lo]) * static_cast<int64_t>(tile_bytes);
        const int64_t rem = static_cast<int64_t>(d[lo].bytes) - off;
        const uint32_t len = static_cast<uint32_t>(rem < tile_bytes ? rem : tile_bytes);
        const char *s = static_cast<const char *>(d[lo].src) + off;
        char *dd = static_cast<char *>(d[lo].dst) + off;
        return Tile{s, dd, len, tile_kind(s, dd, len)};
    }
};

// ---------------------------------------------------------------------------
// Bulk (TMA engine) pipeline, one per warp.
// ---------------------------------------------------------------------------
template <int STAGES, uint32_t STAGE_BYTES, class Src>
__device__ __forceinline__ void warp_bulk_pipeline(const Src &src, int64_t first, int64_t stride,
                                                   char *stage_mem, uint64_t *bars,
                                                   uint32_t *status, uint64_t budget) {
    const int lane = threadIdx.x & 31;
    const int64_t total = src.count();
    if (first >= total) return;
    const int64_t n = (total - 1 - first) / stride + 1;

    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        fence_proxy_async_smem();
    }
    __syncwarp();

    Tile mine{nullptr, nullptr, 0, kSkip};
    int64_t win = -1;
    // Lane-0 record of what each stage holds.
    const char *st_src[STAGES];
    char *st_dst[STAGES];
    uint32_t st_bytes[STAGES];
    uint32_t st_kind[STAGES];
    int64_t issued = 0;
    uint64_t paused = 0;  // lane 0: QoS pause spent so far

    auto issue = [&](int64_t t, int s) {  // warp-collective
        const int64_t w = t >> 5;
        if (w != win) {
            win = w;
            const int64_t tt = (w << 5) + lane;
            mine = tt < n ? src.tile(first + tt * stride) : Tile{nullptr, nullptr, 0, kSkip};
        }
        const int sl = static_cast<int>(t & 31);
        const char *ts = reinterpret_cast<const char *>(
            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(mine.src), sl));
        char *td = reinterpret_cast<char *>(
            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(mine.dst), sl));
        const uint32_t tb = __shfl_sync(0xffffffffu, mine.bytes, sl);
        const uint32_t tk = __shfl_sync(0xffffffffu, mine.kind, sl);
        if (lane == 0) {
            st_src[s] = ts;
            st_dst[s] = td;
            st_bytes[s] = tb;
            st_kind[s] = tk;
            const bool bulk = tk == kBulk;
            qos_gate_wait(src.gate, paused, src.gate_budget);
            mbar_arrive_expect_tx(&bars[s], bulk ? tb : 0u);
            if (bulk) bulk_load(stage_mem + static_cast<size_t>(s) * STAGE_BYTES, ts, tb, &bars[s]);
        }
        ++issued;
    };

    const int64_t pro = n < STAGES ? n : STAGES;
    for (int64_t t = 0; t < pro; ++t) issue(t, static_cast<int>(t));

    int64_t j = 0;
    bool aborted = false;
    for (; j < n; ++j) {
        const int s = static_cast<int>(j % STAGES);
        const uint32_t parity = static_cast<uint32_t>((j / STAGES) & 1);
        uint32_t kind = kSkip;
        const char *isrc = nullptr;
        char *idst = nullptr;
        uint32_t ibytes = 0;
        int ok = 1;
        if (lane == 0) {
            if (!mbar_wait_bounded(&bars[s], parity, budget)) {
                ok = 0;
                atomicOr(status, kStatusLoadTimeout);
            } else {
                kind = st_kind[s];
                if (kind == kBulk) {
                    bulk_store(st_dst[s], stage_mem + static_cast<size_t>(s) * STAGE_BYTES,
                               st_bytes[s]);
                } else if (kind == kBad) {
                    atomicOr(status, kStatusBadIndex);
                }
                isrc = st_src[s];
                idst = st_dst[s];
                ibytes = st_bytes[s];
            }
            bulk_commit();
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            aborted = true;
            break;
        }
        kind = __shfl_sync(0xffffffffu, kind, 0);
        if (kind == kInline) {
            isrc = reinterpret_cast<const char *>(
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(isrc), 0));
            idst = reinterpret_cast<char *>(
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(idst), 0));
            ibytes = __shfl_sync(0xffffffffu, ibytes, 0);
            warp_copy_any(idst, isrc, ibytes);
        }
        if (j >= 1) {
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
            const int64_t t = j - 1 + STAGES;
            if (t < n) issue(t, static_cast<int>((j - 1) % STAGES));
        }
    }
    if (lane == 0) {
        if (aborted) {
            // Drain every load still in flight into this warp's stages before
            // the CTA may exit (bounded again).
            for (int64_t t = j; t < issued; ++t) {
                if (!mbar_wait_bounded(&bars[t % STAGES], static_cast<uint32_t>((t / STAGES) & 1),
                                       budget)) {
                    atomicOr(status, kStatusDrainTimeout);
                    break;
                }
            }
        }
        bulk_wait_all();
    }
    __syncwarp();
}

// Kernel epilogue: closes an H2D QoS window and/or publishes a completion
// flag once the last CTA has drained all of its stores; records the
// launch's device start/end in its trace slot (device memory, optional).
struct Epilogue {
    H2DWindow *win;
    uint32_t *ctr;      // last-CTA detector (self-resetting), required if win or flag
    uint64_t *flag;     // may point into a peer GPU's memory
    uint64_t flag_value;
    KernelStamp *stamp = nullptr;
};


__device__ __forceinline__ void run_epilogue(const Epilogue &ep) {
    if (!ep.win && !ep.flag) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t prev = atomicAdd(ep.ctr, 1u);
        if (prev == gridDim.x - 1) {
            *ep.ctr = 0u;
            __threadfence_system();
            if (ep.flag) st_release_sys_u64(ep.flag, ep.flag_value);
            if (ep.win) {
                uint32_t *gate = *reinterpret_cast<uint32_t *volatile *>(&ep.win->gate);
                if (gate) atomicSub(gate, 1u);
                st_release_sys_u64(&ep.win->end_ns, globaltimer_ns() | 1ull);
            }
        }
    }
}

template <int WARPS, int STAGES, uint32_t STAGE_BYTES, class Src>
__global__ void __launch_bounds__(WARPS * 32, 1)
    bulk_mover_kernel(const __grid_constant__ Src src, uint32_t *status, uint64_t budget,
                      const Epilogue ep) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int warp = threadIdx.x >> 5;
    char *stage_mem = reinterpret_cast<char *>(smem_raw) +
                      static_cast<size_t>(warp) * STAGES * STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(
                         smem_raw + static_cast<size_t>(WARPS) * STAGES * STAGE_BYTES) +
                     warp * STAGES;
    trace_begin(ep.stamp);
    window_open(ep.win);
    warp_bulk_pipeline<STAGES, STAGE_BYTES>(src, static_cast<int64_t>(blockIdx.x) * WARPS + warp,
                                            static_cast<int64_t>(gridDim.x) * WARPS, stage_mem,
                                            bars, status, budget);
    trace_end(ep.stamp);
    run_epilogue(ep);
}

// ---------------------------------------------------------------------------
// Packed gather of small blocks (<= 4 KiB): a warp's stage holds up to 32
// whole blocks of one tile, one per lane. Every lane issues the bulk load of
// its own block into the stage (all completing on the stage's mbarrier, whose
// expected byte count lane 0 sets first), and lane 0 writes the tile to the
// contiguous output with ONE bulk store. A warp keeps STAGES x 32 blocks in
// flight instead of STAGES, so a batch of small blocks is one wave of PCIe
// reads rather than many.
// ---------------------------------------------------------------------------
struct PackedGather {
    const char *pool;
    const int64_t *idx;
    char *out;
    int64_t n, bs, pool_blocks;
    int per;  // blocks per tile (<= 32, per * bs <= stage bytes)
};

// Warp copy of one landed block out of a shared-memory stage (16-byte
// multiples, 16-byte aligned on both sides): shared-space loads, global
// stores.
__device__ __forceinline__ void warp_copy_from_stage(char *dst, const char *stage, uint32_t bytes) {
    const int lane = threadIdx.x & 31;
    for (uint32_t i = static_cast<uint32_t>(lane); i < (bytes >> 4); i += 32) {
        int4 v;
        asm volatile("ld.shared.v4.s32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "r"(smem_u32(stage + (static_cast<size_t>(i) << 4))));
        *reinterpret_cast<int4 *>(dst + (static_cast<size_t>(i) << 4)) = v;
    }
}

template <int STAGES, uint32_t STAGE_BYTES>
__device__ __forceinline__ void warp_packed_gather(const PackedGather &a, int64_t first, int64_t stride,
                                                   char *stage_mem, uint64_t *bars, uint32_t *status,
                                                   uint64_t budget) {
    const int lane = threadIdx.x & 31;
    const int64_t tiles = (a.n + a.per - 1) / a.per;
    if (first >= tiles) return;
    const int64_t n = (tiles - 1 - first) / stride + 1;
    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        fence_proxy_async_smem();
    }
    __syncwarp();
    // Lane-0 record of each stage: first block, block count, bad-index lanes.
    int64_t st_b0[STAGES];
    uint32_t st_cnt[STAGES], st_bad[STAGES];
    int64_t issued = 0;
    const uint32_t bs = static_cast<uint32_t>(a.bs);

    auto issue = [&](int64_t j, int s) {  // warp-collective
        const int64_t b0 = (first + j * stride) * a.per;
        const int64_t left = a.n - b0;
        const uint32_t cnt = static_cast<uint32_t>(left < a.per ? left : a.per);
        int64_t p = -1;
        bool valid = false;
        if (static_cast<uint32_t>(lane) < cnt) {
            p = __ldg(a.idx + b0 + lane);
            valid = p >= 0 && (a.pool_blocks <= 0 || p < a.pool_blocks);
        }
        const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
        if (lane == 0) {
            const uint32_t all = cnt >= 32 ? 0xffffffffu : ((1u << cnt) - 1u);
            st_b0[s] = b0;
            st_cnt[s] = cnt;
            st_bad[s] = all & ~vmask;
            mbar_arrive_expect_tx(&bars[s], static_cast<uint32_t>(__popc(vmask)) * bs);
        }
        __syncwarp();  // the expected byte count is set before any load lands
        if (valid)
            bulk_load(stage_mem + static_cast<size_t>(s) * STAGE_BYTES + static_cast<size_t>(lane) * bs,
                      a.pool + p * a.bs, bs, &bars[s]);
        ++issued;
    };

    const int64_t pro = n < STAGES ? n : STAGES;
    for (int64_t j = 0; j < pro; ++j) issue(j, static_cast<int>(j));

    int64_t j = 0;
    bool aborted = false;
    for (; j < n; ++j) {
        const int s = static_cast<int>(j % STAGES);
        const uint32_t parity = static_cast<uint32_t>((j / STAGES) & 1);
        char *stage = stage_mem + static_cast<size_t>(s) * STAGE_BYTES;
        int ok = 1;
        uint32_t bad = 0, cnt = 0;
        int64_t b0 = 0;
        if (lane == 0) {
            if (!mbar_wait_bounded(&bars[s], parity, budget)) {
                ok = 0;
                atomicOr(status, kStatusLoadTimeout);
            } else {
                bad = st_bad[s];
                cnt = st_cnt[s];
                b0 = st_b0[s];
                if (!bad) bulk_store(a.out + b0 * a.bs, stage, cnt * bs);
                else atomicOr(status, kStatusBadIndex);
            }
            bulk_commit();
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            aborted = true;
            break;
        }
        bad = __shfl_sync(0xffffffffu, bad, 0);
        if (bad) {
            // Slow path: the valid blocks one by one (a bad index leaves its
            // output block untouched, as in the tiled pipeline).
            __syncwarp();  // lane 0 saw the stage land before the lanes read it
            cnt = __shfl_sync(0xffffffffu, cnt, 0);
            b0 = static_cast<int64_t>(__shfl_sync(0xffffffffu, static_cast<long long>(b0), 0));
            for (uint32_t k = 0; k < cnt; ++k)
                if (!((bad >> k) & 1u)) warp_copy_from_stage(a.out + (b0 + k) * a.bs, stage + k * bs, bs);
            __syncwarp();
            if (lane == 0) fence_proxy_async_smem();  // generic reads before the next async fill
        }
        if (j >= 1) {
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
            const int64_t t = j - 1 + STAGES;
            if (t < n) issue(t, static_cast<int>((j - 1) % STAGES));
        }
    }
    if (lane == 0) {
        if (aborted) {
            for (int64_t t = j; t < issued; ++t) {
                if (!mbar_wait_bounded(&bars[t % STAGES], static_cast<uint32_t>((t / STAGES) & 1), budget)) {
                    atomicOr(status, kStatusDrainTimeout);
                    break;
                }
            }
        }
        bulk_wait_all();
    }
    __syncwarp();
}

template <int WARPS, int STAGES, uint32_t STAGE_BYTES>
__global__ void __launch_bounds__(WARPS * 32, 1)
    packed_gather_kernel(const __grid_constant__ PackedGather a, uint32_t *status, uint64_t budget,
                         const Epilogue ep) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int warp = threadIdx.x >> 5;
    char *stage_mem = reinterpret_cast<char *>(smem_raw) + static_cast<size_t>(warp) * STAGES * STAGE_BYTES;
    uint64_t *bars =
        reinterpret_cast<uint64_t *>(smem_raw + static_cast<size_t>(WARPS) * STAGES * STAGE_BYTES) + warp * STAGES;
    trace_begin(ep.stamp);
    window_open(ep.win);
    warp_packed_gather<STAGES, STAGE_BYTES>(a, static_cast<int64_t>(blockIdx.x) * WARPS + warp,
                                            static_cast<int64_t>(gridDim.x) * WARPS, stage_mem, bars, status, budget);
    trace_end(ep.stamp);
    run_epilogue(ep);
}

// Packed scatter of small blocks, the gather's mirror: lane 0 loads a tile
// of up to 32 consecutive source blocks with ONE bulk load, then every lane
// stores its own block to its pool slot (one bulk store per lane, tracked by
// that lane's own bulk groups; every lane commits each round so the groups
// stay aligned across the warp).
struct PackedScatter {
    const char *src;
    const int64_t *idx;
    char *pool;
    int64_t n, bs, pool_blocks;
    int per;
};

template <int STAGES, uint32_t STAGE_BYTES>
__device__ __forceinline__ void warp_packed_scatter(const PackedScatter &a, int64_t first, int64_t stride,
                                                    char *stage_mem, uint64_t *bars, uint32_t *status,
                                                    uint64_t budget) {
    const int lane = threadIdx.x & 31;
    const int64_t tiles = (a.n + a.per - 1) / a.per;
    if (first >= tiles) return;
    const int64_t n = (tiles - 1 - first) / stride + 1;
    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        fence_proxy_async_smem();
    }
    __syncwarp();
    const uint32_t bs = static_cast<uint32_t>(a.bs);
    int64_t issued = 0;

    auto tile_count = [&](int64_t j) -> uint32_t {
        const int64_t left = a.n - (first + j * stride) * a.per;
        return static_cast<uint32_t>(left < a.per ? left : a.per);
    };
    auto issue = [&](int64_t j, int s) {  // lane 0 loads; the others only count
        if (lane == 0) {
            const int64_t b0 = (first + j * stride) * a.per;
            const uint32_t bytes = tile_count(j) * bs;
            mbar_arrive_expect_tx(&bars[s], bytes);
            bulk_load(stage_mem + static_cast<size_t>(s) * STAGE_BYTES, a.src + b0 * a.bs, bytes, &bars[s]);
        }
        ++issued;
    };

    const int64_t pro = n < STAGES ? n : STAGES;
    for (int64_t j = 0; j < pro; ++j) issue(j, static_cast<int>(j));

    int64_t j = 0;
    bool aborted = false;
    for (; j < n; ++j) {
        const int s = static_cast<int>(j % STAGES);
        const uint32_t parity = static_cast<uint32_t>((j / STAGES) & 1);
        int ok = 1;
        if (lane == 0 && !mbar_wait_bounded(&bars[s], parity, budget)) {
            ok = 0;
            atomicOr(status, kStatusLoadTimeout);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            aborted = true;
            break;
        }
        __syncwarp();  // lane 0 saw the tile land before any lane stores from it
        const uint32_t cnt = tile_count(j);
        if (static_cast<uint32_t>(lane) < cnt) {
            const int64_t b = (first + j * stride) * a.per + lane;
            const int64_t p = __ldg(a.idx + b);
            if (p < 0 || (a.pool_blocks > 0 && p >= a.pool_blocks))
                atomicOr(status, kStatusBadIndex);
            else
                bulk_store(a.pool + p * a.bs,
                           stage_mem + static_cast<size_t>(s) * STAGE_BYTES + static_cast<size_t>(lane) * bs, bs);
        }
        bulk_commit();
        if (j >= 1) {
            bulk_wait_read<1>();  // this lane's stores of tile j-1 have read their stage
            __syncwarp();
            const int64_t t = j - 1 + STAGES;
            if (t < n) issue(t, static_cast<int>((j - 1) % STAGES));
        }
    }
    if (lane == 0 && aborted) {
        for (int64_t t = j; t < issued; ++t) {
            if (!mbar_wait_bounded(&bars[t % STAGES], static_cast<uint32_t>((t / STAGES) & 1), budget)) {
                atomicOr(status, kStatusDrainTimeout);
                break;
            }
        }
    }
    bulk_wait_all();
    __syncwarp();
}

template <int WARPS, int STAGES, uint32_t STAGE_BYTES>
__global__ void __launch_bounds__(WARPS * 32, 1)
    packed_scatter_kernel(const __grid_constant__ PackedScatter a, uint32_t *status, uint64_t budget,
                          const Epilogue ep) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int warp = threadIdx.x >> 5;
    char *stage_mem = reinterpret_cast<char *>(smem_raw) + static_cast<size_t>(warp) * STAGES * STAGE_BYTES;
    uint64_t *bars =
        reinterpret_cast<uint64_t *>(smem_raw + static_cast<size_t>(WARPS) * STAGES * STAGE_BYTES) + warp * STAGES;
    trace_begin(ep.stamp);
    window_open(ep.win);
    warp_packed_scatter<STAGES, STAGE_BYTES>(a, static_cast<int64_t>(blockIdx.x) * WARPS + warp,
                                             static_cast<int64_t>(gridDim.x) * WARPS, stage_mem, bars, status,
                                             budget);
    trace_end(ep.stamp);
    run_epilogue(ep);
}

template <class Src>
__global__ void __launch_bounds__(kVecWarps * 32)
    vector_mover_kernel(const __grid_constant__ Src src, uint32_t *status, const Epilogue ep) {
    const int lane = threadIdx.x & 31;
    const int64_t total = src.count();
    const int64_t nw = static_cast<int64_t>(gridDim.x) * kVecWarps;
    uint64_t paused = 0;
    trace_begin(ep.stamp);
    window_open(ep.win);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kVecWarps + (threadIdx.x >> 5); t < total;
         t += nw) {
        if (src.gate) {
            if (lane == 0) qos_gate_wait(src.gate, paused, src.gate_budget);
            __syncwarp();
        }
        const Tile tl = src.tile(t);
        if (tl.kind == kBad) {
            if (lane == 0) atomicOr(status, kStatusBadIndex);
            continue;
        }
        warp_copy_any(tl.dst, tl.src, tl.bytes);
    }
    trace_end(ep.stamp);
    run_epilogue(ep);
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
namespace {

template <int WARPS, int STAGES, uint32_t STAGE_BYTES, class Src>
int launch_bulk_cfg(const Src &src, int64_t tiles, int max_ctas, cudaStream_t st, uint32_t *status,
                    const Epilogue &ep, LaunchInfo *info) {
    constexpr size_t smem = static_cast<size_t>(WARPS) * STAGES * STAGE_BYTES +
                            static_cast<size_t>(WARPS) * STAGES * sizeof(uint64_t);
    int dev = 0;
    cudaGetDevice(&dev);
    static std::mutex mu;
    static uint64_t configured = 0;  // bit per device
    {
        std::lock_guard<std::mutex> g(mu);
        if (dev < 64 && !(configured & (1ull << dev))) {
            cudaError_t e = cudaFuncSetAttribute(bulk_mover_kernel<WARPS, STAGES, STAGE_BYTES, Src>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            configured |= 1ull << dev;
        }
    }
    const int sms = sm_count(dev);
    int cap = max_ctas > 0 ? max_ctas : sms;
    int64_t need = (tiles + WARPS - 1) / WARPS;
    int ctas = static_cast<int>(need < cap ? need : cap);
    if (ctas < 1) ctas = 1;
    if (!status) status = default_status_word(dev);
    bulk_mover_kernel<WARPS, STAGES, STAGE_BYTES, Src><<<ctas, WARPS * 32, smem, st>>>(src, status,
                                                                                       wait_budget_ns(), ep);
    note_launch();
    if (info) *info = LaunchInfo{ctas, WARPS * 32, smem, 1};
    return cudaGetLastError();
}

template <class Src>
int launch_bulk(const Src &src, int64_t tiles, int max_ctas, cudaStream_t st, uint32_t *status,
                const Epilogue &ep, LaunchInfo *info) {
    return launch_bulk_cfg<kWarps, kStages, kStageBytes>(src, tiles, max_ctas, st, status, ep, info);
}

// Stage size of the fabric batch copies (MPCOMM_BULK_STAGE_KB = 16, 32 or
// 64; the shared memory per CTA stays ~192 KiB: 4, 2 or 1 pipelines).
uint32_t batch_stage_bytes() {
    static const uint32_t v = [] {
        const char *e = std::getenv("MPCOMM_BULK_STAGE_KB");
        const long kb = e ? std::atol(e) : 16;
        return static_cast<uint32_t>(kb == 32 || kb == 64 ? kb << 10 : kStageBytes);
    }();
    return v;
}

template <class Src>
int launch_vector(const Src &src, int64_t tiles, int max_ctas, cudaStream_t st, uint32_t *status,
                  const Epilogue &ep, LaunchInfo *info) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = sm_count(dev);
    int cap = (max_ctas > 0 ? max_ctas : sms) * 4;
    int64_t need = (tiles + kVecWarps - 1) / kVecWarps;
    int ctas = static_cast<int>(need < cap ? need : cap);
    if (ctas < 1) ctas = 1;
    if (!status) status = default_status_word(dev);
    vector_mover_kernel<Src><<<ctas, kVecWarps * 32, 0, st>>>(src, status, ep);
    note_launch();
    if (info) *info = LaunchInfo{ctas, kVecWarps * 32, 0, 2};
    return cudaGetLastError();
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Largest block the packed gather kernel takes (a stage holds >= 4 blocks).
constexpr int64_t kPackedMaxBlock = kStageBytes / 4;

int launch_packed_scatter(const PackedScatter &a, int max_ctas, cudaStream_t st, uint32_t *status,
                          const Epilogue &ep, LaunchInfo *info) {
    int dev = 0;
    cudaGetDevice(&dev);
    static std::mutex mu;
    static uint64_t configured = 0;
    {
        std::lock_guard<std::mutex> g(mu);
        if (dev < 64 && !(configured & (1ull << dev))) {
            cudaError_t e = cudaFuncSetAttribute(packed_scatter_kernel<kWarps, kStages, kStageBytes>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(kBulkSmem));
            if (e != cudaSuccess) return e;
            configured |= 1ull << dev;
        }
    }
    const int64_t tiles = (a.n + a.per - 1) / a.per;
    const int cap = max_ctas > 0 ? max_ctas : sm_count(dev);
    const int64_t need = (tiles + kWarps - 1) / kWarps;
    int ctas = static_cast<int>(need < cap ? need : cap);
    if (ctas < 1) ctas = 1;
    if (!status) status = default_status_word(dev);
    packed_scatter_kernel<kWarps, kStages, kStageBytes><<<ctas, kWarps * 32, kBulkSmem, st>>>(a, status,
                                                                                            wait_budget_ns(), ep);
    note_launch();
    if (info) *info = LaunchInfo{ctas, kWarps * 32, kBulkSmem, 4};
    return cudaGetLastError();
}

int launch_packed_gather(const PackedGather &a, int max_ctas, cudaStream_t st, uint32_t *status,
                         const Epilogue &ep, LaunchInfo *info) {
    int dev = 0;
    cudaGetDevice(&dev);
    static std::mutex mu;
    static uint64_t configured = 0;
    {
        std::lock_guard<std::mutex> g(mu);
        if (dev < 64 && !(configured & (1ull << dev))) {
            cudaError_t e = cudaFuncSetAttribute(packed_gather_kernel<kWarps, kStages, kStageBytes>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(kBulkSmem));
            if (e != cudaSuccess) return e;
            configured |= 1ull << dev;
        }
    }
    const int64_t tiles = (a.n + a.per - 1) / a.per;
    const int cap = max_ctas > 0 ? max_ctas : sm_count(dev);
    const int64_t need = (tiles + kWarps - 1) / kWarps;
    int ctas = static_cast<int>(need < cap ? need : cap);
    if (ctas < 1) ctas = 1;
    if (!status) status = default_status_word(dev);
    packed_gather_kernel<kWarps, kStages, kStageBytes><<<ctas, kWarps * 32, kBulkSmem, st>>>(a, status,
                                                                                           wait_budget_ns(), ep);
    note_launch();
    if (info) *info = LaunchInfo{ctas, kWarps * 32, kBulkSmem, 3};
    return cudaGetLastError();
}

// AUTO: the bulk pipeline needs 16-byte aligned spans; tiny blocks are
// better served one warp per block.
int pick_path(int mode, const void *a, const void *b, int64_t bs) {
    const bool ok = aligned16(a) && aligned16(b) && (bs % 16) == 0;
    if (mode == kModeTma) return ok ? 1 : -1;
    if (mode == kModeSm) return 2;
    return (ok && bs >= 1024) ? 1 : 2;
}

}  // namespace

int h2d_gather(const void *pool, int64_t pool_blocks, const int64_t *idx, void *out, int64_t n,
               int64_t bs, int mode, int max_ctas, void *stream, uint32_t *status,
               H2DWindow *window, uint32_t *window_ctr, LaunchInfo *info) {
    if (!pool || !idx || !out || n <= 0 || bs <= 0) return cudaErrorInvalidValue;
    if (window && !window_ctr) return cudaErrorInvalidValue;
    const int path = pick_path(mode, pool, out, bs);
    if (path < 0) return cudaErrorMisalignedAddress;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Packed kernel: small blocks on the bulk path (TMA mode up to 4 KiB;
    // AUTO from 1 KiB, below which the vector kernel measures faster).
    const bool packed = path == 1 && bs <= kPackedMaxBlock && (mode == kModeTma || bs >= 1024);
    if (packed) {
        PackedGather a;
        a.pool = static_cast<const char *>(pool);
        a.idx = idx;
        a.out = static_cast<char *>(out);
        a.n = n;
        a.bs = bs;
        a.pool_blocks = pool_blocks;
        a.per = static_cast<int>(std::min<int64_t>(32, kStageBytes / bs));
        const Epilogue ep{window, window_ctr, nullptr, 0,
                          trace_acquire("h2d_gather", static_cast<uint64_t>(n * bs))};
        return launch_packed_gather(a, max_ctas, st, status, ep, info);
    }
    GatherSrc src;
    src.pool = static_cast<const char *>(pool);
    src.idx = idx;
    src.out = static_cast<char *>(out);
    src.n = n;
    src.bs = bs;
    src.pool_blocks = pool_blocks;
    src.tile_bytes = path == 1 ? kStageBytes : kVecTileBytes;
    src.tpb = (bs + src.tile_bytes - 1) / src.tile_bytes;
    const Epilogue ep{window, window_ctr, nullptr, 0, trace_acquire("h2d_gather", static_cast<uint64_t>(n * bs))};
    return path == 1 ? launch_bulk(src, src.n * src.tpb, max_ctas, st, status, ep, info)
                     : launch_vector(src, src.n * src.tpb, max_ctas, st, status, ep, info);
}

int h2d_scatter(const void *srcp, const int64_t *idx, void *pool, int64_t pool_blocks, int64_t n,
                int64_t bs, int mode, int max_ctas, void *stream, uint32_t *status,
                H2DWindow *window, uint32_t *window_ctr, LaunchInfo *info) {
    if (!pool || !idx || !srcp || n <= 0 || bs <= 0) return cudaErrorInvalidValue;
    if (window && !window_ctr) return cudaErrorInvalidValue;
    const int path = pick_path(mode, pool, srcp, bs);
    if (path < 0) return cudaErrorMisalignedAddress;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Packed kernel for small blocks on the bulk path, as for the gather.
    if (path == 1 && bs <= kPackedMaxBlock && (mode == kModeTma || bs >= 1024)) {
        PackedScatter a;
        a.src = static_cast<const char *>(srcp);
        a.idx = idx;
        a.pool = static_cast<char *>(pool);
        a.n = n;
        a.bs = bs;
        a.pool_blocks = pool_blocks;
        a.per = static_cast<int>(std::min<int64_t>(32, kStageBytes / bs));
        const Epilogue ep{window, window_ctr, nullptr, 0,
                          trace_acquire("h2d_scatter", static_cast<uint64_t>(n * bs))};
        return launch_packed_scatter(a, max_ctas, st, status, ep, info);
    }
    ScatterSrc src;
    src.src = static_cast<const char *>(srcp);
    src.idx = idx;
    src.pool = static_cast<char *>(pool);
    src.n = n;
    src.bs = bs;
    src.pool_blocks = pool_blocks;
    src.tile_bytes = path == 1 ? kStageBytes : kVecTileBytes;
    src.tpb = (bs + src.tile_bytes - 1) / src.tile_bytes;
    const Epilogue ep{window, window_ctr, nullptr, 0, trace_acquire("h2d_scatter", static_cast<uint64_t>(n * bs))};
    return path == 1 ? launch_bulk(src, src.n * src.tpb, max_ctas, st, status, ep, info)
                     : launch_vector(src, src.n * src.tpb, max_ctas, st, status, ep, info);
}

int copy_batch(const CopyDesc *descs, int n, int max_ctas, void *stream, uint32_t *status,
               LaunchInfo *info, int mode, const uint32_t *gate, uint64_t gate_budget_ns, uint64_t *done_flag,
               uint64_t done_value, uint32_t *done_ctr) {
    if (n <= 0 || n > kMaxCopyDescs || !descs) return cudaErrorInvalidValue;
    if (done_flag && !done_ctr) return cudaErrorInvalidValue;
    const bool vec = mode == kModeSm;
    BatchSrc src;
    const uint32_t stage = batch_stage_bytes();
    src.tile_bytes = vec ? kVecTileBytes : stage;
    src.gate = gate_budget_ns ? gate : nullptr;
    src.gate_budget = gate_budget_ns;
    int k = 0;
    int64_t tiles = 0;
    for (int i = 0; i < n; ++i) {
        if (descs[i].bytes == 0) continue;
        src.d[k] = descs[i];
        src.start[k] = tiles;
        tiles += static_cast<int64_t>((descs[i].bytes + src.tile_bytes - 1) / src.tile_bytes);
        ++k;
    }
    if (k == 0) {
        // Nothing to copy: still publish completion, in stream order.
        if (!done_flag) return cudaSuccess;
        src.d[0] = CopyDesc{descs[0].src, descs[0].dst, 0};
        src.start[0] = 0;
        k = 0;
    }
    src.start[k] = tiles;
    src.n = k;
    uint64_t total = 0;
    for (int i = 0; i < n; ++i) total += descs[i].bytes;
    const Epilogue ep{nullptr, done_ctr, done_flag, done_value, trace_acquire("copy_batch", total)};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (vec) return launch_vector(src, tiles, max_ctas, st, status, ep, info);
    if (stage == 32768) return launch_bulk_cfg<2, kStages, 32768>(src, tiles, max_ctas, st, status, ep, info);
    if (stage == 65536) return launch_bulk_cfg<1, kStages, 65536>(src, tiles, max_ctas, st, status, ep, info);
    return launch_bulk(src, tiles, max_ctas, st, status, ep, info);
}

int pxn_gather_forward(const void *pool, int64_t pool_blocks, const int64_t *idx, void *dst,
                       int64_t n, int64_t bs, int max_ctas, void *stream, uint32_t *status,
                       uint64_t *done_flag, uint64_t flag_value, uint32_t *ctr, LaunchInfo *info,
                       H2DWindow *window) {
    if (!pool || !idx || !dst || n <= 0 || bs <= 0) return cudaErrorInvalidValue;
    if ((done_flag || window) && !ctr) return cudaErrorInvalidValue;
    const int path = pick_path(kModeAuto, pool, dst, bs);
    GatherSrc src;
    src.pool = static_cast<const char *>(pool);
    src.idx = idx;
    src.out = static_cast<char *>(dst);
    src.n = n;
    src.bs = bs;
    src.pool_blocks = pool_blocks;
    src.tile_bytes = path == 1 ? kStageBytes : kVecTileBytes;
    src.tpb = (bs + src.tile_bytes - 1) / src.tile_bytes;
    const Epilogue ep{window, ctr, done_flag, flag_value,
                      trace_acquire("pxn_gather_forward", static_cast<uint64_t>(n * bs))};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return path == 1 ? launch_bulk(src, src.n * src.tpb, max_ctas, st, status, ep, info)
                     : launch_vector(src, src.n * src.tpb, max_ctas, st, status, ep, info);
}

}  // namespace kern
}  // namespace mpcomm
