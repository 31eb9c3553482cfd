// Fused H2D gather + one-to-many delivery (rollout-batch broadcast).
//
// One launch on the GPU that owns the host pages: every warp runs a bulk
// pipeline that pulls 16 KiB tiles of the requested pages from mapped host
// DRAM into shared memory (cp.async.bulk, mbarrier complete_tx, no
// multicast qualifier on any load) and delivers each landed tile to every
// consumer GPU straight from shared memory:
//
//  * NVLS sink: all 32 lanes read the tile out of shared memory and issue
//    16-byte `multimem.st` to the multicast address; NVSwitch replicates
//    each store to every GPU bound to the multicast object, so the tile
//    crosses this GPU's NVLinks once however many consumers there are.
//  * P2P sink (no multicast): lane 0 issues one bulk store per destination
//    (up to 8 IPC-mapped peer buffers, the local one included) from the same
//    shared-memory stage.
//
// No byte of the batch is staged in this GPU's HBM first, so the PCIe read
// and the NVLink fan-out overlap tile by tile and the launch costs the
// slower of the two instead of their sum. This replaces the reference's
// tma_gather into local HBM followed by cuMemcpyPeerAsync per consumer
// (src/mpcomm_tma_kernels.cu:144-192, src/mpcomm_pxn.cpp:722-725).
//
// Completion: the last CTA to finish (self-resetting counter) either adds 1
// to a flag inside the multicast object (`multimem.red.release.sys`, so
// every consumer's own copy of the flag increments after its data) or
// stores `flag_value` (release, system scope) to each consumer's flag.
// Consumers wait on their local flag with the bounded wait_flag kernel.
#include <cuda_runtime.h>

#include <mutex>

#include "kernels/common.cuh"

namespace mpcomm {
namespace kern {

namespace {

constexpr int kGbWarps = 4;
constexpr int kGbStages = 3;
constexpr uint32_t kGbStageBytes = 16384;
constexpr size_t kGbSmem = static_cast<size_t>(kGbWarps) * kGbStages * kGbStageBytes +
                           static_cast<size_t>(kGbWarps) * kGbStages * sizeof(uint64_t);
constexpr int kGbMaxDst = kMaxFanoutDsts;

struct GatherBcastArgs {
    const char *pool;
    const int64_t *idx;
    int64_t n, bs, pool_blocks, tpb;
    char *mc;                  // NVLS sink (multicast address), or null
    char *dst[kGbMaxDst];      // P2P sink bases (used when mc is null)
    int ndst;
    uint64_t *mc_flag;         // multicast address of the completion flag (NVLS)
    uint64_t *flag[kGbMaxDst]; // per-consumer flags (P2P)
    int nflag;
    uint64_t flag_value;
    uint32_t *ctr;             // last-CTA counter (zero, self-resetting)
    KernelStamp *stamp;
    H2DWindow *win;            // H2D QoS window of a host-memory source (may be null)
};

// Lane-held description of one tile: source address, byte offset of the tile
// in the delivered batch, length and kind (bulk / bad index / nothing).
struct GbTile {
    const char *src;
    int64_t off;
    uint32_t bytes;
    uint32_t kind;
};

__device__ __forceinline__ GbTile gb_tile(const GatherBcastArgs &a, int64_t t) {
    const int64_t b = t / a.tpb;
    const int64_t off = (t - b * a.tpb) * static_cast<int64_t>(kGbStageBytes);
    const int64_t rem = a.bs - off;
    const uint32_t len = static_cast<uint32_t>(rem < kGbStageBytes ? rem : kGbStageBytes);
    const int64_t p = a.idx ? __ldg(a.idx + b) : b;  // no index list: page i is pool page i
    if (p < 0 || (a.pool_blocks > 0 && p >= a.pool_blocks)) return GbTile{nullptr, 0, len, kBad};
    return GbTile{a.pool + p * a.bs + off, b * a.bs + off, len, kBulk};
}

__device__ __forceinline__ int4 ld_shared_v4(const void *p) {
    int4 v;
    asm volatile("ld.shared.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

__device__ __forceinline__ void multimem_st_v4(void *mc, int4 v) {
    asm volatile("multimem.st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void multimem_red_release_add_u64(uint64_t *mc, uint64_t v) {
    asm volatile("multimem.red.release.sys.global.add.u64 [%0], %1;" ::"l"(mc), "l"(v) : "memory");
}

// Warp-cooperative NVLS delivery of one landed stage: 16 bytes per lane per
// store, 4 stores in flight per lane (a warp covers 2 KiB per round).
__device__ __forceinline__ void mc_deliver(char *mc_dst, const char *stage, uint32_t bytes) {
    const int lane = threadIdx.x & 31;
    const uint32_t n16 = bytes >> 4;
    uint32_t i = lane;
    for (; i + 96 < n16; i += 128) {
        const int4 a = ld_shared_v4(stage + (static_cast<size_t>(i) << 4));
        const int4 b = ld_shared_v4(stage + (static_cast<size_t>(i + 32) << 4));
        const int4 c = ld_shared_v4(stage + (static_cast<size_t>(i + 64) << 4));
        const int4 d = ld_shared_v4(stage + (static_cast<size_t>(i + 96) << 4));
        multimem_st_v4(mc_dst + (static_cast<size_t>(i) << 4), a);
        multimem_st_v4(mc_dst + (static_cast<size_t>(i + 32) << 4), b);
        multimem_st_v4(mc_dst + (static_cast<size_t>(i + 64) << 4), c);
        multimem_st_v4(mc_dst + (static_cast<size_t>(i + 96) << 4), d);
    }
    for (; i < n16; i += 32)
        multimem_st_v4(mc_dst + (static_cast<size_t>(i) << 4), ld_shared_v4(stage + (static_cast<size_t>(i) << 4)));
}

template <bool kMc>
__device__ __forceinline__ void warp_gather_bcast(const GatherBcastArgs &a, int64_t first, int64_t stride,
                                                  char *stage_mem, uint64_t *bars, uint32_t *status,
                                                  uint64_t budget) {
    constexpr int S = kGbStages;
    const int lane = threadIdx.x & 31;
    const int64_t total = a.n * a.tpb;
    if (first >= total) return;
    const int64_t n = (total - 1 - first) / stride + 1;

    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_proxy_async_smem();
    }
    __syncwarp();

    GbTile mine{nullptr, 0, 0, kSkip};
    int64_t win = -1;
    int64_t st_off[S];
    uint32_t st_bytes[S];
    uint32_t st_kind[S];
    int64_t issued = 0;

    auto issue = [&](int64_t t, int s) {  // warp-collective
        const int64_t w = t >> 5;
        if (w != win) {
            win = w;
            const int64_t tt = (w << 5) + lane;
            mine = tt < n ? gb_tile(a, first + tt * stride) : GbTile{nullptr, 0, 0, kSkip};
        }
        const int sl = static_cast<int>(t & 31);
        const char *ts = reinterpret_cast<const char *>(
            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(mine.src), sl));
        const int64_t to = static_cast<int64_t>(__shfl_sync(0xffffffffu, static_cast<long long>(mine.off), sl));
        const uint32_t tb = __shfl_sync(0xffffffffu, mine.bytes, sl);
        const uint32_t tk = __shfl_sync(0xffffffffu, mine.kind, sl);
        if (lane == 0) {
            st_off[s] = to;
            st_bytes[s] = tb;
            st_kind[s] = tk;
            const bool bulk = tk == kBulk;
            mbar_arrive_expect_tx(&bars[s], bulk ? tb : 0u);
            if (bulk) bulk_load(stage_mem + static_cast<size_t>(s) * kGbStageBytes, ts, tb, &bars[s]);
        }
        ++issued;
    };

    const int64_t pro = n < S ? n : S;
    for (int64_t t = 0; t < pro; ++t) issue(t, static_cast<int>(t));

    int64_t j = 0;
    bool aborted = false;
    for (; j < n; ++j) {
        const int s = static_cast<int>(j % S);
        const uint32_t parity = static_cast<uint32_t>((j / S) & 1);
        const char *stage = stage_mem + static_cast<size_t>(s) * kGbStageBytes;
        int ok = 1;
        uint32_t kind = kSkip;
        int64_t off = 0;
        uint32_t bytes = 0;
        if (lane == 0) {
            if (!mbar_wait_bounded(&bars[s], parity, budget)) {
                ok = 0;
                atomicOr(status, kStatusLoadTimeout);
            } else {
                kind = st_kind[s];
                off = st_off[s];
                bytes = st_bytes[s];
                if (kind == kBad) atomicOr(status, kStatusBadIndex);
                if (!kMc) {
                    if (kind == kBulk)
                        for (int k = 0; k < a.ndst; ++k) bulk_store(a.dst[k] + off, stage, bytes);
                    bulk_commit();
                }
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            aborted = true;
            break;
        }
        if (kMc) {
            // Lane 0 observed the stage's mbarrier phase; __syncwarp orders
            // that observation before the other lanes' shared-memory reads.
            __syncwarp();
            kind = __shfl_sync(0xffffffffu, kind, 0);
            if (kind == kBulk) {
                off = static_cast<int64_t>(__shfl_sync(0xffffffffu, static_cast<long long>(off), 0));
                bytes = __shfl_sync(0xffffffffu, bytes, 0);
                mc_deliver(a.mc + off, stage, bytes);
            }
            __syncwarp();  // every lane has read the stage: it may be refilled
            const int64_t t = j + S;
            if (t < n) issue(t, s);
        } else if (j >= 1) {
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
            const int64_t t = j - 1 + S;
            if (t < n) issue(t, static_cast<int>((j - 1) % S));
        }
    }
    if (lane == 0) {
        if (aborted) {
            for (int64_t t = j; t < issued; ++t) {
                if (!mbar_wait_bounded(&bars[t % S], static_cast<uint32_t>((t / S) & 1), budget)) {
                    atomicOr(status, kStatusDrainTimeout);
                    break;
                }
            }
        }
        if (!kMc) bulk_wait_all();
    }
    __syncwarp();
}

template <bool kMc>
__global__ void __launch_bounds__(kGbWarps * 32, 1)
    gather_bcast_kernel(const __grid_constant__ GatherBcastArgs a, uint32_t *status, uint64_t budget) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int warp = threadIdx.x >> 5;
    char *stage_mem = reinterpret_cast<char *>(smem_raw) + static_cast<size_t>(warp) * kGbStages * kGbStageBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw + static_cast<size_t>(kGbWarps) * kGbStages * kGbStageBytes) +
                     warp * kGbStages;
    trace_begin(a.stamp);
    window_open(a.win);
    warp_gather_bcast<kMc>(a, static_cast<int64_t>(blockIdx.x) * kGbWarps + warp,
                           static_cast<int64_t>(gridDim.x) * kGbWarps, stage_mem, bars, status, budget);
    // Every lane's multimem stores (or lane 0's completed bulk stores) are
    // ordered before the CTA's arrival on the completion counter.
    __threadfence_system();
    trace_end(a.stamp);
    if (!a.ctr) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t prev = atomicAdd(a.ctr, 1u);
        if (prev == gridDim.x - 1) {
            *a.ctr = 0u;
            __threadfence_system();
            if (kMc && a.mc_flag) multimem_red_release_add_u64(a.mc_flag, 1ull);
            for (int k = 0; k < a.nflag; ++k) st_release_sys_u64(a.flag[k], a.flag_value);
            if (a.win) {
                uint32_t *gate = *reinterpret_cast<uint32_t *volatile *>(&a.win->gate);
                if (gate) atomicSub(gate, 1u);
                st_release_sys_u64(&a.win->end_ns, globaltimer_ns() | 1ull);
            }
        }
    }
}

template <bool kMc>
cudaError_t configure(int dev) {
    static std::mutex mu;
    static uint64_t done = 0;
    std::lock_guard<std::mutex> g(mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (done & (1ull << dev)) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(gather_bcast_kernel<kMc>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kGbSmem));
    if (e == cudaSuccess) done |= 1ull << dev;
    return e;
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int gather_bcast(const void *pool, int64_t pool_blocks, const int64_t *idx, int64_t n, int64_t bs, void *mc_dst,
                 void *const *dsts, int ndst, uint64_t *mc_flag, uint64_t *const *flags, int nflag,
                 uint64_t flag_value, uint32_t *ctr, int max_ctas, void *stream, uint32_t *status,
                 LaunchInfo *info, H2DWindow *window) {
    if (!pool || n <= 0 || bs <= 0) return cudaErrorInvalidValue;
    if (window && !ctr) return cudaErrorInvalidValue;
    if (!al16(pool) || (bs & 15)) return cudaErrorMisalignedAddress;  // bulk copies need 16-byte spans
    const bool mc = mc_dst != nullptr;
    if (mc) {
        if (!al16(mc_dst)) return cudaErrorMisalignedAddress;
        if (mc_flag && ((reinterpret_cast<uintptr_t>(mc_flag) & 7u) || !ctr)) return cudaErrorInvalidValue;
    } else {
        if (!dsts || ndst <= 0 || ndst > kGbMaxDst) return cudaErrorInvalidValue;
        for (int k = 0; k < ndst; ++k)
            if (!dsts[k] || !al16(dsts[k])) return cudaErrorMisalignedAddress;
    }
    if (nflag < 0 || nflag > kGbMaxDst || (nflag > 0 && (!flags || !ctr))) return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = mc ? configure<true>(dev) : configure<false>(dev);
    if (e != cudaSuccess) return e;

    GatherBcastArgs a{};
    a.pool = static_cast<const char *>(pool);
    a.idx = idx;
    a.n = n;
    a.bs = bs;
    a.pool_blocks = pool_blocks;
    a.tpb = (bs + kGbStageBytes - 1) / kGbStageBytes;
    a.mc = static_cast<char *>(mc_dst);
    a.ndst = mc ? 0 : ndst;
    for (int k = 0; k < a.ndst; ++k) a.dst[k] = static_cast<char *>(dsts[k]);
    a.mc_flag = mc ? mc_flag : nullptr;
    a.nflag = nflag;
    for (int k = 0; k < a.nflag; ++k) a.flag[k] = flags[k];
    a.flag_value = flag_value;
    a.ctr = ((mc && mc_flag) || nflag > 0 || window) ? ctr : nullptr;
    a.win = window;
    const uint64_t bytes = static_cast<uint64_t>(n) * static_cast<uint64_t>(bs);
    a.stamp = trace_acquire(mc ? "gather_bcast_nvls" : "gather_bcast_p2p", bytes);

    const int64_t tiles = n * a.tpb;
    const int cap = max_ctas > 0 ? max_ctas : sm_count(dev);
    const int64_t need = (tiles + kGbWarps - 1) / kGbWarps;
    int ctas = static_cast<int>(need < cap ? need : cap);
    if (ctas < 1) ctas = 1;
    if (!status) status = default_status_word(dev);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (mc)
        gather_bcast_kernel<true><<<ctas, kGbWarps * 32, kGbSmem, st>>>(a, status, wait_budget_ns());
    else
        gather_bcast_kernel<false><<<ctas, kGbWarps * 32, kGbSmem, st>>>(a, status, wait_budget_ns());
    note_launch();
    if (info) *info = LaunchInfo{ctas, kGbWarps * 32, kGbSmem, mc ? 5 : 6};
    return cudaGetLastError();
}

}  // namespace kern
}  // namespace mpcomm
