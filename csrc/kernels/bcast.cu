// One-to-many kernels for the NVSwitch fabric.
//
//  * nvls_broadcast: 16-byte loads from local HBM, `multimem.st` to a
//    multicast address (cuMulticastCreate/BindMem object mapped on every
//    GPU); NVSwitch replicates each store to all bound GPUs, so the source
//    GPU pushes the bytes once over its NVLinks.
//  * p2p_fanout: fallback when multicast is unavailable: the same bytes
//    stored to each peer's IPC-mapped buffer (N x the NVLink egress).
//  * wait_flag: one thread polls a 64-bit flag (peer- or host-written) with
//    acquire semantics under a %globaltimer budget.
#include <cuda_runtime.h>

#include <atomic>

#include "kernels/common.cuh"

namespace mpcomm {
namespace kern {

namespace {

constexpr int kBcastThreads = 512;

// Store flavour / depth of nvls_broadcast (tuning): 0 relaxed.sys x4 loads in
// flight per thread, 1 weak x4, 2 weak x8, 3 relaxed.sys x8.
std::atomic<int> g_nvls_variant{0};

// multimem.st of 16 bytes: relaxed at system scope, or weak (ordered for
// other GPUs by the kernel boundary and whatever synchronisation follows).
template <bool kWeak>
__device__ __forceinline__ void multimem_st_v4(void *mc, int4 v) {
    if (kWeak)
        asm volatile("multimem.st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y), "r"(v.z),
                     "r"(v.w)
                     : "memory");
    else
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y),
                     "r"(v.z), "r"(v.w)
                     : "memory");
}

// Grid-stride broadcast: each thread keeps ILP 16-byte loads in flight, then
// issues their multimem stores (a warp covers 512 contiguous bytes per step).
template <bool kWeak, int ILP>
__global__ void __launch_bounds__(kBcastThreads)
    nvls_broadcast_kernel(const int4 *__restrict__ src, int4 *mc, uint64_t n16, KernelStamp *stamp) {
    trace_begin(stamp);
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + (ILP - 1) * stride < n16; i += ILP * stride) {
        int4 v[ILP];
#pragma unroll
        for (int k = 0; k < ILP; ++k) v[k] = ld_v4(src + i + k * stride);
#pragma unroll
        for (int k = 0; k < ILP; ++k) multimem_st_v4<kWeak>(mc + i + k * stride, v[k]);
    }
    for (; i < n16; i += stride) multimem_st_v4<kWeak>(mc + i, ld_v4(src + i));
    trace_end(stamp);
}

struct FanoutDsts {
    int4 *p[8];
    int n;
};

__global__ void __launch_bounds__(kBcastThreads)
    p2p_fanout_kernel(const int4 *__restrict__ src, const __grid_constant__ FanoutDsts dst,
                      uint64_t n16, KernelStamp *stamp) {
    trace_begin(stamp);
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16;
         i += stride) {
        const int4 v = ld_v4(src + i);
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (k < dst.n) st_v4(dst.p[k] + i, v);
    }
    trace_end(stamp);
}

__global__ void wait_flag_kernel(const uint64_t *flag, uint64_t value, uint64_t budget,
                                 uint32_t *status) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        uint64_t v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
        if (v >= value) return;
        if (globaltimer_ns() - t0 > budget) {
            atomicOr(status, kStatusFlagTimeout);
            return;
        }
        __nanosleep(256);
    }
}

int grid_for(uint64_t n16, int max_ctas) {
    int dev = 0;
    cudaGetDevice(&dev);
    int cap = max_ctas > 0 ? max_ctas : sm_count(dev) * 2;
    uint64_t need = (n16 + kBcastThreads - 1) / kBcastThreads;
    int g = static_cast<int>(need < static_cast<uint64_t>(cap) ? need : cap);
    return g < 1 ? 1 : g;
}

}  // namespace

void set_nvls_variant(int v) { g_nvls_variant.store(v < 0 || v > 3 ? 0 : v, std::memory_order_relaxed); }

int nvls_broadcast(const void *src, void *mc_dst, uint64_t bytes, int max_ctas, void *stream,
                   LaunchInfo *info) {
    if (!src || !mc_dst || bytes == 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(mc_dst)) & 15u)
        return cudaErrorMisalignedAddress;
    if (bytes & 15u) return cudaErrorInvalidValue;  // callers pad to 16 bytes
    const uint64_t n16 = bytes >> 4;
    const int g = grid_for(n16, max_ctas);
    KernelStamp *st = trace_acquire("nvls_broadcast", bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto *sp = static_cast<const int4 *>(src);
    auto *dp = static_cast<int4 *>(mc_dst);
    switch (g_nvls_variant.load(std::memory_order_relaxed)) {
        case 1: nvls_broadcast_kernel<true, 4><<<g, kBcastThreads, 0, s>>>(sp, dp, n16, st); break;
        case 2: nvls_broadcast_kernel<true, 8><<<g, kBcastThreads, 0, s>>>(sp, dp, n16, st); break;
        case 3: nvls_broadcast_kernel<false, 8><<<g, kBcastThreads, 0, s>>>(sp, dp, n16, st); break;
        default: nvls_broadcast_kernel<false, 4><<<g, kBcastThreads, 0, s>>>(sp, dp, n16, st); break;
    }
    note_launch();
    if (info) *info = LaunchInfo{g, kBcastThreads, 0, 3};
    return cudaGetLastError();
}

int p2p_fanout(const void *src, void *const *dsts, int ndst, uint64_t bytes, int max_ctas,
               void *stream, LaunchInfo *info) {
    if (!src || !dsts || ndst <= 0 || ndst > 8 || bytes == 0 || (bytes & 15u))
        return cudaErrorInvalidValue;
    FanoutDsts d{};
    d.n = ndst;
    for (int i = 0; i < ndst; ++i) {
        if (reinterpret_cast<uintptr_t>(dsts[i]) & 15u) return cudaErrorMisalignedAddress;
        d.p[i] = static_cast<int4 *>(dsts[i]);
    }
    const uint64_t n16 = bytes >> 4;
    const int g = grid_for(n16, max_ctas);
    p2p_fanout_kernel<<<g, kBcastThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const int4 *>(src), d, n16, trace_acquire("p2p_fanout", bytes * static_cast<uint64_t>(ndst)));
    note_launch();
    if (info) *info = LaunchInfo{g, kBcastThreads, 0, 4};
    return cudaGetLastError();
}

int wait_flag(const uint64_t *flag, uint64_t value, uint64_t budget_ns, void *stream,
              uint32_t *status) {
    if (!flag) return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!status) status = default_status_word(dev);
    wait_flag_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag, value, budget_ns, status);
    note_launch();
    return cudaGetLastError();
}

}  // namespace kern
}  // namespace mpcomm
