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

#include "kernels/common.cuh"

namespace mpcomm {
namespace kern {

namespace {

constexpr int kBcastThreads = 512;

__device__ __forceinline__ void multimem_st_v4(void *mc, int4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__global__ void __launch_bounds__(kBcastThreads)
    nvls_broadcast_kernel(const int4 *__restrict__ src, int4 *mc, uint64_t n16) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n16; i += 4 * stride) {
        const int4 a = ld_v4(src + i), b = ld_v4(src + i + stride), c = ld_v4(src + i + 2 * stride),
                   d = ld_v4(src + i + 3 * stride);
        multimem_st_v4(mc + i, a);
        multimem_st_v4(mc + i + stride, b);
        multimem_st_v4(mc + i + 2 * stride, c);
        multimem_st_v4(mc + i + 3 * stride, d);
    }
    for (; i < n16; i += stride) multimem_st_v4(mc + i, ld_v4(src + i));
}

struct FanoutDsts {
    int4 *p[8];
    int n;
};

__global__ void __launch_bounds__(kBcastThreads)
    p2p_fanout_kernel(const int4 *__restrict__ src, const __grid_constant__ FanoutDsts dst,
                      uint64_t n16) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16;
         i += stride) {
        const int4 v = ld_v4(src + i);
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (k < dst.n) st_v4(dst.p[k] + i, v);
    }
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

int nvls_broadcast(const void *src, void *mc_dst, uint64_t bytes, int max_ctas, void *stream,
                   LaunchInfo *info) {
    if (!src || !mc_dst || bytes == 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(mc_dst)) & 15u)
        return cudaErrorMisalignedAddress;
    if (bytes & 15u) return cudaErrorInvalidValue;  // callers pad to 16 bytes
    const uint64_t n16 = bytes >> 4;
    const int g = grid_for(n16, max_ctas);
    nvls_broadcast_kernel<<<g, kBcastThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const int4 *>(src), static_cast<int4 *>(mc_dst), n16);
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
        static_cast<const int4 *>(src), d, n16);
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
