// HBM <-> DRAM movers: mapDRAMtoGPU / tmaGather / tmaScatter.
// Parity: reference src/mpcomm.cpp:7774-7938 (mapping + wrappers) and
// src/mpcomm_tma_kernels.cu:301-463 (launchers). Differences: explicit
// stream, launch errors returned, indices bound-checked against the mapped
// pool, SM counts cached per device, no printf, AUTO picks by alignment.
#include <cstring>

#include "core/nvtx.h"
#include "cuda/gpu.h"
#include "engine/impl.h"
#include "mpcomm_log.h"
#include "topo/topology.h"

namespace mpcomm {

uintptr_t MPComm::Impl::mapDRAMtoGPU(void *host, size_t len) {
    if (!host || len == 0) return 0;
    if (gpu::device_count() == 0) {
        MPCOMM_LOG_ERROR("MPComm: mapDRAMtoGPU needs a CUDA device\n");
        return 0;
    }
    void *dptr = nullptr;
    bool pinned = false;
    int e = gpu::host_pin_mapped(host, len, &dptr, &pinned);
    if (e != 0) {
        MPCOMM_LOG_ERROR("MPComm: mapDRAMtoGPU(%p, %zu) failed: %s\n", host, len, gpu::error_string(e));
        return 0;
    }
    std::lock_guard<std::mutex> g(map_mu_);
    auto it = mappings_.find(reinterpret_cast<uintptr_t>(host));
    if (it != mappings_.end()) {
        // Re-mapping the same range keeps the first pin owner.
        pinned = pinned || it->second.pinned_by_us;
    }
    mappings_[reinterpret_cast<uintptr_t>(host)] = Mapping{len, reinterpret_cast<uintptr_t>(dptr), pinned};
    MPCOMM_LOG_DEBUG("MPComm: mapped DRAM %p+%zu (numa %d) -> device %p\n", host, len,
                     topo::numa_node_of_addr(host), dptr);
    return reinterpret_cast<uintptr_t>(dptr);
}

int MPComm::Impl::unmapDRAMfromGPU(void *host) {
    if (!host) return MPCOMM_ERR_INVALID_ARG;
    Mapping m;
    {
        std::lock_guard<std::mutex> g(map_mu_);
        auto it = mappings_.find(reinterpret_cast<uintptr_t>(host));
        if (it == mappings_.end()) return MPCOMM_ERR_INVALID_ARG;
        m = it->second;
        mappings_.erase(it);
    }
    if (m.pinned_by_us && gpu::host_unpin(host) != 0) return MPCOMM_ERR_MEMORY;
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::h2dMove(bool gather, uintptr_t dram, const int64_t *idx, void *gpu_buf, int n,
                          int bs, int max_sm, int mode, void *stream) {
    if (!dram || !idx || !gpu_buf || n <= 0 || bs <= 0) return MPCOMM_ERR_INVALID_ARG;
    if (mode < 0 || mode > 2) return MPCOMM_ERR_INVALID_ARG;
    if (gpu::device_count() == 0) return MPCOMM_ERR_DEVICE;
    // Pool extent (in blocks) when the DRAM pointer lies in a known mapping:
    // enables the device-side index bound check.
    int64_t pool_blocks = 0;
    {
        std::lock_guard<std::mutex> g(map_mu_);
        for (auto &kv : mappings_) {
            const uintptr_t d0 = kv.second.dev_ptr, d1 = d0 + kv.second.len;
            if (dram >= d0 && dram < d1) {
                pool_blocks = static_cast<int64_t>((d1 - dram) / static_cast<uintptr_t>(bs));
                break;
            }
        }
    }
    nvtx::Range range(gather ? "mpcomm::tmaGather" : "mpcomm::tmaScatter");
    kern::H2DWindow *win = nullptr;
    uint32_t *ctr = nullptr;
    const int wgpu = isH2DQoSEnabled() ? gpu::device_of(gpu_buf) : -1;
    if (wgpu >= 0) acquireH2DWindow(wgpu, &win, &ctr);
    // Remote writers into this GPU pause (or pace) before the kernel starts.
    const bool remote = win && cfg_.qos_remote && qosChannelCount() > 0;
    if (remote) broadcastQos(wgpu, qos_bucket_.rate(), qos_bucket_.burst(), false);
    int e;
    if (gather) {
        e = kern::h2d_gather(reinterpret_cast<const void *>(dram), pool_blocks, idx, gpu_buf, n, bs, mode,
                             max_sm, stream, nullptr, win, ctr, nullptr);
    } else {
        e = kern::h2d_scatter(gpu_buf, idx, reinterpret_cast<void *>(dram), pool_blocks, n, bs, mode,
                              max_sm, stream, nullptr, win, ctr, nullptr);
    }
    if (remote) {
        if (e == 0)
            remotePauseForWindow(wgpu, win);  // clear once the window closes
        else
            broadcastQos(wgpu, 0, 0, true);
    }
    if (e != 0) {
        if (win) __atomic_store_n(&win->armed, 0u, __ATOMIC_RELEASE);
        if (e == 716 /* cudaErrorMisalignedAddress */) {
            MPCOMM_LOG_ERROR("MPComm: TMA mode needs 16-byte aligned pool/buffer and block_size\n");
            return MPCOMM_ERR_INVALID_ARG;
        }
        MPCOMM_LOG_ERROR("MPComm: %s launch failed: %s\n", gather ? "tmaGather" : "tmaScatter",
                         gpu::error_string(e));
        return MPCOMM_ERR_DEVICE;
    }
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::setFabricStream(void *stream) {
    for (auto &r : rails_) r->rail->set_stream(stream);
    fabric_stream_ = stream;
    return MPCOMM_SUCCESS;
}

}  // namespace mpcomm
