// Cross-process GPU memory plumbing for one NVSwitch box.
//
//  * CUDA IPC: export/open the allocation that holds a device pointer, so a
//    peer process can store into it from its own kernels (P2P over NVLink).
//  * NVLS multicast: a multicast object bound to one physical allocation per
//    GPU; a kernel's `multimem.st` to the multicast address is replicated by
//    the NVSwitch into every bound allocation. Handles cross processes as
//    POSIX file descriptors (the caller passes them over a Unix socket).
// All driver calls go through cudaGetDriverEntryPoint, so the library still
// loads without a driver. Every function returns 0 or a CUresult.
#ifndef MPCOMM_B200_CSRC_PARALLEL_VMM_H_
#define MPCOMM_B200_CSRC_PARALLEL_VMM_H_

#include <cstddef>
#include <cstdint>
#include <vector>

namespace mpcomm {
namespace vmm {

// IPC handle (64 bytes) of the allocation containing `ptr`; *offset = ptr - base.
int ipc_export(const void *ptr, unsigned char handle[64], uint64_t *offset);
// Maps a peer allocation into this process (peer access enabled lazily).
int ipc_import(const unsigned char handle[64], void **base);
int ipc_release(void *base);

// 1 if `dev` supports multicast objects.
int multicast_supported(int dev);
// Minimum granularity for a multicast object spanning `ndev` devices.
int multicast_granularity(size_t size, int ndev, size_t *gran);
// Creates a multicast object (root only) and exports it as a POSIX fd.
int multicast_create(size_t size, int ndev, uint64_t *mc, int *fd);
// Imports an exported multicast object from its fd.
int multicast_import(int fd, uint64_t *mc);
// Adds `dev` to the object (every participant, before any bind).
int multicast_add_device(uint64_t mc, int dev);
// Allocates `size` bytes on `dev`, binds them to the multicast object at
// offset 0 and maps them at a unicast address (*uc_va, readable by `dev`).
int multicast_bind_local(uint64_t mc, size_t size, int dev, uint64_t *mem, void **uc_va);
// Maps the multicast object itself (*mc_va: target of multimem stores).
int multicast_map(uint64_t mc, size_t size, int dev, void **mc_va);
// Unmaps/unbinds/releases everything created above (any argument may be 0).
int multicast_teardown(uint64_t mc, uint64_t mem, void *uc_va, void *mc_va, size_t size, int dev);

// VMM (cuMemCreate) memory across processes, where CUDA IPC cannot go.
// One allocation of the range a caller registers; a range may be backed by
// several (an allocator that grows a reserved range page by page, e.g.
// PyTorch's expandable segments), mapped back to back.
struct VmmSegment {
    uintptr_t base;
    size_t size;
};
// vmm_segments: the allocations backing [ptr, ptr + len), contiguous and in
// address order, at most `max_segments`. Non-zero for memory that is not
// VMM-mapped or has a hole.
int vmm_segments(const void *ptr, size_t len, size_t max_segments, std::vector<VmmSegment> *out);
// vmm_export_fd: the allocation mapped at `base` as a POSIX file descriptor
// (owned by the caller); fails for allocations created without that handle
// type.
int vmm_export_fd(uintptr_t base, int *fd);
// vmm_offer: offers [ptr, ptr + len) of VMM memory under `key` on this
// process's descriptor server (handles exported afresh per request); 0 with
// the owner's base and span of the allocations behind it, else non-zero.
int vmm_offer(const void *ptr, size_t len, uint64_t key, uintptr_t *base, size_t *span);
void vmm_withdraw(uint64_t key);
// vmm_open: fetches what process `pid` offered under `key` and maps it back
// to back for device `dev`, one allocation at a time as the handles arrive:
// *va stands for the owner's base; *sizes gets the allocation sizes (for
// vmm_unmap). 0, kVmmNotOffered if the key is not (or no longer) offered,
// kVmmUnreachable if the owner did not answer, else the CUresult of the
// failed mapping step.
constexpr int kVmmNotOffered = -3;
constexpr int kVmmUnreachable = -1;
int vmm_open(long pid, uint64_t key, int dev, int timeout_ms, void **va, std::vector<size_t> *sizes);
int vmm_unmap(void *va, const std::vector<size_t> &sizes);

// HBM that a NIC can register through dma-buf (GPUDirect RDMA): a VMM
// allocation of `dev` created with the gpuDirectRDMACapable flag, `size`
// rounded up to the allocation granularity (*alloc_size), mapped read-write
// for `dev`. Registering it with the ib fabric exports it as a dma-buf.
int gdr_alloc(int dev, size_t size, void **ptr, size_t *alloc_size);
int gdr_free(void *ptr, size_t alloc_size);
// Exports [ptr, ptr + size) as a dma-buf file descriptor
// (cuMemGetHandleForAddressRange, DMA_BUF_FD; flags as the driver's).
int dmabuf_export(const void *ptr, size_t size, unsigned long long flags, int *fd);

}  // namespace vmm
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_PARALLEL_VMM_H_
