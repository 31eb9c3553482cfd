// Thin CUDA runtime/driver helpers used by the host library.
//
// The library links the static CUDA runtime and resolves driver entry
// points lazily (cudaGetDriverEntryPoint), so it loads and runs its CPU
// paths on hosts without a GPU driver; every helper reports "no GPU"
// instead of failing to load.
#ifndef MPCOMM_B200_CSRC_CUDA_GPU_H_
#define MPCOMM_B200_CSRC_CUDA_GPU_H_

#include <cstddef>
#include <cstdint>
#include <string>

namespace mpcomm {
namespace gpu {

int device_count();
int current_device();
int set_device(int dev);

struct PtrInfo {
    bool is_device = false;  // device (HBM) memory
    bool is_host_pinned = false;  // page-locked host memory known to CUDA
    int device = -1;
    uintptr_t base = 0;  // allocation base (device memory)
    size_t size = 0;     // allocation size (device memory)
};
// False for plain pageable host memory / no GPU.
bool query_pointer(const void *p, PtrInfo *out);
inline int device_of(const void *p) {
    PtrInfo i;
    return (query_pointer(p, &i) && i.is_device) ? i.device : -1;
}

// "0000:53:00.0" (lowercase) or empty.
std::string pci_bdf(int dev);

// cudaHostRegister(Portable|Mapped) unless already pinned. *registered
// tells whether this call pinned it (and so must unpin it). The device
// pointer equals host_addr on UVA systems.
int host_pin_mapped(void *host_addr, size_t len, void **dev_ptr, bool *registered);
int host_unpin(void *host_addr);
// Pinned + mapped host allocation (for flags, windows, status words).
void *host_alloc_mapped(size_t bytes);
void host_free(void *p);
void *device_alloc(size_t bytes);
void device_free(void *p);
// Synchronous memset / device-to-host copy on a non-blocking stream of the
// current device (never queued behind work on the legacy default stream).
int memset_device(void *p, int v, size_t bytes);
int memset_device_async(void *p, int v, size_t bytes, void *stream);
int copy_d2h_sync(void *dst, const void *src, size_t bytes);
// Copy-engine copy (cudaMemcpyDefault: any UVA addresses, peers included) on
// `stream`; benches use it as the comparator of the data-mover kernels.
int copy_engine_async(void *dst, const void *src, size_t bytes, void *stream);

// CUDA IPC (legacy handles; device memory from cudaMalloc).
constexpr size_t kIpcHandleBytes = 64;
int ipc_get_handle(void *base, unsigned char out[kIpcHandleBytes]);
int ipc_open_handle(const unsigned char h[kIpcHandleBytes], void **ptr);
int ipc_close(void *ptr);
int enable_peer_access(int dev, int peer);

// Streams and events (opaque handles).
void *stream_create(int dev);
// Device ordinal a stream belongs to (-1 on error).
int stream_device(void *s);
void stream_destroy(void *s);
int stream_sync(void *s);
void *event_create(int dev);
void event_destroy(void *e);
int event_record(void *e, void *stream);
// 1 = complete, 0 = pending, <0 = error.
int event_query(void *e);
int event_sync(void *e);
int device_sync();
const char *error_string(int err);
int last_error_clear();

// Driver API entry point by name (nullptr if unavailable).
void *driver_symbol(const char *name);

}  // namespace gpu
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_CUDA_GPU_H_
