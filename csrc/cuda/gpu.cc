#include "cuda/gpu.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cctype>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "mpcomm_log.h"

namespace mpcomm {
namespace gpu {

int device_count() {
    static int n = [] {
        int c = 0;
        if (cudaGetDeviceCount(&c) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return c;
    }();
    return n;
}

int current_device() {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return d;
}

int set_device(int dev) { return cudaSetDevice(dev); }

void *driver_symbol(const char *name) {
    static std::mutex mu;
    static std::unordered_map<std::string, void *> cache;
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(name);
    if (it != cache.end()) return it->second;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        fn = nullptr;
    }
    cache[name] = fn;
    return fn;
}

bool query_pointer(const void *p, PtrInfo *out) {
    *out = PtrInfo{};
    if (!p || device_count() == 0) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
        out->is_device = true;
        out->device = a.device;
        using RangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
        auto fn = reinterpret_cast<RangeFn>(driver_symbol("cuMemGetAddressRange"));
        CUdeviceptr base = 0;
        size_t size = 0;
        if (fn && fn(&base, &size, reinterpret_cast<CUdeviceptr>(p)) == CUDA_SUCCESS) {
            out->base = static_cast<uintptr_t>(base);
            out->size = size;
        }
        return true;
    }
    if (a.type == cudaMemoryTypeHost) {
        out->is_host_pinned = true;
        out->device = a.device;
        return true;
    }
    return false;
}

std::string pci_bdf(int dev) {
    char buf[32] = {0};
    if (cudaDeviceGetPCIBusId(buf, sizeof(buf), dev) != cudaSuccess) {
        cudaGetLastError();
        return std::string();
    }
    std::string s(buf);
    for (auto &c : s) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
    // cudaDeviceGetPCIBusId yields "0000:53:00.0" (domain may be 8 digits).
    if (s.size() > 12 && s[8] == ':') s = s.substr(4);
    return s;
}

int host_pin_mapped(void *host_addr, size_t len, void **dev_ptr, bool *registered) {
    *registered = false;
    PtrInfo info;
    if (!query_pointer(host_addr, &info) || !info.is_host_pinned) {
        cudaError_t e = cudaHostRegister(host_addr, len, cudaHostRegisterPortable | cudaHostRegisterMapped);
        if (e == cudaErrorHostMemoryAlreadyRegistered) {
            cudaGetLastError();
        } else if (e != cudaSuccess) {
            cudaGetLastError();
            return e;
        } else {
            *registered = true;
        }
    }
    void *d = nullptr;
    cudaError_t e = cudaHostGetDevicePointer(&d, host_addr, 0);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (*registered) cudaHostUnregister(host_addr);
        *registered = false;
        return e;
    }
    *dev_ptr = d;
    return 0;
}

int host_unpin(void *host_addr) {
    cudaError_t e = cudaHostUnregister(host_addr);
    if (e != cudaSuccess) cudaGetLastError();
    return e;
}

void *host_alloc_mapped(size_t bytes) {
    void *p = nullptr;
    if (cudaHostAlloc(&p, bytes, cudaHostAllocPortable | cudaHostAllocMapped) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    std::memset(p, 0, bytes);
    return p;
}

void host_free(void *p) {
    if (p) cudaFreeHost(p);
}

void *device_alloc(size_t bytes) {
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

void device_free(void *p) {
    if (p) cudaFree(p);
}

namespace {

// A non-blocking helper stream per device. The synchronous helpers below run
// on it instead of the legacy default stream: work queued on the legacy
// stream (for instance a wait on a collective that needs this very process
// to answer a control message first) would otherwise hold them up.
cudaStream_t helper_stream() {
    static std::mutex mu;
    static cudaStream_t streams[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return nullptr;
    }
    std::lock_guard<std::mutex> g(mu);
    if (!streams[dev] && cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        streams[dev] = nullptr;
    }
    return streams[dev];
}

}  // namespace

int memset_device(void *p, int v, size_t bytes) {
    cudaStream_t s = helper_stream();
    if (!s) return cudaMemset(p, v, bytes);
    cudaError_t e = cudaMemsetAsync(p, v, bytes, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e;
}

int memset_device_async(void *p, int v, size_t bytes, void *stream) {
    return cudaMemsetAsync(p, v, bytes, static_cast<cudaStream_t>(stream));
}

int copy_engine_async(void *dst, const void *src, size_t bytes, void *stream) {
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
}

int copy_d2h_sync(void *dst, const void *src, size_t bytes) {
    cudaStream_t s = helper_stream();
    if (!s) return cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost);
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e;
}

int ipc_get_handle(void *base, unsigned char out[kIpcHandleBytes]) {
    static_assert(sizeof(cudaIpcMemHandle_t) == kIpcHandleBytes, "IPC handle size");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, base);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return e;
    }
    std::memcpy(out, &h, kIpcHandleBytes);
    return 0;
}

int ipc_open_handle(const unsigned char h[kIpcHandleBytes], void **ptr) {
    cudaIpcMemHandle_t hh;
    std::memcpy(&hh, h, kIpcHandleBytes);
    cudaError_t e = cudaIpcOpenMemHandle(ptr, hh, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) cudaGetLastError();
    return e;
}

int ipc_close(void *ptr) { return cudaIpcCloseMemHandle(ptr); }

int enable_peer_access(int dev, int peer) {
    if (dev == peer) return 0;
    int can = 0;
    cudaDeviceCanAccessPeer(&can, dev, peer);
    if (!can) return cudaErrorPeerAccessUnsupported;
    int prev = current_device();
    cudaSetDevice(dev);
    cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        e = cudaSuccess;
    }
    if (prev >= 0) cudaSetDevice(prev);
    return e;
}

void *stream_create(int dev) {
    int prev = current_device();
    cudaSetDevice(dev);
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        s = nullptr;
    }
    if (prev >= 0) cudaSetDevice(prev);
    return s;
}

int stream_device(void *s) {
    int d = -1;
    if (cudaStreamGetDevice(static_cast<cudaStream_t>(s), &d) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return d;
}

void stream_destroy(void *s) {
    if (s) cudaStreamDestroy(static_cast<cudaStream_t>(s));
}

int stream_sync(void *s) { return cudaStreamSynchronize(static_cast<cudaStream_t>(s)); }

void *event_create(int dev) {
    int prev = current_device();
    cudaSetDevice(dev);
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        e = nullptr;
    }
    if (prev >= 0) cudaSetDevice(prev);
    return e;
}

void event_destroy(void *e) {
    if (e) cudaEventDestroy(static_cast<cudaEvent_t>(e));
}

int event_record(void *e, void *stream) {
    return cudaEventRecord(static_cast<cudaEvent_t>(e), static_cast<cudaStream_t>(stream));
}

int event_query(void *e) {
    cudaError_t r = cudaEventQuery(static_cast<cudaEvent_t>(e));
    if (r == cudaSuccess) return 1;
    if (r == cudaErrorNotReady) {
        cudaGetLastError();
        return 0;
    }
    cudaGetLastError();
    return -static_cast<int>(r);
}

int event_sync(void *e) { return cudaEventSynchronize(static_cast<cudaEvent_t>(e)); }

int device_sync() { return cudaDeviceSynchronize(); }

const char *error_string(int err) { return cudaGetErrorString(static_cast<cudaError_t>(err)); }

int last_error_clear() { return cudaGetLastError(); }

}  // namespace gpu
}  // namespace mpcomm
