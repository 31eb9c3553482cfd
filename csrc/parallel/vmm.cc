#include "parallel/vmm.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <unistd.h>

#include <cstring>

#include "ctrl/fdshare.h"
#include "cuda/gpu.h"
#include "mpcomm_log.h"

namespace mpcomm {
namespace vmm {

namespace {

template <typename Fn>
Fn sym(const char *name) {
    return reinterpret_cast<Fn>(gpu::driver_symbol(name));
}

constexpr int kNoDriver = CUDA_ERROR_NOT_FOUND;

int cu_device(int ordinal, CUdevice *out) {
    auto fn = sym<CUresult (*)(CUdevice *, int)>("cuDeviceGet");
    return fn ? fn(out, ordinal) : kNoDriver;
}

CUmulticastObjectProp mc_prop(size_t size, int ndev) {
    CUmulticastObjectProp p;
    std::memset(&p, 0, sizeof(p));
    p.numDevices = static_cast<unsigned>(ndev);
    p.size = size;
    p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    return p;
}

}  // namespace

int ipc_export(const void *ptr, unsigned char handle[64], uint64_t *offset) {
    gpu::PtrInfo pi;
    if (!gpu::query_pointer(ptr, &pi) || !pi.is_device || !pi.base) return CUDA_ERROR_INVALID_VALUE;
    int e = gpu::ipc_get_handle(reinterpret_cast<void *>(pi.base), handle);
    if (e) return e;
    *offset = reinterpret_cast<uintptr_t>(ptr) - pi.base;
    return 0;
}

int ipc_import(const unsigned char handle[64], void **base) { return gpu::ipc_open_handle(handle, base); }

int ipc_release(void *base) { return gpu::ipc_close(base); }

int multicast_supported(int dev) {
    auto fn = sym<CUresult (*)(int *, CUdevice_attribute, CUdevice)>("cuDeviceGetAttribute");
    CUdevice d;
    if (!fn || cu_device(dev, &d)) return 0;
    int v = 0;
    if (fn(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, d) != CUDA_SUCCESS) return 0;
    return v;
}

int multicast_granularity(size_t size, int ndev, size_t *gran) {
    auto fn = sym<CUresult (*)(size_t *, const CUmulticastObjectProp *, CUmulticastGranularity_flags)>(
        "cuMulticastGetGranularity");
    if (!fn) return kNoDriver;
    CUmulticastObjectProp p = mc_prop(size, ndev);
    return fn(gran, &p, CU_MULTICAST_GRANULARITY_MINIMUM);
}

int multicast_create(size_t size, int ndev, uint64_t *mc, int *fd) {
    auto create = sym<CUresult (*)(CUmemGenericAllocationHandle *, const CUmulticastObjectProp *)>(
        "cuMulticastCreate");
    auto exp = sym<CUresult (*)(void *, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                                unsigned long long)>("cuMemExportToShareableHandle");
    if (!create || !exp) return kNoDriver;
    CUmulticastObjectProp p = mc_prop(size, ndev);
    CUmemGenericAllocationHandle h = 0;
    CUresult r = create(&h, &p);
    if (r != CUDA_SUCCESS) return r;
    int f = -1;
    r = exp(&f, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
    if (r != CUDA_SUCCESS) {
        auto rel = sym<CUresult (*)(CUmemGenericAllocationHandle)>("cuMemRelease");
        if (rel) rel(h);
        return r;
    }
    *mc = h;
    *fd = f;
    return 0;
}

int multicast_import(int fd, uint64_t *mc) {
    auto imp = sym<CUresult (*)(CUmemGenericAllocationHandle *, void *, CUmemAllocationHandleType)>(
        "cuMemImportFromShareableHandle");
    if (!imp) return kNoDriver;
    CUmemGenericAllocationHandle h = 0;
    CUresult r = imp(&h, reinterpret_cast<void *>(static_cast<uintptr_t>(fd)),
                     CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
    if (r == CUDA_SUCCESS) *mc = h;
    return r;
}

int multicast_add_device(uint64_t mc, int dev) {
    auto fn = sym<CUresult (*)(CUmemGenericAllocationHandle, CUdevice)>("cuMulticastAddDevice");
    CUdevice d;
    if (!fn) return kNoDriver;
    int e = cu_device(dev, &d);
    return e ? e : fn(mc, d);
}

namespace {

int map_rw(CUmemGenericAllocationHandle h, size_t size, int dev, void **va) {
    auto reserve = sym<CUresult (*)(CUdeviceptr *, size_t, size_t, CUdeviceptr, unsigned long long)>(
        "cuMemAddressReserve");
    auto map = sym<CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long)>(
        "cuMemMap");
    auto access = sym<CUresult (*)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t)>("cuMemSetAccess");
    auto unmap = sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemUnmap");
    auto vfree = sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemAddressFree");
    if (!reserve || !map || !access || !unmap || !vfree) return kNoDriver;
    CUdeviceptr p = 0;
    CUresult r = reserve(&p, size, 0, 0, 0);
    if (r != CUDA_SUCCESS) return r;
    r = map(p, size, 0, h, 0);
    if (r != CUDA_SUCCESS) {
        vfree(p, size);
        return r;
    }
    CUmemAccessDesc a;
    std::memset(&a, 0, sizeof(a));
    a.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    a.location.id = dev;
    a.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    r = access(p, size, &a, 1);
    if (r != CUDA_SUCCESS) {
        unmap(p, size);
        vfree(p, size);
        return r;
    }
    *va = reinterpret_cast<void *>(p);
    return 0;
}

}  // namespace

int multicast_bind_local(uint64_t mc, size_t size, int dev, uint64_t *mem, void **uc_va) {
    auto create = sym<CUresult (*)(CUmemGenericAllocationHandle *, size_t, const CUmemAllocationProp *,
                                   unsigned long long)>("cuMemCreate");
    auto bind = sym<CUresult (*)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle, size_t,
                                 size_t, unsigned long long)>("cuMulticastBindMem");
    auto rel = sym<CUresult (*)(CUmemGenericAllocationHandle)>("cuMemRelease");
    if (!create || !bind || !rel) return kNoDriver;
    CUmemAllocationProp p;
    std::memset(&p, 0, sizeof(p));
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = dev;
    p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    CUmemGenericAllocationHandle h = 0;
    CUresult r = create(&h, size, &p, 0);
    if (r != CUDA_SUCCESS) return r;
    r = bind(mc, 0, h, 0, size, 0);
    if (r != CUDA_SUCCESS) {
        rel(h);
        return r;
    }
    int e = map_rw(h, size, dev, uc_va);
    if (e) {
        rel(h);
        return e;
    }
    *mem = h;
    return 0;
}

int multicast_map(uint64_t mc, size_t size, int dev, void **mc_va) { return map_rw(mc, size, dev, mc_va); }

int vmm_segments(const void *ptr, size_t len, size_t max_segments, std::vector<VmmSegment> *out) {
    auto retain = sym<CUresult (*)(CUmemGenericAllocationHandle *, void *)>("cuMemRetainAllocationHandle");
    auto range = sym<CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr)>("cuMemGetAddressRange");
    auto rel = sym<CUresult (*)(CUmemGenericAllocationHandle)>("cuMemRelease");
    if (!retain || !range || !rel) return kNoDriver;
    out->clear();
    const CUdeviceptr end = reinterpret_cast<CUdeviceptr>(ptr) + len;
    CUdeviceptr p = reinterpret_cast<CUdeviceptr>(ptr);
    while (p < end) {
        CUdeviceptr b = 0;
        size_t n = 0;
        CUresult r = range(&b, &n, p);
        if (r != CUDA_SUCCESS) return r;
        // Contiguous: after the first, each allocation starts where the
        // previous one ended.
        if (n == 0 || (!out->empty() && b != p) || out->size() >= max_segments) return -1;
        // One allocation per range: its first and last bytes share a handle.
        CUmemGenericAllocationHandle h = 0, last = 0;
        r = retain(&h, reinterpret_cast<void *>(b));
        if (r != CUDA_SUCCESS) return r;
        r = retain(&last, reinterpret_cast<void *>(b + n - 1));
        if (r == CUDA_SUCCESS) rel(last);
        rel(h);
        if (r != CUDA_SUCCESS) return r;
        if (last != h) return -1;
        out->push_back(VmmSegment{static_cast<uintptr_t>(b), n});
        p = b + n;
    }
    return out->empty() ? -1 : 0;
}

int vmm_export_fd(uintptr_t base, int *fd) {
    auto retain = sym<CUresult (*)(CUmemGenericAllocationHandle *, void *)>("cuMemRetainAllocationHandle");
    auto exp = sym<CUresult (*)(void *, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                                unsigned long long)>("cuMemExportToShareableHandle");
    auto rel = sym<CUresult (*)(CUmemGenericAllocationHandle)>("cuMemRelease");
    if (!retain || !exp || !rel) return kNoDriver;
    CUmemGenericAllocationHandle h = 0;
    CUresult r = retain(&h, reinterpret_cast<void *>(base));
    if (r != CUDA_SUCCESS) return r;
    int f = -1;
    r = exp(&f, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
    rel(h);
    if (r != CUDA_SUCCESS) return r;
    *fd = f;
    return 0;
}

namespace {

// Maps imported allocations back to back into one reserved range, one at a
// time (so a caller never holds more than one handle), then grants `dev`
// access to the whole range. abort() undoes whatever was mapped.
class BackToBack {
 public:
    BackToBack()
        : imp_(sym<CUresult (*)(CUmemGenericAllocationHandle *, void *, CUmemAllocationHandleType)>(
              "cuMemImportFromShareableHandle")),
          reserve_(sym<CUresult (*)(CUdeviceptr *, size_t, size_t, CUdeviceptr, unsigned long long)>(
              "cuMemAddressReserve")),
          map_(sym<CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long)>(
              "cuMemMap")),
          access_(sym<CUresult (*)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t)>("cuMemSetAccess")),
          unmap_(sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemUnmap")),
          vfree_(sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemAddressFree")),
          rel_(sym<CUresult (*)(CUmemGenericAllocationHandle)>("cuMemRelease")) {}

    int begin(size_t total) {
        if (!imp_ || !reserve_ || !map_ || !access_ || !unmap_ || !vfree_ || !rel_) return kNoDriver;
        if (total == 0) return CUDA_ERROR_INVALID_VALUE;
        total_ = total;
        return reserve_(&base_, total, 0, 0, 0);
    }
    // The next allocation, at `offset` (must continue where the last ended).
    int add(int fd, size_t offset, size_t size) {
        if (!base_ || offset != mapped_ || size == 0 || offset + size > total_) return CUDA_ERROR_INVALID_VALUE;
        CUmemGenericAllocationHandle h = 0;
        CUresult r = imp_(&h, reinterpret_cast<void *>(static_cast<uintptr_t>(fd)), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
        if (r != CUDA_SUCCESS) return r;
        r = map_(base_ + mapped_, size, 0, h, 0);
        rel_(h);  // the mapping holds the allocation from here on
        if (r != CUDA_SUCCESS) return r;
        sizes_.push_back(size);
        mapped_ += size;
        return 0;
    }
    int finish(int dev, void **va, std::vector<size_t> *sizes) {
        if (mapped_ != total_) return CUDA_ERROR_INVALID_VALUE;
        CUmemAccessDesc a;
        std::memset(&a, 0, sizeof(a));
        a.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        a.location.id = dev;
        a.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        const CUresult r = access_(base_, total_, &a, 1);
        if (r != CUDA_SUCCESS) return r;
        *va = reinterpret_cast<void *>(base_);
        if (sizes) *sizes = sizes_;
        base_ = 0;  // handed over
        return 0;
    }
    void abort() {
        if (!base_) return;
        size_t off = 0;
        for (size_t n : sizes_) {
            unmap_(base_ + off, n);
            off += n;
        }
        vfree_(base_, total_);
        base_ = 0;
    }
    ~BackToBack() { abort(); }

 private:
    CUresult (*imp_)(CUmemGenericAllocationHandle *, void *, CUmemAllocationHandleType);
    CUresult (*reserve_)(CUdeviceptr *, size_t, size_t, CUdeviceptr, unsigned long long);
    CUresult (*map_)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
    CUresult (*access_)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t);
    CUresult (*unmap_)(CUdeviceptr, size_t);
    CUresult (*vfree_)(CUdeviceptr, size_t);
    CUresult (*rel_)(CUmemGenericAllocationHandle);
    CUdeviceptr base_ = 0;
    size_t total_ = 0, mapped_ = 0;
    std::vector<size_t> sizes_;
};

}  // namespace

int multicast_teardown(uint64_t mc, uint64_t mem, void *uc_va, void *mc_va, size_t size, int dev) {
    auto unmap = sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemUnmap");
    auto vfree = sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemAddressFree");
    auto unbind = sym<CUresult (*)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t)>("cuMulticastUnbind");
    auto rel = sym<CUresult (*)(CUmemGenericAllocationHandle)>("cuMemRelease");
    if (!unmap || !vfree || !rel) return kNoDriver;
    for (void *va : {mc_va, uc_va}) {
        if (!va) continue;
        unmap(reinterpret_cast<CUdeviceptr>(va), size);
        vfree(reinterpret_cast<CUdeviceptr>(va), size);
    }
    CUdevice d;
    if (mc && mem && unbind && cu_device(dev, &d) == 0) unbind(mc, d, 0, size);
    if (mem) rel(mem);
    if (mc) rel(mc);
    return 0;
}

int gdr_alloc(int dev, size_t size, void **ptr, size_t *alloc_size) {
    auto gran = sym<CUresult (*)(size_t *, const CUmemAllocationProp *, CUmemAllocationGranularity_flags)>(
        "cuMemGetAllocationGranularity");
    auto create = sym<CUresult (*)(CUmemGenericAllocationHandle *, size_t, const CUmemAllocationProp *,
                                   unsigned long long)>("cuMemCreate");
    auto rel = sym<CUresult (*)(CUmemGenericAllocationHandle)>("cuMemRelease");
    if (!gran || !create || !rel) return kNoDriver;
    if (size == 0) return CUDA_ERROR_INVALID_VALUE;
    CUmemAllocationProp p;
    std::memset(&p, 0, sizeof(p));
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = dev;
    p.allocFlags.gpuDirectRDMACapable = 1;
    p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;  // reachable by peer processes
    size_t g = 0;
    CUresult r = gran(&g, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
    if (r != CUDA_SUCCESS) return r;
    if (g == 0) g = 2u << 20;
    const size_t n = (size + g - 1) / g * g;
    CUmemGenericAllocationHandle h = 0;
    r = create(&h, n, &p, 0);
    if (r != CUDA_SUCCESS) return r;
    // The mapping holds a reference; the creation handle is released now,
    // so unmapping frees the memory.
    const int e = map_rw(h, n, dev, ptr);
    rel(h);
    if (e) return e;
    *alloc_size = n;
    return 0;
}

int gdr_free(void *ptr, size_t alloc_size) {
    auto unmap = sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemUnmap");
    auto vfree = sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemAddressFree");
    if (!unmap || !vfree) return kNoDriver;
    if (!ptr) return 0;
    CUresult r = unmap(reinterpret_cast<CUdeviceptr>(ptr), alloc_size);
    if (r != CUDA_SUCCESS) return r;
    return vfree(reinterpret_cast<CUdeviceptr>(ptr), alloc_size);
}

int dmabuf_export(const void *ptr, size_t size, unsigned long long flags, int *fd) {
    auto fn = sym<CUresult (*)(void *, CUdeviceptr, size_t, CUmemRangeHandleType, unsigned long long)>(
        "cuMemGetHandleForAddressRange");
    if (!fn) return kNoDriver;
    return fn(fd, reinterpret_cast<CUdeviceptr>(ptr), size, CU_MEM_RANGE_HANDLE_TYPE_DMA_BUF_FD, flags);
}

int vmm_offer(const void *ptr, size_t len, uint64_t key, uintptr_t *base, size_t *span) {
    std::vector<VmmSegment> segs;
    int e = vmm_segments(ptr, len, ctrl::kFdMaxSegments, &segs);
    if (e) return e;
    int fd = -1;
    if ((e = vmm_export_fd(segs[0].base, &fd))) return e;  // created without a POSIX handle type?
    close(fd);
    const uintptr_t b = segs[0].base;
    ctrl::FdOffer o;
    std::vector<uintptr_t> bases;
    for (const auto &g : segs) {
        ctrl::FdSegment f;
        f.offset = g.base - b;
        f.size = g.size;
        o.segments.push_back(f);
        bases.push_back(g.base);
    }
    o.export_fd = [bases](size_t i) {
        int f = -1;
        return i < bases.size() && vmm_export_fd(bases[i], &f) == 0 ? f : -1;
    };
    if (ctrl::fd_offer(ctrl::fd_service_name(getpid()), key, std::move(o)) != 0) return -1;
    *base = b;
    *span = segs.back().base + segs.back().size - b;
    return 0;
}

void vmm_withdraw(uint64_t key) { ctrl::fd_withdraw(key); }

int vmm_open(long pid, uint64_t key, int dev, int timeout_ms, void **va, std::vector<size_t> *sizes) {
    BackToBack m;
    int e = 0;
    const int fr = ctrl::fd_fetch(
        ctrl::fd_service_name(pid), key, timeout_ms,
        [&](size_t, uint64_t bytes) { return (e = m.begin(static_cast<size_t>(bytes))) == 0; },
        [&](const ctrl::FdSegment &g) {
            return (e = m.add(g.fd, static_cast<size_t>(g.offset), static_cast<size_t>(g.size))) == 0;
        });
    if (e) return e;
    if (fr) return fr == 1 ? kVmmNotOffered : kVmmUnreachable;
    return m.finish(dev, va, sizes);
}

int vmm_unmap(void *va, const std::vector<size_t> &sizes) {
    auto unmap = sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemUnmap");
    auto vfree = sym<CUresult (*)(CUdeviceptr, size_t)>("cuMemAddressFree");
    if (!unmap || !vfree) return kNoDriver;
    const CUdeviceptr p = reinterpret_cast<CUdeviceptr>(va);
    size_t off = 0;
    for (size_t n : sizes) {
        unmap(p + off, n);
        off += n;
    }
    return vfree(p, off);
}

}  // namespace vmm
}  // namespace mpcomm
