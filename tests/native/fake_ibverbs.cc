// In-process stand-in for libibverbs, loaded by the "ib" fabric through
// MPCOMM_IBVERBS_LIB in CPU tests. Two devices (mlx5_0, mlx5_1), port 1
// ACTIVE, one non-zero GID each. RC QPs follow the INIT/RTR/RTS/ERR state
// machine; post_send (ops slot 25) executes RDMA WRITE/READ immediately with
// rkey and bounds checks against the destination device's registrations and
// queues one completion per WR on the send CQ, drained by poll_cq (slot 11).
// A QP in ERR flushes WRs with status 5 (IBV_WC_WR_FLUSH_ERR).
// ibv_reg_dmabuf_mr accepts a dma-buf fd (as exported by the CUDA driver
// for device memory) and registers the iova range; WRs touching such a
// region are executed with the driver's UVA cuMemCpy in the region's
// context, so GPU tests exercise the GPUDirect registration path
// (cuMemGetHandleForAddressRange -> ibv_reg_dmabuf_mr) on real HBM without
// a NIC. fake_ibv_dmabuf_registrations() counts those registrations.
// Built as a shared library by CMake; it shares the ABI declarations of
// csrc/transport/ib_verbs.h, so it checks the backend's logic, not the
// system ABI.
#include <cuda.h>
#include <dlfcn.h>
#include <cstdio>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <vector>

#include "transport/ib_verbs.h"

using namespace mpcomm::ibv;

namespace {

struct FakeDevice {
    char name[32];
    int index;
};

struct FakeCtx {
    Context ctx;  // must be first: the backend sees Context*
    FakeDevice *dev;
};

struct FakeCq {
    Cq cq;
    std::deque<Wc> wcs;
};

struct FakeQp {
    Qp qp;
    FakeCtx *owner;
    uint32_t dest_qpn = 0;
};

struct FakeMr {
    Mr mr;
    FakeCtx *owner;
    bool device = false;  // GPU memory (dma-buf, or plain reg_mr of a device pointer)
};

std::mutex g_mu;
FakeDevice g_devs[2] = {{"mlx5_0", 0}, {"mlx5_1", 1}};
// FAKE_IBV_DEVICE_PREFIX renames the devices (e.g. "bnxt_re" -> bnxt_re0/1).
void name_devices() {
    static std::once_flag once;
    std::call_once(once, [] {
        const char *p = std::getenv("FAKE_IBV_DEVICE_PREFIX");
        if (!p || !*p) return;
        for (int i = 0; i < 2; ++i) std::snprintf(g_devs[i].name, sizeof(g_devs[i].name), "%s%d", p, i);
    });
}
// Vendor UDP source-port calls (0 = mlx5dv, 1 = bnxt_re_dv) and their ports.
std::atomic<int> g_sport_calls[2];
std::mutex g_sport_mu;
std::vector<uint16_t> g_sports;
int record_sport(int vendor, Qp *qp, uint16_t port) {
    if (!qp || port == 0) return 22;
    g_sport_calls[vendor].fetch_add(1);
    std::lock_guard<std::mutex> g(g_sport_mu);
    g_sports.push_back(port);
    return 0;
}
std::map<uint32_t, FakeQp *> g_qps;
std::map<uint32_t, FakeMr *> g_mrs;  // key -> region (lkey == rkey)
uint32_t g_next_qpn = 0x300, g_next_key = 0x4000;

std::atomic<int> g_dmabuf_regs{0};

FakeMr *mr_find(uint32_t key, uint64_t addr, uint64_t len) {
    auto it = g_mrs.find(key);
    if (it == g_mrs.end()) return nullptr;
    const Mr &m = it->second->mr;
    const uint64_t a = reinterpret_cast<uint64_t>(m.addr);
    return addr >= a && addr + len <= a + m.length ? it->second : nullptr;
}

// CUDA driver entry points, resolved when the first dma-buf region arrives.
struct CuApi {
    CUresult (*memcpy)(CUdeviceptr, CUdeviceptr, size_t) = nullptr;
    CUresult (*ptr_attr)(void *, CUpointer_attribute, CUdeviceptr) = nullptr;
    CUresult (*push)(CUcontext) = nullptr;
    CUresult (*pop)(CUcontext *) = nullptr;
};
const CuApi *cu();

// True for device memory of a CUDA context in this process (the driver
// must already be loaded; CPU-only processes never see device pointers).
bool is_device_ptr(const void *p) {
    const CuApi *api = cu();
    if (!api) return false;
    unsigned int type = 0;
    return api->ptr_attr(&type, CU_POINTER_ATTRIBUTE_MEMORY_TYPE, reinterpret_cast<CUdeviceptr>(p)) ==
               CUDA_SUCCESS &&
           type == CU_MEMORYTYPE_DEVICE;
}

const CuApi *cu() {
    static CuApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_NOLOAD);  // only if the process uses CUDA
        if (h) {
            api.memcpy = reinterpret_cast<decltype(api.memcpy)>(dlsym(h, "cuMemcpy"));
            api.ptr_attr = reinterpret_cast<decltype(api.ptr_attr)>(dlsym(h, "cuPointerGetAttribute"));
            api.push = reinterpret_cast<decltype(api.push)>(dlsym(h, "cuCtxPushCurrent_v2"));
            api.pop = reinterpret_cast<decltype(api.pop)>(dlsym(h, "cuCtxPopCurrent_v2"));
        }
    });
    return api.memcpy && api.ptr_attr && api.push && api.pop ? &api : nullptr;
}

// The "NIC DMA": host memmove, or a UVA copy in the device region's context.
bool move_bytes(void *dst, const void *src, size_t n, const FakeMr *dev_mr) {
    if (!dev_mr) {
        std::memmove(dst, src, n);
        return true;
    }
    const CuApi *api = cu();
    if (!api) return false;
    CUcontext ctx = nullptr;
    if (api->ptr_attr(&ctx, CU_POINTER_ATTRIBUTE_CONTEXT, reinterpret_cast<CUdeviceptr>(dev_mr->mr.addr)) !=
            CUDA_SUCCESS ||
        !ctx || api->push(ctx) != CUDA_SUCCESS)
        return false;
    const bool ok = api->memcpy(reinterpret_cast<CUdeviceptr>(dst), reinterpret_cast<CUdeviceptr>(src), n) ==
                    CUDA_SUCCESS;
    CUcontext popped = nullptr;
    api->pop(&popped);
    return ok;
}

int fake_post_send(Qp *qp, SendWr *wr, SendWr **bad) {
    std::lock_guard<std::mutex> g(g_mu);
    FakeQp *q = reinterpret_cast<FakeQp *>(qp);
    FakeCq *cq = reinterpret_cast<FakeCq *>(qp->send_cq);
    for (SendWr *w = wr; w; w = w->next) {
        Wc c;
        std::memset(&c, 0, sizeof(c));
        c.wr_id = w->wr_id;
        c.qp_num = qp->qp_num;
        c.opcode = w->opcode;
        if (qp->state == kQpsErr) {
            c.status = 5;
        } else if (qp->state != kQpsRts || w->num_sge != 1) {
            if (bad) *bad = w;
            return 22;  // EINVAL, nothing queued from here on
        } else {
            const Sge &s = w->sg_list[0];
            auto peer = g_qps.find(q->dest_qpn);
            FakeMr *lm = mr_find(s.lkey, s.addr, s.length);
            FakeMr *rm = lm ? mr_find(w->wr.rkey, w->wr.remote_addr, s.length) : nullptr;
            if (!lm) {
                c.status = 4;  // local protection error
            } else if (peer == g_qps.end() || peer->second->qp.state == kQpsErr) {
                c.status = 12;  // retry exceeded
            } else if (!rm) {
                c.status = 10;  // remote access error
            } else {
                void *local = reinterpret_cast<void *>(s.addr);
                void *remote = reinterpret_cast<void *>(w->wr.remote_addr);
                const FakeMr *dev = lm->device ? lm : (rm->device ? rm : nullptr);
                const bool ok = w->opcode == kWrRdmaWrite ? move_bytes(remote, local, s.length, dev)
                                                          : move_bytes(local, remote, s.length, dev);
                c.status = ok ? 0 : 4;
                c.byte_len = ok ? s.length : 0;
            }
        }
        if (w->send_flags & kSendSignaled) cq->wcs.push_back(c);
    }
    return 0;
}

int fake_poll_cq(Cq *cq, int n, Wc *wc) {
    std::lock_guard<std::mutex> g(g_mu);
    FakeCq *f = reinterpret_cast<FakeCq *>(cq);
    int k = 0;
    while (k < n && !f->wcs.empty()) {
        wc[k++] = f->wcs.front();
        f->wcs.pop_front();
    }
    return k;
}

}  // namespace

extern "C" {

Device **ibv_get_device_list(int *n) {
    name_devices();
    Device **l = static_cast<Device **>(std::calloc(3, sizeof(Device *)));
    l[0] = reinterpret_cast<Device *>(&g_devs[0]);
    l[1] = reinterpret_cast<Device *>(&g_devs[1]);
    if (n) *n = 2;
    return l;
}
void ibv_free_device_list(Device **l) { std::free(l); }
const char *ibv_get_device_name(Device *d) { return reinterpret_cast<FakeDevice *>(d)->name; }

Context *ibv_open_device(Device *d) {
    FakeCtx *c = new FakeCtx();
    std::memset(&c->ctx, 0, sizeof(c->ctx));
    c->ctx.device = d;
    c->ctx.ops[11] = reinterpret_cast<void *>(&fake_poll_cq);
    c->ctx.ops[25] = reinterpret_cast<void *>(&fake_post_send);
    c->dev = reinterpret_cast<FakeDevice *>(d);
    return &c->ctx;
}
int ibv_close_device(Context *c) {
    delete reinterpret_cast<FakeCtx *>(c);
    return 0;
}
int ibv_query_port(Context *c, uint8_t port, PortAttr *a) {
    std::memset(a, 0, 64);
    if (port != 1) return 22;
    a->state = kPortActive;
    a->gid_tbl_len = 4;
    a->lid = static_cast<uint16_t>(reinterpret_cast<FakeCtx *>(c)->dev->index + 1);
    return 0;
}
int ibv_query_gid(Context *c, uint8_t, int index, Gid *g) {
    std::memset(g, 0, sizeof(*g));
    if (index < 0 || index >= 4) return 22;
    g->raw[0] = 0xfe;
    g->raw[1] = 0x80;
    g->raw[14] = static_cast<uint8_t>(index);
    g->raw[15] = static_cast<uint8_t>(reinterpret_cast<FakeCtx *>(c)->dev->index + 1);
    return 0;
}
Pd *ibv_alloc_pd(Context *c) { return reinterpret_cast<Pd *>(c); }
int ibv_dealloc_pd(Pd *) { return 0; }
Cq *ibv_create_cq(Context *c, int, void *, CompChannel *, int) {
    FakeCq *f = new FakeCq();
    f->cq.context = c;
    return &f->cq;
}
int ibv_destroy_cq(Cq *cq) {
    delete reinterpret_cast<FakeCq *>(cq);
    return 0;
}
Mr *ibv_reg_mr(Pd *pd, void *addr, size_t len, int) {
    std::lock_guard<std::mutex> g(g_mu);
    FakeMr *m = new FakeMr();
    m->owner = reinterpret_cast<FakeCtx *>(pd);
    m->mr.context = &m->owner->ctx;
    m->mr.pd = pd;
    m->mr.addr = addr;
    m->mr.length = len;
    m->mr.lkey = m->mr.rkey = g_next_key++;
    m->device = is_device_ptr(addr);  // nvidia-peermem style registration of HBM
    g_mrs[m->mr.lkey] = m;
    return &m->mr;
}
// GPUDirect registration of a dma-buf (device memory exported by the CUDA
// driver): `iova` is the virtual address WRs use, `offset` the start within
// the dma-buf. The fd must be open; the fake keeps no reference to it.
Mr *ibv_reg_dmabuf_mr(Pd *pd, uint64_t offset, size_t len, uint64_t iova, int fd, int) {
    struct stat st;
    if (fd < 0 || fstat(fd, &st) != 0 || len == 0 || !cu()) {
        errno = EINVAL;
        return nullptr;
    }
    (void)offset;
    std::lock_guard<std::mutex> g(g_mu);
    FakeMr *m = new FakeMr();
    m->owner = reinterpret_cast<FakeCtx *>(pd);
    m->mr.context = &m->owner->ctx;
    m->mr.pd = pd;
    m->mr.addr = reinterpret_cast<void *>(iova);
    m->mr.length = len;
    m->mr.lkey = m->mr.rkey = g_next_key++;
    m->device = true;
    g_mrs[m->mr.lkey] = m;
    g_dmabuf_regs.fetch_add(1);
    return &m->mr;
}
int fake_ibv_dmabuf_registrations() { return g_dmabuf_regs.load(); }
int mlx5dv_modify_qp_udp_sport(Qp *qp, uint16_t port) { return record_sport(0, qp, port); }
int bnxt_re_dv_modify_qp_udp_sport(Qp *qp, uint16_t port) { return record_sport(1, qp, port); }
int fake_ibv_sport_calls(int vendor) { return vendor == 0 || vendor == 1 ? g_sport_calls[vendor].load() : -1; }
// Copies up to `max` recorded ports into `out`; returns how many were recorded.
int fake_ibv_sports(uint16_t *out, int max) {
    std::lock_guard<std::mutex> g(g_sport_mu);
    for (int i = 0; i < max && i < static_cast<int>(g_sports.size()); ++i) out[i] = g_sports[i];
    return static_cast<int>(g_sports.size());
}
int ibv_dereg_mr(Mr *mr) {
    std::lock_guard<std::mutex> g(g_mu);
    g_mrs.erase(mr->lkey);
    delete reinterpret_cast<FakeMr *>(mr);
    return 0;
}
Qp *ibv_create_qp(Pd *pd, QpInitAttr *a) {
    std::lock_guard<std::mutex> g(g_mu);
    FakeQp *q = new FakeQp();
    std::memset(&q->qp, 0, sizeof(q->qp));
    q->owner = reinterpret_cast<FakeCtx *>(pd);
    q->qp.context = &q->owner->ctx;
    q->qp.pd = pd;
    q->qp.send_cq = a->send_cq;
    q->qp.recv_cq = a->recv_cq;
    q->qp.qp_num = g_next_qpn++;
    q->qp.state = kQpsReset;
    q->qp.qp_type = a->qp_type;
    g_qps[q->qp.qp_num] = q;
    return &q->qp;
}
int ibv_modify_qp(Qp *qp, QpAttr *a, int mask) {
    std::lock_guard<std::mutex> g(g_mu);
    FakeQp *q = reinterpret_cast<FakeQp *>(qp);
    if (!(mask & kQpState)) return 22;
    const uint32_t from = qp->state, to = a->qp_state;
    const bool legal = to == kQpsErr || to == kQpsReset || (from == kQpsReset && to == kQpsInit) ||
                       (from == kQpsInit && to == kQpsRtr) || (from == kQpsRtr && to == kQpsRts);
    if (!legal) return 22;
    if (to == kQpsRtr) {
        if (!(mask & kQpDestQpn) || !(mask & kQpAv) || !a->ah_attr.is_global) return 22;
        q->dest_qpn = a->dest_qp_num;
    }
    qp->state = to;
    return 0;
}
int ibv_destroy_qp(Qp *qp) {
    std::lock_guard<std::mutex> g(g_mu);
    g_qps.erase(qp->qp_num);
    delete reinterpret_cast<FakeQp *>(qp);
    return 0;
}

}  // extern "C"
