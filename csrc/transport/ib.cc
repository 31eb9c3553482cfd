// "ib" backend: ibverbs RC one-sided RDMA WRITE/READ.
//
// libibverbs is opened with dlopen at run time (ib_verbs.h), so this file
// builds everywhere and the backend is simply unavailable on hosts without
// rdma-core or RDMA devices. QP parameters follow the reference
// (src/mpcomm.cpp:3854-3976): RC, 1 SGE, max_send_wr=MPCOMM_MAX_SEND_WR,
// MTU 4096, max_rd/dest_rd_atomic 16, min_rnr_timer 12, timeout 14,
// retry 7, rnr_retry 7, GRH hop_limit 16 with traffic class DSCP<<2.
// GPU memory is registered through dma-buf (cuMemGetHandleForAddressRange
// + ibv_reg_dmabuf_mr) with plain ibv_reg_mr (nvidia-peermem) as the
// fallback. On mlx5 devices each QP gets its own RoCE UDP source port
// (ECMP spreading) when libmlx5 exports mlx5dv_modify_qp_udp_sport.
#include <cuda.h>
#include <dlfcn.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <map>
#include <vector>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "cuda/gpu.h"
#include "mpcomm.h"
#include "mpcomm_log.h"
#include "topo/topology.h"
#include "transport/fabric.h"
#include "transport/ib_verbs.h"

namespace mpcomm {
namespace ibv {

const Api *load() {
    static Api api;
    static const Api *ok = [] () -> const Api * {
        const char *path = std::getenv("MPCOMM_IBVERBS_LIB");
        void *h = dlopen(path && *path ? path : "libibverbs.so.1", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return nullptr;
        auto sym = [&](const char *n) { return dlsym(h, n); };
#define MPCOMM_IBV_SYM(field, name) \
    api.field = reinterpret_cast<decltype(api.field)>(sym(name));
        MPCOMM_IBV_SYM(get_device_list, "ibv_get_device_list")
        MPCOMM_IBV_SYM(free_device_list, "ibv_free_device_list")
        MPCOMM_IBV_SYM(get_device_name, "ibv_get_device_name")
        MPCOMM_IBV_SYM(open_device, "ibv_open_device")
        MPCOMM_IBV_SYM(close_device, "ibv_close_device")
        MPCOMM_IBV_SYM(query_port, "ibv_query_port")
        MPCOMM_IBV_SYM(query_gid, "ibv_query_gid")
        MPCOMM_IBV_SYM(alloc_pd, "ibv_alloc_pd")
        MPCOMM_IBV_SYM(dealloc_pd, "ibv_dealloc_pd")
        MPCOMM_IBV_SYM(create_cq, "ibv_create_cq")
        MPCOMM_IBV_SYM(destroy_cq, "ibv_destroy_cq")
        MPCOMM_IBV_SYM(reg_mr, "ibv_reg_mr")
        MPCOMM_IBV_SYM(reg_dmabuf_mr, "ibv_reg_dmabuf_mr")
        MPCOMM_IBV_SYM(dereg_mr, "ibv_dereg_mr")
        MPCOMM_IBV_SYM(create_qp, "ibv_create_qp")
        MPCOMM_IBV_SYM(modify_qp, "ibv_modify_qp")
        MPCOMM_IBV_SYM(destroy_qp, "ibv_destroy_qp")
#undef MPCOMM_IBV_SYM
        if (!api.get_device_list || !api.open_device || !api.alloc_pd || !api.create_cq ||
            !api.reg_mr || !api.create_qp || !api.modify_qp || !api.query_port || !api.query_gid)
            return nullptr;
        return &api;
    }();
    return ok;
}

}  // namespace ibv

namespace fabric {
namespace {

std::string gid_to_string(const ibv::Gid &g) {
    char buf[64];
    snprintf(buf, sizeof(buf),
             "%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x:%02x",
             g.raw[0], g.raw[1], g.raw[2], g.raw[3], g.raw[4], g.raw[5], g.raw[6], g.raw[7], g.raw[8],
             g.raw[9], g.raw[10], g.raw[11], g.raw[12], g.raw[13], g.raw[14], g.raw[15]);
    return buf;
}

bool string_to_gid(const std::string &s, ibv::Gid *g) {
    unsigned v[16];
    if (sscanf(s.c_str(), "%x:%x:%x:%x:%x:%x:%x:%x:%x:%x:%x:%x:%x:%x:%x:%x", &v[0], &v[1], &v[2], &v[3],
               &v[4], &v[5], &v[6], &v[7], &v[8], &v[9], &v[10], &v[11], &v[12], &v[13], &v[14],
               &v[15]) != 16)
        return false;
    for (int i = 0; i < 16; ++i) g->raw[i] = static_cast<uint8_t>(v[i]);
    return true;
}

bool gid_zero(const ibv::Gid &g) {
    for (auto b : g.raw)
        if (b) return false;
    return true;
}

using UdpSportFn = int (*)(ibv::Qp *, uint16_t);

// UDP source port of a RoCE v2 QP (ECMP spreading across fabric paths),
// set through the NIC vendor's direct-verbs call: mlx5dv_modify_qp_udp_sport
// for mlx5 devices, bnxt_re_dv_modify_qp_udp_sport for Broadcom bnxt_re
// devices (the reference calls one or the other depending on its build,
// src/mpcomm.cpp:3954-3967). MPCOMM_IBV_DV_LIB names one library to look
// both symbols up in instead of the vendors' own.
UdpSportFn udp_sport_fn(const std::string &device) {
    struct Fns {
        UdpSportFn mlx5 = nullptr, bnxt = nullptr;
    };
    static const Fns fns = [] {
        Fns f;
        auto look = [](const char *lib, const char *sym) -> UdpSportFn {
            void *h = dlopen(lib, RTLD_NOW | RTLD_GLOBAL);
            return h ? reinterpret_cast<UdpSportFn>(dlsym(h, sym)) : nullptr;
        };
        const char *over = std::getenv("MPCOMM_IBV_DV_LIB");
        if (over && *over) {
            f.mlx5 = look(over, "mlx5dv_modify_qp_udp_sport");
            f.bnxt = look(over, "bnxt_re_dv_modify_qp_udp_sport");
            return f;
        }
        f.mlx5 = look("libmlx5.so.1", "mlx5dv_modify_qp_udp_sport");
        for (const char *lib : {"libbnxt_re.so.1", "libbnxt_re.so", "libbnxt_re-rdmav34.so"})
            if (!f.bnxt) f.bnxt = look(lib, "bnxt_re_dv_modify_qp_udp_sport");
        return f;
    }();
    return device.compare(0, 7, "bnxt_re") == 0 ? fns.bnxt : fns.mlx5;
}

// Source port of the i-th QP: MPCOMM_UDP_SPORTS (comma list) cycled in QP
// order, else spread over the dynamic range 49152-65535 by a multiplicative
// hash so consecutive QPs land far apart.
uint16_t udp_sport_for(uint32_t i) {
    static const std::vector<uint16_t> list = [] {
        std::vector<uint16_t> v;
        const char *e = std::getenv("MPCOMM_UDP_SPORTS");
        for (const char *p = e; p && *p;) {
            char *end = nullptr;
            const long x = std::strtol(p, &end, 10);
            if (end == p) break;
            if (x > 0 && x < 65536) v.push_back(static_cast<uint16_t>(x));
            p = *end == ',' ? end + 1 : end;
        }
        return v;
    }();
    if (!list.empty()) return list[i % list.size()];
    return static_cast<uint16_t>(49152 + (i * 40503u) % 16384);
}

class IbRail;

class IbQp final : public QueuePair {
 public:
    IbQp(IbRail *rail, ibv::Qp *qp) : rail_(rail), qp_(qp) {}
    ~IbQp() override;
    uint32_t qp_num() const override { return qp_->qp_num; }
    QpState state() const override { return state_; }
    int to_init() override;
    int to_rtr(const EndpointInfo &remote) override;
    int to_rts() override;
    int to_err() override;
    int recover() override;
    int post(const WorkRequest *wrs, size_t n) override;

 private:
    IbRail *rail_;
    ibv::Qp *qp_;
    QpState state_ = QpState::kReset;
    EndpointInfo remote_;
};

class IbRail final : public Rail {
 public:
    IbRail(const ibv::Api *api, ibv::Device *dev, const Config &cfg) : api_(api), cfg_(cfg) {
        name_ = api_->get_device_name(dev);
        ctx_ = api_->open_device(dev);
        if (!ctx_) return;
        ibv::PortAttr pa;
        std::memset(&pa, 0, sizeof(pa));
        if (api_->query_port(ctx_, port_, &pa) != 0 || pa.state != ibv::kPortActive) {
            MPCOMM_LOG_WARN("MPComm[ib]: %s port %u not active, skipped\n", name_.c_str(), port_);
            return;
        }
        lid_ = pa.lid;
        gid_index_ = cfg.gid_index;
        if (gid_index_ < 0) {
            for (int i = 0; i < pa.gid_tbl_len && i < 256; ++i) {
                ibv::Gid g;
                if (api_->query_gid(ctx_, port_, i, &g) == 0 && !gid_zero(g)) {
                    gid_index_ = i;
                    break;
                }
            }
        }
        if (gid_index_ < 0 || api_->query_gid(ctx_, port_, gid_index_, &gid_) != 0 || gid_zero(gid_)) {
            MPCOMM_LOG_WARN("MPComm[ib]: %s has no usable GID at index %d, skipped\n", name_.c_str(),
                            gid_index_);
            return;
        }
        pd_ = api_->alloc_pd(ctx_);
        cq_ = pd_ ? api_->create_cq(ctx_, 4096, nullptr, nullptr, 0) : nullptr;
        numa_ = topo::ib_numa_node(name_);
        pci_path_ = topo::ib_realpath(name_);
        ok_ = pd_ && cq_;
    }
    ~IbRail() override {
        if (cq_) api_->destroy_cq(cq_);
        if (pd_) api_->dealloc_pd(pd_);
        if (ctx_) api_->close_device(ctx_);
    }
    bool ok() const { return ok_; }
    const std::string &name() const override { return name_; }
    std::string gid() const override { return gid_to_string(gid_); }
    uint16_t lid() const override { return lid_; }
    int numa_node() const override { return numa_; }
    std::string pci_path() const override { return pci_path_; }
    bool port_active() const override {
        ibv::PortAttr pa;
        std::memset(&pa, 0, sizeof(pa));
        return api_->query_port(ctx_, port_, &pa) == 0 && pa.state == ibv::kPortActive;
    }

    int register_memory(void *addr, size_t len, MemKey *out) override {
        const int access = ibv::kAccessLocalWrite | ibv::kAccessRemoteRead | ibv::kAccessRemoteWrite;
        ibv::Mr *mr = nullptr;
        gpu::PtrInfo pi;
        if (gpu::query_pointer(addr, &pi) && pi.is_device && api_->reg_dmabuf_mr) {
            using HandleFn = CUresult (*)(void *, CUdeviceptr, size_t, CUmemRangeHandleType,
                                          unsigned long long);
            auto fn = reinterpret_cast<HandleFn>(gpu::driver_symbol("cuMemGetHandleForAddressRange"));
            // Export the whole allocation (the driver refuses sub-ranges of a
            // cudaMalloc allocation on this platform) and register the
            // buffer at its offset in it; 64 KiB-aligned span otherwise.
            const uintptr_t page = 64 * 1024;
            uintptr_t a0 = reinterpret_cast<uintptr_t>(addr) & ~(page - 1);
            size_t span = ((reinterpret_cast<uintptr_t>(addr) + len + page - 1) & ~(page - 1)) - a0;
            if (pi.base && pi.size && pi.base <= reinterpret_cast<uintptr_t>(addr) &&
                reinterpret_cast<uintptr_t>(addr) + len <= pi.base + pi.size) {
                a0 = pi.base;
                span = pi.size;
            }
            int fd = -1;
            // flags 0, then 1 (CU_MEM_RANGE_FLAG_DMA_BUF_MAPPING_TYPE_PCIE, CUDA 12.8+: a
            // PCIe BAR1 mapping, which some platforms require for NIC access).
            bool exported = false;
            for (unsigned long long flags = 0; fn && !exported && flags <= 1; ++flags)
                exported = fn(&fd, static_cast<CUdeviceptr>(a0), span, CU_MEM_RANGE_HANDLE_TYPE_DMA_BUF_FD,
                              flags) == CUDA_SUCCESS;
            if (exported) {
                mr = api_->reg_dmabuf_mr(pd_, reinterpret_cast<uintptr_t>(addr) - a0, len,
                                         reinterpret_cast<uintptr_t>(addr), fd, access);
                ::close(fd);
            }
        }
        if (!mr) mr = api_->reg_mr(pd_, addr, len, access);  // host memory, or nvidia-peermem
        if (!mr) {
            MPCOMM_PLOG_ERROR("MPComm[ib]: ibv_reg_mr(%p, %zu) on %s failed", addr, len, name_.c_str());
            return MPCOMM_ERR_MEMORY;
        }
        std::lock_guard<std::mutex> g(mu_);
        mrs_[mr->lkey] = mr;
        out->lkey = mr->lkey;
        out->rkey = mr->rkey;
        return 0;
    }
    int deregister_memory(void *, const MemKey &k) override {
        std::lock_guard<std::mutex> g(mu_);
        auto it = mrs_.find(k.lkey);
        if (it == mrs_.end()) return MPCOMM_ERR_INVALID_ARG;
        api_->dereg_mr(it->second);
        mrs_.erase(it);
        return 0;
    }
    std::unique_ptr<QueuePair> create_qp() override {
        ibv::QpInitAttr a;
        std::memset(&a, 0, sizeof(a));
        a.send_cq = cq_;
        a.recv_cq = cq_;
        a.qp_type = ibv::kQptRc;
        a.sq_sig_all = 0;
        a.cap.max_send_wr = static_cast<uint32_t>(cfg_.max_send_wr);
        a.cap.max_recv_wr = 1;
        a.cap.max_send_sge = 1;
        a.cap.max_recv_sge = 1;
        ibv::Qp *qp = api_->create_qp(pd_, &a);
        if (!qp) {
            MPCOMM_PLOG_ERROR("MPComm[ib]: ibv_create_qp on %s failed", name_.c_str());
            return nullptr;
        }
        return std::make_unique<IbQp>(this, qp);
    }
    int poll(WorkCompletion *out, int max) override {
        ibv::Wc wc[64];
        int total = 0;
        while (total < max) {
            int want = std::min(max - total, 64);
            int n = ibv::poll_cq(cq_, want, wc);
            if (n <= 0) break;
            for (int i = 0; i < n; ++i)
                out[total++] = WorkCompletion{wc[i].wr_id, static_cast<int>(wc[i].status), wc[i].byte_len};
            if (n < want) break;
        }
        return total;
    }

    const ibv::Api *api_;
    const Config &cfg_;
    uint8_t port_ = 1;
    int gid_index_ = 3;
    ibv::Gid gid_{};

 private:
    std::string name_, pci_path_;
    ibv::Context *ctx_ = nullptr;
    ibv::Pd *pd_ = nullptr;
    ibv::Cq *cq_ = nullptr;
    uint16_t lid_ = 0;
    int numa_ = -1;
    bool ok_ = false;
    std::mutex mu_;
    std::map<uint32_t, ibv::Mr *> mrs_;
};

IbQp::~IbQp() { rail_->api_->destroy_qp(qp_); }

int IbQp::to_init() {
    ibv::QpAttr a;
    std::memset(&a, 0, sizeof(a));
    a.qp_state = ibv::kQpsInit;
    a.port_num = rail_->port_;
    a.pkey_index = 0;
    a.qp_access_flags =
        ibv::kAccessLocalWrite | ibv::kAccessRemoteRead | ibv::kAccessRemoteWrite | ibv::kAccessRemoteAtomic;
    if (rail_->api_->modify_qp(qp_, &a, ibv::kQpState | ibv::kQpPkeyIndex | ibv::kQpPort | ibv::kQpAccessFlags))
        return MPCOMM_ERR_CONNECTION;
    state_ = QpState::kInit;
    return 0;
}

int IbQp::to_rtr(const EndpointInfo &remote) {
    ibv::QpAttr a;
    std::memset(&a, 0, sizeof(a));
    a.qp_state = ibv::kQpsRtr;
    a.path_mtu = ibv::kMtu4096;
    a.dest_qp_num = remote.qp_num;
    a.rq_psn = 0;
    a.max_dest_rd_atomic = 16;
    a.min_rnr_timer = 12;
    if (!string_to_gid(remote.gid, &a.ah_attr.grh.dgid)) return MPCOMM_ERR_CONNECTION;
    a.ah_attr.grh.sgid_index = static_cast<uint8_t>(rail_->gid_index_);
    a.ah_attr.grh.hop_limit = 16;
    a.ah_attr.grh.traffic_class = static_cast<uint8_t>(rail_->cfg_.roce_dscp << 2);
    a.ah_attr.dlid = remote.lid;
    a.ah_attr.is_global = 1;
    a.ah_attr.port_num = rail_->port_;
    if (rail_->api_->modify_qp(qp_, &a,
                               ibv::kQpState | ibv::kQpAv | ibv::kQpPathMtu | ibv::kQpDestQpn |
                                   ibv::kQpRqPsn | ibv::kQpMaxDestRdAtomic | ibv::kQpMinRnrTimer)) {
        MPCOMM_PLOG_ERROR("MPComm[ib]: QP %u -> RTR failed (remote %s qpn %u)", qp_->qp_num,
                          remote.gid.c_str(), remote.qp_num);
        return MPCOMM_ERR_CONNECTION;
    }
    remote_ = remote;
    state_ = QpState::kRtr;
    return 0;
}

int IbQp::to_rts() {
    ibv::QpAttr a;
    std::memset(&a, 0, sizeof(a));
    a.qp_state = ibv::kQpsRts;
    a.timeout = 14;
    a.retry_cnt = 7;
    a.rnr_retry = 7;
    a.sq_psn = 0;
    a.max_rd_atomic = 16;
    if (rail_->api_->modify_qp(qp_, &a,
                               ibv::kQpState | ibv::kQpTimeout | ibv::kQpRetryCnt | ibv::kQpRnrRetry |
                                   ibv::kQpSqPsn | ibv::kQpMaxQpRdAtomic))
        return MPCOMM_ERR_CONNECTION;
    if (UdpSportFn fn = udp_sport_fn(rail_->name())) {
        static std::atomic<uint32_t> k{0};
        if (fn(qp_, udp_sport_for(k.fetch_add(1))) != 0)
            MPCOMM_LOG_DEBUG("MPComm[ib]: UDP source port not set on %s\n", rail_->name().c_str());
    }
    state_ = QpState::kRts;
    return 0;
}

int IbQp::to_err() {
    ibv::QpAttr a;
    std::memset(&a, 0, sizeof(a));
    a.qp_state = ibv::kQpsErr;
    if (rail_->api_->modify_qp(qp_, &a, ibv::kQpState)) return MPCOMM_ERR_CONNECTION;
    state_ = QpState::kErr;
    return 0;
}

int IbQp::recover() {
    ibv::QpAttr a;
    std::memset(&a, 0, sizeof(a));
    a.qp_state = ibv::kQpsReset;
    if (rail_->api_->modify_qp(qp_, &a, ibv::kQpState)) return MPCOMM_ERR_CONNECTION;
    state_ = QpState::kReset;
    EndpointInfo r = remote_;
    if (to_init() || to_rtr(r) || to_rts()) return MPCOMM_ERR_CONNECTION;
    return 0;
}

int IbQp::post(const WorkRequest *wrs, size_t n) {
    if (n == 0) return 0;
    std::vector<ibv::SendWr> w(n);
    std::vector<ibv::Sge> s(n);
    std::memset(w.data(), 0, n * sizeof(ibv::SendWr));
    for (size_t i = 0; i < n; ++i) {
        s[i].addr = wrs[i].local_addr;
        s[i].length = wrs[i].length;
        s[i].lkey = wrs[i].lkey;
        w[i].wr_id = wrs[i].wr_id;
        w[i].next = i + 1 < n ? &w[i + 1] : nullptr;
        w[i].sg_list = &s[i];
        w[i].num_sge = 1;
        w[i].opcode = wrs[i].op == Opcode::kWrite ? ibv::kWrRdmaWrite : ibv::kWrRdmaRead;
        w[i].send_flags = ibv::kSendSignaled;
        w[i].wr.remote_addr = wrs[i].remote_addr;
        w[i].wr.rkey = wrs[i].rkey;
    }
    ibv::SendWr *bad = nullptr;
    return ibv::post_send(qp_, w.data(), &bad) == 0 ? 0 : MPCOMM_ERR_TRANSFER;
}

class IbBackend final : public Backend {
 public:
    const char *name() const override { return "ib"; }
    int open(const Config &cfg, const std::vector<std::string> &filter,
             std::vector<std::unique_ptr<Rail>> *rails) override {
        const ibv::Api *api = ibv::load();
        if (!api) {
            MPCOMM_LOG_ERROR("MPComm[ib]: libibverbs not available\n");
            return MPCOMM_ERR_DEVICE;
        }
        int n = 0;
        ibv::Device **list = api->get_device_list(&n);
        if (!list) return MPCOMM_ERR_DEVICE;
        for (int i = 0; i < n; ++i) {
            std::string nm = api->get_device_name(list[i]);
            if (!filter.empty()) {
                bool ok = false;
                for (auto &f : filter) ok |= (f == nm);
                if (!ok) continue;
            }
            auto r = std::make_unique<IbRail>(api, list[i], cfg);
            if (r->ok()) rails->push_back(std::move(r));
        }
        api->free_device_list(list);
        return rails->empty() ? MPCOMM_ERR_DEVICE : MPCOMM_SUCCESS;
    }
};

}  // namespace

bool ib_available() {
    static const bool ok = [] {
        if (topo::ib_device_names().empty() && !std::getenv("MPCOMM_IBVERBS_LIB")) return false;
        return ibv::load() != nullptr;
    }();
    return ok;
}

std::unique_ptr<Backend> make_ib_backend() { return std::make_unique<IbBackend>(); }

}  // namespace fabric
}  // namespace mpcomm
