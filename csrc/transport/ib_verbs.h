// Minimal ibverbs ABI shim, resolved at run time (dlopen "libibverbs.so.1").
//
// No rdma-core headers are needed to build. The struct layouts below are
// the stable x86-64 ABI of libibverbs (unchanged since the 1.1 ABI): only
// the fields this library touches are declared, and every struct the
// library allocates is over-sized with zeroed padding. ibv_post_send and
// ibv_poll_cq are inline in rdma-core (they dispatch through the context
// ops table), so they are reached the same way here: ops slots 25
// (post_send) and 11 (poll_cq).
#ifndef MPCOMM_B200_CSRC_TRANSPORT_IB_VERBS_H_
#define MPCOMM_B200_CSRC_TRANSPORT_IB_VERBS_H_

#include <cstddef>
#include <cstdint>

namespace mpcomm {
namespace ibv {

struct Device;   // opaque
struct Pd;       // opaque
struct CompChannel;

struct Context {
    Device *device;
    void *ops[32];  // ibv_context_ops (function pointers)
};

struct Cq {
    Context *context;
};

struct Mr {
    Context *context;
    Pd *pd;
    void *addr;
    size_t length;
    uint32_t handle;
    uint32_t lkey;
    uint32_t rkey;
};

struct Qp {
    Context *context;
    void *qp_context;
    Pd *pd;
    Cq *send_cq;
    Cq *recv_cq;
    void *srq;
    uint32_t handle;
    uint32_t qp_num;
    uint32_t state;
    uint32_t qp_type;
};

union Gid {
    uint8_t raw[16];
    struct {
        uint64_t subnet_prefix;
        uint64_t interface_id;
    } global;
};

struct Wc {
    uint64_t wr_id;
    uint32_t status;
    uint32_t opcode;
    uint32_t vendor_err;
    uint32_t byte_len;
    uint32_t imm_data;
    uint32_t qp_num;
    uint32_t src_qp;
    uint32_t wc_flags;
    uint16_t pkey_index;
    uint16_t slid;
    uint8_t sl;
    uint8_t dlid_path_bits;
};
static_assert(sizeof(Wc) == 48, "ibv_wc size");

struct Sge {
    uint64_t addr;
    uint32_t length;
    uint32_t lkey;
};

struct RdmaWr {  // the `rdma` member of ibv_send_wr's wr union, padded to the union's 32 bytes
    uint64_t remote_addr;
    uint32_t rkey;
    uint32_t pad_rdma;
    uint64_t pad_atomic[2];
};

struct SendWr {
    uint64_t wr_id;
    SendWr *next;
    Sge *sg_list;
    int num_sge;
    uint32_t opcode;
    uint32_t send_flags;
    uint32_t imm_data;
    RdmaWr wr;
    uint32_t qp_type_xrc;
    uint32_t pad0;
    unsigned char tail[64];  // bind_mw / tso union
};

struct QpCap {
    uint32_t max_send_wr, max_recv_wr, max_send_sge, max_recv_sge, max_inline_data;
};

struct QpInitAttr {
    void *qp_context;
    Cq *send_cq;
    Cq *recv_cq;
    void *srq;
    QpCap cap;
    uint32_t qp_type;
    int sq_sig_all;
    unsigned char tail[64];
};

struct GlobalRoute {
    Gid dgid;
    uint32_t flow_label;
    uint8_t sgid_index;
    uint8_t hop_limit;
    uint8_t traffic_class;
};

struct AhAttr {
    GlobalRoute grh;
    uint16_t dlid;
    uint8_t sl;
    uint8_t src_path_bits;
    uint8_t static_rate;
    uint8_t is_global;
    uint8_t port_num;
};
static_assert(sizeof(AhAttr) == 32, "ibv_ah_attr size");

struct QpAttr {
    uint32_t qp_state;
    uint32_t cur_qp_state;
    uint32_t path_mtu;
    uint32_t path_mig_state;
    uint32_t qkey;
    uint32_t rq_psn;
    uint32_t sq_psn;
    uint32_t dest_qp_num;
    uint32_t qp_access_flags;
    QpCap cap;
    AhAttr ah_attr;
    AhAttr alt_ah_attr;
    uint16_t pkey_index;
    uint16_t alt_pkey_index;
    uint8_t en_sqd_async_notify;
    uint8_t sq_draining;
    uint8_t max_rd_atomic;
    uint8_t max_dest_rd_atomic;
    uint8_t min_rnr_timer;
    uint8_t port_num;
    uint8_t timeout;
    uint8_t retry_cnt;
    uint8_t rnr_retry;
    uint8_t alt_port_num;
    uint8_t alt_timeout;
    uint32_t rate_limit;
    unsigned char tail[64];
};
static_assert(offsetof(QpAttr, ah_attr) == 56, "ibv_qp_attr.ah_attr offset");
static_assert(offsetof(QpAttr, pkey_index) == 120, "ibv_qp_attr.pkey_index offset");

struct PortAttr {  // ibv_port_attr prefix; buffer over-sized
    uint32_t state;
    uint32_t max_mtu;
    uint32_t active_mtu;
    int gid_tbl_len;
    uint32_t port_cap_flags;
    uint32_t max_msg_sz;
    uint32_t bad_pkey_cntr;
    uint32_t qkey_viol_cntr;
    uint16_t pkey_tbl_len;
    uint16_t lid;
    uint16_t sm_lid;
    uint8_t lmc, max_vl_num, sm_sl, subnet_timeout, init_type_reply, active_width, active_speed,
        phys_state, link_layer, flags;
    unsigned char tail[192];
};

enum : uint32_t {
    kQpsReset = 0, kQpsInit = 1, kQpsRtr = 2, kQpsRts = 3, kQpsErr = 6,
    kQptRc = 2,
    kMtu4096 = 5,
    kAccessLocalWrite = 1, kAccessRemoteWrite = 2, kAccessRemoteRead = 4, kAccessRemoteAtomic = 8,
    kWrRdmaWrite = 0, kWrRdmaRead = 4,
    kSendSignaled = 2,
    kPortActive = 4,
};
enum : int {
    kQpState = 1, kQpAccessFlags = 8, kQpPkeyIndex = 16, kQpPort = 32, kQpAv = 128,
    kQpPathMtu = 256, kQpTimeout = 512, kQpRetryCnt = 1024, kQpRnrRetry = 2048, kQpRqPsn = 4096,
    kQpMaxQpRdAtomic = 8192, kQpMinRnrTimer = 32768, kQpSqPsn = 65536,
    kQpMaxDestRdAtomic = 131072, kQpDestQpn = 1048576,
};

struct Api {
    Device **(*get_device_list)(int *);
    void (*free_device_list)(Device **);
    const char *(*get_device_name)(Device *);
    Context *(*open_device)(Device *);
    int (*close_device)(Context *);
    int (*query_port)(Context *, uint8_t, PortAttr *);
    int (*query_gid)(Context *, uint8_t, int, Gid *);
    Pd *(*alloc_pd)(Context *);
    int (*dealloc_pd)(Pd *);
    Cq *(*create_cq)(Context *, int, void *, CompChannel *, int);
    int (*destroy_cq)(Cq *);
    Mr *(*reg_mr)(Pd *, void *, size_t, int);
    Mr *(*reg_dmabuf_mr)(Pd *, uint64_t, size_t, uint64_t, int, int);  // may be null
    int (*dereg_mr)(Mr *);
    Qp *(*create_qp)(Pd *, QpInitAttr *);
    int (*modify_qp)(Qp *, QpAttr *, int);
    int (*destroy_qp)(Qp *);
};

// Layout checks against rdma-core's infiniband/verbs.h on LP64 (x86-64 and
// aarch64 Linux): the size and the offset of every field this library reads
// or writes. Structs this library allocates (SendWr, QpInitAttr, QpAttr,
// PortAttr) may be larger than the real ones; providers read only the real
// fields.
static_assert(offsetof(Context, ops) == 8, "ibv_context.ops");
static_assert(sizeof(Context::ops) == 32 * sizeof(void *), "ibv_context_ops has 32 slots");
static_assert(offsetof(Cq, context) == 0, "ibv_cq.context");
static_assert(offsetof(Mr, addr) == 16 && offsetof(Mr, length) == 24, "ibv_mr.addr/length");
static_assert(offsetof(Mr, handle) == 32 && offsetof(Mr, lkey) == 36 && offsetof(Mr, rkey) == 40, "ibv_mr keys");
static_assert(sizeof(Mr) == 48, "ibv_mr size");
static_assert(offsetof(Qp, send_cq) == 24 && offsetof(Qp, srq) == 40, "ibv_qp queues");
static_assert(offsetof(Qp, handle) == 48 && offsetof(Qp, qp_num) == 52, "ibv_qp.qp_num");
static_assert(offsetof(Qp, state) == 56 && offsetof(Qp, qp_type) == 60, "ibv_qp.state/qp_type");
static_assert(sizeof(Gid) == 16, "ibv_gid size");
static_assert(offsetof(Wc, status) == 8 && offsetof(Wc, opcode) == 12, "ibv_wc.status/opcode");
static_assert(offsetof(Wc, byte_len) == 20 && offsetof(Wc, qp_num) == 28, "ibv_wc.byte_len/qp_num");
static_assert(offsetof(Wc, wc_flags) == 36 && offsetof(Wc, pkey_index) == 40, "ibv_wc.wc_flags");
static_assert(offsetof(Wc, sl) == 44 && offsetof(Wc, dlid_path_bits) == 45, "ibv_wc tail");
static_assert(sizeof(Sge) == 16 && offsetof(Sge, length) == 8 && offsetof(Sge, lkey) == 12, "ibv_sge");
static_assert(offsetof(SendWr, next) == 8 && offsetof(SendWr, sg_list) == 16, "ibv_send_wr list");
static_assert(offsetof(SendWr, num_sge) == 24 && offsetof(SendWr, opcode) == 28, "ibv_send_wr.opcode");
static_assert(offsetof(SendWr, send_flags) == 32 && offsetof(SendWr, imm_data) == 36, "ibv_send_wr flags");
static_assert(offsetof(SendWr, wr) == 40 && sizeof(RdmaWr) == 32, "ibv_send_wr.wr union");
static_assert(offsetof(RdmaWr, rkey) == 8, "ibv_send_wr.wr.rdma.rkey");
static_assert(offsetof(SendWr, qp_type_xrc) == 72 && offsetof(SendWr, tail) == 80, "ibv_send_wr.qp_type");
static_assert(sizeof(SendWr) >= 128, "ibv_send_wr size (bind_mw member is 48 bytes)");
static_assert(sizeof(QpCap) == 20, "ibv_qp_cap size");
static_assert(offsetof(QpInitAttr, send_cq) == 8 && offsetof(QpInitAttr, srq) == 24, "ibv_qp_init_attr queues");
static_assert(offsetof(QpInitAttr, cap) == 32 && offsetof(QpInitAttr, qp_type) == 52, "ibv_qp_init_attr.cap");
static_assert(offsetof(QpInitAttr, sq_sig_all) == 56 && sizeof(QpInitAttr) >= 64, "ibv_qp_init_attr size");
static_assert(sizeof(GlobalRoute) == 24 && offsetof(GlobalRoute, flow_label) == 16, "ibv_global_route");
static_assert(offsetof(GlobalRoute, sgid_index) == 20 && offsetof(GlobalRoute, traffic_class) == 22,
              "ibv_global_route.traffic_class");
static_assert(offsetof(AhAttr, dlid) == 24 && offsetof(AhAttr, is_global) == 29 && offsetof(AhAttr, port_num) == 30,
              "ibv_ah_attr fields");
static_assert(offsetof(QpAttr, path_mtu) == 8 && offsetof(QpAttr, rq_psn) == 20, "ibv_qp_attr psn");
static_assert(offsetof(QpAttr, sq_psn) == 24 && offsetof(QpAttr, dest_qp_num) == 28, "ibv_qp_attr.dest_qp_num");
static_assert(offsetof(QpAttr, qp_access_flags) == 32 && offsetof(QpAttr, cap) == 36, "ibv_qp_attr.cap");
static_assert(offsetof(QpAttr, alt_ah_attr) == 88, "ibv_qp_attr.alt_ah_attr");
static_assert(offsetof(QpAttr, max_rd_atomic) == 126 && offsetof(QpAttr, max_dest_rd_atomic) == 127,
              "ibv_qp_attr rd_atomic");
static_assert(offsetof(QpAttr, min_rnr_timer) == 128 && offsetof(QpAttr, port_num) == 129, "ibv_qp_attr.port");
static_assert(offsetof(QpAttr, timeout) == 130 && offsetof(QpAttr, retry_cnt) == 131 &&
                  offsetof(QpAttr, rnr_retry) == 132, "ibv_qp_attr retries");
static_assert(offsetof(QpAttr, rate_limit) == 136 && sizeof(QpAttr) >= 144, "ibv_qp_attr size");
static_assert(offsetof(PortAttr, gid_tbl_len) == 12 && offsetof(PortAttr, lid) == 34, "ibv_port_attr.lid");
static_assert(offsetof(PortAttr, active_mtu) == 8 && offsetof(PortAttr, link_layer) == 46, "ibv_port_attr.link_layer");

// Loads libibverbs once; nullptr if unavailable. MPCOMM_IBVERBS_LIB
// overrides the library path (tests load a fake provider through it).
const Api *load();

inline int post_send(Qp *qp, SendWr *wr, SendWr **bad) {
    using Fn = int (*)(Qp *, SendWr *, SendWr **);
    return reinterpret_cast<Fn>(qp->context->ops[25])(qp, wr, bad);
}
inline int poll_cq(Cq *cq, int n, Wc *wc) {
    using Fn = int (*)(Cq *, int, Wc *);
    return reinterpret_cast<Fn>(cq->context->ops[11])(cq, n, wc);
}

}  // namespace ibv
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_TRANSPORT_IB_VERBS_H_
