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

struct SendWr {
    uint64_t wr_id;
    SendWr *next;
    Sge *sg_list;
    int num_sge;
    uint32_t opcode;
    uint32_t send_flags;
    uint32_t imm_data;
    struct {
        uint64_t remote_addr;
        uint32_t rkey;
        uint32_t pad_rdma;
        uint64_t pad_atomic[2];
    } wr;
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
