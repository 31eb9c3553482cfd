// Fabric backends: the data-plane contract the transfer engine drives.
//
// The engine is written against RDMA RC semantics (the reference drives
// ibverbs directly, src/mpcomm.cpp:3850-3976, 6808-6840, 7213-7357): a rail
// (NIC) owns a completion queue and memory registrations; queue pairs are
// connected pairwise through endpoint info exchanged on the TCP control
// plane; a posted one-sided WRITE/READ produces exactly one completion
// carrying its wr_id. Every backend here honours that contract, so the
// engine, handshake and buffer registry are backend-agnostic:
//
//   lo   in-process loopback rails (memcpy by a per-rail engine thread)
//   sock software RDMA over TCP between processes (per-rail server thread)
//   nvl  B200 GPU fabric: one rail per GPU; WRs batched into launches of the
//        sm_100a bulk-copy kernel over HBM / NVLink peers / mapped host DRAM
//   ib   ibverbs RC (libibverbs loaded with dlopen at runtime)
#ifndef MPCOMM_B200_CSRC_TRANSPORT_FABRIC_H_
#define MPCOMM_B200_CSRC_TRANSPORT_FABRIC_H_

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "core/config.h"

namespace mpcomm {
namespace fabric {

enum class Opcode : uint8_t { kWrite = 0, kRead = 1 };

// Completion status values mirror ibv_wc_status numbering for the codes the
// engine distinguishes, so logs read the same across backends.
enum WcStatus : int {
    kWcSuccess = 0,
    kWcLocProtErr = 4,
    kWcFlushErr = 5,
    kWcRemAccessErr = 10,
    kWcRetryExcErr = 12,
    kWcGeneralErr = 21,
};

struct WorkRequest {
    uint64_t wr_id;
    Opcode op;
    uintptr_t local_addr;
    uint32_t lkey;
    uintptr_t remote_addr;
    uint32_t rkey;
    uint32_t length;
};

struct WorkCompletion {
    uint64_t wr_id;
    int status;
    uint32_t byte_len;
};

// Address of one QP as carried by the handshake's RemoteEndpointInfo.
struct EndpointInfo {
    std::string gid;
    uint16_t lid = 0;
    uint32_t qp_num = 0;
};

enum class QpState { kReset, kInit, kRtr, kRts, kErr };

class QueuePair;

// A WRITE whose source is a list of pages of a pool (host DRAM mapped for
// the device, or device memory): page i = pool + indices[i] * page_bytes,
// written contiguously from remote_addr. `indices` is device memory of the
// rail's GPU and stays valid until the completion.
struct PagedWrite {
    uint64_t wr_id;
    uintptr_t pool;
    uint64_t pool_pages;     // index bound (0 = unchecked)
    const int64_t *indices;
    uint32_t count;
    uint32_t page_bytes;
    uintptr_t remote_addr;
    uint32_t rkey;
    void *h2d_window;        // kern::H2DWindow of a host pool read (may be null)
};

// One destination of a one-to-many WRITE (post_fanout): the QP of that
// destination's connection (on the same local rail as the posting QP), the
// remote address and its rkey.
struct FanoutTarget {
    QueuePair *qp;
    uintptr_t remote_addr;
    uint32_t rkey;
};

struct MemKey {
    uint32_t lkey = 0;
    uint32_t rkey = 0;
};

class QueuePair {
 public:
    virtual ~QueuePair() = default;
    virtual uint32_t qp_num() const = 0;
    virtual QpState state() const = 0;
    virtual int to_init() = 0;
    virtual int to_rtr(const EndpointInfo &remote) = 0;
    virtual int to_rts() = 0;
    // Moves the QP to ERR: outstanding and future WRs complete with
    // kWcFlushErr (fault injection, host side).
    virtual int to_err() = 0;
    // RESET -> INIT -> RTR -> RTS against the remote saved by to_rtr().
    virtual int recover() = 0;
    // Queues WRs; returns 0 or a negative MPCommError (nothing queued).
    virtual int post(const WorkRequest *wrs, size_t n) = 0;
    // Rings the doorbell for everything posted since the last flush. For
    // the nvl backend this is where a kernel launch happens.
    virtual void flush() {}
    // One-to-many WRITE: wr.length bytes at wr.local_addr (wr.lkey) to every
    // target, moved by ONE device operation that reads the source once
    // (wr.remote_addr and wr.rkey are ignored). One completion carries
    // wr.wr_id, on this QP's rail. Only rails with max_fanout() >= n accept
    // it; others return MPCOMM_ERR_INVALID_ARG and queue nothing.
    // `h2d_window` (a kern::H2DWindow, may be null) is the QoS window the
    // device operation opens and closes when its source is host memory.
    virtual int post_fanout(const WorkRequest & /*wr*/, const FanoutTarget * /*targets*/, size_t /*n*/,
                            void * /*h2d_window*/) {
        return -7;  // MPCOMM_ERR_INVALID_ARG
    }
    // Paged WRITE (gather from a pool + write to the peer in one device
    // operation; one completion carrying w.wr_id). Rails without
    // supports_paged() return MPCOMM_ERR_INVALID_ARG.
    virtual int post_paged(const PagedWrite & /*w*/) { return -7; }
};

class Rail {
 public:
    virtual ~Rail() = default;
    virtual const std::string &name() const = 0;
    virtual std::string gid() const = 0;
    virtual uint16_t lid() const { return 0; }
    virtual int numa_node() const = 0;
    // sysfs realpath of the device (PCIe-affinity by longest common prefix).
    virtual std::string pci_path() const { return std::string(); }
    // GPU ordinal served by this rail (nvl) or -1.
    virtual int gpu_ordinal() const { return -1; }
    virtual bool port_active() const { return true; }
    virtual int register_memory(void *addr, size_t len, MemKey *out) = 0;
    virtual int deregister_memory(void *addr, const MemKey &key) = 0;
    virtual std::unique_ptr<QueuePair> create_qp() = 0;
    // Non-blocking; returns the number of completions written.
    virtual int poll(WorkCompletion *out, int max) = 0;
    // Chunk size and per-QP depth this rail moves efficiently.
    virtual size_t preferred_chunk(const Config &cfg) const { return cfg.max_rdma_transfer_size; }
    virtual size_t preferred_outstanding(const Config &cfg) const {
        return cfg.max_outstanding_per_qp;
    }
    // Routes kernel launches (nvl) into a caller stream; others ignore it.
    virtual int set_stream(void * /*stream*/) { return 0; }
    // True when QPs of this rail accept post_paged.
    virtual bool supports_paged() const { return false; }
    // Largest number of destinations one post_fanout may carry (0 = none).
    virtual size_t max_fanout() const { return 0; }
    // Source and destination alignment a one-to-many WRITE needs (bytes).
    virtual size_t fanout_alignment() const { return 1; }
    // Marks the registration `key` (covering [uc_addr, uc_addr + len)) as
    // this process's copy of an NVLS multicast group: `mc_addr` is this
    // process's mapping of the group's multicast address for offset 0 of
    // uc_addr, `token` names the group across processes, `members` counts
    // the GPUs bound to it. A one-to-many WRITE whose destinations are
    // exactly the group's other members (at one common offset) is then
    // issued as multicast stores. Unsupported rails return
    // MPCOMM_ERR_INVALID_ARG.
    virtual int set_multicast(const MemKey & /*key*/, uintptr_t /*uc_addr*/, size_t /*len*/, uintptr_t /*mc_addr*/,
                              uint64_t /*token*/, int /*members*/) {
        return -7;
    }
    // Device QoS gate for H2D copies (nvl): while *gate != 0 the rail's copy
    // kernels pause before each tile, at most budget_ns per pipeline.
    // Null disables it. Other fabrics ignore it.
    virtual void set_qos_gate(const uint32_t * /*gate*/, uint64_t /*budget_ns*/) {}
};

class Backend {
 public:
    virtual ~Backend() = default;
    virtual const char *name() const = 0;
    // Opens rails, honouring `filter` (empty = all). Returns 0 or an error.
    virtual int open(const Config &cfg, const std::vector<std::string> &filter,
                     std::vector<std::unique_ptr<Rail>> *rails) = 0;
};

std::unique_ptr<Backend> make_loopback_backend();
std::unique_ptr<Backend> make_sock_backend();
std::unique_ptr<Backend> make_nvl_backend();
std::unique_ptr<Backend> make_ib_backend();
// True when at least one ibverbs device is present and libibverbs loads.
bool ib_available();
// Number of CUDA devices visible (0 without driver/GPU).
int nvl_device_count();

}  // namespace fabric
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_TRANSPORT_FABRIC_H_
