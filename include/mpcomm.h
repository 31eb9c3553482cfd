// mpcomm — memory-pool communication for Blackwell (B200, sm_100a) systems.
//
// Public C++ API. Class, enum, struct and method names and signatures follow
// UCL-MPComm's `mpcomm::MPComm` (reference include/mpcomm.h:30-625) so that
// code written against it compiles unchanged; behaviour differences and B200
// extensions are documented beside each declaration.
//
// Data plane. A transfer is split into chunks; each chunk is one work request
// (WR) posted to a "rail" (a NIC in RDMA terms) and one of its queue pairs.
// Rails come from a pluggable fabric backend chosen at init():
//   * "nvl"  — B200 GPU fabric: one rail per visible GPU. A WR is moved by a
//              hand-written sm_100a bulk-copy kernel between HBM, peer HBM
//              (NVLink/NVSwitch, CUDA IPC mapped) and pinned host DRAM (PCIe).
//   * "lo"   — in-process loopback rails (host memory only; CPU memcpy).
//   * "sock" — software RDMA over TCP between processes (host memory).
//   * "ib"   — ibverbs RC one-sided WRITE/READ (dlopen'd libibverbs).
// Selection: MPCOMM_FABRIC=nvl|lo|sock|ib|auto (default auto: ib when verbs
// devices exist, else nvl when a GPU exists, else lo+sock).
#ifndef MPCOMM_B200_INCLUDE_MPCOMM_H_
#define MPCOMM_B200_INCLUDE_MPCOMM_H_

#include <stddef.h>
#include <stdint.h>

#include <memory>
#include <string>
#include <vector>

namespace mpcomm {

// ---------------------------------------------------------------------------
// Error codes (values identical to reference include/mpcomm.h:30-41).
// ---------------------------------------------------------------------------
enum MPCommError {
    MPCOMM_SUCCESS = 0,
    MPCOMM_ERR_DEVICE = -1,
    MPCOMM_ERR_CONTEXT = -2,
    MPCOMM_ERR_MEMORY = -3,
    MPCOMM_ERR_CONNECTION = -4,
    MPCOMM_ERR_TRANSFER = -5,
    MPCOMM_ERR_TIMEOUT = -6,
    MPCOMM_ERR_INVALID_ARG = -7,
    MPCOMM_ERR_INVALID_HANDLE = -8,
    MPCOMM_ERR_PENDING = -9,
};

using TransferHandle = uint64_t;
struct MulticastGroup;  // defined after MPComm
static constexpr TransferHandle INVALID_TRANSFER_HANDLE = 0;

// H2D kernel selection for tmaGather/tmaScatter (values as reference
// include/mpcomm.h:63-67).
//   AUTO - bulk-copy (TMA) pipeline when every block address is 16-byte
//          aligned and block_size % 16 == 0, else the vector SM kernel.
//   SM   - vector LDG/STG kernel, one warp per block; any alignment.
//   TMA  - cp.async.bulk pipeline through shared memory; needs 16-byte
//          alignment (returns MPCOMM_ERR_INVALID_ARG otherwise, never falls
//          back silently).
enum H2DMode {
    H2D_MODE_AUTO = 0,
    H2D_MODE_SM = 1,
    H2D_MODE_TMA = 2,
};

// Real defaults (the reference header's prose and constants disagree; these
// are the values the library uses).
static constexpr size_t MPCOMM_DEFAULT_MAX_RDMA_TRANSFER_SIZE = 128ULL << 10;
static constexpr size_t MPCOMM_DEFAULT_QPS_PER_CONNECTION = 4;
static constexpr size_t MPCOMM_DEFAULT_MAX_OUTSTANDING_PER_QP = 2;
static constexpr int MPCOMM_DEFAULT_GID_INDEX = 3;
// GPU-fabric rails move far larger chunks per WR: one WR is one slice of a
// kernel launch, and a launch must be long enough to hide ~4 us of launch
// latency at NVLink/HBM bandwidth.
static constexpr size_t MPCOMM_DEFAULT_NVL_CHUNK_SIZE = 32ULL << 20;
static constexpr size_t MPCOMM_DEFAULT_NVL_OUTSTANDING_PER_QP = 4;

struct NumaTopology {
    int numa_node;
    std::vector<std::string> local_nics;
    std::vector<std::string> remote_nics;
};

struct NicTopologyInfo {
    std::string nic_name;
    int numa_node;
};

struct RemoteBufferEntry {
    uint64_t addr;
    uint64_t length;
    int numa_node;
    int gpu_device_id = -1;
    std::vector<size_t> pcie_affine_nic_indices;
    std::vector<uint32_t> rkeys;
};

struct PublishedBufferEntry {
    uint64_t addr;
    uint64_t length;
    int numa_node;
    int gpu_device_id = -1;
    std::vector<size_t> pcie_affine_nic_indices;
    std::vector<uint32_t> rkeys;
};

struct PublishedBufferInfo {
    std::vector<PublishedBufferEntry> buffers;
};

struct RemoteBufferInfo {
    std::string host_id;
    std::vector<RemoteBufferEntry> buffers;
};

struct TransferResult {
    int error_code;
    size_t bytes_transferred;
    double elapsed_ms;
};

class MPComm {
 public:
    MPComm();
    ~MPComm();
    MPComm(const MPComm &) = delete;
    MPComm &operator=(const MPComm &) = delete;
    MPComm(MPComm &&) noexcept;
    MPComm &operator=(MPComm &&) noexcept;

    // ---- lifecycle / memory -------------------------------------------
    // init() opens the fabric's rails, binds the TCP control listener
    // (tcp_port 0 = ephemeral), discovers topology and starts one worker per
    // NUMA node. Unlike the reference, init() succeeds without any RDMA NIC:
    // the H2D API needs no rail at all.
    int init(const std::string &local_host_id,
             const std::string &device_names = "",
             int tcp_port = 0);
    void shutdown();
    int registerMemory(void *addr, size_t length);
    int unregisterMemory(void *addr);

    // ---- control plane -------------------------------------------------
    int connect(const std::string &remote_host_id,
                const std::string &remote_tcp_addr,
                int remote_tcp_port);
    int startAcceptThread();
    void stopAcceptThread();
    int updateRemoteMemoryInfo(const std::string &remote_host_id,
                               const std::vector<uint32_t> &rkeys);
    int publishBuffer(void *addr, size_t length, int numa_node = -1);
    int unpublishBuffer(void *addr);
    void unpublishAllBuffers();
    int queryRemoteBuffer(const std::string &remote_host_id,
                          const std::string &remote_tcp_addr,
                          int remote_tcp_port,
                          RemoteBufferInfo &out_info);
    int queryRemoteBufferByNuma(const std::string &remote_host_id,
                                const std::string &remote_tcp_addr,
                                int remote_tcp_port,
                                int numa_node,
                                RemoteBufferEntry &out_entry);
    // Returns a snapshot owned by this object; valid until the next
    // publish/unpublish call (the reference returned a live pointer read
    // without a lock).
    const PublishedBufferInfo *getPublishedBufferInfo() const;
    size_t getPublishedBufferCount() const;
    uint32_t getRkey(size_t nic_index, void *addr) const;

    // ---- async transfers -----------------------------------------------
    // A local buffer that is not registered is moved through the two-stage
    // staging pool (multi-threaded copy into registered slabs, then the
    // zero-copy engine) unless MPCOMM_STAGING_ENABLE=0.
    TransferHandle scatterAsync(uintptr_t local_addr,
                                const std::vector<std::string> &host_list,
                                const std::vector<uintptr_t> &remote_addrs,
                                const std::vector<size_t> &lengths);
    TransferHandle gatherAsync(uintptr_t local_addr,
                               const std::vector<std::string> &host_list,
                               const std::vector<uintptr_t> &remote_addrs,
                               const std::vector<size_t> &lengths);
    TransferHandle broadcastAsync(uintptr_t local_addr, size_t length,
                                  const std::vector<std::string> &host_list,
                                  const std::vector<uintptr_t> &remote_addrs);
    TransferHandle putAsync(uintptr_t local_addr,
                            const std::string &remote_host_id,
                            uintptr_t remote_addr, size_t length);
    TransferHandle getAsync(uintptr_t local_addr,
                            const std::string &remote_host_id,
                            uintptr_t remote_addr, size_t length);
    bool isTransferComplete(TransferHandle handle);
    int waitTransfer(TransferHandle handle, int timeout_ms = -1);
    TransferResult getTransferResult(TransferHandle handle);
    void releaseTransfer(TransferHandle handle);

    // ---- introspection -------------------------------------------------
    size_t getNumNics() const;
    const std::string &getLocalHostId() const;
    int getTcpPort() const;
    std::string getGid(size_t nic_index) const;
    std::string getDeviceName(size_t nic_index) const;
    std::vector<std::string> getActiveDevices() const;
    static const char *getNicFilterEnvVarName();
    size_t getMaxRdmaTransferSize() const;

    // ---- QoS / throttle ------------------------------------------------
    void setNicThrottle(size_t max_outstanding_per_qp, size_t chunk_size);
    void clearNicThrottle();
    // H2D-window QoS: while a tmaGather/tmaScatter kernel of this process is
    // running on GPU g (window opened and closed by the kernel itself through
    // host-mapped flags), new posts of GATHER/READ chunks on rails that are
    // PCIe-affine to g are paused (rate 0) or paced by a shared token bucket.
    void enableH2DQoS(uint64_t rate_bytes_per_sec = 0, uint64_t burst_bytes = 0);
    void setH2DQoSPolicy(uint64_t rate_bytes_per_sec, uint64_t burst_bytes = 0);
    bool isH2DQoSEnabled() const;
    // Extension: device timestamps (%globaltimer, ns) of the most recently
    // closed H2D window on GPU `gpu`: first CTA start and last CTA end of a
    // tmaGather/tmaScatter launched while QoS was enabled. False if none.
    bool getLastH2DWindow(int gpu, uint64_t *begin_ns, uint64_t *end_ns) const;

    // QoS control channel (extension; the reference's wire format, which it
    // declares but never opens). openQosChannel(host) connects to a host
    // this object connect()ed to; policies sent over it make that host
    // defer (rate 0) or pace its RDMA WRITEs into this host's GPU `gpu`
    // (-1 = any) until cleared or until the channel closes (fail-open).
    // With MPCOMM_QOS_REMOTE=1 each QoS-windowed tmaGather/tmaScatter sends
    // the enableH2DQoS rate to every open channel and clears it when its
    // H2D window closes.
    int openQosChannel(const std::string &host_id);
    int closeQosChannel(const std::string &host_id);
    int sendQosPolicy(const std::string &host_id, int gpu, uint64_t rate_bytes_per_sec, uint64_t burst_bytes = 0);
    int clearQosPolicy(const std::string &host_id, int gpu = -1);
    struct RemoteQosPolicy {
        std::string peer_host_id;
        int gpu_device_id;
        uint64_t rate_bytes_per_sec;
        uint64_t burst_bytes;
        uint64_t generation;
    };
    // Policies peers have sent to this object, and how many WRITE chunk
    // posts they deferred so far.
    std::vector<RemoteQosPolicy> getRemoteQosPolicies() const;
    uint64_t getRemoteQosDeferCount() const;
    void disableH2DQoS();
    uint64_t getNicCompletedBytes() const;
    // Extension: completed bytes per rail, in getActiveDevices() order (how
    // striping spread the traffic, e.g. over the PXN proxy rails).
    std::vector<uint64_t> getRailCompletedBytes() const;

    struct PcieDomainStats {
        int gpu_device_id;
        uint64_t posted_bytes;
        uint64_t completed_bytes;
        uint64_t in_flight_bytes;
        uint64_t in_flight_bytes_max;
        uint64_t post_count;
        uint64_t defer_count;
    };
    std::vector<PcieDomainStats> getPcieDomainStats() const;
    void resetPcieDomainStats();
    bool isPcieDomainStatEnabled() const;
    static const char *getPcieStatEnableEnvVarName();
    bool getThrottleLatency(uint64_t *set_ns, uint64_t *worker_seen_ns,
                            uint64_t *drained_ns,
                            size_t *snapshot_outstanding_wqes) const;
    size_t getQpsPerConnection() const;
    static const char *getQpsPerConnectionEnvVarName();

    // ---- topology ------------------------------------------------------
    // GPU <-> rail PCIe affinity self-check (extension; the reference prints
    // it at init, src/mpcomm.cpp:3192-3251): for every visible GPU, the
    // rails sysfs places under the same PCIe switch (used for PCIe-domain
    // accounting and rail choice) beside the rail the name-suffix heuristic
    // would pick (suffix N serves GPU N), and whether they agree. Logged at
    // INFO by init(); empty without GPUs.
    struct PcieAffinityCheck {
        int gpu_device_id;
        std::vector<std::string> sysfs_rails;
        std::string suffix_rail;  // empty when no rail has suffix N
        bool agrees;
    };
    std::vector<PcieAffinityCheck> getPcieAffinitySelfCheck() const;
    const std::vector<NumaTopology> &getNumaTopology() const;
    const std::vector<NicTopologyInfo> &getNicTopology() const;
    int getNicNumaNode(const std::string &nic_name) const;
    int getNumaNodeForAddr(void *addr) const;
    std::vector<size_t> getLocalNicIndicesForNuma(int numa_node) const;
    int getGpuNumaNode(int gpu_device_id) const;

    // ---- HBM <-> DRAM --------------------------------------------------
    uintptr_t mapDRAMtoGPU(void *host_addr, size_t length);
    int unmapDRAMfromGPU(void *host_addr);
    // Launch on the current device's legacy default stream (reference
    // behaviour) but check the launch and return its error.
    int tmaGather(uintptr_t dram_dev_ptr, const int64_t *indices,
                  void *gpu_dst, int num_blocks, int block_size,
                  int max_sm_count = 0, H2DMode mode = H2D_MODE_AUTO);
    int tmaScatter(void *gpu_src, const int64_t *indices,
                   uintptr_t dram_dev_ptr, int num_blocks, int block_size,
                   int max_sm_count = 0, H2DMode mode = H2D_MODE_AUTO);

    // ---- B200 extensions (no reference counterpart) --------------------
    // Same as tmaGather/tmaScatter on an explicit cudaStream_t.
    int tmaGatherOnStream(uintptr_t dram_dev_ptr, const int64_t *indices,
                          void *gpu_dst, int num_blocks, int block_size,
                          int max_sm_count, H2DMode mode, void *stream);
    int tmaScatterOnStream(void *gpu_src, const int64_t *indices,
                           uintptr_t dram_dev_ptr, int num_blocks,
                           int block_size, int max_sm_count, H2DMode mode,
                           void *stream);
    // Route every GPU-fabric copy kernel of this object into `stream` (a
    // cudaStream_t of the rail's device; nullptr restores the per-QP
    // internal streams). Lets callers bracket transfers with CUDA events.
    int setFabricStream(void *stream);
    // Paged PUT, the fused PXN gather + forward as a transfer: page i =
    // dram_dev_ptr + indices[i] * block_size (a pool mapped with
    // mapDRAMtoGPU, or device memory) is written to remote_addr +
    // i * block_size of `remote_host_id` (a published buffer, typically
    // another GPU's HBM). The GPU that holds `indices` (device memory, kept
    // valid until the transfer completes) gathers the pages into shared
    // memory and stores them straight into the destination over NVLink, one
    // launch per chunk of pages, on its GPU-fabric rail; with H2D QoS on,
    // each launch reading host memory opens a QoS window on that GPU. Use a
    // GPU close to the pool's NUMA node (the reference routes traffic
    // through such a proxy GPU, src/mpcomm.cpp:5135-5403). Tracked like any
    // transfer (waitTransfer, getTransferResult).
    TransferHandle putPagesAsync(uintptr_t dram_dev_ptr, const int64_t *indices, int num_blocks,
                                 int block_size, const std::string &remote_host_id, uintptr_t remote_addr);
    // Number of this library's GPU kernels launched so far (all objects).
    static uint64_t getKernelLaunchCount();
    // Extension: device start/end of recent data-mover launches, from the
    // kernel trace ring (enable with MPCOMM_KERNEL_TRACE=<slots per device>;
    // empty when off). Reading it synchronises with the devices.
    struct KernelTraceRecord {
        uint64_t seq;
        int device;
        std::string kind;
        uint64_t bytes;
        uint64_t begin_ns, end_ns;  // %globaltimer of the device
    };
    static std::vector<KernelTraceRecord> getKernelTrace();
    // Name of the fabric backend in use ("nvl", "lo", "sock", "ib").
    std::string getFabricName() const;
    // Registers this process's copy of an NVLS multicast group buffer (GPU
    // fabric): [uc_addr, uc_addr + length) is bound to the group at offset
    // 0, `mc_addr` is this process's mapping of the group's multicast
    // address, `group_token` (non-zero) names the group in every member
    // process and `group_size` counts its GPUs. Every member registers its
    // copy (then publishes it as usual). A broadcastAsync whose destinations
    // are exactly the group's other members at one common offset is then
    // sent as NVLS multicast stores, one launch per chunk (the switch
    // replicates each store; the source crosses this GPU's NVLinks once).
    // The sending GPU's own copy at that offset receives the bytes too.
    // Broadcasts to other destination sets use one launch per chunk that
    // stores to each destination (up to 8). Both fused forms need 16-byte
    // aligned addresses and lengths; MPCOMM_FUSED_BROADCAST=0 turns them off.
    int registerMulticastMemory(void *uc_addr, size_t length, void *mc_addr, uint64_t group_token,
                                int group_size);
    // registerMulticastMemory for a group formed by createMulticastGroup /
    // joinMulticastGroup (below).
    int registerMulticastGroup(const MulticastGroup &group);

    class Impl;  // opaque implementation type

 private:
    std::unique_ptr<Impl> impl_;
};

// ---------------------------------------------------------------------------
// NVLS multicast groups between processes of one box (B200 extension; no
// launcher or collective library needed). One process creates the group,
// `members - 1` others join it under the same name, in any order and each on
// its current CUDA device; both calls return once every member has bound a
// copy of `bytes` (rounded up to the multicast granularity) and mapped the
// group's multicast address, or fail after `timeout_ms` (the group object is
// handed over an abstract Unix socket named after the group, so every member
// must share the creator's network namespace). Returns MPCOMM_SUCCESS,
// MPCOMM_ERR_DEVICE (a driver call failed, e.g. no multicast support) or
// MPCOMM_ERR_CONNECTION (a member did not arrive, or left, in time).
// ---------------------------------------------------------------------------
struct MulticastGroup {
    void *uc_addr = nullptr;  // this member's copy (publish it like any buffer)
    void *mc_addr = nullptr;  // multicast address: a store here reaches every copy
    size_t length = 0;        // bytes of each copy
    uint64_t token = 0;       // group identity (the same in every member)
    int members = 0;
    int device = -1;
    uint64_t mc_handle = 0, mem_handle = 0;  // driver handles (released by releaseMulticastGroup)
};
int createMulticastGroup(const std::string &name, size_t bytes, int members, MulticastGroup *out,
                         int timeout_ms = 60000);
int joinMulticastGroup(const std::string &name, size_t bytes, int members, MulticastGroup *out,
                       int timeout_ms = 60000);
// Unmaps and releases this member's part (unregister the copy first).
int releaseMulticastGroup(MulticastGroup *group);

}  // namespace mpcomm

#endif  // MPCOMM_B200_INCLUDE_MPCOMM_H_
