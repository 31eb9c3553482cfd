// MPComm::Impl — the engine behind the public facade.
//
// Threads:
//   * caller threads: submit transfers (lock-free push into a worker ring),
//     wait/poll, register memory, connect, publish.
//   * one worker per NUMA node (<= kMaxNumaNodes), pinned to that node's
//     CPUs: drains its ring, posts chunks to rails/QPs under flow control
//     and QoS gates, polls completion queues, routes completions by wr_id,
//     retires transfers, probes quarantined rails (worker 0).
//   * the accept thread: connect handshakes, buffer queries, QoS channels.
//   * staging copy threads (non-zero-copy path).
// Parity map (reference src/mpcomm.cpp): submit :4929-5479, worker loop
// :5969-7061, completion routing :7213-7357, completion API :5563-5740,
// quarantine :7068-7155, fault injection :5802-5929, throttle :2375-2401,
// H2D QoS :2403-2622, PCIe domain stats :1091-1212.
#ifndef MPCOMM_B200_CSRC_ENGINE_IMPL_H_
#define MPCOMM_B200_CSRC_ENGINE_IMPL_H_

#include <array>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "core/config.h"
#include "core/core.h"
#include "ctrl/wire.h"
#include "kernels/launch.h"
#include "mpcomm.h"
#include "transport/fabric.h"

namespace mpcomm {

class StagingEngine;

enum class Direction { kScatter, kGather, kBroadcast };

using Clock = std::chrono::steady_clock;

struct RailSlot {
    std::unique_ptr<fabric::Rail> rail;
    std::string name;
    std::string gid;
    int numa = 0;
    int gpu = -1;  // PCIe-affine GPU (nvl: the rail's own GPU)
    std::string pci_path;
    std::atomic<bool> quarantined{false};
    std::atomic<uint64_t> quarantine_since_ns{0};
    std::atomic<uint64_t> completed_bytes{0};
};

struct Region {
    uintptr_t addr = 0;
    size_t len = 0;
    std::vector<fabric::MemKey> keys;  // per rail
    int numa = -1;
    int gpu = -1;
    std::vector<size_t> affine_rails;
};

struct QpGroup {
    size_t local_rail = 0;
    size_t remote_rail = 0;
    std::vector<std::unique_ptr<fabric::QueuePair>> qps;
};

struct Connection {
    std::string host_id;
    std::string tcp_addr;  // control-plane address (active side; empty when accepted)
    int tcp_port = 0;
    std::vector<RemoteEndpointInfo> nic_endpoints;  // indexed by remote rail
    std::vector<int> remote_nic_numa;
    int remote_numa_count = 0;
    std::vector<std::string> remote_nic_names;
    std::map<size_t, std::vector<size_t>> local_to_remote;
    std::map<std::pair<size_t, size_t>, std::unique_ptr<QpGroup>> groups;
    std::map<uint64_t, RemoteBufferEntry> remote_buffers;
    mutable std::mutex mu;  // remote_buffers / endpoint rkeys

    uint32_t rkey_for(uint64_t raddr, size_t remote_rail) const;
    int remote_gpu_for(uint64_t raddr) const;
    QpGroup *group_for(size_t local_rail) const;
};

struct Transfer {
    uint64_t handle = 0;
    uint64_t nvtx = 0;  // NVTX range of the transfer's lifetime (0 = none)
    Direction dir = Direction::kScatter;
    fabric::Opcode op = fabric::Opcode::kWrite;
    uintptr_t local_addr = 0;
    std::vector<std::string> hosts;
    std::vector<uintptr_t> remote_addrs;
    std::vector<size_t> lengths;
    std::vector<std::shared_ptr<Connection>> conns;
    std::vector<int> remote_gpu;  // per host (SCATTER PCIe accounting)
    ChunkPlan plan;
    std::vector<size_t> candidates;
    int numa = 0;
    int local_gpu = -1;
    int owner = 0;  // worker id
    size_t outstanding_limit = 2;
    bool composite = false;  // completion driven by the staging engine
    // Fused broadcast: every chunk is ONE one-to-many WRITE on fanout_rail
    // (plan = the chunks of one destination; each completion covers all).
    bool fanout = false;
    size_t fanout_rail = 0;
    bool host_source = false;  // local buffer in host memory (H2D QoS window)
    // Paged PUT: the source is pages of a pool (indices on the GPU of
    // paged_rail); chunk k covers pages [k * pages_per_chunk, ...).
    bool paged = false;
    size_t paged_rail = 0;
    uintptr_t pool = 0;
    uint64_t pool_pages = 0;
    const int64_t *indices = nullptr;
    uint32_t page_bytes = 0;
    size_t pages_per_chunk = 0;

    // Worker-owned progress.
    size_t next_chunk = 0;
    std::deque<size_t> retry;
    size_t in_flight = 0;
    size_t repost_budget = 0;
    bool aborted = false;
    std::array<fabric::MemKey, kMaxRails> lkeys{};
    std::array<bool, kMaxRails> lkey_ok{};

    std::atomic<size_t> done_chunks{0};
    std::atomic<uint64_t> bytes{0};
    std::array<std::atomic<uint64_t>, kMaxRails> rail_bytes{};
    std::atomic<int> error{0};
    std::atomic<bool> finished{false};
    // bit 0: finished, bit 1: released by the user. Whichever side sets the
    // second bit returns the handle to the pool (in-flight completions never
    // see a recycled handle).
    std::atomic<int> life{0};

    Clock::time_point t_start, t_queued, t_worker, t_first_post, t_all_posted, t_end;
    bool first_posted = false;
};

struct PcieDomain {
    std::atomic<uint64_t> posted{0}, completed{0}, inflight_max{0}, post_count{0}, defer_count{0};
    std::atomic<bool> seen{false};
};

class MPComm::Impl {
 public:
    Impl();
    ~Impl();

    // ---- lifecycle / memory (impl_core.cc) ----
    int init(const std::string &host_id, const std::string &device_names, int tcp_port);
    void shutdown();
    int registerMemory(void *addr, size_t len);
    int registerMulticastMemory(void *uc, size_t len, void *mc, uint64_t token, int members);
    int unregisterMemory(void *addr);
    uint32_t getRkey(size_t nic, void *addr) const;
    bool lookupRegion(uintptr_t addr, size_t len, Region *out) const;

    // ---- control plane (impl_ctrl.cc) ----
    int connect(const std::string &id, const std::string &addr, int port);
    int startAcceptThread();
    void stopAcceptThread();
    int updateRemoteMemoryInfo(const std::string &id, const std::vector<uint32_t> &rkeys);
    int publishBuffer(void *addr, size_t len, int numa);
    int unpublishBuffer(void *addr);
    void unpublishAllBuffers();
    int queryRemoteBuffer(const std::string &id, const std::string &addr, int port,
                          RemoteBufferInfo &out);
    int queryRemoteBufferByNuma(const std::string &id, const std::string &addr, int port, int numa,
                                RemoteBufferEntry &out);
    const PublishedBufferInfo *getPublishedBufferInfo() const;
    size_t getPublishedBufferCount() const;

    // ---- transfers (impl_xfer.cc) ----
    TransferHandle submit(uintptr_t local, const std::vector<std::string> &hosts,
                          const std::vector<uintptr_t> &raddrs, const std::vector<size_t> &lens,
                          Direction dir);
    TransferHandle submitPaged(uintptr_t dram_dev_ptr, const int64_t *indices, int num_blocks, int block_size,
                               const std::string &host, uintptr_t raddr);
    bool isTransferComplete(TransferHandle h);
    int waitTransfer(TransferHandle h, int timeout_ms);
    TransferResult getTransferResult(TransferHandle h);
    void releaseTransfer(TransferHandle h);
    // Composite (staged) transfer plumbing.
    std::shared_ptr<Transfer> newCompositeTransfer(Direction dir, uintptr_t local,
                                                   const std::vector<std::string> &hosts,
                                                   const std::vector<uintptr_t> &raddrs,
                                                   const std::vector<size_t> &lens);
    std::shared_ptr<Transfer> findTransfer(TransferHandle h) const;
    // Marks t finished (error already set) and frees the handle if released.
    void finishTransfer(Transfer *t);
    StagingEngine *staging() { return staging_.get(); }

    // ---- QoS / stats (impl_qos.cc) ----
    void setNicThrottle(size_t outstanding, size_t chunk);
    void clearNicThrottle();
    void enableH2DQoS(uint64_t rate, uint64_t burst);
    void setH2DQoSPolicy(uint64_t rate, uint64_t burst);
    bool isH2DQoSEnabled() const { return h2d_qos_enabled_.load(std::memory_order_acquire); }
    void disableH2DQoS();
    uint64_t getNicCompletedBytes() const { return nic_completed_bytes_.load(); }
    std::vector<uint64_t> railCompletedBytes() const {
        std::vector<uint64_t> v;
        for (const auto &r : rails_) v.push_back(r->completed_bytes.load(std::memory_order_relaxed));
        return v;
    }
    std::vector<MPComm::PcieDomainStats> getPcieDomainStats() const;
    void resetPcieDomainStats();
    bool isPcieDomainStatEnabled() const { return cfg_.pcie_stat_enable; }
    bool getThrottleLatency(uint64_t *set, uint64_t *seen, uint64_t *drained, size_t *snap) const;
    // True while an H2D kernel window is open on GPU `gpu` (device-written).
    bool h2dWindowOpen(int gpu) const;
    bool lastH2DWindow(int gpu, uint64_t *begin_ns, uint64_t *end_ns) const;
    // Arms a window slot for one H2D launch on `gpu`; returns device-visible
    // pointers (nullptr when QoS is off).
    bool acquireH2DWindow(int gpu, kern::H2DWindow **win, uint32_t **ctr);
    bool ensureWindowPoolLocked();
    uint32_t *deviceGateLocked(int gpu);
    void applyDeviceGates();

    // ---- QoS control channel (impl_qos_channel.cc) ----
    int openQosChannel(const std::string &host_id);
    int closeQosChannel(const std::string &host_id);
    int sendQosPolicy(const std::string &host_id, int gpu, uint64_t rate, uint64_t burst, bool clear);
    struct RemoteQosView {
        std::string peer;
        int gpu;
        uint64_t rate, burst, generation;
    };
    std::vector<RemoteQosView> remoteQosPolicies() const;
    uint64_t remoteQosDefers() const { return remote_qos_defers_.load(std::memory_order_relaxed); }
    size_t qosChannelCount() const;

    // ---- H2D (impl_h2d.cc) ----
    uintptr_t mapDRAMtoGPU(void *host, size_t len);
    int unmapDRAMfromGPU(void *host);
    int h2dMove(bool gather, uintptr_t dram, const int64_t *idx, void *gpu_buf, int n, int bs,
                int max_sm, int mode, void *stream);
    int setFabricStream(void *stream);
    void *fabricStream() const { return fabric_stream_; }

    // ---- topology / introspection (impl_core.cc) ----
    size_t numNics() const { return rails_.size(); }
    const std::string &hostId() const { return host_id_; }
    int tcpPort() const { return tcp_port_; }
    std::string gid(size_t i) const { return i < rails_.size() ? rails_[i]->gid : std::string(); }
    std::string deviceName(size_t i) const {
        return i < rails_.size() ? rails_[i]->name : std::string();
    }
    std::vector<std::string> activeDevices() const;
    size_t maxRdmaTransferSize() const { return cfg_.max_rdma_transfer_size; }
    size_t qpsPerConnection() const { return cfg_.qps_per_connection; }
    const std::vector<NumaTopology> &numaTopology() const { return numa_topology_; }
    const std::vector<NicTopologyInfo> &nicTopology() const { return nic_topology_; }
    int nicNumaNode(const std::string &name) const;
    int numaNodeForAddr(void *addr) const;
    std::vector<size_t> localNicsForNuma(int numa) const;
    int gpuNumaNode(int gpu) const;
    std::vector<MPComm::PcieAffinityCheck> pcieAffinitySelfCheck() const;
    std::string fabricName() const { return fabric_name_; }
    const Config &config() const { return cfg_; }
    RailSlot *rail(size_t i) { return rails_[i].get(); }

 private:
    friend class StagingEngine;
    struct Worker;

    // impl_core.cc
    void discoverTopology();
    void writeConfigFile() const;
    int numaForAddr(uintptr_t addr) const;
    std::vector<size_t> affineRailsForGpu(int gpu) const;

    // impl_ctrl.cc
    void acceptLoop();
    void handleConnect(int fd, uint32_t remote_nics);
    void handleBufferQuery(int fd);
    void handleQosChannel(int fd);
    std::vector<std::pair<size_t, size_t>> pairRails(const std::vector<std::string> &local,
                                                     const std::vector<std::string> &remote,
                                                     bool local_is_active) const;
    std::shared_ptr<Connection> connection(const std::string &id) const;

    // impl_xfer.cc
    void workerLoop(Worker *w);
    void wakeWorker(Worker *w);
    void postChunks(Worker *w, Transfer *t, std::vector<fabric::QueuePair *> *touched);
    void postFanoutChunks(Worker *w, Transfer *t, std::vector<fabric::QueuePair *> *touched);
    void postPagedChunks(Worker *w, Transfer *t, std::vector<fabric::QueuePair *> *touched);
    void handleCompletion(Worker *w, const fabric::WorkCompletion &wc);
    void retire(Worker *w);
    void probeQuarantine();
    void maybeInjectFault();
    size_t effectiveChunk(const std::vector<size_t> &candidates) const;
    void quarantine(size_t rail, int status);
    void pcieOnPosted(int gpu, uint64_t bytes);
    void pcieOnCompleted(int gpu, uint64_t bytes);
    bool qosAllowPost(const Transfer &t, size_t rail, size_t bytes);

    // impl_qos_channel.cc
    struct QosOutChannel;
    struct RemoteQosPolicy {
        std::string peer, peer_ip;
        int gpu = -1;
        uint64_t rate = 0, burst = 0, generation = 0;
        TokenBucket bucket;
    };
    struct QosRestoreItem {
        int gpu;
        const kern::H2DWindow *win;
        std::chrono::steady_clock::time_point deadline;
    };
    void qosRxLoop(int fd, std::string peer, std::string peer_ip);
    bool qosAllowRemoteWrite(const Connection &conn, uint64_t raddr, size_t bytes);
    void broadcastQos(int gpu, uint64_t rate, uint64_t burst, bool clear);
    void stopQosChannels();
    void remotePauseForWindow(int gpu, const kern::H2DWindow *win);
    void qosRestoreLoop();

    mutable std::mutex qos_out_mu_;
    std::map<std::string, std::shared_ptr<QosOutChannel>> qos_out_;  // channels we opened
    mutable std::mutex qos_in_mu_;
    std::vector<std::unique_ptr<RemoteQosPolicy>> qos_in_;  // policies peers sent us
    std::atomic<int> qos_in_active_{0};
    std::atomic<uint64_t> remote_qos_defers_{0};
    std::atomic<uint64_t> qos_generation_{0};
    std::mutex qos_rx_mu_;
    std::atomic<bool> qos_rx_running_{true};
    std::vector<std::thread> qos_rx_threads_;
    std::vector<int> qos_rx_fds_;
    std::mutex qos_restore_mu_;
    std::condition_variable qos_restore_cv_;
    std::deque<QosRestoreItem> qos_restore_q_;
    bool qos_restore_running_ = false;
    std::thread qos_restore_thread_;

    Config cfg_;
    bool initialized_ = false;
    std::string host_id_;
    std::string fabric_name_;
    std::unique_ptr<fabric::Backend> backend_;
    std::vector<std::unique_ptr<RailSlot>> rails_;

    std::vector<NumaTopology> numa_topology_;
    std::vector<NicTopologyInfo> nic_topology_;
    int num_numa_ = 1;

    mutable std::shared_mutex regions_mu_;
    std::map<uintptr_t, Region> regions_;

    mutable std::mutex pub_mu_;
    std::vector<PublishedBufferEntry> published_;
    mutable PublishedBufferInfo published_snapshot_;

    mutable std::mutex conn_mu_;
    std::map<std::string, std::shared_ptr<Connection>> connections_;

    int listen_fd_ = -1;
    int tcp_port_ = 0;
    std::thread accept_thread_;
    std::atomic<bool> accept_running_{false};

    HandlePool handles_;
    mutable std::mutex xfer_mu_;
    std::unordered_map<uint64_t, std::shared_ptr<Transfer>> transfers_;
    std::unique_ptr<std::atomic<Transfer *>[]> handle_table_;
    // waitTransfer blocks here after a short spin; finishTransfer notifies.
    std::mutex done_mu_;
    std::condition_variable done_cv_;
    std::atomic<int> done_waiters_{0};
    // Submitted transfers not yet taken by their worker (keeps them alive
    // even if the user releases the handle immediately).
    std::mutex admit_mu_;
    std::unordered_map<uint64_t, std::shared_ptr<Transfer>> admit_;

    std::vector<std::unique_ptr<Worker>> workers_;
    std::atomic<bool> running_{false};
    Clock::time_point init_time_;

    // throttle
    std::atomic<bool> throttle_enabled_{false};
    std::atomic<size_t> throttle_outstanding_{0};
    std::atomic<size_t> throttle_chunk_{0};
    std::atomic<uint64_t> throttle_epoch_{0};
    std::atomic<uint64_t> throttle_set_ns_{0};
    std::atomic<uint64_t> throttle_seen_ns_{0};
    std::atomic<uint64_t> throttle_drained_ns_{0};
    std::atomic<size_t> throttle_snapshot_{0};
    std::atomic<bool> throttle_drain_pending_{false};

    // H2D QoS
    std::atomic<bool> h2d_qos_enabled_{false};
    std::atomic<bool> device_gates_on_{false};
    TokenBucket qos_bucket_;
    struct WindowPool;
    std::unique_ptr<WindowPool> windows_;
    std::atomic<WindowPool *> windows_live_{nullptr};  // published once created
    std::atomic<uint64_t> nic_completed_bytes_{0};

    // PCIe domains
    std::array<PcieDomain, kMaxGpuDomains> pcie_;

    // fault injection state (worker 0)
    bool fault_injected_ = false;
    bool fault_recovered_ = false;
    std::vector<fabric::QueuePair *> fault_qps_;

    std::unique_ptr<StagingEngine> staging_;

    // mapDRAMtoGPU registry
    struct Mapping {
        size_t len;
        uintptr_t dev_ptr;
        bool pinned_by_us;
    };
    std::mutex map_mu_;
    std::map<uintptr_t, Mapping> mappings_;
    void *fabric_stream_ = nullptr;

    std::atomic<uint64_t> stats_counter_{0};
};

constexpr int kSlotsPerGpu = 64;

struct MPComm::Impl::WindowPool {
    kern::H2DWindow *slots = nullptr;  // [kMaxGpuDomains][kSlotsPerGpu], host-mapped
    uint32_t *ctrs[kMaxGpuDomains] = {nullptr};  // device counters per GPU
    uint32_t *gates[kMaxGpuDomains] = {nullptr};  // open-window count per GPU (device memory)
    ~WindowPool();
};

struct MPComm::Impl::Worker {
    int id = 0;
    int numa = 0;
    MpscRing queue{4096};
    std::thread thread;
    std::vector<std::shared_ptr<Transfer>> active;
    std::mutex inbox_mu;
    std::vector<fabric::WorkCompletion> inbox;
    std::atomic<bool> inbox_nonempty{false};
    // Idle sleep with a doorbell: submitters (and workers forwarding
    // completions) bump `doorbell` and wake the worker when it sleeps, so a
    // transfer that arrives after a quiet period starts at once.
    std::mutex wake_mu;
    std::condition_variable wake_cv;
    std::atomic<uint64_t> doorbell{0};
    std::atomic<bool> sleeping{false};
    std::array<size_t, kMaxRails> rail_posted{}, rail_completed{};
    std::array<std::array<size_t, kMaxQpsPerRail>, kMaxRails> qp_posted{}, qp_completed{};
    uint64_t seen_epoch = 0;
    std::array<size_t, kMaxRails> drain_mark{};
    bool drain_armed = false;
    uint64_t loops = 0;
};

}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_ENGINE_IMPL_H_
