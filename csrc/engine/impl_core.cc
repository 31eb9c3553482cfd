// Lifecycle, memory registration, topology (MPComm::Impl).
// Parity: reference src/mpcomm.cpp:1575-1911 (init/shutdown),
// :2171-2318 (register/unregister/getRkey), :2849-3369 (topology).
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <ctime>
#include <fstream>

#include "cuda/gpu.h"
#include "engine/impl.h"
#include "engine/staging.h"
#include "mpcomm_log.h"
#include "topo/topology.h"

namespace mpcomm {

#ifndef MPCOMM_VERSION_STRING
#define MPCOMM_VERSION_STRING "0.1.0"
#endif

MPComm::Impl::Impl() : cfg_(Config::from_env()) {
    handle_table_.reset(new std::atomic<Transfer *>[HandlePool::kMax + 1]);
    for (size_t i = 0; i <= HandlePool::kMax; ++i) handle_table_[i].store(nullptr);
}

MPComm::Impl::~Impl() { shutdown(); }

namespace {

std::vector<std::string> split_csv(const std::string &s) {
    std::vector<std::string> out;
    std::string cur;
    for (char c : s) {
        if (c == ',') {
            if (!cur.empty()) out.push_back(cur);
            cur.clear();
        } else if (c != ' ') {
            cur.push_back(c);
        }
    }
    if (!cur.empty()) out.push_back(cur);
    return out;
}

}  // namespace

int MPComm::Impl::init(const std::string &host_id, const std::string &device_names, int tcp_port) {
    if (initialized_) {
        MPCOMM_LOG_WARN("MPComm: init called twice; keeping the first initialisation\n");
        return MPCOMM_SUCCESS;
    }
    host_id_ = host_id;
    qos_rx_running_.store(true, std::memory_order_release);

    // Backend selection.
    std::string fab = cfg_.fabric;
    if (fab == "auto") {
        if (fabric::ib_available()) fab = "ib";
        else if (fabric::nvl_device_count() > 0) fab = "nvl";
        else fab = "lo";
    }
    if (fab == "ib") backend_ = fabric::make_ib_backend();
    else if (fab == "nvl") backend_ = fabric::make_nvl_backend();
    else if (fab == "sock") backend_ = fabric::make_sock_backend();
    else if (fab == "lo") backend_ = fabric::make_loopback_backend();
    else {
        MPCOMM_LOG_ERROR("MPComm: unknown MPCOMM_FABRIC=%s\n", fab.c_str());
        return MPCOMM_ERR_INVALID_ARG;
    }
    fabric_name_ = fab;

    // MPCOMM_NIC_FILTER overrides the init() device list (reference :1942-1959).
    std::vector<std::string> filter = split_csv(cfg_.nic_filter.empty() ? device_names : cfg_.nic_filter);
    if (filter.empty() && fab == "nvl" && !cfg_.pxn_enable) {
        // One rail for the calling thread's current GPU: opening a rail (a
        // CUDA context + streams) on every GPU from every rank is wasteful.
        // With PXN every visible GPU becomes a rail (proxy egress/ingress).
        int dev = gpu::current_device();
        filter.push_back("nvl_" + std::to_string(dev < 0 ? 0 : dev));
    }
    std::vector<std::unique_ptr<fabric::Rail>> opened;
    int rc = backend_->open(cfg_, filter, &opened);
    if (rc != MPCOMM_SUCCESS || opened.empty()) {
        MPCOMM_LOG_WARN("MPComm: fabric '%s' opened no rails; transfers are unavailable "
                        "(H2D movers still work)\n", fab.c_str());
    }
    if (opened.size() > kMaxRails) {
        MPCOMM_LOG_WARN("MPComm: %zu rails found, using the first %zu\n", opened.size(), kMaxRails);
        opened.resize(kMaxRails);
    }
    for (auto &r : opened) {
        auto slot = std::make_unique<RailSlot>();
        slot->name = r->name();
        slot->gid = r->gid();
        slot->numa = r->numa_node() < 0 ? 0 : r->numa_node();
        slot->gpu = r->gpu_ordinal();
        slot->pci_path = r->pci_path();
        slot->rail = std::move(r);
        rails_.push_back(std::move(slot));
    }
    // PCIe affinity of non-GPU rails: GPU whose sysfs path shares the
    // longest prefix with the rail's (reference :3256-3369).
    {
        std::vector<std::string> paths;
        for (auto &s : rails_) paths.push_back(s->gpu < 0 ? s->pci_path : std::string());
        for (int g = 0; g < gpu::device_count(); ++g) {
            for (size_t i : topo::best_affinity(topo::pci_realpath(gpu::pci_bdf(g)), paths))
                if (rails_[i]->gpu < 0) rails_[i]->gpu = g;
        }
    }

    listen_fd_ = net::listen_tcp(tcp_port, 64, &tcp_port_);
    if (listen_fd_ < 0) {
        rails_.clear();
        return MPCOMM_ERR_CONNECTION;
    }

    discoverTopology();

    running_ = true;
    init_time_ = Clock::now();
    const int nworkers = std::max(1, std::min(num_numa_, static_cast<int>(kMaxNumaNodes)));
    for (int i = 0; i < nworkers; ++i) {
        auto w = std::make_unique<Worker>();
        w->id = i;
        w->numa = i;
        workers_.push_back(std::move(w));
    }
    for (auto &w : workers_) {
        Worker *wp = w.get();
        wp->thread = std::thread([this, wp] { workerLoop(wp); });
    }
    staging_ = std::make_unique<StagingEngine>(this);
    if (cfg_.h2d_qos_enable) enableH2DQoS(cfg_.h2d_qos_rate_bps, cfg_.h2d_qos_burst_bytes);
    writeConfigFile();
    initialized_ = true;
    MPCOMM_LOG_INFO("MPComm: initialised host '%s' fabric=%s rails=%zu tcp_port=%d numa=%d workers=%zu\n",
                    host_id_.c_str(), fabric_name_.c_str(), rails_.size(), tcp_port_, num_numa_,
                    workers_.size());
    return MPCOMM_SUCCESS;
}

void MPComm::Impl::shutdown() {
    if (!initialized_ && workers_.empty() && rails_.empty()) return;
    stopAcceptThread();
    stopQosChannels();
    if (staging_) staging_.reset();
    running_ = false;
    for (auto &w : workers_) wakeWorker(w.get());
    for (auto &w : workers_)
        if (w->thread.joinable()) w->thread.join();
    workers_.clear();
    {
        std::lock_guard<std::mutex> g(xfer_mu_);
        for (auto &kv : transfers_) handle_table_[kv.first].store(nullptr);
        transfers_.clear();
    }
    {
        std::lock_guard<std::mutex> g(conn_mu_);
        connections_.clear();  // destroys QPs before their rails
    }
    fault_qps_.clear();
    {
        std::unique_lock<std::shared_mutex> g(regions_mu_);
        for (auto &kv : regions_)
            for (size_t i = 0; i < rails_.size() && i < kv.second.keys.size(); ++i)
                rails_[i]->rail->deregister_memory(reinterpret_cast<void *>(kv.first), kv.second.keys[i]);
        regions_.clear();
    }
    {
        std::lock_guard<std::mutex> g(map_mu_);
        for (auto &kv : mappings_)
            if (kv.second.pinned_by_us) gpu::host_unpin(reinterpret_cast<void *>(kv.first));
        mappings_.clear();
    }
    rails_.clear();
    if (listen_fd_ >= 0) {
        ::close(listen_fd_);
        listen_fd_ = -1;
    }
    windows_live_.store(nullptr);
    windows_.reset();
    initialized_ = false;
}

int MPComm::Impl::registerMemory(void *addr, size_t len) {
    if (!initialized_) return MPCOMM_ERR_CONTEXT;
    if (!addr || len == 0) return MPCOMM_ERR_INVALID_ARG;
    const uintptr_t a = reinterpret_cast<uintptr_t>(addr);
    {
        std::shared_lock<std::shared_mutex> g(regions_mu_);
        auto it = regions_.find(a);
        if (it != regions_.end() && it->second.len == len) return MPCOMM_SUCCESS;
    }
    gpu::PtrInfo pi;
    const bool known = gpu::query_pointer(addr, &pi);
    const bool is_dev = known && pi.is_device;
    if (is_dev && fabric_name_ != "nvl" && fabric_name_ != "ib") {
        MPCOMM_LOG_ERROR("MPComm: fabric '%s' cannot reach GPU memory %p\n", fabric_name_.c_str(), addr);
        return MPCOMM_ERR_MEMORY;
    }
    Region r;
    r.addr = a;
    r.len = len;
    r.keys.resize(rails_.size());
    for (size_t i = 0; i < rails_.size(); ++i) {
        int e = rails_[i]->rail->register_memory(addr, len, &r.keys[i]);
        if (e != MPCOMM_SUCCESS) {
            MPCOMM_LOG_ERROR("MPComm: registration of %p+%zu failed on %s\n", addr, len,
                             rails_[i]->name.c_str());
            for (size_t k = 0; k < i; ++k) rails_[k]->rail->deregister_memory(addr, r.keys[k]);
            return MPCOMM_ERR_MEMORY;
        }
    }
    if (is_dev) {
        r.gpu = pi.device;
        r.numa = gpuNumaNode(pi.device);
        r.affine_rails = affineRailsForGpu(pi.device);
    } else {
        r.numa = topo::numa_node_of_addr(addr);
    }
    std::unique_lock<std::shared_mutex> g(regions_mu_);
    auto it = regions_.find(a);
    if (it != regions_.end()) {
        // Re-registration with a new length replaces the old keys.
        for (size_t i = 0; i < rails_.size() && i < it->second.keys.size(); ++i)
            rails_[i]->rail->deregister_memory(addr, it->second.keys[i]);
        regions_.erase(it);
    }
    regions_.emplace(a, std::move(r));
    MPCOMM_LOG_DEBUG("MPComm: registered %p+%zu (%s) on %zu rails\n", addr, len,
                     is_dev ? "gpu" : "host", rails_.size());
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::registerMulticastMemory(void *uc, size_t len, void *mc, uint64_t token, int members) {
    if (!uc || !mc || !len || !token || members < 2) return MPCOMM_ERR_INVALID_ARG;
    int e = registerMemory(uc, len);
    if (e != MPCOMM_SUCCESS) return e;
    Region r;
    if (!lookupRegion(reinterpret_cast<uintptr_t>(uc), len, &r)) return MPCOMM_ERR_MEMORY;
    int ok = 0;
    for (size_t i = 0; i < rails_.size() && i < r.keys.size(); ++i)
        if (rails_[i]->rail->set_multicast(r.keys[i], reinterpret_cast<uintptr_t>(uc), len,
                                           reinterpret_cast<uintptr_t>(mc), token, members) == 0)
            ++ok;
    if (!ok) {
        MPCOMM_LOG_ERROR("MPComm: fabric '%s' cannot use multicast memory %p\n", fabric_name_.c_str(), uc);
        return MPCOMM_ERR_INVALID_ARG;
    }
    MPCOMM_LOG_DEBUG("MPComm: %p+%zu registered as a copy of multicast group %llx (%d GPUs)\n", uc, len,
                     static_cast<unsigned long long>(token), members);
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::unregisterMemory(void *addr) {
    if (!initialized_) return MPCOMM_ERR_CONTEXT;
    std::unique_lock<std::shared_mutex> g(regions_mu_);
    auto it = regions_.find(reinterpret_cast<uintptr_t>(addr));
    if (it == regions_.end()) return MPCOMM_ERR_INVALID_ARG;
    for (size_t i = 0; i < rails_.size() && i < it->second.keys.size(); ++i)
        rails_[i]->rail->deregister_memory(addr, it->second.keys[i]);
    regions_.erase(it);
    return MPCOMM_SUCCESS;
}

bool MPComm::Impl::lookupRegion(uintptr_t addr, size_t len, Region *out) const {
    std::shared_lock<std::shared_mutex> g(regions_mu_);
    auto it = regions_.upper_bound(addr);
    if (it == regions_.begin()) return false;
    --it;
    if (addr < it->second.addr || addr + len > it->second.addr + it->second.len) return false;
    if (out) *out = it->second;
    return true;
}

uint32_t MPComm::Impl::getRkey(size_t nic, void *addr) const {
    Region r;
    if (!lookupRegion(reinterpret_cast<uintptr_t>(addr), 1, &r)) return 0;
    return nic < r.keys.size() ? r.keys[nic].rkey : 0;
}

void MPComm::Impl::discoverTopology() {
    num_numa_ = topo::numa_node_count();
    numa_topology_.clear();
    for (int n = 0; n < num_numa_; ++n) {
        NumaTopology t;
        t.numa_node = n;
        for (auto &r : rails_) (r->numa == n ? t.local_nics : t.remote_nics).push_back(r->name);
        numa_topology_.push_back(std::move(t));
    }
    nic_topology_.clear();
    for (auto &r : rails_) nic_topology_.push_back(NicTopologyInfo{r->name, r->numa});
    const auto rows = pcieAffinitySelfCheck();
    if (rows.empty()) return;
    size_t mismatches = 0;
    MPCOMM_LOG_INFO("MPComm: GPU <-> rail PCIe affinity (sysfs, used for accounting) vs name-suffix heuristic:\n");
    for (const auto &row : rows) {
        std::string sys;
        for (const auto &n : row.sysfs_rails) sys += (sys.empty() ? "" : ",") + n;
        if (!row.agrees) ++mismatches;
        MPCOMM_LOG_INFO("MPComm:   GPU%-2d sysfs=[%s] suffix=[%s] %s\n", row.gpu_device_id,
                        sys.empty() ? "-" : sys.c_str(), row.suffix_rail.empty() ? "-" : row.suffix_rail.c_str(),
                        row.agrees ? "match" : "MISMATCH");
    }
    if (mismatches)
        MPCOMM_LOG_INFO("MPComm:   %zu GPU(s) disagree with the suffix heuristic; accounting follows sysfs\n",
                        mismatches);
}

std::vector<MPComm::PcieAffinityCheck> MPComm::Impl::pcieAffinitySelfCheck() const {
    std::vector<MPComm::PcieAffinityCheck> out;
    const int ngpu = gpu::device_count();
    for (int g = 0; g < ngpu && g < static_cast<int>(kMaxGpuDomains); ++g) {
        MPComm::PcieAffinityCheck row;
        row.gpu_device_id = g;
        const auto affine = affineRailsForGpu(g);
        for (size_t r : affine) row.sysfs_rails.push_back(rails_[r]->name);
        size_t heur = SIZE_MAX;
        for (size_t r = 0; r < rails_.size(); ++r)
            if (topo::name_suffix(rails_[r]->name) == g) {
                heur = r;
                break;
            }
        if (heur != SIZE_MAX) row.suffix_rail = rails_[heur]->name;
        row.agrees = !affine.empty() && heur != SIZE_MAX && affine[0] == heur;
        out.push_back(std::move(row));
    }
    return out;
}

void MPComm::Impl::writeConfigFile() const {
    if (cfg_.config_file.empty()) return;
    std::ofstream f(cfg_.config_file);
    if (!f) {
        MPCOMM_LOG_WARN("MPComm: cannot write %s\n", cfg_.config_file.c_str());
        return;
    }
    char ts[64];
    std::time_t now = std::time(nullptr);
    struct tm tmv;
    localtime_r(&now, &tmv);
    std::strftime(ts, sizeof(ts), "%Y-%m-%d %H:%M:%S", &tmv);
    f << "{\"TIMESTAMP\": \"" << ts << "\", \"MPCOMM_VERSION\": \"" << MPCOMM_VERSION_STRING
      << "\", \"PLATFORM\": \"cuda\", \"FABRIC\": \"" << fabric_name_ << "\"}\n";
}

std::vector<size_t> MPComm::Impl::affineRailsForGpu(int g) const {
    std::vector<size_t> out;
    if (g < 0) return out;
    for (size_t i = 0; i < rails_.size(); ++i)
        if (rails_[i]->gpu == g) out.push_back(i);
    return out;
}

std::vector<std::string> MPComm::Impl::activeDevices() const {
    std::vector<std::string> v;
    for (auto &r : rails_) v.push_back(r->name);
    return v;
}

int MPComm::Impl::nicNumaNode(const std::string &name) const {
    for (auto &r : rails_)
        if (r->name == name) return r->numa;
    return -1;
}

int MPComm::Impl::gpuNumaNode(int g) const {
    if (g < 0) return -1;
    return topo::pci_numa_node(gpu::pci_bdf(g));
}

int MPComm::Impl::numaNodeForAddr(void *addr) const {
    Region r;
    if (lookupRegion(reinterpret_cast<uintptr_t>(addr), 1, &r) && r.numa >= 0) return r.numa;
    gpu::PtrInfo pi;
    if (gpu::query_pointer(addr, &pi) && pi.is_device) return gpuNumaNode(pi.device);
    return topo::numa_node_of_addr(addr);
}

int MPComm::Impl::numaForAddr(uintptr_t addr) const {
    const int nw = static_cast<int>(workers_.size());
    if (nw <= 1) return 0;
    Region r;
    if (lookupRegion(addr, 1, &r) && r.numa >= 0) return r.numa % nw;
    return static_cast<int>((addr >> 12) % static_cast<uintptr_t>(nw));
}

std::vector<size_t> MPComm::Impl::localNicsForNuma(int numa) const {
    std::vector<size_t> out;
    for (size_t i = 0; i < rails_.size(); ++i)
        if (rails_[i]->numa == numa) out.push_back(i);
    return out;
}

}  // namespace mpcomm
