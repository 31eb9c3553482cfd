// Python binding: module `mpcomm._mpcomm`, re-exported by the `mpcomm`
// package. Method names, argument names, defaults and return shapes follow
// the reference module (python/mpcomm_py.cpp:687-900); addresses are ints.
// The GIL is released in every call that can block (wait, connect, query,
// H2D launches) — the reference released it only in wait_transfer.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <string>
#include <vector>

#include "cuda/gpu.h"
#include "kernels/launch.h"
#include "mpcomm.h"
#include "parallel/vmm.h"
#include "topo/topology.h"
#include "transport/loopback_hooks.h"

namespace py = pybind11;
using namespace mpcomm;

namespace {

class PyMPComm {
 public:
    int init(const std::string &id, const std::string &devs, int port) {
        py::gil_scoped_release r;
        return c_.init(id, devs, port);
    }
    void shutdown() {
        py::gil_scoped_release r;
        c_.shutdown();
    }
    int register_memory(uintptr_t a, size_t l) {
        py::gil_scoped_release r;
        return c_.registerMemory(reinterpret_cast<void *>(a), l);
    }
    int unregister_memory(uintptr_t a) { return c_.unregisterMemory(reinterpret_cast<void *>(a)); }
    py::list get_pcie_affinity_self_check() const {
        py::list out;
        for (const auto &r : c_.getPcieAffinitySelfCheck()) {
            py::dict d;
            d["gpu"] = r.gpu_device_id;
            d["sysfs_rails"] = r.sysfs_rails;
            d["suffix_rail"] = r.suffix_rail;
            d["agrees"] = r.agrees;
            out.append(d);
        }
        return out;
    }
    int register_multicast_memory(uintptr_t uc, size_t l, uintptr_t mc, uint64_t token, int members) {
        py::gil_scoped_release r;
        return c_.registerMulticastMemory(reinterpret_cast<void *>(uc), l, reinterpret_cast<void *>(mc), token,
                                          members);
    }
    int connect(const std::string &id, const std::string &addr, int port) {
        py::gil_scoped_release r;
        return c_.connect(id, addr, port);
    }
    int start_accept_thread() { return c_.startAcceptThread(); }
    void stop_accept_thread() {
        py::gil_scoped_release r;
        c_.stopAcceptThread();
    }
    int update_remote_memory_info(const std::string &id, const std::vector<uint32_t> &k) {
        return c_.updateRemoteMemoryInfo(id, k);
    }
    uint32_t get_rkey(size_t nic, uintptr_t a) { return c_.getRkey(nic, reinterpret_cast<void *>(a)); }
    std::vector<uint32_t> get_all_rkeys(uintptr_t a) {
        std::vector<uint32_t> v;
        for (size_t i = 0; i < c_.getNumNics(); ++i) v.push_back(c_.getRkey(i, reinterpret_cast<void *>(a)));
        return v;
    }
    uint64_t scatter_async(uintptr_t l, const std::vector<std::string> &h, const std::vector<uintptr_t> &r,
                           const std::vector<size_t> &n) {
        return c_.scatterAsync(l, h, r, n);
    }
    uint64_t gather_async(uintptr_t l, const std::vector<std::string> &h, const std::vector<uintptr_t> &r,
                          const std::vector<size_t> &n) {
        return c_.gatherAsync(l, h, r, n);
    }
    uint64_t broadcast_async(uintptr_t l, size_t len, const std::vector<std::string> &h,
                             const std::vector<uintptr_t> &r) {
        return c_.broadcastAsync(l, len, h, r);
    }
    uint64_t put_async(uintptr_t l, const std::string &h, uintptr_t r, size_t n) { return c_.putAsync(l, h, r, n); }
    uint64_t get_async(uintptr_t l, const std::string &h, uintptr_t r, size_t n) { return c_.getAsync(l, h, r, n); }
    uint64_t put_pages_async(uintptr_t dram, uintptr_t idx, int n, int bs, const std::string &h, uintptr_t r) {
        return c_.putPagesAsync(dram, reinterpret_cast<const int64_t *>(idx), n, bs, h, r);
    }
    uint64_t mp_replicate_async(const std::string &type, const std::vector<std::string> &h, uintptr_t l,
                                const std::vector<uintptr_t> &r, const std::vector<size_t> &n) {
        if (type == "scatter") return c_.scatterAsync(l, h, r, n);
        if (type == "gather") return c_.gatherAsync(l, h, r, n);
        if (type == "broadcast") return n.empty() ? INVALID_TRANSFER_HANDLE : c_.broadcastAsync(l, n[0], h, r);
        return INVALID_TRANSFER_HANDLE;
    }
    bool is_transfer_complete(uint64_t h) { return c_.isTransferComplete(h); }
    int wait_transfer(uint64_t h, int timeout_ms) {
        py::gil_scoped_release r;
        return c_.waitTransfer(h, timeout_ms);
    }
    py::dict get_transfer_result(uint64_t h) {
        TransferResult t = c_.getTransferResult(h);
        py::dict d;
        d["error_code"] = t.error_code;
        d["bytes_transferred"] = t.bytes_transferred;
        d["elapsed_ms"] = t.elapsed_ms;
        return d;
    }
    void release_transfer(uint64_t h) { c_.releaseTransfer(h); }
    size_t get_num_nics() const { return c_.getNumNics(); }
    std::string get_local_host_id() const { return c_.getLocalHostId(); }
    int get_tcp_port() const { return c_.getTcpPort(); }
    std::string get_gid(size_t i) const { return c_.getGid(i); }
    std::string get_device_name(size_t i) const { return c_.getDeviceName(i); }
    std::vector<std::string> get_active_devices() const { return c_.getActiveDevices(); }
    size_t get_qps_per_connection() const { return c_.getQpsPerConnection(); }
    size_t get_max_rdma_transfer_size() const { return c_.getMaxRdmaTransferSize(); }
    void set_nic_throttle(size_t o, size_t c) { c_.setNicThrottle(o, c); }
    void clear_nic_throttle() { c_.clearNicThrottle(); }
    void enable_h2d_qos(uint64_t r, uint64_t b) { c_.enableH2DQoS(r, b); }
    void set_h2d_qos_policy(uint64_t r, uint64_t b) { c_.setH2DQoSPolicy(r, b); }
    bool is_h2d_qos_enabled() const { return c_.isH2DQoSEnabled(); }
    int open_qos_channel(const std::string &h) { return c_.openQosChannel(h); }
    int close_qos_channel(const std::string &h) { return c_.closeQosChannel(h); }
    int send_qos_policy(const std::string &h, int gpu, uint64_t rate, uint64_t burst) {
        return c_.sendQosPolicy(h, gpu, rate, burst);
    }
    int clear_qos_policy(const std::string &h, int gpu) { return c_.clearQosPolicy(h, gpu); }
    py::list get_remote_qos_policies() const {
        py::list out;
        for (auto &p : c_.getRemoteQosPolicies()) {
            py::dict d;
            d["peer_host_id"] = p.peer_host_id;
            d["gpu_device_id"] = p.gpu_device_id;
            d["rate_bytes_per_sec"] = p.rate_bytes_per_sec;
            d["burst_bytes"] = p.burst_bytes;
            d["generation"] = p.generation;
            out.append(d);
        }
        return out;
    }
    uint64_t get_remote_qos_defer_count() const { return c_.getRemoteQosDeferCount(); }
    py::object get_last_h2d_window(int gpu) const {
        uint64_t b = 0, e = 0;
        if (!c_.getLastH2DWindow(gpu, &b, &e)) return py::none();
        py::dict d;
        d["begin_ns"] = b;
        d["end_ns"] = e;
        d["duration_us"] = e > b ? (e - b) / 1000.0 : 0.0;
        return d;
    }
    void disable_h2d_qos() { c_.disableH2DQoS(); }
    uint64_t get_nic_completed_bytes() const { return c_.getNicCompletedBytes(); }
    std::vector<uint64_t> get_rail_completed_bytes() const { return c_.getRailCompletedBytes(); }
    py::list get_pcie_domain_stats() const {
        py::list out;
        for (auto &s : c_.getPcieDomainStats()) {
            py::dict d;
            d["gpu"] = s.gpu_device_id;
            d["posted_bytes"] = s.posted_bytes;
            d["completed_bytes"] = s.completed_bytes;
            d["in_flight_bytes"] = s.in_flight_bytes;
            d["in_flight_bytes_max"] = s.in_flight_bytes_max;
            d["post_count"] = s.post_count;
            d["defer_count"] = s.defer_count;
            out.append(d);
        }
        return out;
    }
    void reset_pcie_domain_stats() { c_.resetPcieDomainStats(); }
    bool is_pcie_domain_stat_enabled() const { return c_.isPcieDomainStatEnabled(); }
    py::dict get_throttle_latency() const {
        uint64_t s = 0, w = 0, d = 0;
        size_t snap = 0;
        const bool drained = c_.getThrottleLatency(&s, &w, &d, &snap);
        py::dict r;
        r["set_ns"] = s;
        r["worker_seen_ns"] = w;
        r["drained_ns"] = d;
        r["snapshot_outstanding_wqes"] = snap;
        r["drained"] = drained;
        r["worker_us"] = w > s ? (w - s) / 1000.0 : 0.0;
        r["drain_us"] = (drained && d > w && w > 0) ? (d - w) / 1000.0 : 0.0;
        r["effective_us"] = (drained && d > s) ? (d - s) / 1000.0 : 0.0;
        return r;
    }
    int write_bytes_to_buffer(uintptr_t a, const py::bytes &data, size_t len) {
        std::string s = data;
        if (s.size() < len) return MPCOMM_ERR_INVALID_ARG;
        std::memcpy(reinterpret_cast<void *>(a), s.data(), len);
        return MPCOMM_SUCCESS;
    }
    py::bytes read_bytes_from_buffer(uintptr_t a, size_t len) {
        return py::bytes(reinterpret_cast<const char *>(a), len);
    }
    int publish_buffer(uintptr_t a, size_t l, int numa) {
        return c_.publishBuffer(reinterpret_cast<void *>(a), l, numa);
    }
    int unpublish_buffer(uintptr_t a) { return c_.unpublishBuffer(reinterpret_cast<void *>(a)); }
    void unpublish_all_buffers() { c_.unpublishAllBuffers(); }
    size_t get_published_buffer_count() { return c_.getPublishedBufferCount(); }

    static py::dict entry_dict(uint64_t addr, uint64_t len, int numa, int gpu, const std::vector<size_t> &aff,
                               const std::vector<uint32_t> &rkeys) {
        py::dict d;
        d["addr"] = addr;
        d["length"] = len;
        d["numa_node"] = numa;
        d["gpu_device_id"] = gpu;
        d["pcie_affine_nic_indices"] = aff;
        d["rkeys"] = rkeys;
        return d;
    }
    py::dict query_remote_buffers(const std::string &id, const std::string &addr, int port) {
        RemoteBufferInfo info;
        int rc;
        {
            py::gil_scoped_release r;
            rc = c_.queryRemoteBuffer(id, addr, port, info);
        }
        py::dict out;
        if (rc != 0) return out;
        out["host_id"] = info.host_id;
        py::list bl;
        for (auto &b : info.buffers)
            bl.append(entry_dict(b.addr, b.length, b.numa_node, b.gpu_device_id, b.pcie_affine_nic_indices, b.rkeys));
        out["buffers"] = bl;
        return out;
    }
    py::dict query_remote_buffer_by_numa(const std::string &id, const std::string &addr, int port, int numa) {
        RemoteBufferEntry e;
        int rc;
        {
            py::gil_scoped_release r;
            rc = c_.queryRemoteBufferByNuma(id, addr, port, numa, e);
        }
        if (rc != 0) return py::dict();
        return entry_dict(e.addr, e.length, e.numa_node, e.gpu_device_id, e.pcie_affine_nic_indices, e.rkeys);
    }
    py::dict get_published_buffer_info() {
        py::dict out;
        const PublishedBufferInfo *info = c_.getPublishedBufferInfo();
        if (!info || info->buffers.empty()) return out;
        py::list bl;
        for (auto &b : info->buffers)
            bl.append(entry_dict(b.addr, b.length, b.numa_node, b.gpu_device_id, b.pcie_affine_nic_indices, b.rkeys));
        out["buffers"] = bl;
        return out;
    }
    py::list get_numa_topology() const {
        py::list out;
        for (auto &t : c_.getNumaTopology()) {
            py::dict d;
            d["numa_node"] = t.numa_node;
            d["local_nics"] = t.local_nics;
            d["remote_nics"] = t.remote_nics;
            out.append(d);
        }
        return out;
    }
    py::list get_nic_topology() const {
        py::list out;
        for (auto &t : c_.getNicTopology()) {
            py::dict d;
            d["nic_name"] = t.nic_name;
            d["numa_node"] = t.numa_node;
            out.append(d);
        }
        return out;
    }
    int get_nic_numa_node(const std::string &n) const { return c_.getNicNumaNode(n); }
    int get_numa_node_for_addr(uintptr_t a) const { return c_.getNumaNodeForAddr(reinterpret_cast<void *>(a)); }
    std::vector<size_t> get_local_nic_indices_for_numa(int n) const { return c_.getLocalNicIndicesForNuma(n); }
    int get_gpu_numa_node(int g) const { return c_.getGpuNumaNode(g); }
    uintptr_t map_dram_to_gpu(uintptr_t h, size_t l) {
        py::gil_scoped_release r;
        return c_.mapDRAMtoGPU(reinterpret_cast<void *>(h), l);
    }
    int unmap_dram_from_gpu(uintptr_t h) {
        py::gil_scoped_release r;
        return c_.unmapDRAMfromGPU(reinterpret_cast<void *>(h));
    }
    int tma_gather(uintptr_t dram, uintptr_t idx, uintptr_t dst, int n, int bs, int max_sm, int mode,
                   uintptr_t stream) {
        py::gil_scoped_release r;
        return c_.tmaGatherOnStream(dram, reinterpret_cast<const int64_t *>(idx), reinterpret_cast<void *>(dst),
                                    n, bs, max_sm, static_cast<H2DMode>(mode), reinterpret_cast<void *>(stream));
    }
    int tma_scatter(uintptr_t src, uintptr_t idx, uintptr_t dram, int n, int bs, int max_sm, int mode,
                    uintptr_t stream) {
        py::gil_scoped_release r;
        return c_.tmaScatterOnStream(reinterpret_cast<void *>(src), reinterpret_cast<const int64_t *>(idx), dram,
                                     n, bs, max_sm, static_cast<H2DMode>(mode), reinterpret_cast<void *>(stream));
    }
    int set_fabric_stream(uintptr_t s) { return c_.setFabricStream(reinterpret_cast<void *>(s)); }
    std::string get_fabric_name() const { return c_.getFabricName(); }

 private:
    MPComm c_;
};

int check(int e) { return e; }

}  // namespace

PYBIND11_MODULE(_mpcomm, m) {
    m.doc() = "mpcomm native module: memory-pool communication for B200 (sm_100a)";

    py::enum_<MPCommError>(m, "MPCommError")
        .value("SUCCESS", MPCOMM_SUCCESS)
        .value("ERR_DEVICE", MPCOMM_ERR_DEVICE)
        .value("ERR_CONTEXT", MPCOMM_ERR_CONTEXT)
        .value("ERR_MEMORY", MPCOMM_ERR_MEMORY)
        .value("ERR_CONNECTION", MPCOMM_ERR_CONNECTION)
        .value("ERR_TRANSFER", MPCOMM_ERR_TRANSFER)
        .value("ERR_TIMEOUT", MPCOMM_ERR_TIMEOUT)
        .value("ERR_INVALID_ARG", MPCOMM_ERR_INVALID_ARG)
        .value("ERR_INVALID_HANDLE", MPCOMM_ERR_INVALID_HANDLE)
        .value("ERR_PENDING", MPCOMM_ERR_PENDING)
        .export_values();
    m.attr("INVALID_TRANSFER_HANDLE") = INVALID_TRANSFER_HANDLE;
    m.attr("H2D_MODE_AUTO") = static_cast<int>(H2D_MODE_AUTO);
    m.attr("H2D_MODE_SM") = static_cast<int>(H2D_MODE_SM);
    m.attr("H2D_MODE_TMA") = static_cast<int>(H2D_MODE_TMA);

    using C = PyMPComm;
    py::class_<C>(m, "MPComm")
        .def(py::init<>())
        .def("init", &C::init, py::arg("local_host_id"), py::arg("device_names") = "", py::arg("tcp_port") = 0)
        .def("shutdown", &C::shutdown)
        .def("register_memory", &C::register_memory, py::arg("addr"), py::arg("length"))
        .def("unregister_memory", &C::unregister_memory, py::arg("addr"))
        .def("get_pcie_affinity_self_check", &C::get_pcie_affinity_self_check,
             "Per GPU: rails under the same PCIe switch (sysfs) vs the name-suffix heuristic.")
        .def("register_multicast_memory", &C::register_multicast_memory, py::arg("uc_addr"), py::arg("length"),
             py::arg("mc_addr"), py::arg("group_token"), py::arg("group_size"),
             "Registers this process's copy of an NVLS multicast group buffer; broadcast_async to the group's "
             "other members then goes out as multicast stores.")
        .def("connect", &C::connect, py::arg("remote_host_id"), py::arg("remote_tcp_addr"),
             py::arg("remote_tcp_port"))
        .def("start_accept_thread", &C::start_accept_thread)
        .def("stop_accept_thread", &C::stop_accept_thread)
        .def("update_remote_memory_info", &C::update_remote_memory_info, py::arg("remote_host_id"),
             py::arg("rkeys"))
        .def("get_rkey", &C::get_rkey, py::arg("nic_index"), py::arg("addr"))
        .def("get_all_rkeys", &C::get_all_rkeys, py::arg("addr"))
        .def("scatter_async", &C::scatter_async, py::arg("local_addr"), py::arg("host_list"),
             py::arg("remote_addrs"), py::arg("lengths"))
        .def("gather_async", &C::gather_async, py::arg("local_addr"), py::arg("host_list"),
             py::arg("remote_addrs"), py::arg("lengths"))
        .def("broadcast_async", &C::broadcast_async, py::arg("local_addr"), py::arg("length"),
             py::arg("host_list"), py::arg("remote_addrs"))
        .def("put_async", &C::put_async, py::arg("local_addr"), py::arg("remote_host_id"),
             py::arg("remote_addr"), py::arg("length"))
        .def("get_async", &C::get_async, py::arg("local_addr"), py::arg("remote_host_id"),
             py::arg("remote_addr"), py::arg("length"))
        .def("put_pages_async", &C::put_pages_async, py::arg("dram_dev_ptr"), py::arg("indices_ptr"),
             py::arg("num_blocks"), py::arg("block_size"), py::arg("remote_host_id"), py::arg("remote_addr"),
             "Paged PUT: the GPU holding the int64 indices gathers pool pages and writes them to the remote range "
             "in one launch per chunk of pages (fused PXN gather + forward).")
        .def("mp_replicate_async", &C::mp_replicate_async, py::arg("comm_type"), py::arg("host_list"),
             py::arg("local_addr"), py::arg("remote_addrs"), py::arg("lengths"))
        .def("is_transfer_complete", &C::is_transfer_complete, py::arg("handle"))
        .def("wait_transfer", &C::wait_transfer, py::arg("handle"), py::arg("timeout_ms") = -1)
        .def("get_transfer_result", &C::get_transfer_result, py::arg("handle"))
        .def("release_transfer", &C::release_transfer, py::arg("handle"))
        .def("get_num_nics", &C::get_num_nics)
        .def("get_local_host_id", &C::get_local_host_id)
        .def("get_tcp_port", &C::get_tcp_port)
        .def("get_gid", &C::get_gid, py::arg("nic_index"))
        .def("get_device_name", &C::get_device_name, py::arg("nic_index"))
        .def("get_active_devices", &C::get_active_devices)
        .def_static("get_nic_filter_env_var_name", [] { return std::string(MPComm::getNicFilterEnvVarName()); })
        .def_static("get_qps_per_connection_env_var_name",
                    [] { return std::string(MPComm::getQpsPerConnectionEnvVarName()); })
        .def_static("get_pcie_stat_enable_env_var_name",
                    [] { return std::string(MPComm::getPcieStatEnableEnvVarName()); })
        .def("get_qps_per_connection", &C::get_qps_per_connection)
        .def("get_max_rdma_transfer_size", &C::get_max_rdma_transfer_size)
        .def("set_nic_throttle", &C::set_nic_throttle, py::arg("max_outstanding_per_qp"), py::arg("chunk_size") = 0)
        .def("clear_nic_throttle", &C::clear_nic_throttle)
        .def("enable_h2d_qos", &C::enable_h2d_qos, py::arg("rate_bytes_per_sec") = 0, py::arg("burst_bytes") = 0)
        .def("set_h2d_qos_policy", &C::set_h2d_qos_policy, py::arg("rate_bytes_per_sec"), py::arg("burst_bytes") = 0)
        .def("is_h2d_qos_enabled", &C::is_h2d_qos_enabled)
        .def("open_qos_channel", &C::open_qos_channel, py::arg("host_id"))
        .def("close_qos_channel", &C::close_qos_channel, py::arg("host_id"))
        .def("send_qos_policy", &C::send_qos_policy, py::arg("host_id"), py::arg("gpu") = -1,
             py::arg("rate_bytes_per_sec") = 0, py::arg("burst_bytes") = 0)
        .def("clear_qos_policy", &C::clear_qos_policy, py::arg("host_id"), py::arg("gpu") = -1)
        .def("get_remote_qos_policies", &C::get_remote_qos_policies)
        .def("get_remote_qos_defer_count", &C::get_remote_qos_defer_count)
        .def("get_last_h2d_window", &C::get_last_h2d_window, py::arg("gpu") = 0)
        .def("disable_h2d_qos", &C::disable_h2d_qos)
        .def("get_nic_completed_bytes", &C::get_nic_completed_bytes)
        .def("get_rail_completed_bytes", &C::get_rail_completed_bytes)
        .def("get_pcie_domain_stats", &C::get_pcie_domain_stats)
        .def("reset_pcie_domain_stats", &C::reset_pcie_domain_stats)
        .def("is_pcie_domain_stat_enabled", &C::is_pcie_domain_stat_enabled)
        .def("get_throttle_latency", &C::get_throttle_latency)
        .def("write_bytes_to_buffer", &C::write_bytes_to_buffer, py::arg("addr"), py::arg("data"), py::arg("length"))
        .def("read_bytes_from_buffer", &C::read_bytes_from_buffer, py::arg("addr"), py::arg("length"))
        .def("publish_buffer", &C::publish_buffer, py::arg("addr"), py::arg("length"), py::arg("numa_node") = -1)
        .def("unpublish_buffer", &C::unpublish_buffer, py::arg("addr"))
        .def("unpublish_all_buffers", &C::unpublish_all_buffers)
        .def("get_published_buffer_count", &C::get_published_buffer_count)
        .def("query_remote_buffers", &C::query_remote_buffers, py::arg("remote_host_id"),
             py::arg("remote_tcp_addr"), py::arg("remote_tcp_port"))
        .def("query_remote_buffer_by_numa", &C::query_remote_buffer_by_numa, py::arg("remote_host_id"),
             py::arg("remote_tcp_addr"), py::arg("remote_tcp_port"), py::arg("numa_node") = -1)
        .def("query_remote_buffer",
             [](C &c, const std::string &id, const std::string &a, int p) {
                 return c.query_remote_buffer_by_numa(id, a, p, -1);
             },
             py::arg("remote_host_id"), py::arg("remote_tcp_addr"), py::arg("remote_tcp_port"))
        .def("get_published_buffer_info", &C::get_published_buffer_info)
        .def("get_numa_topology", &C::get_numa_topology)
        .def("get_nic_topology", &C::get_nic_topology)
        .def("get_nic_numa_node", &C::get_nic_numa_node, py::arg("nic_name"))
        .def("get_numa_node_for_addr", &C::get_numa_node_for_addr, py::arg("addr"))
        .def("get_local_nic_indices_for_numa", &C::get_local_nic_indices_for_numa, py::arg("numa_node"))
        .def("get_gpu_numa_node", &C::get_gpu_numa_node, py::arg("gpu_device_id"))
        .def("map_dram_to_gpu", &C::map_dram_to_gpu, py::arg("host_addr"), py::arg("length"))
        .def("unmap_dram_from_gpu", &C::unmap_dram_from_gpu, py::arg("host_addr"))
        .def("tma_gather", &C::tma_gather, py::arg("dram_dev_ptr"), py::arg("indices_ptr"), py::arg("gpu_dst_ptr"),
             py::arg("num_blocks"), py::arg("block_size"), py::arg("max_sm_count") = 0, py::arg("mode") = 0,
             py::arg("stream") = 0,
             "Gather blocks from mapped DRAM into HBM. mode: 0=AUTO, 1=SM, 2=TMA. stream: cudaStream_t "
             "(0 = legacy default stream).")
        .def("tma_scatter", &C::tma_scatter, py::arg("gpu_src_ptr"), py::arg("indices_ptr"),
             py::arg("dram_dev_ptr"), py::arg("num_blocks"), py::arg("block_size"), py::arg("max_sm_count") = 0,
             py::arg("mode") = 0, py::arg("stream") = 0)
        .def("set_fabric_stream", &C::set_fabric_stream, py::arg("stream"))
        .def("get_fabric_name", &C::get_fabric_name)
        .def_static("get_kernel_launch_count", [] { return MPComm::getKernelLaunchCount(); });

    // ---- kernel entry points (used by mpcomm.ops) ----
    m.def("crc32_blocks",
          [](uintptr_t data, int64_t n, int64_t bs, uintptr_t out, uintptr_t stream) {
              py::gil_scoped_release r;
              return check(kern::crc32_blocks(reinterpret_cast<const void *>(data), n, bs,
                                              reinterpret_cast<uint32_t *>(out), reinterpret_cast<void *>(stream)));
          },
          py::arg("data"), py::arg("num_blocks"), py::arg("block_size"), py::arg("out"), py::arg("stream") = 0);
    m.def("crc32_host",
          [](py::bytes b, uint32_t crc) {
              std::string s = b;
              return kern::crc32_host(s.data(), s.size(), crc);
          },
          py::arg("data"), py::arg("crc") = 0);
    m.def("crc32_host_ptr",
          [](uintptr_t p, size_t len, uint32_t crc) {
              py::gil_scoped_release r;
              return kern::crc32_host(reinterpret_cast<const void *>(p), len, crc);
          },
          py::arg("addr"), py::arg("length"), py::arg("crc") = 0);
    m.def("paged_gather",
          [](uintptr_t pool, int64_t pool_blocks, uintptr_t idx, uintptr_t out, int64_t n, int64_t bs, int mode,
             int max_ctas, uintptr_t stream) {
              kern::LaunchInfo li;
              int e;
              {
                  py::gil_scoped_release r;
                  e = kern::h2d_gather(reinterpret_cast<const void *>(pool), pool_blocks,
                                       reinterpret_cast<const int64_t *>(idx), reinterpret_cast<void *>(out), n, bs,
                                       mode, max_ctas, reinterpret_cast<void *>(stream), nullptr, nullptr, nullptr,
                                       &li);
              }
              return py::make_tuple(e, li.ctas, li.path);
          },
          py::arg("pool"), py::arg("pool_blocks"), py::arg("indices"), py::arg("out"), py::arg("num_blocks"),
          py::arg("block_size"), py::arg("mode") = 0, py::arg("max_ctas") = 0, py::arg("stream") = 0);
    m.def("paged_scatter",
          [](uintptr_t src, uintptr_t idx, uintptr_t pool, int64_t pool_blocks, int64_t n, int64_t bs, int mode,
             int max_ctas, uintptr_t stream) {
              kern::LaunchInfo li;
              int e;
              {
                  py::gil_scoped_release r;
                  e = kern::h2d_scatter(reinterpret_cast<const void *>(src), reinterpret_cast<const int64_t *>(idx),
                                        reinterpret_cast<void *>(pool), pool_blocks, n, bs, mode, max_ctas,
                                        reinterpret_cast<void *>(stream), nullptr, nullptr, nullptr, &li);
              }
              return py::make_tuple(e, li.ctas, li.path);
          },
          py::arg("src"), py::arg("indices"), py::arg("pool"), py::arg("pool_blocks"), py::arg("num_blocks"),
          py::arg("block_size"), py::arg("mode") = 0, py::arg("max_ctas") = 0, py::arg("stream") = 0);
    m.def("copy_spans",
          [](const std::vector<uintptr_t> &src, const std::vector<uintptr_t> &dst, const std::vector<uint64_t> &len,
             int max_ctas, uintptr_t stream, int mode, uintptr_t gate, uint64_t gate_budget_ns) {
              if (src.size() != dst.size() || src.size() != len.size() || src.size() > kern::kMaxCopyDescs)
                  return static_cast<int>(MPCOMM_ERR_INVALID_ARG);
              std::vector<kern::CopyDesc> d(src.size());
              for (size_t i = 0; i < src.size(); ++i)
                  d[i] = kern::CopyDesc{reinterpret_cast<const void *>(src[i]), reinterpret_cast<void *>(dst[i]), len[i]};
              py::gil_scoped_release r;
              return kern::copy_batch(d.data(), static_cast<int>(d.size()), max_ctas,
                                      reinterpret_cast<void *>(stream), nullptr, nullptr, mode,
                                      reinterpret_cast<const uint32_t *>(gate), gate_budget_ns);
          },
          py::arg("src"), py::arg("dst"), py::arg("lengths"), py::arg("max_ctas") = 0, py::arg("stream") = 0,
          py::arg("mode") = 0, py::arg("gate") = 0, py::arg("gate_budget_ns") = 0);
    m.def("pxn_gather_forward",
          [](uintptr_t pool, int64_t pool_blocks, uintptr_t idx, uintptr_t dst, int64_t n, int64_t bs, int max_ctas,
             uintptr_t stream, uintptr_t flag, uint64_t flag_value, uintptr_t ctr) {
              py::gil_scoped_release r;
              return kern::pxn_gather_forward(reinterpret_cast<const void *>(pool), pool_blocks,
                                              reinterpret_cast<const int64_t *>(idx), reinterpret_cast<void *>(dst), n,
                                              bs, max_ctas, reinterpret_cast<void *>(stream), nullptr,
                                              reinterpret_cast<uint64_t *>(flag), flag_value,
                                              reinterpret_cast<uint32_t *>(ctr), nullptr);
          },
          py::arg("pool"), py::arg("pool_blocks"), py::arg("indices"), py::arg("dst"), py::arg("num_blocks"),
          py::arg("block_size"), py::arg("max_ctas") = 0, py::arg("stream") = 0, py::arg("done_flag") = 0,
          py::arg("flag_value") = 1, py::arg("counter") = 0);
    m.def("gather_bcast",
          [](uintptr_t pool, int64_t pool_blocks, uintptr_t idx, int64_t n, int64_t bs, uintptr_t mc,
             const std::vector<uintptr_t> &dsts, uintptr_t mc_flag, const std::vector<uintptr_t> &flags,
             uint64_t flag_value, uintptr_t ctr, int max_ctas, uintptr_t stream, uintptr_t status) {
              std::vector<void *> d;
              for (auto p : dsts) d.push_back(reinterpret_cast<void *>(p));
              std::vector<uint64_t *> f;
              for (auto p : flags) f.push_back(reinterpret_cast<uint64_t *>(p));
              py::gil_scoped_release r;
              return kern::gather_bcast(reinterpret_cast<const void *>(pool), pool_blocks,
                                        reinterpret_cast<const int64_t *>(idx), n, bs, reinterpret_cast<void *>(mc),
                                        d.data(), static_cast<int>(d.size()), reinterpret_cast<uint64_t *>(mc_flag),
                                        f.data(), static_cast<int>(f.size()), flag_value,
                                        reinterpret_cast<uint32_t *>(ctr), max_ctas, reinterpret_cast<void *>(stream),
                                        reinterpret_cast<uint32_t *>(status), nullptr);
          },
          py::arg("pool"), py::arg("pool_blocks"), py::arg("indices"), py::arg("num_blocks"), py::arg("block_size"),
          py::arg("mc_dst") = 0, py::arg("dsts") = std::vector<uintptr_t>{}, py::arg("mc_flag") = 0,
          py::arg("flags") = std::vector<uintptr_t>{}, py::arg("flag_value") = 1, py::arg("counter") = 0,
          py::arg("max_ctas") = 0, py::arg("stream") = 0, py::arg("status") = 0);
    m.def("nvls_broadcast",
          [](uintptr_t src, uintptr_t mc, uint64_t bytes, int max_ctas, uintptr_t stream) {
              py::gil_scoped_release r;
              return kern::nvls_broadcast(reinterpret_cast<const void *>(src), reinterpret_cast<void *>(mc), bytes,
                                          max_ctas, reinterpret_cast<void *>(stream), nullptr);
          },
          py::arg("src"), py::arg("mc_dst"), py::arg("bytes"), py::arg("max_ctas") = 0, py::arg("stream") = 0);
    m.def("p2p_fanout",
          [](uintptr_t src, const std::vector<uintptr_t> &dsts, uint64_t bytes, int max_ctas, uintptr_t stream) {
              std::vector<void *> d;
              for (auto p : dsts) d.push_back(reinterpret_cast<void *>(p));
              py::gil_scoped_release r;
              return kern::p2p_fanout(reinterpret_cast<const void *>(src), d.data(), static_cast<int>(d.size()),
                                      bytes, max_ctas, reinterpret_cast<void *>(stream), nullptr);
          },
          py::arg("src"), py::arg("dsts"), py::arg("bytes"), py::arg("max_ctas") = 0, py::arg("stream") = 0);
    m.def("wait_flag",
          [](uintptr_t flag, uint64_t value, uint64_t budget_ns, uintptr_t stream, uintptr_t status) {
              py::gil_scoped_release r;
              return kern::wait_flag(reinterpret_cast<const uint64_t *>(flag), value, budget_ns,
                                     reinterpret_cast<void *>(stream), reinterpret_cast<uint32_t *>(status));
          },
          py::arg("flag"), py::arg("value"), py::arg("budget_ns"), py::arg("stream") = 0, py::arg("status") = 0);
    m.def("kernel_launch_count", [] { return kern::launch_count(); });
    m.def(
        "copy_roundtrip_us",
        [](uintptr_t src, uintptr_t dst, size_t bytes, int iters, int ctas) {
            // The floor under one engine WR: a copy_batch launch that stores
            // its done word into pinned host memory, timed from the launch
            // call until this thread sees the word (the engine's path minus
            // the engine). Spins are bounded (1 s per launch).
            py::list out;
            auto *word = static_cast<uint64_t *>(gpu::host_alloc_mapped(64));
            auto *ctr = static_cast<uint32_t *>(gpu::device_alloc(64));
            void *stream = gpu::stream_create(gpu::current_device());
            if (!word || !ctr || !stream || gpu::memset_device(ctr, 0, 64) != 0) {
                if (word) gpu::host_free(word);
                if (ctr) gpu::device_free(ctr);
                if (stream) gpu::stream_destroy(stream);
                return out;
            }
            {
                py::gil_scoped_release r;
                kern::CopyDesc d{reinterpret_cast<const void *>(src), reinterpret_cast<void *>(dst), bytes};
                using C = std::chrono::steady_clock;
                std::vector<double> us;
                for (int i = 1; i <= iters; ++i) {
                    const auto t0 = C::now();
                    if (kern::copy_batch(&d, 1, ctas, stream, nullptr, nullptr, kern::kModeAuto, nullptr, 0, word,
                                         static_cast<uint64_t>(i), ctr) != 0)
                        break;
                    bool seen = false;
                    while (C::now() - t0 < std::chrono::seconds(1))
                        if (__atomic_load_n(word, __ATOMIC_ACQUIRE) >= static_cast<uint64_t>(i)) {
                            seen = true;
                            break;
                        }
                    if (!seen) break;
                    us.push_back(std::chrono::duration<double, std::micro>(C::now() - t0).count());
                }
                gpu::stream_sync(stream);
                py::gil_scoped_acquire a;
                for (double v : us) out.append(v);
            }
            gpu::stream_destroy(stream);
            gpu::device_free(ctr);
            gpu::host_free(word);
            return out;
        },
        py::arg("src"), py::arg("dst"), py::arg("bytes"), py::arg("iters") = 200, py::arg("ctas") = 4,
        "Per-launch round trips (us) of one copy_batch launch to its host-visible done word: the floor under "
        "an engine transfer of `bytes`.");
    m.def("kernel_trace", [] {
        std::vector<kern::TraceRecord> raw;
        int e;
        {
            py::gil_scoped_release r;
            e = kern::kernel_trace(&raw);
        }
        if (e != 0) throw std::runtime_error(std::string("kernel_trace: ") + gpu::error_string(e));
        py::list out;
        for (const auto &t : raw) {
            py::dict d;
            d["seq"] = t.seq;
            d["device"] = t.dev;
            d["kind"] = t.kind ? t.kind : "";
            d["bytes"] = t.bytes;
            d["begin_ns"] = t.begin_ns;
            d["end_ns"] = t.end_ns;
            d["duration_us"] = (t.end_ns - t.begin_ns) / 1000.0;
            out.append(d);
        }
        return out;
    });
    m.def("kernel_trace_reset", [] { kern::kernel_trace_reset(); });
    m.def("_set_nvls_variant", [](int v) { kern::set_nvls_variant(v); });
    m.def("kernel_trace_slots", [] { return kern::kernel_trace_slots(); });
    m.def("kernel_wait_budget_ns", [] { return kern::wait_budget_ns(); });

    // ---- cross-process GPU memory (mpcomm.parallel) ----
    m.def("ipc_export", [](uintptr_t ptr) {
        unsigned char h[64] = {0};
        uint64_t off = 0;
        int e = vmm::ipc_export(reinterpret_cast<const void *>(ptr), h, &off);
        return py::make_tuple(e, py::bytes(reinterpret_cast<const char *>(h), 64), off);
    });
    m.def("ipc_import", [](py::bytes handle) -> py::tuple {
        std::string s = handle;
        if (s.size() != 64) return py::make_tuple(static_cast<int>(MPCOMM_ERR_INVALID_ARG), 0);
        void *base = nullptr;
        int e = vmm::ipc_import(reinterpret_cast<const unsigned char *>(s.data()), &base);
        return py::make_tuple(e, reinterpret_cast<uintptr_t>(base));
    });
    m.def("ipc_release", [](uintptr_t base) { return vmm::ipc_release(reinterpret_cast<void *>(base)); });
    m.def("host_register", [](uintptr_t ptr, size_t len) {
        void *d = nullptr;
        bool pinned = false;
        int e;
        {
            py::gil_scoped_release r;
            e = gpu::host_pin_mapped(reinterpret_cast<void *>(ptr), len, &d, &pinned);
        }
        return py::make_tuple(e, reinterpret_cast<uintptr_t>(d), pinned);
    });
    m.def("host_unregister", [](uintptr_t ptr) { return gpu::host_unpin(reinterpret_cast<void *>(ptr)); });
    m.def(
        "host_bandwidth",
        [](size_t bytes, int threads, int node, int reps) {
            topo::HostBandwidth b;
            bool ok;
            {
                py::gil_scoped_release r;
                ok = topo::host_bandwidth(bytes, threads, node, reps, &b);
            }
            py::dict d;
            if (!ok) return d;
            d["write_gbs"] = b.write_gbs;
            d["read_gbs"] = b.read_gbs;
            d["threads"] = b.threads;
            return d;
        },
        py::arg("bytes"), py::arg("threads") = 0, py::arg("node") = -1, py::arg("reps") = 3,
        "Host DRAM write (memset) and read bandwidth of `threads` CPU threads over a `bytes` buffer, GB/s; "
        "no device involved. Empty dict if the buffer cannot be allocated.");
    m.def(
        "copy_engine_async",
        [](uintptr_t dst, uintptr_t src, size_t bytes, uintptr_t stream) {
            return gpu::copy_engine_async(reinterpret_cast<void *>(dst), reinterpret_cast<const void *>(src), bytes,
                                          reinterpret_cast<void *>(stream));
        },
        py::arg("dst"), py::arg("src"), py::arg("bytes"), py::arg("stream") = 0,
        "cudaMemcpyAsync(cudaMemcpyDefault) on `stream` (the copy engine; a comparator for the benches).");
    m.def("enable_peer_access", &gpu::enable_peer_access, py::arg("device"), py::arg("peer"),
          "Lets kernels on `device` access memory of `peer` (0 or a CUDA error).");
    m.def("multicast_supported", &vmm::multicast_supported, py::arg("device"));
    m.def("multicast_granularity", [](size_t size, int ndev) {
        size_t g = 0;
        int e = vmm::multicast_granularity(size, ndev, &g);
        return py::make_tuple(e, g);
    });
    m.def("multicast_create", [](size_t size, int ndev) {
        uint64_t mc = 0;
        int fd = -1;
        int e = vmm::multicast_create(size, ndev, &mc, &fd);
        return py::make_tuple(e, mc, fd);
    });
    m.def("multicast_import", [](int fd) {
        uint64_t mc = 0;
        int e = vmm::multicast_import(fd, &mc);
        return py::make_tuple(e, mc);
    });
    m.def("multicast_add_device", &vmm::multicast_add_device, py::arg("mc"), py::arg("device"));
    m.def("multicast_bind_local", [](uint64_t mc, size_t size, int dev) {
        uint64_t mem = 0;
        void *va = nullptr;
        int e = vmm::multicast_bind_local(mc, size, dev, &mem, &va);
        return py::make_tuple(e, mem, reinterpret_cast<uintptr_t>(va));
    });
    m.def("multicast_map", [](uint64_t mc, size_t size, int dev) {
        void *va = nullptr;
        int e = vmm::multicast_map(mc, size, dev, &va);
        return py::make_tuple(e, reinterpret_cast<uintptr_t>(va));
    });
    m.def(
        "gdr_alloc",
        [](int dev, size_t size) {
            void *p = nullptr;
            size_t n = 0;
            int e = vmm::gdr_alloc(dev, size, &p, &n);
            return py::make_tuple(e, reinterpret_cast<uintptr_t>(p), n);
        },
        py::arg("device"), py::arg("size"),
        "(err, ptr, alloc_size): HBM created for GPUDirect RDMA (dma-buf exportable), mapped for `device`.");
    m.def("gdr_free", [](uintptr_t p, size_t n) { return vmm::gdr_free(reinterpret_cast<void *>(p), n); },
          py::arg("ptr"), py::arg("alloc_size"));
    m.def(
        "dmabuf_export_rc",
        [](uintptr_t p, size_t n, unsigned long long flags) {
            int fd = -1;
            int e = vmm::dmabuf_export(reinterpret_cast<void *>(p), n, flags, &fd);
            if (e == 0 && fd >= 0) ::close(fd);
            return e;
        },
        py::arg("ptr"), py::arg("size"), py::arg("flags") = 0,
        "Driver result of exporting [ptr, ptr+size) as a dma-buf (the fd is closed again).");
    m.def(
        "vmm_segments",
        [](uintptr_t ptr, size_t len) {
            std::vector<vmm::VmmSegment> segs;
            const int e = vmm::vmm_segments(reinterpret_cast<void *>(ptr), len, 1u << 20, &segs);
            py::list out;
            for (const auto &g : segs) out.append(py::make_tuple(g.base, g.size));
            return py::make_tuple(e, out);
        },
        py::arg("ptr"), py::arg("length"),
        "(err, [(base, size), ...]): the VMM allocations behind [ptr, ptr+length) (err != 0 for memory that is "
        "not VMM-mapped, e.g. cudaMalloc).");
    m.def(
        "vmm_offer",
        [](uintptr_t ptr, size_t len) {
            static std::atomic<uint64_t> next{1ull << 40};  // apart from the fabric's registration keys
            const uint64_t key = next++;
            uintptr_t base = 0;
            size_t span = 0;
            const int e = vmm::vmm_offer(reinterpret_cast<void *>(ptr), len, key, &base, &span);
            return py::make_tuple(e, e ? 0 : key, base, span);
        },
        py::arg("ptr"), py::arg("length"),
        "(err, key, base, span): offers VMM memory [ptr, ptr+length) to peer processes of this host (what CUDA IPC "
        "cannot export); a peer maps it with vmm_open(pid, key, device), where its address stands for `base`.");
    m.def("vmm_withdraw", &vmm::vmm_withdraw, py::arg("key"));
    m.def(
        "vmm_open",
        [](long pid, uint64_t key, int dev, int timeout_ms) {
            void *va = nullptr;
            std::vector<size_t> sizes;
            int e;
            {
                py::gil_scoped_release r;
                e = vmm::vmm_open(pid, key, dev, timeout_ms, &va, &sizes);
            }
            return py::make_tuple(e, reinterpret_cast<uintptr_t>(va), sizes);
        },
        py::arg("pid"), py::arg("key"), py::arg("device"), py::arg("timeout_ms") = 5000,
        "(err, va, sizes): maps what process `pid` offered under `key` for `device`; release with vmm_unmap.");
    m.def(
        "vmm_unmap",
        [](uintptr_t va, const std::vector<size_t> &sizes) { return vmm::vmm_unmap(reinterpret_cast<void *>(va), sizes); },
        py::arg("va"), py::arg("sizes"));
    m.def(
        "multicast_group",
        [](const std::string &name, size_t bytes, int members, bool create, int timeout_ms) {
            mpcomm::MulticastGroup g;
            int e;
            {
                py::gil_scoped_release r;
                e = create ? mpcomm::createMulticastGroup(name, bytes, members, &g, timeout_ms)
                           : mpcomm::joinMulticastGroup(name, bytes, members, &g, timeout_ms);
            }
            py::dict d;
            if (e == 0) {
                d["uc_addr"] = reinterpret_cast<uintptr_t>(g.uc_addr);
                d["mc_addr"] = reinterpret_cast<uintptr_t>(g.mc_addr);
                d["length"] = g.length;
                d["token"] = g.token;
                d["members"] = g.members;
                d["device"] = g.device;
                d["mc_handle"] = g.mc_handle;
                d["mem_handle"] = g.mem_handle;
            }
            return py::make_tuple(e, d);
        },
        py::arg("name"), py::arg("bytes"), py::arg("members"), py::arg("create"), py::arg("timeout_ms") = 60000,
        "(err, group): create (create=True, one process) or join an NVLS multicast group of `members` GPUs by "
        "name, on the current device, without a launcher; err is an MPCOMM_ERR_* code. Release with "
        "multicast_teardown(mc_handle, mem_handle, uc_addr, mc_addr, length, device).");
    m.def("multicast_teardown", [](uint64_t mc, uint64_t mem, uintptr_t uc, uintptr_t mcva, size_t size, int dev) {
        return vmm::multicast_teardown(mc, mem, reinterpret_cast<void *>(uc), reinterpret_cast<void *>(mcva), size,
                                       dev);
    });

    // ---- host-side fault hooks of the loopback fabric (tests) ----
    m.def("_lo_inject_wc_errors", &fabric::loopback_inject_wc_errors, py::arg("gid"), py::arg("count"));
    m.def("_lo_set_port_active", &fabric::loopback_set_port_active, py::arg("gid"), py::arg("active"));
    m.def("_lo_set_wr_delay_us", &fabric::loopback_set_wr_delay_us, py::arg("gid"), py::arg("us"));
}
