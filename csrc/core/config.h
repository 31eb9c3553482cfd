// Environment configuration, read once per MPComm object at construction.
// An out-of-range or unparsable value logs a warning and keeps the default
// (reference behaviour, src/mpcomm.cpp:1372-1569). Every variable the
// reference reads is accepted here with the same name and range; the ones
// marked (b200) are new.
#ifndef MPCOMM_B200_CSRC_CORE_CONFIG_H_
#define MPCOMM_B200_CSRC_CORE_CONFIG_H_

#include <cstddef>
#include <cstdint>
#include <string>

namespace mpcomm {

struct Config {
    // ---- data plane (reference) ----
    std::string nic_filter;                  // MPCOMM_NIC_FILTER (CSV)
    size_t max_rdma_transfer_size = 128 << 10;   // MPCOMM_MAX_RDMA_TRANSFER_SIZE
    bool max_rdma_transfer_size_set = false;
    size_t qps_per_connection = 4;           // MPCOMM_QPS_PER_CONNECTION [1,16]
    size_t max_outstanding_per_qp = 2;       // MPCOMM_MAX_OUTSTANDING_PER_QP [1,8192]
    bool max_outstanding_set = false;
    int gid_index = 3;                       // MPCOMM_GID_INDEX [-1,255]
    int roce_dscp = 0;                       // MPCOMM_ROCE_DSCP [0,63]
    size_t poll_batch_size = 64;             // MPCOMM_POLL_BATCH_SIZE [1,256]
    int max_send_wr = 512;                   // MPCOMM_MAX_SEND_WR [1,8192]
    size_t max_idle_spins = 10000;           // MPCOMM_MAX_IDLE_SPINS [1,1e7]
    size_t transfer_stats_interval = 0;      // MPCOMM_TRANSFER_STATS_INTERVAL
    bool pcie_stat_enable = false;           // MPCOMM_PCIE_STAT_ENABLE
    bool h2d_qos_enable = false;             // MPCOMM_H2D_QOS_ENABLE
    uint64_t h2d_qos_rate_bps = 0;           // MPCOMM_H2D_QOS_RATE_BPS
    uint64_t h2d_qos_burst_bytes = 0;        // MPCOMM_H2D_QOS_BURST_BYTES
    // Device-side pause of background GPU-fabric H2D copies while an H2D
    // window is open (rate 0 only): total pause per copy pipeline, us.
    uint64_t qos_device_pause_us = 2000;     // MPCOMM_QOS_DEVICE_PAUSE_US (0 = host gating only)
    // Send pause/clear frames to every peer with an open QoS control channel
    // around each QoS-windowed tmaGather/tmaScatter.
    bool qos_remote = false;                 // MPCOMM_QOS_REMOTE
    size_t nic_probe_interval = 10000;       // MPCOMM_NIC_PROBE_INTERVAL (loops)
    double nic_quarantine_sec = 5.0;         // MPCOMM_NIC_QUARANTINE_SEC
    // ---- fault injection (host side only) ----
    double fault_after_sec = -1.0;           // MPCOMM_FAULT_INJECT_AFTER_SEC
    int fault_nic = 0;                       // MPCOMM_FAULT_INJECT_NIC
    std::string fault_mode = "single_qp";    // MPCOMM_FAULT_INJECT_MODE
    double fault_recover_after_sec = -1.0;   // MPCOMM_FAULT_INJECT_RECOVER_AFTER_SEC
    bool fault_tolerate = false;             // MPCOMM_FAULT_INJECT_TOLERATE
    // ---- PXN ----
    bool pxn_enable = false;                 // MPCOMM_PXN_ENABLE
    size_t pxn_buffer_size = 256ull << 20;   // MPCOMM_PXN_BUFFER_SIZE
    double pxn_nvlink_alpha = 1.0;           // MPCOMM_PXN_NVLINK_ALPHA
    bool pxn_bench_sequential = false;       // MPCOMM_PXN_BENCH_SEQUENTIAL
    size_t pxn_proxy_nics = 0;               // MPCOMM_PXN_PROXY_NICS (0 = all)
    // ---- (b200) ----
    std::string fabric = "auto";             // MPCOMM_FABRIC
    size_t nvl_chunk_size = 32ull << 20;     // MPCOMM_NVL_CHUNK_SIZE
    size_t nvl_outstanding_per_qp = 4;       // MPCOMM_NVL_OUTSTANDING_PER_QP
    int nvl_ctas_per_qp = 0;                 // MPCOMM_NVL_CTAS_PER_QP (0 = SMs/qps)
    int loopback_nics = 2;                   // MPCOMM_LOOPBACK_NICS [1,16]
    bool staging_enable = true;              // MPCOMM_STAGING_ENABLE
    size_t staging_slab_bytes = 4ull << 20;  // MPCOMM_STAGING_SLAB_BYTES
    size_t staging_slabs = 16;               // MPCOMM_STAGING_SLABS
    size_t staging_threads = 4;              // MPCOMM_STAGING_THREADS
    size_t staging_device_slab_bytes = 32ull << 20;  // MPCOMM_STAGING_DEVICE_SLAB_BYTES
    std::string nic_pairing = "suffix";      // MPCOMM_NIC_PAIRING suffix|index
    bool repost_on_failure = true;           // MPCOMM_REPOST_ON_FAILURE
    bool fused_broadcast = true;             // MPCOMM_FUSED_BROADCAST
    size_t paged_chunk_size = 1ull << 30;    // MPCOMM_PAGED_CHUNK_SIZE (bytes of pages per launch)
    std::string config_file;                 // MPCOMM_CONFIG_FILE (version json)

    // Reads all variables from the process environment.
    static Config from_env();
};

}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_CORE_CONFIG_H_
