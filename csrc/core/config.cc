#include "core/config.h"

#include <cerrno>
#include <cstdlib>
#include <cstring>

#include "mpcomm_log.h"

namespace mpcomm {
namespace {

const char *env(const char *name) {
    const char *v = std::getenv(name);
    return (v && *v) ? v : nullptr;
}

template <typename T>
bool read_int(const char *name, long long lo, long long hi, T *out) {
    const char *v = env(name);
    if (!v) return false;
    errno = 0;
    char *end = nullptr;
    long long x = std::strtoll(v, &end, 0);
    if (errno || !end || *end || x < lo || x > hi) {
        MPCOMM_LOG_WARN("MPComm: ignoring %s=%s (valid range [%lld, %lld])\n", name, v, lo, hi);
        return false;
    }
    *out = static_cast<T>(x);
    return true;
}

bool read_u64(const char *name, uint64_t *out) {
    const char *v = env(name);
    if (!v) return false;
    errno = 0;
    char *end = nullptr;
    unsigned long long x = std::strtoull(v, &end, 0);
    if (errno || !end || *end || v[0] == '-') {
        MPCOMM_LOG_WARN("MPComm: ignoring %s=%s (expected unsigned integer)\n", name, v);
        return false;
    }
    *out = x;
    return true;
}

bool read_double(const char *name, double lo, double hi, double *out) {
    const char *v = env(name);
    if (!v) return false;
    errno = 0;
    char *end = nullptr;
    double x = std::strtod(v, &end);
    if (errno || !end || *end || x < lo || x > hi) {
        MPCOMM_LOG_WARN("MPComm: ignoring %s=%s (valid range [%g, %g])\n", name, v, lo, hi);
        return false;
    }
    *out = x;
    return true;
}

// Any value other than "0" enables (reference :1499-1507 semantics).
bool read_flag(const char *name, bool *out) {
    const char *v = env(name);
    if (!v) return false;
    *out = std::strcmp(v, "0") != 0;
    return true;
}

bool read_str(const char *name, std::string *out) {
    const char *v = env(name);
    if (!v) return false;
    *out = v;
    return true;
}

}  // namespace

Config Config::from_env() {
    Config c;
    read_str("MPCOMM_NIC_FILTER", &c.nic_filter);
    c.max_rdma_transfer_size_set =
        read_int("MPCOMM_MAX_RDMA_TRANSFER_SIZE", 1, 1ll << 40, &c.max_rdma_transfer_size);
    read_int("MPCOMM_QPS_PER_CONNECTION", 1, 16, &c.qps_per_connection);
    c.max_outstanding_set =
        read_int("MPCOMM_MAX_OUTSTANDING_PER_QP", 1, 8192, &c.max_outstanding_per_qp);
    read_int("MPCOMM_GID_INDEX", -1, 255, &c.gid_index);
    read_int("MPCOMM_ROCE_DSCP", 0, 63, &c.roce_dscp);
    read_int("MPCOMM_POLL_BATCH_SIZE", 1, 256, &c.poll_batch_size);
    read_int("MPCOMM_MAX_SEND_WR", 1, 8192, &c.max_send_wr);
    read_int("MPCOMM_MAX_IDLE_SPINS", 1, 10000000, &c.max_idle_spins);
    read_int("MPCOMM_TRANSFER_STATS_INTERVAL", 0, 1ll << 40, &c.transfer_stats_interval);
    read_flag("MPCOMM_PCIE_STAT_ENABLE", &c.pcie_stat_enable);
    read_flag("MPCOMM_H2D_QOS_ENABLE", &c.h2d_qos_enable);
    read_u64("MPCOMM_H2D_QOS_RATE_BPS", &c.h2d_qos_rate_bps);
    read_u64("MPCOMM_H2D_QOS_BURST_BYTES", &c.h2d_qos_burst_bytes);
    read_u64("MPCOMM_QOS_DEVICE_PAUSE_US", &c.qos_device_pause_us);
    read_flag("MPCOMM_QOS_REMOTE", &c.qos_remote);
    read_int("MPCOMM_NIC_PROBE_INTERVAL", 1, 1ll << 40, &c.nic_probe_interval);
    read_double("MPCOMM_NIC_QUARANTINE_SEC", 0.0, 1e6, &c.nic_quarantine_sec);
    read_double("MPCOMM_FAULT_INJECT_AFTER_SEC", 0.0, 1e9, &c.fault_after_sec);
    read_int("MPCOMM_FAULT_INJECT_NIC", 0, 255, &c.fault_nic);
    if (read_str("MPCOMM_FAULT_INJECT_MODE", &c.fault_mode) && c.fault_mode != "single_qp" &&
        c.fault_mode != "all_qp" && c.fault_mode != "all_nic") {
        MPCOMM_LOG_WARN("MPComm: unknown MPCOMM_FAULT_INJECT_MODE=%s, using single_qp\n",
                        c.fault_mode.c_str());
        c.fault_mode = "single_qp";
    }
    read_double("MPCOMM_FAULT_INJECT_RECOVER_AFTER_SEC", 0.0, 1e9, &c.fault_recover_after_sec);
    read_flag("MPCOMM_FAULT_INJECT_TOLERATE", &c.fault_tolerate);
    read_flag("MPCOMM_PXN_ENABLE", &c.pxn_enable);
    read_int("MPCOMM_PXN_BUFFER_SIZE", 1 << 20, 1ll << 40, &c.pxn_buffer_size);
    read_double("MPCOMM_PXN_NVLINK_ALPHA", 0.0, 1e6, &c.pxn_nvlink_alpha);
    read_flag("MPCOMM_PXN_BENCH_SEQUENTIAL", &c.pxn_bench_sequential);
    read_int("MPCOMM_PXN_PROXY_NICS", 0, 16, &c.pxn_proxy_nics);
    read_str("MPCOMM_FABRIC", &c.fabric);
    read_int("MPCOMM_NVL_CHUNK_SIZE", 4096, 1ll << 40, &c.nvl_chunk_size);
    read_int("MPCOMM_NVL_OUTSTANDING_PER_QP", 1, 1024, &c.nvl_outstanding_per_qp);
    read_int("MPCOMM_NVL_CTAS_PER_QP", 0, 4096, &c.nvl_ctas_per_qp);
    read_int("MPCOMM_LOOPBACK_NICS", 1, 16, &c.loopback_nics);
    read_flag("MPCOMM_STAGING_ENABLE", &c.staging_enable);
    read_int("MPCOMM_STAGING_SLAB_BYTES", 4096, 1ll << 32, &c.staging_slab_bytes);
    read_int("MPCOMM_STAGING_SLABS", 2, 4096, &c.staging_slabs);
    read_int("MPCOMM_STAGING_THREADS", 1, 256, &c.staging_threads);
    read_int("MPCOMM_STAGING_DEVICE_SLAB_BYTES", 4096, 1ll << 32, &c.staging_device_slab_bytes);
    if (read_str("MPCOMM_NIC_PAIRING", &c.nic_pairing) && c.nic_pairing != "suffix" &&
        c.nic_pairing != "index") {
        MPCOMM_LOG_WARN("MPComm: unknown MPCOMM_NIC_PAIRING=%s, using suffix\n",
                        c.nic_pairing.c_str());
        c.nic_pairing = "suffix";
    }
    read_flag("MPCOMM_REPOST_ON_FAILURE", &c.repost_on_failure);
    read_flag("MPCOMM_FUSED_BROADCAST", &c.fused_broadcast);
    read_int("MPCOMM_PAGED_CHUNK_SIZE", 4096, 1ll << 30, &c.paged_chunk_size);
    read_str("MPCOMM_CONFIG_FILE", &c.config_file);
    return c;
}

}  // namespace mpcomm
