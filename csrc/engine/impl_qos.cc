// QoS: legacy throttle, H2D-window post pacing, PCIe-domain accounting.
//
// H2D windows. Each tmaGather/tmaScatter launch (while QoS is enabled)
// takes a slot in pinned, device-mapped host memory; the kernel itself
// stamps begin_ns when its first CTA starts and end_ns (system-scope
// release) when its last CTA has drained its stores. Workers consult the
// slots of a rail's PCIe-affine GPU before posting a READ chunk: while a
// window is open the chunk is paused (rate 0) or paced by the shared token
// bucket, and posting resumes by itself when the kernel closes the window.
// The reference declares this behaviour (include/mpcomm.h:437-446) but its
// tmaGather never triggers it (src/mpcomm.cpp:7892-7894).
#include <algorithm>
#include <cstring>

#include "cuda/gpu.h"
#include "engine/impl.h"
#include "mpcomm_log.h"

namespace mpcomm {

MPComm::Impl::WindowPool::~WindowPool() {
    gpu::host_free(slots);
    for (auto *c : ctrs) gpu::device_free(c);
    for (auto *g : gates) gpu::device_free(g);
}

void MPComm::Impl::setNicThrottle(size_t outstanding, size_t chunk) {
    throttle_outstanding_.store(outstanding, std::memory_order_relaxed);
    throttle_chunk_.store(chunk, std::memory_order_relaxed);
    throttle_seen_ns_.store(0, std::memory_order_relaxed);
    throttle_drained_ns_.store(0, std::memory_order_relaxed);
    throttle_snapshot_.store(0, std::memory_order_relaxed);
    throttle_drain_pending_.store(true, std::memory_order_relaxed);
    throttle_enabled_.store(true, std::memory_order_relaxed);
    throttle_set_ns_.store(monotonic_raw_ns(), std::memory_order_relaxed);
    throttle_epoch_.fetch_add(1, std::memory_order_release);
    MPCOMM_LOG_INFO("MPComm: rail throttle set (outstanding_per_qp=%zu, chunk=%zu)\n", outstanding, chunk);
}

void MPComm::Impl::clearNicThrottle() {
    throttle_drain_pending_.store(false, std::memory_order_relaxed);
    throttle_enabled_.store(false, std::memory_order_relaxed);
    throttle_outstanding_.store(0, std::memory_order_relaxed);
    throttle_chunk_.store(0, std::memory_order_relaxed);
    throttle_epoch_.fetch_add(1, std::memory_order_release);
}

bool MPComm::Impl::getThrottleLatency(uint64_t *set, uint64_t *seen, uint64_t *drained,
                                      size_t *snap) const {
    if (set) *set = throttle_set_ns_.load();
    if (seen) *seen = throttle_seen_ns_.load();
    const uint64_t d = throttle_drained_ns_.load();
    if (drained) *drained = d;
    if (snap) *snap = throttle_snapshot_.load();
    return d != 0;
}

void MPComm::Impl::enableH2DQoS(uint64_t rate, uint64_t burst) {
    h2d_qos_enabled_.store(true, std::memory_order_release);
    setH2DQoSPolicy(rate, burst);
    MPCOMM_LOG_INFO("MPComm: H2D QoS enabled (rate=%lu B/s, burst=%lu B, device pause %s)\n",
                    static_cast<unsigned long>(rate), static_cast<unsigned long>(qos_bucket_.burst()),
                    device_gates_on_.load() ? "on" : "off");
}

void MPComm::Impl::setH2DQoSPolicy(uint64_t rate, uint64_t burst) {
    if (burst == 0 && rate != 0) burst = default_qos_burst(rate);
    qos_bucket_.configure(rate, burst);
    applyDeviceGates();
}

void MPComm::Impl::disableH2DQoS() {
    h2d_qos_enabled_.store(false, std::memory_order_release);
    applyDeviceGates();
}

// Device gating: with QoS on and rate 0 (pause), every GPU rail's H2D copy
// kernels watch their GPU's open-window counter and yield within one tile
// (host gating alone stops new posts but cannot recall launched chunks).
// A paced rate (> 0) stays host-side: the token bucket meters chunks.
void MPComm::Impl::applyDeviceGates() {
    const bool on = isH2DQoSEnabled() && qos_bucket_.rate() == 0 && cfg_.qos_device_pause_us > 0;
    std::lock_guard<std::mutex> lk(map_mu_);
    for (auto &r : rails_) {
        const int g = r->gpu;
        uint32_t *gate = (on && g >= 0 && ensureWindowPoolLocked()) ? deviceGateLocked(g) : nullptr;
        r->rail->set_qos_gate(gate, gate ? cfg_.qos_device_pause_us * 1000ull : 0);
    }
    device_gates_on_.store(on, std::memory_order_release);
}

bool MPComm::Impl::ensureWindowPoolLocked() {
    if (windows_) return true;
    windows_ = std::make_unique<WindowPool>();
    windows_->slots = static_cast<kern::H2DWindow *>(
        gpu::host_alloc_mapped(sizeof(kern::H2DWindow) * kMaxGpuDomains * kSlotsPerGpu));
    if (!windows_->slots) {
        windows_.reset();
        return false;
    }
    windows_live_.store(windows_.get(), std::memory_order_release);
    return true;
}

uint32_t *MPComm::Impl::deviceGateLocked(int g) {
    if (g < 0 || g >= static_cast<int>(kMaxGpuDomains)) return nullptr;
    WindowPool &p = *windows_;
    if (!p.gates[g]) {
        int prev = gpu::current_device();
        gpu::set_device(g);
        p.gates[g] = static_cast<uint32_t *>(gpu::device_alloc(128));
        if (p.gates[g]) gpu::memset_device(p.gates[g], 0, 128);
        if (prev >= 0) gpu::set_device(prev);
    }
    return p.gates[g];
}

bool MPComm::Impl::acquireH2DWindow(int g, kern::H2DWindow **win, uint32_t **ctr) {
    *win = nullptr;
    *ctr = nullptr;
    if (!isH2DQoSEnabled() || g < 0 || g >= static_cast<int>(kMaxGpuDomains)) return false;
    std::lock_guard<std::mutex> lk(map_mu_);
    if (!ensureWindowPoolLocked()) return false;
    WindowPool &p = *windows_;
    if (!p.ctrs[g]) {
        int prev = gpu::current_device();
        gpu::set_device(g);
        p.ctrs[g] = static_cast<uint32_t *>(gpu::device_alloc(sizeof(uint32_t) * kSlotsPerGpu));
        if (p.ctrs[g]) gpu::memset_device(p.ctrs[g], 0, sizeof(uint32_t) * kSlotsPerGpu);
        if (prev >= 0) gpu::set_device(prev);
        if (!p.ctrs[g]) return false;
    }
    for (int i = 0; i < kSlotsPerGpu; ++i) {
        kern::H2DWindow *s = &p.slots[g * kSlotsPerGpu + i];
        const uint32_t armed = __atomic_load_n(&s->armed, __ATOMIC_ACQUIRE);
        const uint64_t end = __atomic_load_n(&s->end_ns, __ATOMIC_ACQUIRE);
        if (armed && end == 0) continue;  // in use (pending or running)
        __atomic_store_n(&s->begin_ns, 0ull, __ATOMIC_RELAXED);
        __atomic_store_n(&s->end_ns, 0ull, __ATOMIC_RELAXED);
        s->gpu = g;
        s->gate = device_gates_on_.load(std::memory_order_acquire) ? deviceGateLocked(g) : nullptr;
        __atomic_store_n(&s->armed, 1u, __ATOMIC_RELEASE);
        *win = s;
        *ctr = p.ctrs[g] + i;
        return true;
    }
    return false;  // all slots busy: the launch runs without a window
}

bool MPComm::Impl::h2dWindowOpen(int g) const {
    const WindowPool *wp = windows_live_.load(std::memory_order_acquire);
    if (g < 0 || g >= static_cast<int>(kMaxGpuDomains) || !wp) return false;
    const kern::H2DWindow *base = &wp->slots[g * kSlotsPerGpu];
    for (int i = 0; i < kSlotsPerGpu; ++i) {
        const kern::H2DWindow *s = base + i;
        if (!__atomic_load_n(&s->armed, __ATOMIC_ACQUIRE)) continue;
        if (__atomic_load_n(&s->begin_ns, __ATOMIC_ACQUIRE) != 0 &&
            __atomic_load_n(&s->end_ns, __ATOMIC_ACQUIRE) == 0)
            return true;
    }
    return false;
}

bool MPComm::Impl::lastH2DWindow(int g, uint64_t *begin_ns, uint64_t *end_ns) const {
    const WindowPool *wp = windows_live_.load(std::memory_order_acquire);
    if (g < 0 || g >= static_cast<int>(kMaxGpuDomains) || !wp) return false;
    uint64_t best_b = 0, best_e = 0;
    for (int i = 0; i < kSlotsPerGpu; ++i) {
        const kern::H2DWindow *s = &wp->slots[g * kSlotsPerGpu + i];
        const uint64_t e = __atomic_load_n(&s->end_ns, __ATOMIC_ACQUIRE);
        const uint64_t b = __atomic_load_n(&s->begin_ns, __ATOMIC_ACQUIRE);
        if (e > best_e && b != 0) {
            best_e = e;
            best_b = b;
        }
    }
    if (!best_e) return false;
    *begin_ns = best_b;
    *end_ns = best_e;
    return true;
}

bool MPComm::Impl::qosAllowPost(const Transfer &t, size_t rail, size_t bytes) {
    if (!h2d_qos_enabled_.load(std::memory_order_relaxed)) return true;
    if (t.op != fabric::Opcode::kRead) return true;  // READ posts land in local HBM/DRAM
    const int g = rails_[rail]->gpu;
    if (g < 0 || !h2dWindowOpen(g)) return true;
    return qos_bucket_.consume(bytes);
}

void MPComm::Impl::pcieOnPosted(int g, uint64_t bytes) {
    if (g < 0 || g >= static_cast<int>(kMaxGpuDomains)) return;
    PcieDomain &d = pcie_[g];
    d.seen.store(true, std::memory_order_relaxed);
    const uint64_t posted = d.posted.fetch_add(bytes, std::memory_order_relaxed) + bytes;
    d.post_count.fetch_add(1, std::memory_order_relaxed);
    const uint64_t done = d.completed.load(std::memory_order_acquire);
    const uint64_t inflight = posted > done ? posted - done : 0;
    uint64_t m = d.inflight_max.load(std::memory_order_relaxed);
    while (inflight > m && !d.inflight_max.compare_exchange_weak(m, inflight)) {
    }
}

void MPComm::Impl::pcieOnCompleted(int g, uint64_t bytes) {
    if (g < 0 || g >= static_cast<int>(kMaxGpuDomains)) return;
    pcie_[g].completed.fetch_add(bytes, std::memory_order_release);
}

std::vector<MPComm::PcieDomainStats> MPComm::Impl::getPcieDomainStats() const {
    std::vector<MPComm::PcieDomainStats> out;
    for (size_t g = 0; g < kMaxGpuDomains; ++g) {
        const PcieDomain &d = pcie_[g];
        if (!d.seen.load()) continue;
        MPComm::PcieDomainStats s;
        s.gpu_device_id = static_cast<int>(g);
        s.posted_bytes = d.posted.load();
        s.completed_bytes = d.completed.load();
        s.in_flight_bytes = s.posted_bytes > s.completed_bytes ? s.posted_bytes - s.completed_bytes : 0;
        s.in_flight_bytes_max = d.inflight_max.load();
        s.post_count = d.post_count.load();
        s.defer_count = d.defer_count.load();
        out.push_back(s);
    }
    return out;
}

void MPComm::Impl::resetPcieDomainStats() {
    for (auto &d : pcie_) {
        const uint64_t posted = d.posted.load(), done = d.completed.load();
        const uint64_t inflight = posted > done ? posted - done : 0;
        // Keep live in-flight state: re-base both counters on it.
        d.completed.fetch_sub(done, std::memory_order_relaxed);
        d.posted.fetch_sub(posted - inflight, std::memory_order_relaxed);
        d.inflight_max.store(inflight);
        d.post_count.store(0);
        d.defer_count.store(0);
    }
}

}  // namespace mpcomm
