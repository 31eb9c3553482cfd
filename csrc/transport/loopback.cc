// "lo" backend: in-process loopback rails.
//
// Each rail runs one engine thread that executes posted WRs in order:
// validates lkey against its own registrations and rkey against the
// connected peer rail's registrations (bounds included), memcpy's the bytes
// and pushes one completion per WR onto the rail's CQ. A QP moved to ERR
// flushes queued and future WRs with kWcFlushErr, exactly like RC verbs.
// Test hooks (loopback_hooks.h) inject completion errors and port-down
// states on the host, which is how quarantine, recovery and re-post are
// exercised without touching any device.
#include <sys/types.h>
#include <unistd.h>

#include <atomic>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <shared_mutex>
#include <thread>
#include <unordered_map>
#include <vector>

#include "mpcomm.h"
#include "mpcomm_log.h"
#include "transport/fabric.h"
#include "transport/loopback_hooks.h"

namespace mpcomm {
namespace fabric {
namespace {

class LoRail;
class LoQp;

struct MrEntry {
    uintptr_t addr;
    size_t len;
};

// Process-wide directory of loopback rails and QPs (by gid / qp_num).
struct Directory {
    std::mutex mu;
    std::unordered_map<std::string, LoRail *> rails;
    std::atomic<uint32_t> next_rail{0};
    std::atomic<uint32_t> next_qpn{0x100};
    static Directory &get() {
        static Directory d;
        return d;
    }
};

struct PendingWr {
    WorkRequest wr;
    LoQp *qp;
    std::vector<FanoutTarget> fan;  // one-to-many WRITE (empty: a plain WR)
};

class LoRail final : public Rail {
 public:
    LoRail(std::string name, int numa)
        : name_(std::move(name)), numa_(numa) {
        char buf[64];
        snprintf(buf, sizeof(buf), "lo:%d:%u", static_cast<int>(getpid()),
                 Directory::get().next_rail.fetch_add(1));
        gid_ = buf;
        {
            std::lock_guard<std::mutex> g(Directory::get().mu);
            Directory::get().rails[gid_] = this;
        }
        thread_ = std::thread([this] { run(); });
    }
    ~LoRail() override {
        {
            std::lock_guard<std::mutex> g(Directory::get().mu);
            Directory::get().rails.erase(gid_);
        }
        {
            std::lock_guard<std::mutex> g(qmu_);
            stop_ = true;
        }
        qcv_.notify_all();
        thread_.join();
    }

    const std::string &name() const override { return name_; }
    std::string gid() const override { return gid_; }
    int numa_node() const override { return numa_; }
    bool port_active() const override { return active_.load(); }

    int register_memory(void *addr, size_t len, MemKey *out) override {
        std::unique_lock<std::shared_mutex> g(mrmu_);
        uint32_t key = next_key_++;
        mrs_[key] = MrEntry{reinterpret_cast<uintptr_t>(addr), len};
        out->lkey = key;
        out->rkey = key;
        return MPCOMM_SUCCESS;
    }
    int deregister_memory(void *, const MemKey &key) override {
        std::unique_lock<std::shared_mutex> g(mrmu_);
        return mrs_.erase(key.lkey) ? MPCOMM_SUCCESS : MPCOMM_ERR_INVALID_ARG;
    }
    bool check(uint32_t key, uintptr_t addr, size_t len) const {
        std::shared_lock<std::shared_mutex> g(mrmu_);
        auto it = mrs_.find(key);
        if (it == mrs_.end()) return false;
        return addr >= it->second.addr && addr + len <= it->second.addr + it->second.len;
    }

    std::unique_ptr<QueuePair> create_qp() override;
    // One-to-many WRITEs: one completion after the bytes reached every target.
    size_t max_fanout() const override { return 8; }

    int poll(WorkCompletion *out, int max) override {
        std::lock_guard<std::mutex> g(cqmu_);
        int n = 0;
        while (n < max && !cq_.empty()) {
            out[n++] = cq_.front();
            cq_.pop_front();
        }
        return n;
    }

    void enqueue(const WorkRequest *wrs, size_t n, LoQp *qp) {
        {
            std::lock_guard<std::mutex> g(qmu_);
            for (size_t i = 0; i < n; ++i) work_.push_back(PendingWr{wrs[i], qp, {}});
        }
        qcv_.notify_one();
    }
    void enqueue_fanout(const WorkRequest &wr, const FanoutTarget *t, size_t n, LoQp *qp) {
        {
            std::lock_guard<std::mutex> g(qmu_);
            work_.push_back(PendingWr{wr, qp, std::vector<FanoutTarget>(t, t + n)});
        }
        qcv_.notify_one();
    }
    void complete(uint64_t wr_id, int status, uint32_t len) {
        std::lock_guard<std::mutex> g(cqmu_);
        cq_.push_back(WorkCompletion{wr_id, status, len});
    }
    // Drops queued work of `qp` with flush errors (QP destroyed or ERR).
    void flush_qp(LoQp *qp, bool report);

    // ---- hooks ----
    std::atomic<int> inject_errors{0};
    std::atomic<bool> active_{true};
    std::atomic<uint64_t> wr_delay_us{0};

 private:
    void run();

    std::string name_, gid_;
    int numa_;
    mutable std::shared_mutex mrmu_;
    std::map<uint32_t, MrEntry> mrs_;
    uint32_t next_key_ = 0x1000;
    std::mutex qmu_;
    std::condition_variable qcv_;
    std::deque<PendingWr> work_;
    bool stop_ = false;
    std::mutex cqmu_;
    std::deque<WorkCompletion> cq_;
    std::thread thread_;
};

class LoQp final : public QueuePair {
 public:
    explicit LoQp(LoRail *rail) : rail_(rail), qpn_(Directory::get().next_qpn.fetch_add(1)) {}
    ~LoQp() override { rail_->flush_qp(this, false); }

    uint32_t qp_num() const override { return qpn_; }
    QpState state() const override { return state_.load(); }
    int to_init() override {
        state_ = QpState::kInit;
        return 0;
    }
    int to_rtr(const EndpointInfo &remote) override {
        if (state_.load() != QpState::kInit) return MPCOMM_ERR_CONNECTION;
        remote_ = remote;
        state_ = QpState::kRtr;
        return 0;
    }
    int to_rts() override {
        if (state_.load() != QpState::kRtr) return MPCOMM_ERR_CONNECTION;
        state_ = QpState::kRts;
        return 0;
    }
    int to_err() override {
        state_ = QpState::kErr;
        rail_->flush_qp(this, true);
        return 0;
    }
    int recover() override {
        rail_->flush_qp(this, true);
        state_ = QpState::kReset;
        to_init();
        EndpointInfo r = remote_;
        if (to_rtr(r) || to_rts()) return MPCOMM_ERR_CONNECTION;
        return 0;
    }
    int post(const WorkRequest *wrs, size_t n) override {
        QpState s = state_.load();
        if (s != QpState::kRts && s != QpState::kErr) return MPCOMM_ERR_CONNECTION;
        rail_->enqueue(wrs, n, this);
        return 0;
    }
    int post_fanout(const WorkRequest &wr, const FanoutTarget *targets, size_t n, void *) override {
        QpState s = state_.load();
        if (s != QpState::kRts && s != QpState::kErr) return MPCOMM_ERR_CONNECTION;
        if (n == 0 || n > 8 || wr.op != Opcode::kWrite) return MPCOMM_ERR_INVALID_ARG;
        for (size_t i = 0; i < n; ++i) {
            auto *q = dynamic_cast<LoQp *>(targets[i].qp);
            if (!q || q->rail_ != rail_) return MPCOMM_ERR_INVALID_ARG;
        }
        rail_->enqueue_fanout(wr, targets, n, this);
        return 0;
    }
    const EndpointInfo &remote() const { return remote_; }

 private:
    friend class LoRail;
    LoRail *rail_;
    uint32_t qpn_;
    std::atomic<QpState> state_{QpState::kReset};
    EndpointInfo remote_;
};

std::unique_ptr<QueuePair> LoRail::create_qp() { return std::make_unique<LoQp>(this); }

void LoRail::flush_qp(LoQp *qp, bool report) {
    std::deque<PendingWr> keep, drop;
    {
        std::lock_guard<std::mutex> g(qmu_);
        for (auto &p : work_) (p.qp == qp ? drop : keep).push_back(p);
        work_.swap(keep);
    }
    if (report)
        for (auto &p : drop) complete(p.wr.wr_id, kWcFlushErr, 0);
}

void LoRail::run() {
    for (;;) {
        PendingWr p;
        {
            std::unique_lock<std::mutex> g(qmu_);
            qcv_.wait(g, [&] { return stop_ || !work_.empty(); });
            if (stop_) return;
            p = work_.front();
            work_.pop_front();
        }
        uint64_t delay = wr_delay_us.load(std::memory_order_relaxed);
        if (delay) std::this_thread::sleep_for(std::chrono::microseconds(delay));
        const WorkRequest &wr = p.wr;
        if (p.qp->state() == QpState::kErr) {
            complete(wr.wr_id, kWcFlushErr, 0);
            continue;
        }
        if (!active_.load() ) {
            complete(wr.wr_id, kWcRetryExcErr, 0);
            continue;
        }
        int inj = inject_errors.load();
        if (inj > 0 && inject_errors.compare_exchange_strong(inj, inj - 1)) {
            complete(wr.wr_id, kWcRemAccessErr, 0);
            continue;
        }
        if (!check(wr.lkey, wr.local_addr, wr.length)) {
            complete(wr.wr_id, kWcLocProtErr, 0);
            continue;
        }
        if (!p.fan.empty()) {
            int st = kWcSuccess;
            for (const auto &t : p.fan) {
                auto *q = static_cast<LoQp *>(t.qp);
                LoRail *peer = nullptr;
                {
                    std::lock_guard<std::mutex> g(Directory::get().mu);
                    auto it = Directory::get().rails.find(q->remote().gid);
                    if (it != Directory::get().rails.end()) peer = it->second;
                }
                if (q->state() == QpState::kErr) st = kWcFlushErr;
                else if (!peer || !peer->port_active()) st = kWcRetryExcErr;
                else if (!peer->check(t.rkey, t.remote_addr, wr.length)) st = kWcRemAccessErr;
                if (st != kWcSuccess) break;
                std::memmove(reinterpret_cast<void *>(t.remote_addr), reinterpret_cast<const void *>(wr.local_addr),
                             wr.length);
            }
            complete(wr.wr_id, st, st == kWcSuccess ? wr.length : 0);
            continue;
        }
        LoRail *peer = nullptr;
        {
            std::lock_guard<std::mutex> g(Directory::get().mu);
            auto it = Directory::get().rails.find(p.qp->remote().gid);
            if (it != Directory::get().rails.end()) peer = it->second;
        }
        if (!peer || !peer->port_active()) {
            complete(wr.wr_id, kWcRetryExcErr, 0);
            continue;
        }
        if (!peer->check(wr.rkey, wr.remote_addr, wr.length)) {
            complete(wr.wr_id, kWcRemAccessErr, 0);
            continue;
        }
        void *dst = reinterpret_cast<void *>(wr.op == Opcode::kWrite ? wr.remote_addr : wr.local_addr);
        const void *src =
            reinterpret_cast<const void *>(wr.op == Opcode::kWrite ? wr.local_addr : wr.remote_addr);
        std::memmove(dst, src, wr.length);
        complete(wr.wr_id, kWcSuccess, wr.length);
    }
}

class LoBackend final : public Backend {
 public:
    const char *name() const override { return "lo"; }
    int open(const Config &cfg, const std::vector<std::string> &filter,
             std::vector<std::unique_ptr<Rail>> *rails) override {
        for (int i = 0; i < cfg.loopback_nics; ++i) {
            std::string nm = "lo_" + std::to_string(i);
            if (!filter.empty()) {
                bool ok = false;
                for (auto &f : filter) ok |= (f == nm);
                if (!ok) continue;
            }
            rails->push_back(std::make_unique<LoRail>(nm, 0));
        }
        return rails->empty() ? MPCOMM_ERR_DEVICE : MPCOMM_SUCCESS;
    }
};

}  // namespace

std::unique_ptr<Backend> make_loopback_backend() { return std::make_unique<LoBackend>(); }

// ---- host-side fault hooks --------------------------------------------------
int loopback_inject_wc_errors(const std::string &gid, int count) {
    std::lock_guard<std::mutex> g(Directory::get().mu);
    auto it = Directory::get().rails.find(gid);
    if (it == Directory::get().rails.end()) return MPCOMM_ERR_INVALID_ARG;
    it->second->inject_errors.store(count);
    return MPCOMM_SUCCESS;
}

int loopback_set_port_active(const std::string &gid, bool active) {
    std::lock_guard<std::mutex> g(Directory::get().mu);
    auto it = Directory::get().rails.find(gid);
    if (it == Directory::get().rails.end()) return MPCOMM_ERR_INVALID_ARG;
    it->second->active_.store(active);
    return MPCOMM_SUCCESS;
}

int loopback_set_wr_delay_us(const std::string &gid, uint64_t us) {
    std::lock_guard<std::mutex> g(Directory::get().mu);
    auto it = Directory::get().rails.find(gid);
    if (it == Directory::get().rails.end()) return MPCOMM_ERR_INVALID_ARG;
    it->second->wr_delay_us.store(us);
    return MPCOMM_SUCCESS;
}

}  // namespace fabric
}  // namespace mpcomm
