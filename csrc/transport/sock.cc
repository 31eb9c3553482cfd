// "sock" backend: software one-sided RDMA over TCP, for host memory across
// processes (CPU-only hosts, multi-process tests, soft-RoCE-like drills).
//
// Each rail listens on MPCOMM_SOCK_ADDR (default 127.0.0.1), ephemeral
// port; gid = "sock:<ip>:<port>:<n>". to_rtr() opens one TCP stream from
// this QP to the peer rail, announcing the peer QP number; the peer's
// server thread then executes this QP's requests against its own
// registrations — the target CPU plays the role of the remote NIC:
//   WRITE: {hdr} + payload  -> target checks rkey/bounds, stores, acks
//   READ:  {hdr}            -> target checks, replies status + payload
// A sender thread per QP executes posted WRs in order and produces one
// completion each on the rail CQ. to_err() flushes like RC verbs.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <sys/socket.h>
#include <unistd.h>

#include <atomic>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <shared_mutex>
#include <thread>

#include "ctrl/wire.h"
#include "mpcomm.h"
#include "mpcomm_log.h"
#include "transport/fabric.h"

namespace mpcomm {
namespace fabric {
namespace {

constexpr uint32_t kHelloMagic = 0x4D505348;  // "MPSH"
constexpr uint32_t kReqMagic = 0x4D505352;    // "MPSR"

struct Hello {
    uint32_t magic;
    uint32_t target_qpn;
    uint32_t source_qpn;
};

struct ReqHdr {
    uint32_t magic;
    uint32_t op;  // 0 write, 1 read
    uint32_t rkey;
    uint32_t length;
    uint64_t raddr;
};

std::string sock_addr() {
    const char *e = std::getenv("MPCOMM_SOCK_ADDR");
    return (e && *e) ? e : "127.0.0.1";
}

class SockRail;

class SockQp final : public QueuePair {
 public:
    SockQp(SockRail *rail, uint32_t qpn);
    ~SockQp() override;
    uint32_t qp_num() const override { return qpn_; }
    QpState state() const override { return state_.load(); }
    int to_init() override {
        state_ = QpState::kInit;
        return 0;
    }
    int to_rtr(const EndpointInfo &remote) override;
    int to_rts() override {
        if (state_.load() != QpState::kRtr) return MPCOMM_ERR_CONNECTION;
        state_ = QpState::kRts;
        return 0;
    }
    int to_err() override;
    int recover() override {
        to_err();
        close_fd();
        state_ = QpState::kInit;
        EndpointInfo r = remote_;
        if (to_rtr(r) != 0) return MPCOMM_ERR_CONNECTION;
        return to_rts();
    }
    int post(const WorkRequest *wrs, size_t n) override;

 private:
    void run();
    void close_fd();
    SockRail *rail_;
    uint32_t qpn_;
    std::atomic<QpState> state_{QpState::kReset};
    EndpointInfo remote_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::deque<WorkRequest> q_;
    bool stop_ = false;
    int fd_ = -1;
    std::thread thread_;
};

class SockRail final : public Rail {
 public:
    SockRail(std::string name, int index, int dscp) : name_(std::move(name)), tos_((dscp & 63) << 2) {
        int port = 0;
        listen_fd_ = net::listen_tcp(0, 128, &port);
        gid_ = "sock:" + sock_addr() + ":" + std::to_string(port) + ":" + std::to_string(index);
        if (listen_fd_ >= 0) accept_thread_ = std::thread([this] { accept_loop(); });
    }
    ~SockRail() override {
        stop_ = true;
        if (listen_fd_ >= 0) {
            ::shutdown(listen_fd_, SHUT_RDWR);
            ::close(listen_fd_);
        }
        if (accept_thread_.joinable()) accept_thread_.join();
        std::vector<std::thread> servers;
        {
            std::lock_guard<std::mutex> g(srv_mu_);
            for (int fd : server_fds_) ::shutdown(fd, SHUT_RDWR);
            servers.swap(servers_);
        }
        for (auto &t : servers)
            if (t.joinable()) t.join();
    }
    bool ok() const { return listen_fd_ >= 0; }
    // DSCP marking of this rail's data connections (MPCOMM_ROCE_DSCP, the
    // same knob the ib fabric puts in the GRH traffic class): IP_TOS, or
    // IPV6_TCLASS for IPv6 sockets, on both ends.
    void mark(int fd) const {
        if (!tos_ || fd < 0) return;
        sockaddr_storage ss{};
        socklen_t sl = sizeof(ss);
        const bool v6 = getsockname(fd, reinterpret_cast<sockaddr *>(&ss), &sl) == 0 && ss.ss_family == AF_INET6;
        const int level = v6 ? IPPROTO_IPV6 : IPPROTO_IP, opt = v6 ? IPV6_TCLASS : IP_TOS;
        int tos = tos_, got = -1;
        socklen_t gl = sizeof(got);
        if (setsockopt(fd, level, opt, &tos, sizeof(tos)) != 0 || getsockopt(fd, level, opt, &got, &gl) != 0 ||
            (got & 0xFC) != tos_) {
            MPCOMM_LOG_WARN("MPComm[sock]: %s: cannot set traffic class 0x%02x on fd %d\n", name_.c_str(), tos_, fd);
            return;
        }
        MPCOMM_LOG_DEBUG("MPComm[sock]: %s: data connection fd %d traffic class 0x%02x (DSCP %d)\n", name_.c_str(),
                         fd, got & 0xFC, (got & 0xFC) >> 2);
    }
    const std::string &name() const override { return name_; }
    std::string gid() const override { return gid_; }
    int numa_node() const override { return 0; }
    bool port_active() const override { return active.load(); }

    int register_memory(void *addr, size_t len, MemKey *out) override {
        std::unique_lock<std::shared_mutex> g(mrmu_);
        uint32_t k = next_key_++;
        mrs_[k] = std::make_pair(reinterpret_cast<uintptr_t>(addr), len);
        out->lkey = out->rkey = k;
        return 0;
    }
    int deregister_memory(void *, const MemKey &k) override {
        std::unique_lock<std::shared_mutex> g(mrmu_);
        return mrs_.erase(k.lkey) ? 0 : MPCOMM_ERR_INVALID_ARG;
    }
    bool check(uint32_t key, uintptr_t a, size_t len) const {
        std::shared_lock<std::shared_mutex> g(mrmu_);
        auto it = mrs_.find(key);
        return it != mrs_.end() && a >= it->second.first && a + len <= it->second.first + it->second.second;
    }
    std::unique_ptr<QueuePair> create_qp() override {
        return std::make_unique<SockQp>(this, next_qpn_.fetch_add(1));
    }
    int poll(WorkCompletion *out, int max) override {
        std::lock_guard<std::mutex> g(cqmu_);
        int n = 0;
        while (n < max && !cq_.empty()) {
            out[n++] = cq_.front();
            cq_.pop_front();
        }
        return n;
    }
    void complete(uint64_t id, int st, uint32_t len) {
        std::lock_guard<std::mutex> g(cqmu_);
        cq_.push_back(WorkCompletion{id, st, len});
    }
    std::atomic<bool> active{true};

 private:
    void accept_loop() {
        while (!stop_) {
            int fd = ::accept(listen_fd_, nullptr, nullptr);
            if (fd < 0) {
                if (stop_) return;
                continue;
            }
            mark(fd);
            std::lock_guard<std::mutex> g(srv_mu_);
            server_fds_.push_back(fd);
            servers_.emplace_back([this, fd] { serve(fd); });
        }
    }
    // Executes the peer QP's one-sided requests against our registrations.
    void serve(int fd) {
        Hello h;
        if (!net::recv_pod(fd, &h) || h.magic != kHelloMagic) {
            ::close(fd);
            return;
        }
        std::vector<char> sink;  // discard buffer of rejected writes
        for (;;) {
            ReqHdr r;
            if (!net::recv_pod(fd, &r) || r.magic != kReqMagic) break;
            const bool ok = active.load() && check(r.rkey, r.raddr, r.length);
            int32_t st = ok ? kWcSuccess : kWcRemAccessErr;
            if (r.op == 0) {
                if (ok) {
                    if (!net::recv_all(fd, reinterpret_cast<void *>(r.raddr), r.length)) break;
                } else {
                    // Rejected write: drain its payload in bounded pieces (the
                    // length comes from the peer; never size a buffer by it).
                    sink.resize(64 * 1024);
                    uint64_t left = r.length;
                    bool io = true;
                    while (left && io) {
                        const size_t k = left < sink.size() ? static_cast<size_t>(left) : sink.size();
                        io = net::recv_all(fd, sink.data(), k);
                        left -= k;
                    }
                    if (!io) break;
                }
                if (!net::send_pod(fd, st)) break;
            } else {
                if (!net::send_pod(fd, st)) break;
                if (ok && !net::send_all(fd, reinterpret_cast<const void *>(r.raddr), r.length)) break;
            }
        }
        ::close(fd);
    }

    std::string name_, gid_;
    int listen_fd_ = -1;
    std::atomic<bool> stop_{false};
    std::thread accept_thread_;
    int tos_ = 0;
    std::mutex srv_mu_;
    std::vector<int> server_fds_;
    std::vector<std::thread> servers_;
    mutable std::shared_mutex mrmu_;
    std::map<uint32_t, std::pair<uintptr_t, size_t>> mrs_;
    uint32_t next_key_ = 0x2000;
    std::atomic<uint32_t> next_qpn_{0x200};
    std::mutex cqmu_;
    std::deque<WorkCompletion> cq_;
};

SockQp::SockQp(SockRail *rail, uint32_t qpn) : rail_(rail), qpn_(qpn) {
    thread_ = std::thread([this] { run(); });
}

SockQp::~SockQp() {
    {
        std::lock_guard<std::mutex> g(mu_);
        stop_ = true;
        q_.clear();
    }
    cv_.notify_all();
    close_fd();
    thread_.join();
}

void SockQp::close_fd() {
    std::lock_guard<std::mutex> g(mu_);
    if (fd_ >= 0) {
        ::shutdown(fd_, SHUT_RDWR);
        ::close(fd_);
        fd_ = -1;
    }
}

int SockQp::to_rtr(const EndpointInfo &remote) {
    // gid: sock:<ip>:<port>:<n>
    if (remote.gid.compare(0, 5, "sock:") != 0) return MPCOMM_ERR_CONNECTION;
    size_t a = remote.gid.find(':', 5), b = a == std::string::npos ? a : remote.gid.find(':', a + 1);
    if (a == std::string::npos || b == std::string::npos) return MPCOMM_ERR_CONNECTION;
    std::string ip = remote.gid.substr(5, a - 5);
    int port = std::atoi(remote.gid.substr(a + 1, b - a - 1).c_str());
    int fd = net::connect_tcp(ip, port, 0);
    if (fd < 0) return MPCOMM_ERR_CONNECTION;
    rail_->mark(fd);
    Hello h{kHelloMagic, remote.qp_num, qpn_};
    if (!net::send_pod(fd, h)) {
        ::close(fd);
        return MPCOMM_ERR_CONNECTION;
    }
    {
        std::lock_guard<std::mutex> g(mu_);
        fd_ = fd;
        remote_ = remote;
    }
    state_ = QpState::kRtr;
    return 0;
}

int SockQp::to_err() {
    state_ = QpState::kErr;
    std::deque<WorkRequest> drop;
    {
        std::lock_guard<std::mutex> g(mu_);
        drop.swap(q_);
    }
    for (auto &w : drop) rail_->complete(w.wr_id, kWcFlushErr, 0);
    return 0;
}

int SockQp::post(const WorkRequest *wrs, size_t n) {
    QpState s = state_.load();
    if (s != QpState::kRts && s != QpState::kErr) return MPCOMM_ERR_CONNECTION;
    if (s == QpState::kErr) {
        for (size_t i = 0; i < n; ++i) rail_->complete(wrs[i].wr_id, kWcFlushErr, 0);
        return 0;
    }
    {
        std::lock_guard<std::mutex> g(mu_);
        for (size_t i = 0; i < n; ++i) q_.push_back(wrs[i]);
    }
    cv_.notify_one();
    return 0;
}

void SockQp::run() {
    for (;;) {
        WorkRequest w;
        int fd;
        {
            std::unique_lock<std::mutex> g(mu_);
            cv_.wait(g, [&] { return stop_ || !q_.empty(); });
            if (stop_) return;
            w = q_.front();
            q_.pop_front();
            fd = fd_;
        }
        if (state_.load() == QpState::kErr) {
            rail_->complete(w.wr_id, kWcFlushErr, 0);
            continue;
        }
        if (!rail_->check(w.lkey, w.local_addr, w.length)) {
            rail_->complete(w.wr_id, kWcLocProtErr, 0);
            continue;
        }
        if (!rail_->active.load() || fd < 0) {
            rail_->complete(w.wr_id, kWcRetryExcErr, 0);
            continue;
        }
        ReqHdr r{kReqMagic, w.op == Opcode::kWrite ? 0u : 1u, w.rkey, w.length, w.remote_addr};
        int32_t st = kWcRetryExcErr;
        bool io = net::send_pod(fd, r);
        if (io && w.op == Opcode::kWrite) {
            io = net::send_all(fd, reinterpret_cast<const void *>(w.local_addr), w.length) &&
                 net::recv_pod(fd, &st);
        } else if (io) {
            io = net::recv_pod(fd, &st);
            if (io && st == kWcSuccess)
                io = net::recv_all(fd, reinterpret_cast<void *>(w.local_addr), w.length);
        }
        if (!io) {
            st = kWcRetryExcErr;
            state_ = QpState::kErr;  // a broken stream leaves the QP unusable
        }
        rail_->complete(w.wr_id, st, st == kWcSuccess ? w.length : 0);
    }
}

class SockBackend final : public Backend {
 public:
    const char *name() const override { return "sock"; }
    int open(const Config &cfg, const std::vector<std::string> &filter,
             std::vector<std::unique_ptr<Rail>> *rails) override {
        for (int i = 0; i < cfg.loopback_nics; ++i) {
            std::string nm = "sock_" + std::to_string(i);
            if (!filter.empty()) {
                bool ok = false;
                for (auto &f : filter) ok |= (f == nm);
                if (!ok) continue;
            }
            auto r = std::make_unique<SockRail>(nm, i, cfg.roce_dscp);
            if (r->ok()) rails->push_back(std::move(r));
        }
        return rails->empty() ? MPCOMM_ERR_DEVICE : MPCOMM_SUCCESS;
    }
};

}  // namespace

std::unique_ptr<Backend> make_sock_backend() { return std::make_unique<SockBackend>(); }

}  // namespace fabric
}  // namespace mpcomm
