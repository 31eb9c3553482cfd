// QoS control channel: a host that is about to pull bytes into a GPU over
// PCIe (an H2D gather) tells the peers that WRITE into that GPU to pause or
// pace those writes, and lifts the policy when it is done.
//
// Wire format (host-endian, the reference's: src/mpcomm.cpp:215-248): the
// opener connects to the peer's control port, sends the u32 0x4D505143 and
// a QosControlHello {version, host_id[128]}, then any number of 112-byte
// QosControlFrame (magic 0x4D505146, version, type update/clear, target GPU
// (-1 = all), rate, burst, generation). The receiver keeps one policy per
// (opener, target GPU); its workers consult it before posting a WRITE chunk
// to that opener (rate 0 = deferred, else a token bucket). When the channel
// drops the opener's policies are removed: fail-open.
//
// The reference declares this channel but never opens it, rejects it in the
// accept loop and paces remote WRITEs with a stub that always allows
// (src/mpcomm.cpp:2624-2799, 4524-4531); here it is live, and with
// MPCOMM_QOS_REMOTE=1 each QoS-windowed tmaGather/tmaScatter sends the
// update itself and the clear once its H2D window has closed (50 ms cap).
#include <netinet/in.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>

#include "engine/impl.h"
#include "mpcomm_log.h"

namespace mpcomm {

struct MPComm::Impl::QosOutChannel {
    int fd = -1;
    std::mutex send_mu;
};

namespace {
std::string ip_of(const std::string &id_or_addr) { return id_or_addr.substr(0, id_or_addr.rfind(':')); }
}  // namespace

int MPComm::Impl::openQosChannel(const std::string &host_id) {
    if (!initialized_) return MPCOMM_ERR_CONTEXT;
    std::string addr;
    int port = 0;
    {
        std::lock_guard<std::mutex> g(conn_mu_);
        auto it = connections_.find(host_id);
        if (it == connections_.end() || it->second->tcp_addr.empty()) {
            MPCOMM_LOG_ERROR("MPComm: openQosChannel(%s): connect() to that host first\n", host_id.c_str());
            return MPCOMM_ERR_CONNECTION;
        }
        addr = it->second->tcp_addr;
        port = it->second->tcp_port;
    }
    int fd = net::connect_tcp(addr, port, net::ctrl_timeout_ms());
    if (fd < 0) return MPCOMM_ERR_CONNECTION;
    QosControlHello hello{};
    hello.version = kQosControlVersion;
    std::strncpy(hello.host_id, host_id_.c_str(), sizeof(hello.host_id) - 1);
    if (!net::send_pod(fd, kMsgTypeQosControlOpen) || !net::send_pod(fd, hello)) {
        ::close(fd);
        return MPCOMM_ERR_CONNECTION;
    }
    auto ch = std::make_shared<QosOutChannel>();
    ch->fd = fd;
    std::shared_ptr<QosOutChannel> old;
    {
        std::lock_guard<std::mutex> g(qos_out_mu_);
        auto &slot = qos_out_[host_id];
        old = slot;
        slot = ch;
    }
    if (old) {
        std::lock_guard<std::mutex> g(old->send_mu);
        ::close(old->fd);
        old->fd = -1;
    }
    MPCOMM_LOG_INFO("MPComm: QoS control channel open to %s\n", host_id.c_str());
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::closeQosChannel(const std::string &host_id) {
    std::shared_ptr<QosOutChannel> ch;
    {
        std::lock_guard<std::mutex> g(qos_out_mu_);
        auto it = qos_out_.find(host_id);
        if (it == qos_out_.end()) return MPCOMM_ERR_INVALID_ARG;
        ch = it->second;
        qos_out_.erase(it);
    }
    std::lock_guard<std::mutex> g(ch->send_mu);
    if (ch->fd >= 0) ::close(ch->fd);
    ch->fd = -1;
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::sendQosPolicy(const std::string &host_id, int gpu, uint64_t rate, uint64_t burst, bool clear) {
    std::shared_ptr<QosOutChannel> ch;
    {
        std::lock_guard<std::mutex> g(qos_out_mu_);
        auto it = qos_out_.find(host_id);
        if (it == qos_out_.end()) return MPCOMM_ERR_INVALID_ARG;
        ch = it->second;
    }
    QosControlFrame f{};
    f.magic = kQosControlFrameMagic;
    f.version = kQosControlVersion;
    f.type = static_cast<uint32_t>(clear ? QosFrameType::kClear : QosFrameType::kUpdate);
    f.target_gpu_device = gpu;
    f.rate_bytes_per_sec = rate;
    f.burst_bytes = burst ? burst : default_qos_burst(rate);
    f.generation = qos_generation_.fetch_add(1, std::memory_order_relaxed) + 1;
    std::lock_guard<std::mutex> g(ch->send_mu);
    if (ch->fd < 0 || !net::send_pod(ch->fd, f)) {
        MPCOMM_LOG_WARN("MPComm: QoS control channel to %s lost\n", host_id.c_str());
        if (ch->fd >= 0) ::close(ch->fd);
        ch->fd = -1;
        std::lock_guard<std::mutex> g2(qos_out_mu_);
        auto it = qos_out_.find(host_id);
        if (it != qos_out_.end() && it->second == ch) qos_out_.erase(it);
        return MPCOMM_ERR_CONNECTION;
    }
    return MPCOMM_SUCCESS;
}

void MPComm::Impl::broadcastQos(int gpu, uint64_t rate, uint64_t burst, bool clear) {
    std::vector<std::string> peers;
    {
        std::lock_guard<std::mutex> g(qos_out_mu_);
        for (auto &kv : qos_out_) peers.push_back(kv.first);
    }
    for (auto &p : peers) sendQosPolicy(p, gpu, rate, burst, clear);
}

size_t MPComm::Impl::qosChannelCount() const {
    std::lock_guard<std::mutex> g(qos_out_mu_);
    return qos_out_.size();
}

// ---- receiving side ---------------------------------------------------------
void MPComm::Impl::handleQosChannel(int fd) {
    QosControlHello hello{};
    if (!net::recv_pod(fd, &hello)) return;
    hello.host_id[sizeof(hello.host_id) - 1] = 0;
    if (hello.version != kQosControlVersion) {
        MPCOMM_LOG_WARN("MPComm: QoS control channel from %s: version %u unsupported\n", hello.host_id,
                        hello.version);
        return;
    }
    int port = 0;
    const std::string peer_ip = ip_of(net::peer_id(fd, &port));
    int keep = ::dup(fd);  // the accept loop closes `fd` when this returns
    if (keep < 0) return;
    std::lock_guard<std::mutex> g(qos_rx_mu_);
    if (!qos_rx_running_.load()) {
        ::close(keep);
        return;
    }
    qos_rx_fds_.push_back(keep);
    qos_rx_threads_.emplace_back(&MPComm::Impl::qosRxLoop, this, keep, std::string(hello.host_id), peer_ip);
    MPCOMM_LOG_INFO("MPComm: QoS control channel from %s (%s)\n", hello.host_id, peer_ip.c_str());
}

void MPComm::Impl::qosRxLoop(int fd, std::string peer, std::string peer_ip) {
    while (qos_rx_running_.load(std::memory_order_acquire)) {
        pollfd p{fd, POLLIN, 0};
        const int r = ::poll(&p, 1, 100);
        if (r == 0) continue;
        if (r < 0 && errno == EINTR) continue;
        QosControlFrame f{};
        if (r < 0 || !net::recv_pod(fd, &f)) break;
        if (f.magic != kQosControlFrameMagic || f.version != kQosControlVersion) {
            MPCOMM_LOG_WARN("MPComm: bad QoS control frame from %s; closing the channel\n", peer.c_str());
            break;
        }
        std::lock_guard<std::mutex> g(qos_in_mu_);
        if (f.type == static_cast<uint32_t>(QosFrameType::kClear)) {
            qos_in_.erase(std::remove_if(qos_in_.begin(), qos_in_.end(),
                                         [&](const std::unique_ptr<RemoteQosPolicy> &q) {
                                             return q->peer == peer &&
                                                    (f.target_gpu_device < 0 || q->gpu == f.target_gpu_device);
                                         }),
                          qos_in_.end());
        } else if (f.type == static_cast<uint32_t>(QosFrameType::kUpdate)) {
            RemoteQosPolicy *pol = nullptr;
            for (auto &q : qos_in_)
                if (q->peer == peer && q->gpu == f.target_gpu_device) pol = q.get();
            if (!pol) {
                qos_in_.push_back(std::make_unique<RemoteQosPolicy>());
                pol = qos_in_.back().get();
                pol->peer = peer;
                pol->peer_ip = peer_ip;
                pol->gpu = f.target_gpu_device;
            }
            if (f.generation >= pol->generation) {
                pol->rate = f.rate_bytes_per_sec;
                pol->burst = f.burst_bytes;
                pol->generation = f.generation;
                pol->bucket.configure(pol->rate, pol->burst);
            }
        }
        qos_in_active_.store(static_cast<int>(qos_in_.size()), std::memory_order_release);
    }
    // Fail-open: the peer's policies go with its channel.
    {
        std::lock_guard<std::mutex> g(qos_in_mu_);
        qos_in_.erase(std::remove_if(qos_in_.begin(), qos_in_.end(),
                                     [&](const std::unique_ptr<RemoteQosPolicy> &q) { return q->peer == peer; }),
                      qos_in_.end());
        qos_in_active_.store(static_cast<int>(qos_in_.size()), std::memory_order_release);
    }
    ::shutdown(fd, SHUT_RDWR);
    MPCOMM_LOG_INFO("MPComm: QoS control channel from %s closed; its policies are lifted\n", peer.c_str());
}

bool MPComm::Impl::qosAllowRemoteWrite(const Connection &conn, uint64_t raddr, size_t bytes) {
    if (qos_in_active_.load(std::memory_order_acquire) == 0) return true;
    std::lock_guard<std::mutex> g(qos_in_mu_);
    // Policies of the peer named like this connection; if none carries that
    // name, those from the connection's address.
    bool by_id = false;
    for (auto &q : qos_in_) by_id |= q->peer == conn.host_id;
    const std::string ip = ip_of(conn.tcp_addr.empty() ? conn.host_id : conn.tcp_addr + ":0");
    int gpu = -2;
    for (auto &q : qos_in_) {
        if (by_id ? q->peer != conn.host_id : q->peer_ip != ip) continue;
        if (q->gpu >= 0) {
            if (gpu == -2) gpu = conn.remote_gpu_for(raddr);
            if (gpu != q->gpu) continue;
        }
        if (q->rate == 0 || !q->bucket.consume(bytes)) {
            remote_qos_defers_.fetch_add(1, std::memory_order_relaxed);
            return false;
        }
    }
    return true;
}

std::vector<MPComm::Impl::RemoteQosView> MPComm::Impl::remoteQosPolicies() const {
    std::vector<RemoteQosView> out;
    std::lock_guard<std::mutex> g(qos_in_mu_);
    for (auto &q : qos_in_) out.push_back(RemoteQosView{q->peer, q->gpu, q->rate, q->burst, q->generation});
    return out;
}

void MPComm::Impl::stopQosChannels() {
    {
        std::lock_guard<std::mutex> g(qos_out_mu_);
        for (auto &kv : qos_out_) {
            std::lock_guard<std::mutex> g2(kv.second->send_mu);
            if (kv.second->fd >= 0) ::close(kv.second->fd);
            kv.second->fd = -1;
        }
        qos_out_.clear();
    }
    std::vector<std::thread> threads;
    std::vector<int> fds;
    {
        std::lock_guard<std::mutex> g(qos_rx_mu_);
        qos_rx_running_.store(false, std::memory_order_release);
        threads.swap(qos_rx_threads_);
        fds.swap(qos_rx_fds_);
    }
    for (auto &t : threads)
        if (t.joinable()) t.join();
    for (int fd : fds) ::close(fd);
    {
        std::lock_guard<std::mutex> g(qos_restore_mu_);
        qos_restore_running_ = false;
    }
    qos_restore_cv_.notify_all();
    if (qos_restore_thread_.joinable()) qos_restore_thread_.join();
}

// ---- automatic remote pause around H2D windows (MPCOMM_QOS_REMOTE=1) --------
void MPComm::Impl::remotePauseForWindow(int gpu, const kern::H2DWindow *win) {
    std::lock_guard<std::mutex> g(qos_restore_mu_);
    if (!qos_restore_running_) {
        qos_restore_running_ = true;
        qos_restore_thread_ = std::thread(&MPComm::Impl::qosRestoreLoop, this);
    }
    qos_restore_q_.push_back(QosRestoreItem{gpu, win, std::chrono::steady_clock::now() + std::chrono::milliseconds(50)});
    qos_restore_cv_.notify_one();
}

void MPComm::Impl::qosRestoreLoop() {
    std::unique_lock<std::mutex> lk(qos_restore_mu_);
    while (qos_restore_running_) {
        if (qos_restore_q_.empty()) {
            qos_restore_cv_.wait(lk);
            continue;
        }
        QosRestoreItem it = qos_restore_q_.front();
        // The window's end stamp is written by the kernel's last CTA into
        // host-mapped memory; the deadline bounds the pause if it never lands.
        const bool closed = __atomic_load_n(&it.win->end_ns, __ATOMIC_ACQUIRE) != 0;
        if (!closed && std::chrono::steady_clock::now() < it.deadline) {
            qos_restore_cv_.wait_for(lk, std::chrono::microseconds(20));
            continue;
        }
        qos_restore_q_.pop_front();
        bool still_open = false;
        for (auto &o : qos_restore_q_) still_open |= o.gpu == it.gpu;
        if (still_open) continue;  // a later window on this GPU keeps the pause
        lk.unlock();
        broadcastQos(it.gpu, 0, 0, true);
        lk.lock();
    }
}

}  // namespace mpcomm
