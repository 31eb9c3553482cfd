// Control plane: connect/accept handshake, buffer publish and query.
// Wire format and message order: see ctrl/wire.h (byte-compatible with the
// reference, src/mpcomm.cpp:3375-3848 and 3982-4896).
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <set>

#include "core/nvtx.h"
#include "cuda/gpu.h"
#include "engine/impl.h"
#include "mpcomm_log.h"
#include "topo/topology.h"

namespace mpcomm {

// ---- Connection helpers -----------------------------------------------------
uint32_t Connection::rkey_for(uint64_t raddr, size_t remote_rail) const {
    std::lock_guard<std::mutex> g(mu);
    auto it = remote_buffers.upper_bound(raddr);
    if (it != remote_buffers.begin()) {
        --it;
        const RemoteBufferEntry &e = it->second;
        if (raddr >= e.addr && raddr < e.addr + e.length && remote_rail < e.rkeys.size() &&
            e.rkeys[remote_rail] != 0)
            return e.rkeys[remote_rail];
    }
    return remote_rail < nic_endpoints.size() ? nic_endpoints[remote_rail].rkey : 0;
}

int Connection::remote_gpu_for(uint64_t raddr) const {
    std::lock_guard<std::mutex> g(mu);
    auto it = remote_buffers.upper_bound(raddr);
    if (it == remote_buffers.begin()) return -1;
    --it;
    const RemoteBufferEntry &e = it->second;
    return (raddr >= e.addr && raddr < e.addr + e.length) ? e.gpu_device_id : -1;
}

QpGroup *Connection::group_for(size_t local_rail) const {
    auto it = local_to_remote.find(local_rail);
    if (it == local_to_remote.end() || it->second.empty()) return nullptr;
    auto g = groups.find({local_rail, it->second[0]});
    return g == groups.end() ? nullptr : g->second.get();
}

std::shared_ptr<Connection> MPComm::Impl::connection(const std::string &id) const {
    std::lock_guard<std::mutex> g(conn_mu_);
    auto it = connections_.find(id);
    return it == connections_.end() ? nullptr : it->second;
}

// Pairs of (active rail, passive rail) in the order the active side walks
// them. suffix mode: rail with suffix N -> peer suffix N (primary) and N-4 /
// N+4 (cross-NUMA secondary), as the reference; a rail with neither falls
// back to peer (index mod count) so differently named fabrics still pair.
// index mode: rail i -> peer (i mod count).
std::vector<std::pair<size_t, size_t>> MPComm::Impl::pairRails(
    const std::vector<std::string> &active, const std::vector<std::string> &passive, bool) const {
    std::vector<std::pair<size_t, size_t>> out;
    if (passive.empty()) return out;
    std::map<int, size_t> by_suffix;
    for (size_t i = 0; i < passive.size(); ++i) {
        int s = topo::name_suffix(passive[i]);
        if (s >= 0 && !by_suffix.count(s)) by_suffix[s] = i;
    }
    for (size_t a = 0; a < active.size(); ++a) {
        std::vector<size_t> t;
        if (cfg_.nic_pairing == "suffix") {
            int s = topo::name_suffix(active[a]);
            auto p = by_suffix.find(s);
            if (s >= 0 && p != by_suffix.end()) t.push_back(p->second);
            int cross = s >= 4 ? s - 4 : s + 4;
            auto c = by_suffix.find(cross);
            if (s >= 0 && c != by_suffix.end() && (t.empty() || t[0] != c->second)) t.push_back(c->second);
        }
        if (t.empty()) t.push_back(a % passive.size());
        for (size_t r : t) out.emplace_back(a, r);
    }
    return out;
}

namespace {

bool send_names(int fd, const std::vector<std::string> &names) {
    for (auto &n : names) {
        uint32_t len = static_cast<uint32_t>(n.size());
        if (!net::send_pod(fd, len) || (len && !net::send_all(fd, n.data(), len))) return false;
    }
    return true;
}

bool recv_names(int fd, size_t count, std::vector<std::string> *names) {
    names->assign(count, std::string());
    for (size_t i = 0; i < count; ++i) {
        uint32_t len = 0;
        if (!net::recv_pod(fd, &len) || len > 4096) return false;
        std::string s(len, '\0');
        if (len && !net::recv_all(fd, &s[0], len)) return false;
        (*names)[i] = s.c_str();
    }
    return true;
}

RemoteEndpointInfo make_info(const std::string &gid, uint16_t lid, uint32_t qpn, uint64_t addr,
                             uint64_t length) {
    RemoteEndpointInfo e;
    std::memset(&e, 0, sizeof(e));
    std::strncpy(e.gid, gid.c_str(), sizeof(e.gid) - 1);
    e.lid = lid;
    e.qp_num = qpn;
    e.addr = addr;
    e.length = length;
    return e;
}

fabric::EndpointInfo to_ep(const RemoteEndpointInfo &r) {
    fabric::EndpointInfo e;
    char g[65];
    std::memcpy(g, r.gid, 64);
    g[64] = 0;
    e.gid = g;
    e.lid = r.lid;
    e.qp_num = r.qp_num;
    return e;
}

}  // namespace

int MPComm::Impl::connect(const std::string &id, const std::string &addr, int port) {
    nvtx::Range range("mpcomm::connect");
    if (!initialized_) return MPCOMM_ERR_CONTEXT;
    int fd = net::connect_tcp(addr, port, net::ctrl_timeout_ms());
    if (fd < 0) return MPCOMM_ERR_CONNECTION;
    auto fail = [&](const char *what) {
        MPCOMM_LOG_ERROR("MPComm: connect to %s (%s:%d) failed: %s\n", id.c_str(), addr.c_str(), port, what);
        ::close(fd);
        return MPCOMM_ERR_CONNECTION;
    };
    auto conn = std::make_shared<Connection>();
    conn->host_id = id;
    conn->tcp_addr = addr;
    conn->tcp_port = port;

    const uint32_t nn = static_cast<uint32_t>(rails_.size());
    uint32_t rn = 0;
    if (!net::send_pod(fd, nn) || !net::recv_pod(fd, &rn)) return fail("nic count");
    if (rn > kMaxConnectNicCount) return fail("bad remote nic count");
    int32_t numa_count = static_cast<int32_t>(numa_topology_.size());
    std::vector<int32_t> nic_numa(nn);
    for (uint32_t i = 0; i < nn; ++i) nic_numa[i] = rails_[i]->numa;
    if (!net::send_pod(fd, numa_count) ||
        (nn && !net::send_all(fd, nic_numa.data(), nn * sizeof(int32_t))))
        return fail("numa map");
    int32_t rnuma = 0;
    std::vector<int32_t> rnic_numa(rn);
    if (!net::recv_pod(fd, &rnuma) || (rn && !net::recv_all(fd, rnic_numa.data(), rn * sizeof(int32_t))))
        return fail("remote numa map");
    conn->remote_numa_count = rnuma;
    conn->remote_nic_numa.assign(rnic_numa.begin(), rnic_numa.end());
    std::vector<std::string> lnames = activeDevices(), rnames;
    if (!send_names(fd, lnames) || !recv_names(fd, rn, &rnames)) return fail("nic names");
    conn->remote_nic_names = rnames;
    const uint32_t qps = static_cast<uint32_t>(cfg_.qps_per_connection);
    uint32_t rqps = 0;
    if (!net::send_pod(fd, qps) || !net::recv_pod(fd, &rqps)) return fail("qp count");
    const size_t actual = std::max<size_t>(1, std::min<size_t>(qps, rqps));
    conn->nic_endpoints.assign(rn, RemoteEndpointInfo{});

    size_t total = 0, skipped = 0;
    for (auto pr : pairRails(lnames, rnames, true)) {
        const size_t l = pr.first, r = pr.second;
        auto group = std::make_unique<QpGroup>();
        group->local_rail = l;
        group->remote_rail = r;
        bool ok = true;
        for (size_t q = 0; q < actual; ++q) {
            auto qp = rails_[l]->rail->create_qp();
            if (!qp || qp->to_init() != 0) return fail("qp create");
            RemoteEndpointInfo mine =
                make_info(rails_[l]->gid, rails_[l]->rail->lid(), qp->qp_num(), r, l);
            RemoteEndpointInfo theirs;
            if (!net::send_pod(fd, mine) || !net::recv_pod(fd, &theirs)) return fail("endpoint exchange");
            int rc = qp->to_rtr(to_ep(theirs));
            if (rc == 0) rc = qp->to_rts();
            uint8_t status = rc == 0 ? 0 : 1;
            if (!net::send_pod(fd, status)) return fail("qp status");
            if (rc != 0) {
                MPCOMM_LOG_WARN("MPComm: skipping rail pair %s->%s (QP transition failed)\n",
                                lnames[l].c_str(), rnames[r].c_str());
                ok = false;
                break;
            }
            group->qps.push_back(std::move(qp));
            if (q == 0) conn->nic_endpoints[r] = theirs;
        }
        if (!ok) {
            ++skipped;
            continue;
        }
        conn->groups[{l, r}] = std::move(group);
        conn->local_to_remote[l].push_back(r);
        ++total;
    }
    ::close(fd);
    if (total == 0) {
        MPCOMM_LOG_ERROR("MPComm: no rail pair connected to %s (%zu skipped)\n", id.c_str(), skipped);
        return MPCOMM_ERR_CONNECTION;
    }
    {
        std::lock_guard<std::mutex> g(conn_mu_);
        connections_[id] = conn;
    }
    MPCOMM_LOG_INFO("MPComm: connected to %s: %zu rail pairs x %zu QPs (%zu skipped)\n", id.c_str(),
                    total, actual, skipped);
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::startAcceptThread() {
    if (listen_fd_ < 0) return MPCOMM_ERR_CONNECTION;
    if (accept_running_.exchange(true)) return MPCOMM_SUCCESS;
    accept_thread_ = std::thread([this] { acceptLoop(); });
    return MPCOMM_SUCCESS;
}

void MPComm::Impl::stopAcceptThread() {
    if (!accept_running_.exchange(false)) {
        if (accept_thread_.joinable()) accept_thread_.join();
        return;
    }
    // Unblock accept() by connecting to ourselves (reference behaviour); the
    // loop sees accept_running_ == false and exits.
    int fd = net::connect_tcp("127.0.0.1", tcp_port_, 2000);
    if (fd >= 0) ::close(fd);
    if (accept_thread_.joinable()) accept_thread_.join();
}

namespace {
constexpr int kFirstWordTimeoutMs = 2000;
}  // namespace

void MPComm::Impl::acceptLoop() {
    while (accept_running_.load()) {
        int fd = ::accept4(listen_fd_, nullptr, nullptr, SOCK_CLOEXEC);
        if (fd < 0) {
            if (!accept_running_.load()) break;
            continue;
        }
        if (!accept_running_.load()) {
            ::close(fd);
            break;
        }
        // Connections are served one at a time (as the reference does), so a
        // client that connects and stays silent (a port scanner, a half-open
        // peer) may hold the loop only briefly: every legitimate client sends
        // its first word right after connecting.
        const int full = net::ctrl_timeout_ms();
        net::set_timeouts(fd, full > 0 && full < kFirstWordTimeoutMs ? full : kFirstWordTimeoutMs);
        int one = 1;
        setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
        uint32_t msg = 0;
        if (!net::recv_pod(fd, &msg)) {
            ::close(fd);
            continue;
        }
        net::set_timeouts(fd, full);
        if (msg == kMsgTypeBufferQuery) {
            handleBufferQuery(fd);
        } else if (msg == kMsgTypeQosControlOpen) {
            handleQosChannel(fd);
        } else if (msg < kMaxConnectNicCount) {
            handleConnect(fd, msg);
        } else {
            MPCOMM_LOG_WARN("MPComm: unknown control message 0x%08x\n", msg);
        }
        ::close(fd);
    }
}

void MPComm::Impl::handleConnect(int fd, uint32_t rn) {
    int peer_port = 0;
    const std::string peer = net::peer_id(fd, &peer_port);
    auto conn = std::make_shared<Connection>();
    conn->host_id = peer;
    conn->tcp_port = peer_port;
    const uint32_t nn = static_cast<uint32_t>(rails_.size());
    if (!net::send_pod(fd, nn)) return;
    int32_t rnuma = 0;
    std::vector<int32_t> rnic_numa(rn);
    if (!net::recv_pod(fd, &rnuma) || (rn && !net::recv_all(fd, rnic_numa.data(), rn * sizeof(int32_t))))
        return;
    int32_t numa_count = static_cast<int32_t>(numa_topology_.size());
    std::vector<int32_t> nic_numa(nn);
    for (uint32_t i = 0; i < nn; ++i) nic_numa[i] = rails_[i]->numa;
    if (!net::send_pod(fd, numa_count) || (nn && !net::send_all(fd, nic_numa.data(), nn * sizeof(int32_t))))
        return;
    conn->remote_numa_count = rnuma;
    conn->remote_nic_numa.assign(rnic_numa.begin(), rnic_numa.end());
    std::vector<std::string> rnames, lnames = activeDevices();
    if (!recv_names(fd, rn, &rnames) || !send_names(fd, lnames)) return;
    conn->remote_nic_names = rnames;
    uint32_t rqps = 0;
    const uint32_t qps = static_cast<uint32_t>(cfg_.qps_per_connection);
    if (!net::recv_pod(fd, &rqps) || !net::send_pod(fd, qps)) return;
    const size_t actual = std::max<size_t>(1, std::min<size_t>(qps, rqps));
    conn->nic_endpoints.assign(rn, RemoteEndpointInfo{});

    const size_t expected = pairRails(rnames, lnames, false).size();
    size_t handled = 0;
    bool success = true;
    while (handled < expected && success) {
        RemoteEndpointInfo theirs;
        if (!net::recv_pod(fd, &theirs)) {
            success = false;
            break;
        }
        const size_t l = static_cast<size_t>(theirs.addr);    // our rail
        const size_t r = static_cast<size_t>(theirs.length);  // their rail
        if (l >= nn || r >= rn) {
            MPCOMM_LOG_WARN("MPComm: bad rail indices %zu/%zu from %s\n", l, r, peer.c_str());
            success = false;
            break;
        }
        auto group = std::make_unique<QpGroup>();
        group->local_rail = l;
        group->remote_rail = r;
        bool skipped = false;
        for (size_t q = 0; q < actual && success; ++q) {
            if (q > 0 && !net::recv_pod(fd, &theirs)) {
                success = false;
                break;
            }
            auto qp = rails_[l]->rail->create_qp();
            if (!qp || qp->to_init() != 0) {
                success = false;
                break;
            }
            RemoteEndpointInfo mine = make_info(rails_[l]->gid, rails_[l]->rail->lid(), qp->qp_num(), 0, 0);
            uint8_t status = 0;
            if (!net::send_pod(fd, mine) || !net::recv_pod(fd, &status)) {
                success = false;
                break;
            }
            if (status != 0) {
                skipped = true;
                break;
            }
            if (qp->to_rtr(to_ep(theirs)) != 0 || qp->to_rts() != 0) {
                success = false;
                break;
            }
            group->qps.push_back(std::move(qp));
            if (q == 0) {
                theirs.addr = 0;
                conn->nic_endpoints[r] = theirs;
            }
        }
        ++handled;
        if (skipped || !success) continue;
        conn->groups[{l, r}] = std::move(group);
        conn->local_to_remote[l].push_back(r);
    }
    if (success) {
        std::lock_guard<std::mutex> g(conn_mu_);
        connections_[peer] = conn;
        MPCOMM_LOG_INFO("MPComm: accepted connection from %s (%zu rail pairs)\n", peer.c_str(),
                        conn->groups.size());
    }
}

int MPComm::Impl::updateRemoteMemoryInfo(const std::string &id, const std::vector<uint32_t> &rkeys) {
    if (!initialized_) return MPCOMM_ERR_CONTEXT;
    auto c = connection(id);
    if (!c) return MPCOMM_ERR_CONNECTION;
    std::lock_guard<std::mutex> g(c->mu);
    if (rkeys.size() != c->nic_endpoints.size()) return MPCOMM_ERR_INVALID_ARG;
    for (size_t i = 0; i < rkeys.size(); ++i) c->nic_endpoints[i].rkey = rkeys[i];
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::publishBuffer(void *addr, size_t len, int numa) {
    if (!initialized_) return MPCOMM_ERR_CONTEXT;
    if (!addr || len == 0) return MPCOMM_ERR_INVALID_ARG;
    Region r;
    if (!lookupRegion(reinterpret_cast<uintptr_t>(addr), len, &r)) {
        MPCOMM_LOG_ERROR("MPComm: publishBuffer(%p) — buffer not registered\n", addr);
        return MPCOMM_ERR_MEMORY;
    }
    PublishedBufferEntry e;
    e.addr = reinterpret_cast<uint64_t>(addr);
    e.length = len;
    e.numa_node = numa >= 0 ? numa : numaNodeForAddr(addr);
    e.gpu_device_id = gpu::device_of(addr);
    if (e.gpu_device_id >= 0) e.pcie_affine_nic_indices = affineRailsForGpu(e.gpu_device_id);
    const uintptr_t off = reinterpret_cast<uintptr_t>(addr) - r.addr;
    (void)off;  // keys cover the whole region; the rkey is the region's
    for (size_t i = 0; i < r.keys.size(); ++i) e.rkeys.push_back(r.keys[i].rkey);
    std::lock_guard<std::mutex> g(pub_mu_);
    for (auto &p : published_) {
        if (p.addr == e.addr) {
            p = e;
            return MPCOMM_SUCCESS;
        }
    }
    published_.push_back(std::move(e));
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::unpublishBuffer(void *addr) {
    if (!initialized_) return MPCOMM_ERR_CONTEXT;
    std::lock_guard<std::mutex> g(pub_mu_);
    for (auto it = published_.begin(); it != published_.end(); ++it) {
        if (it->addr == reinterpret_cast<uint64_t>(addr)) {
            published_.erase(it);
            return MPCOMM_SUCCESS;
        }
    }
    return MPCOMM_ERR_INVALID_ARG;
}

void MPComm::Impl::unpublishAllBuffers() {
    std::lock_guard<std::mutex> g(pub_mu_);
    published_.clear();
}

size_t MPComm::Impl::getPublishedBufferCount() const {
    std::lock_guard<std::mutex> g(pub_mu_);
    return published_.size();
}

const PublishedBufferInfo *MPComm::Impl::getPublishedBufferInfo() const {
    std::lock_guard<std::mutex> g(pub_mu_);
    if (published_.empty()) return nullptr;
    published_snapshot_.buffers = published_;
    return &published_snapshot_;
}

void MPComm::Impl::handleBufferQuery(int fd) {
    std::vector<PublishedBufferEntry> bufs;
    {
        std::lock_guard<std::mutex> g(pub_mu_);
        bufs = published_;
    }
    const uint32_t nb = static_cast<uint32_t>(bufs.size());
    if (!net::send_pod(fd, nb) || nb == 0) return;
    const uint32_t nn = static_cast<uint32_t>(rails_.size());
    if (!net::send_pod(fd, nn)) return;
    for (uint32_t i = 0; i < nn; ++i) {
        char g[64];
        std::memset(g, 0, sizeof(g));
        std::strncpy(g, rails_[i]->gid.c_str(), sizeof(g) - 1);
        if (!net::send_all(fd, g, sizeof(g))) return;
    }
    for (auto &b : bufs) {
        const int32_t numa = b.numa_node, gpu_id = b.gpu_device_id;
        const uint32_t aff = static_cast<uint32_t>(std::min(b.pcie_affine_nic_indices.size(), kMaxRails));
        if (!net::send_pod(fd, b.addr) || !net::send_pod(fd, b.length) || !net::send_pod(fd, numa) ||
            !net::send_pod(fd, gpu_id) || !net::send_pod(fd, aff))
            return;
        for (uint32_t i = 0; i < aff; ++i) {
            uint32_t v = static_cast<uint32_t>(b.pcie_affine_nic_indices[i]);
            if (!net::send_pod(fd, v)) return;
        }
        for (uint32_t i = 0; i < nn; ++i) {
            uint32_t k = i < b.rkeys.size() ? b.rkeys[i] : 0;
            if (!net::send_pod(fd, k)) return;
        }
    }
}

int MPComm::Impl::queryRemoteBuffer(const std::string &id, const std::string &addr, int port,
                                    RemoteBufferInfo &out) {
    if (!initialized_) return MPCOMM_ERR_CONTEXT;
    int fd = net::connect_tcp(addr, port, net::ctrl_timeout_ms());
    if (fd < 0) return MPCOMM_ERR_CONNECTION;
    auto fail = [&](int code) {
        ::close(fd);
        return code;
    };
    const uint32_t msg = kMsgTypeBufferQuery;
    uint32_t nb = 0;
    if (!net::send_pod(fd, msg) || !net::recv_pod(fd, &nb)) return fail(MPCOMM_ERR_CONNECTION);
    if (nb == 0) {
        MPCOMM_LOG_ERROR("MPComm: %s has no published buffers\n", id.c_str());
        return fail(MPCOMM_ERR_INVALID_ARG);
    }
    uint32_t nn = 0;
    if (!net::recv_pod(fd, &nn) || nn > 4096) return fail(MPCOMM_ERR_CONNECTION);
    std::vector<std::string> gids(nn);
    for (uint32_t i = 0; i < nn; ++i) {
        char g[65];
        if (!net::recv_all(fd, g, 64)) return fail(MPCOMM_ERR_CONNECTION);
        g[64] = 0;
        gids[i] = g;
    }
    out.host_id = id;
    out.buffers.clear();
    for (uint32_t b = 0; b < nb; ++b) {
        RemoteBufferEntry e;
        int32_t numa = 0, gpu_id = -1;
        uint32_t aff = 0;
        if (!net::recv_pod(fd, &e.addr) || !net::recv_pod(fd, &e.length) || !net::recv_pod(fd, &numa) ||
            !net::recv_pod(fd, &gpu_id) || !net::recv_pod(fd, &aff) || aff > kMaxRails)
            return fail(MPCOMM_ERR_CONNECTION);
        e.numa_node = numa;
        e.gpu_device_id = gpu_id;
        for (uint32_t i = 0; i < aff; ++i) {
            uint32_t v = 0;
            if (!net::recv_pod(fd, &v)) return fail(MPCOMM_ERR_CONNECTION);
            e.pcie_affine_nic_indices.push_back(v);
        }
        e.rkeys.resize(nn);
        for (uint32_t i = 0; i < nn; ++i)
            if (!net::recv_pod(fd, &e.rkeys[i])) return fail(MPCOMM_ERR_CONNECTION);
        out.buffers.push_back(std::move(e));
    }
    ::close(fd);

    // Store into the connection with rkeys re-ordered to our endpoint view
    // (match by GID string, reference :3657-3676).
    auto conn = connection(id);
    if (conn) {
        std::lock_guard<std::mutex> g(conn->mu);
        conn->remote_buffers.clear();
        const size_t eps = conn->nic_endpoints.size();
        for (auto &b : out.buffers) {
            RemoteBufferEntry r = b;
            r.rkeys.assign(eps, 0);
            for (size_t ep = 0; ep < eps; ++ep) {
                std::string eg(conn->nic_endpoints[ep].gid,
                               strnlen(conn->nic_endpoints[ep].gid, sizeof(conn->nic_endpoints[ep].gid)));
                for (uint32_t k = 0; k < nn; ++k)
                    if (!eg.empty() && gids[k] == eg) {
                        r.rkeys[ep] = b.rkeys[k];
                        break;
                    }
            }
            conn->remote_buffers[b.addr] = r;
        }
        const auto &first = out.buffers[0];
        for (size_t ep = 0; ep < eps; ++ep) {
            std::string eg(conn->nic_endpoints[ep].gid,
                           strnlen(conn->nic_endpoints[ep].gid, sizeof(conn->nic_endpoints[ep].gid)));
            for (uint32_t k = 0; k < nn; ++k)
                if (!eg.empty() && gids[k] == eg) {
                    conn->nic_endpoints[ep].rkey = first.rkeys[k];
                    break;
                }
        }
    }
    return MPCOMM_SUCCESS;
}

int MPComm::Impl::queryRemoteBufferByNuma(const std::string &id, const std::string &addr, int port,
                                          int numa, RemoteBufferEntry &out) {
    RemoteBufferInfo all;
    int rc = queryRemoteBuffer(id, addr, port, all);
    if (rc != MPCOMM_SUCCESS) return rc;
    if (all.buffers.empty()) return MPCOMM_ERR_INVALID_ARG;
    if (numa >= 0) {
        for (auto &b : all.buffers)
            if (b.numa_node == numa) {
                out = b;
                return MPCOMM_SUCCESS;
            }
        MPCOMM_LOG_WARN("MPComm: no buffer tagged %d on %s, using the first\n", numa, id.c_str());
    }
    out = all.buffers[0];
    return MPCOMM_SUCCESS;
}

}  // namespace mpcomm
