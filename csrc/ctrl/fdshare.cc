#include "ctrl/fdshare.h"

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cstdio>
#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>

#include "mpcomm_log.h"

namespace mpcomm {
namespace ctrl {
namespace {

enum : uint8_t { kOk = 0, kNoKey = 1, kDenied = 2 };

// Reply: messages of this header, `count` wire segments and `count`
// descriptors (SCM_RIGHTS), until `total` segments have been sent. A refusal
// is one header with count = total = 0.
struct ReplyHeader {
    uint8_t status;
    uint8_t pad[3];
    uint32_t count;
    uint32_t total;
    uint32_t pad2;
};
struct WireSegment {
    uint64_t offset;
    uint64_t size;
};
constexpr size_t kPerMessage = 64;

socklen_t abstract_addr(const std::string &name, sockaddr_un *a) {
    std::memset(a, 0, sizeof(*a));
    a->sun_family = AF_UNIX;
    const size_t n = std::min(name.size(), sizeof(a->sun_path) - 2);
    std::memcpy(a->sun_path + 1, name.data(), n);
    return static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + n);
}

bool wait_in(int fd, int ms) {
    pollfd p{fd, POLLIN, 0};
    for (;;) {
        const int r = poll(&p, 1, ms);
        if (r > 0) return (p.revents & POLLIN) != 0;
        if (r == 0 || errno != EINTR) return false;
    }
}

bool send_part(int c, uint8_t st, const std::vector<FdSegment> &segs, size_t first, size_t n) {
    char buf[sizeof(ReplyHeader) + kPerMessage * sizeof(WireSegment)];
    ReplyHeader h{};
    h.status = st;
    h.count = static_cast<uint32_t>(n);
    h.total = static_cast<uint32_t>(segs.size());
    std::memcpy(buf, &h, sizeof(h));
    for (size_t i = 0; i < n; ++i) {
        WireSegment w{segs[first + i].offset, segs[first + i].size};
        std::memcpy(buf + sizeof(h) + i * sizeof(w), &w, sizeof(w));
    }
    iovec io{buf, sizeof(h) + n * sizeof(WireSegment)};
    msghdr m{};
    m.msg_iov = &io;
    m.msg_iovlen = 1;
    alignas(cmsghdr) char ctl[CMSG_SPACE(kPerMessage * sizeof(int))];
    if (n) {
        std::memset(ctl, 0, sizeof(ctl));
        m.msg_control = ctl;
        m.msg_controllen = CMSG_SPACE(n * sizeof(int));
        cmsghdr *c0 = CMSG_FIRSTHDR(&m);
        c0->cmsg_level = SOL_SOCKET;
        c0->cmsg_type = SCM_RIGHTS;
        c0->cmsg_len = CMSG_LEN(n * sizeof(int));
        for (size_t i = 0; i < n; ++i) std::memcpy(CMSG_DATA(c0) + i * sizeof(int), &segs[first + i].fd, sizeof(int));
    }
    return sendmsg(c, &m, MSG_NOSIGNAL) == static_cast<ssize_t>(io.iov_len);
}

class Server {
 public:
    // Never destroyed: offers may be withdrawn by other objects' destructors
    // at exit, after function-local statics are gone; the thread ends with
    // the process.
    static Server &get() {
        static Server *s = new Server;
        return *s;
    }

    int offer(const std::string &name, uint64_t key, FdProvider p) {
        std::lock_guard<std::mutex> g(mu_);
        if (lfd_ < 0 && start(name) != 0) return -1;
        offers_[key] = std::move(p);
        return 0;
    }

    void withdraw(uint64_t key) {
        std::lock_guard<std::mutex> g(mu_);
        offers_.erase(key);
    }

 private:
    int start(const std::string &name) {
        int s = socket(AF_UNIX, SOCK_SEQPACKET | SOCK_CLOEXEC, 0);
        sockaddr_un a;
        const socklen_t n = abstract_addr(name, &a);
        if (s < 0 || bind(s, reinterpret_cast<sockaddr *>(&a), n) != 0 || listen(s, 64) != 0) {
            MPCOMM_LOG_WARN("MPComm: descriptor server '%s' cannot listen: %s\n", name.c_str(), std::strerror(errno));
            if (s >= 0) close(s);
            return -1;
        }
        lfd_ = s;
        std::thread([this] { run(); }).detach();
        return 0;
    }

    void run() {
        for (;;) {
            if (!wait_in(lfd_, -1)) {
                std::this_thread::sleep_for(std::chrono::milliseconds(100));
                continue;
            }
            const int c = accept4(lfd_, nullptr, nullptr, SOCK_CLOEXEC);
            if (c < 0) continue;
            serve(c);
            close(c);
        }
    }

    // One request: u64 key in; the segments out, when the key is offered,
    // its provider succeeds and the peer runs as our user.
    void serve(int c) {
        uint64_t key = 0;
        if (!wait_in(c, 1000) || recv(c, &key, sizeof(key), 0) != static_cast<ssize_t>(sizeof(key))) return;
        ucred cred{};
        socklen_t cl = sizeof(cred);
        uint8_t st = kOk;
        if (getsockopt(c, SOL_SOCKET, SO_PEERCRED, &cred, &cl) != 0 || cred.uid != geteuid()) st = kDenied;
        std::vector<FdSegment> segs;
        if (st == kOk) {
            FdProvider p;
            {
                std::lock_guard<std::mutex> g(mu_);
                auto it = offers_.find(key);
                if (it != offers_.end()) p = it->second;
            }
            if (!p || !p(&segs) || segs.empty() || segs.size() > kFdMaxSegments) st = kNoKey;
        }
        if (st != kOk) {
            for (auto &s : segs) close(s.fd);
            segs.clear();
            send_part(c, st, segs, 0, 0);
            return;
        }
        for (size_t i = 0; i < segs.size(); i += kPerMessage)
            if (!send_part(c, kOk, segs, i, std::min(kPerMessage, segs.size() - i))) break;
        for (auto &s : segs) close(s.fd);
    }

    std::mutex mu_;
    std::map<uint64_t, FdProvider> offers_;
    int lfd_ = -1;
};

}  // namespace

std::string fd_service_name(long pid) {
    static const std::string boot = [] {
        std::string s;
        if (FILE *f = std::fopen("/proc/sys/kernel/random/boot_id", "r")) {
            int c;
            while ((c = std::fgetc(f)) != EOF && s.size() < 8)
                if (std::isxdigit(c)) s.push_back(static_cast<char>(c));
            std::fclose(f);
        }
        return s.empty() ? std::string("00000000") : s;
    }();
    return "mpcomm-fd." + boot + "." + std::to_string(pid);
}

int fd_offer(const std::string &name, uint64_t key, FdProvider provider) {
    return Server::get().offer(name, key, std::move(provider));
}

void fd_withdraw(uint64_t key) { Server::get().withdraw(key); }

int fd_fetch(const std::string &name, uint64_t key, int timeout_ms, std::vector<FdSegment> *out) {
    out->clear();
    int s = socket(AF_UNIX, SOCK_SEQPACKET | SOCK_CLOEXEC, 0);
    if (s < 0) return -1;
    sockaddr_un a;
    const socklen_t n = abstract_addr(name, &a);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    auto left = [&] {
        const auto d = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - std::chrono::steady_clock::now());
        return static_cast<int>(std::max<int64_t>(0, d.count()));
    };
    int rc = -1;
    if (connect(s, reinterpret_cast<sockaddr *>(&a), n) == 0 &&
        send(s, &key, sizeof(key), MSG_NOSIGNAL) == static_cast<ssize_t>(sizeof(key))) {
        size_t total = SIZE_MAX;
        while (out->size() < total) {
            char buf[sizeof(ReplyHeader) + kPerMessage * sizeof(WireSegment)];
            alignas(cmsghdr) char ctl[CMSG_SPACE(kPerMessage * sizeof(int))];
            iovec io{buf, sizeof(buf)};
            msghdr m{};
            m.msg_iov = &io;
            m.msg_iovlen = 1;
            m.msg_control = ctl;
            m.msg_controllen = sizeof(ctl);
            if (!wait_in(s, left())) break;
            const ssize_t got = recvmsg(s, &m, MSG_CMSG_CLOEXEC);
            if (got < static_cast<ssize_t>(sizeof(ReplyHeader))) break;
            ReplyHeader h;
            std::memcpy(&h, buf, sizeof(h));
            // Descriptors first, so every one that arrived is closed on error.
            std::vector<int> fds;
            for (cmsghdr *c = CMSG_FIRSTHDR(&m); c; c = CMSG_NXTHDR(&m, c)) {
                if (c->cmsg_level != SOL_SOCKET || c->cmsg_type != SCM_RIGHTS) continue;
                const size_t k = (c->cmsg_len - CMSG_LEN(0)) / sizeof(int);
                for (size_t i = 0; i < k; ++i) {
                    int f;
                    std::memcpy(&f, CMSG_DATA(c) + i * sizeof(int), sizeof(int));
                    fds.push_back(f);
                }
            }
            const bool shaped = h.status == kOk && h.count == fds.size() && h.count <= kPerMessage &&
                                (m.msg_flags & MSG_CTRUNC) == 0 &&
                                static_cast<size_t>(got) == sizeof(h) + h.count * sizeof(WireSegment) &&
                                h.total > 0 && h.total <= kFdMaxSegments &&
                                (total == SIZE_MAX || h.total == total) && out->size() + h.count <= h.total;
            if (!shaped) {
                for (int f : fds) close(f);
                if (h.status == kNoKey || h.status == kDenied) rc = h.status == kNoKey ? 1 : -1;
                break;
            }
            total = h.total;
            for (size_t i = 0; i < h.count; ++i) {
                WireSegment w;
                std::memcpy(&w, buf + sizeof(h) + i * sizeof(w), sizeof(w));
                out->push_back(FdSegment{w.offset, w.size, fds[i]});
            }
        }
        if (total != SIZE_MAX && out->size() == total) rc = 0;
    }
    close(s);
    if (rc != 0) {
        for (auto &f : *out) close(f.fd);
        out->clear();
    }
    return rc;
}

}  // namespace ctrl
}  // namespace mpcomm
