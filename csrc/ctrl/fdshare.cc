#include "ctrl/fdshare.h"

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <thread>

#include "mpcomm_log.h"

namespace mpcomm {
namespace ctrl {
namespace {

enum : uint8_t { kOk = 0, kNoKey = 1, kDenied = 2 };

// Reply: messages of this header, `count` wire segments and `count`
// descriptors (SCM_RIGHTS), until `total` segments have been sent. A
// refusal, or an export that fails part-way, is a header with that status
// and count 0.
struct ReplyHeader {
    uint8_t status;
    uint8_t pad[3];
    uint32_t count;
    uint32_t total;
    uint32_t pad2;
    uint64_t total_bytes;
};
struct WireSegment {
    uint64_t offset;
    uint64_t size;
};
constexpr size_t kPerMessage = 64;
constexpr size_t kMsgBytes = sizeof(ReplyHeader) + kPerMessage * sizeof(WireSegment);

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

bool send_part(int c, const ReplyHeader &hdr, const FdSegment *segs, size_t n) {
    char buf[kMsgBytes];
    ReplyHeader h = hdr;
    h.count = static_cast<uint32_t>(n);
    std::memcpy(buf, &h, sizeof(h));
    for (size_t i = 0; i < n; ++i) {
        WireSegment w{segs[i].offset, segs[i].size};
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
        for (size_t i = 0; i < n; ++i) std::memcpy(CMSG_DATA(c0) + i * sizeof(int), &segs[i].fd, sizeof(int));
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

    int offer(const std::string &name, uint64_t key, FdOffer o) {
        std::lock_guard<std::mutex> g(mu_);
        if (lfd_ < 0 && start(name) != 0) return -1;
        offers_[key] = std::make_shared<const FdOffer>(std::move(o));
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

    // One request: u64 key in; the segments out, exported and sent one
    // message at a time, when the key is offered and the peer runs as our
    // user.
    void serve(int c) {
        uint64_t key = 0;
        if (!wait_in(c, 1000) || recv(c, &key, sizeof(key), 0) != static_cast<ssize_t>(sizeof(key))) return;
        ucred cred{};
        socklen_t cl = sizeof(cred);
        ReplyHeader h{};
        h.status = kOk;
        if (getsockopt(c, SOL_SOCKET, SO_PEERCRED, &cred, &cl) != 0 || cred.uid != geteuid()) h.status = kDenied;
        std::shared_ptr<const FdOffer> o;
        if (h.status == kOk) {
            std::lock_guard<std::mutex> g(mu_);
            auto it = offers_.find(key);
            if (it != offers_.end()) o = it->second;
        }
        if (h.status == kOk && (!o || o->segments.empty() || o->segments.size() > kFdMaxSegments || !o->export_fd))
            h.status = kNoKey;
        if (h.status != kOk) {
            send_part(c, h, nullptr, 0);
            return;
        }
        h.total = static_cast<uint32_t>(o->segments.size());
        for (const auto &s : o->segments) h.total_bytes += s.size;
        FdSegment part[kPerMessage];
        for (size_t i = 0; i < o->segments.size(); i += kPerMessage) {
            const size_t n = std::min(kPerMessage, o->segments.size() - i);
            size_t ok = 0;
            for (; ok < n; ++ok) {
                part[ok] = o->segments[i + ok];
                part[ok].fd = o->export_fd(i + ok);
                if (part[ok].fd < 0) break;
            }
            const bool sent = ok == n && send_part(c, h, part, n);
            for (size_t k = 0; k < ok; ++k) close(part[k].fd);
            if (ok != n) {
                ReplyHeader e = h;
                e.status = kNoKey;
                send_part(c, e, nullptr, 0);
            }
            if (!sent) return;
        }
    }

    std::mutex mu_;
    std::map<uint64_t, std::shared_ptr<const FdOffer>> offers_;
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

int fd_offer(const std::string &name, uint64_t key, FdOffer offer) {
    return Server::get().offer(name, key, std::move(offer));
}

void fd_withdraw(uint64_t key) { Server::get().withdraw(key); }

int fd_fetch(const std::string &name, uint64_t key, int timeout_ms,
             const std::function<bool(size_t count, uint64_t bytes)> &on_begin,
             const std::function<bool(const FdSegment &)> &on_segment) {
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
        size_t total = SIZE_MAX, got_segments = 0;
        uint64_t total_bytes = 0;
        bool stop = false;
        while (!stop && got_segments < total) {
            char buf[kMsgBytes];
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
            // Every descriptor that arrived is closed, whatever happens next.
            int fds[kPerMessage];
            size_t nfd = 0;
            for (cmsghdr *c = CMSG_FIRSTHDR(&m); c; c = CMSG_NXTHDR(&m, c)) {
                if (c->cmsg_level != SOL_SOCKET || c->cmsg_type != SCM_RIGHTS) continue;
                const size_t k = (c->cmsg_len - CMSG_LEN(0)) / sizeof(int);
                for (size_t i = 0; i < k; ++i) {
                    int f;
                    std::memcpy(&f, CMSG_DATA(c) + i * sizeof(int), sizeof(int));
                    if (nfd < kPerMessage) fds[nfd++] = f;
                    else close(f);
                }
            }
            const bool shaped = h.status == kOk && h.count == nfd && h.count > 0 && h.count <= kPerMessage &&
                                (m.msg_flags & MSG_CTRUNC) == 0 &&
                                static_cast<size_t>(got) == sizeof(h) + h.count * sizeof(WireSegment) &&
                                h.total > 0 && h.total <= kFdMaxSegments &&
                                (total == SIZE_MAX || (h.total == total && h.total_bytes == total_bytes)) &&
                                got_segments + h.count <= h.total;
            if (!shaped) {
                for (size_t i = 0; i < nfd; ++i) close(fds[i]);
                if (h.status == kNoKey) rc = 1;
                break;
            }
            if (total == SIZE_MAX) {
                total = h.total;
                total_bytes = h.total_bytes;
                if (!on_begin(total, total_bytes)) stop = true;
            }
            for (size_t i = 0; i < h.count; ++i) {
                WireSegment w;
                std::memcpy(&w, buf + sizeof(h) + i * sizeof(w), sizeof(w));
                if (!stop && !on_segment(FdSegment{w.offset, w.size, fds[i]})) stop = true;
                close(fds[i]);
            }
            got_segments += h.count;
        }
        if (!stop && total != SIZE_MAX && got_segments == total) rc = 0;
    }
    close(s);
    return rc;
}

}  // namespace ctrl
}  // namespace mpcomm
