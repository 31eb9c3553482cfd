#include "ctrl/fdshare.h"

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>

#include "mpcomm_log.h"

namespace mpcomm {
namespace ctrl {
namespace {

enum : uint8_t { kOk = 0, kNoKey = 1, kDenied = 2 };

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

class Server {
 public:
    static Server &get() {
        static Server s;
        return s;
    }

    int offer(const std::string &name, uint64_t key, int fd) {
        std::lock_guard<std::mutex> g(mu_);
        if (lfd_ < 0 && start(name) != 0) {
            close(fd);
            return -1;
        }
        auto it = fds_.find(key);
        if (it != fds_.end()) close(it->second);
        fds_[key] = fd;
        return 0;
    }

    void withdraw(uint64_t key) {
        std::lock_guard<std::mutex> g(mu_);
        auto it = fds_.find(key);
        if (it == fds_.end()) return;
        close(it->second);
        fds_.erase(it);
    }

    ~Server() {
        stop_ = true;
        if (th_.joinable()) th_.join();
        if (lfd_ >= 0) close(lfd_);
        for (auto &kv : fds_) close(kv.second);
    }

 private:
    int start(const std::string &name) {
        int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
        sockaddr_un a;
        const socklen_t n = abstract_addr(name, &a);
        if (s < 0 || bind(s, reinterpret_cast<sockaddr *>(&a), n) != 0 || listen(s, 64) != 0) {
            MPCOMM_LOG_WARN("MPComm: descriptor server '%s' cannot listen: %s\n", name.c_str(), std::strerror(errno));
            if (s >= 0) close(s);
            return -1;
        }
        lfd_ = s;
        th_ = std::thread([this] { run(); });
        return 0;
    }

    void run() {
        while (!stop_.load()) {
            if (!wait_in(lfd_, 100)) continue;
            const int c = accept4(lfd_, nullptr, nullptr, SOCK_CLOEXEC);
            if (c < 0) continue;
            serve(c);
            close(c);
        }
    }

    // One request: u64 key in; one status byte out, with the descriptor
    // attached when the key is known and the peer runs as our user.
    void serve(int c) {
        uint64_t key = 0;
        if (!wait_in(c, 1000) || recv(c, &key, sizeof(key), MSG_WAITALL) != static_cast<ssize_t>(sizeof(key)))
            return;
        ucred cred{};
        socklen_t cl = sizeof(cred);
        uint8_t st = kOk;
        if (getsockopt(c, SOL_SOCKET, SO_PEERCRED, &cred, &cl) != 0 || cred.uid != geteuid()) st = kDenied;
        std::lock_guard<std::mutex> g(mu_);
        auto it = fds_.find(key);
        if (st == kOk && it == fds_.end()) st = kNoKey;
        msghdr m{};
        iovec io{&st, 1};
        m.msg_iov = &io;
        m.msg_iovlen = 1;
        char ctl[CMSG_SPACE(sizeof(int))];
        if (st == kOk) {
            std::memset(ctl, 0, sizeof(ctl));
            m.msg_control = ctl;
            m.msg_controllen = sizeof(ctl);
            cmsghdr *h = CMSG_FIRSTHDR(&m);
            h->cmsg_level = SOL_SOCKET;
            h->cmsg_type = SCM_RIGHTS;
            h->cmsg_len = CMSG_LEN(sizeof(int));
            std::memcpy(CMSG_DATA(h), &it->second, sizeof(int));
        }
        sendmsg(c, &m, MSG_NOSIGNAL);
    }

    std::mutex mu_;
    std::map<uint64_t, int> fds_;
    int lfd_ = -1;
    std::thread th_;
    std::atomic<bool> stop_{false};
};

}  // namespace

int fd_offer(const std::string &name, uint64_t key, int fd) { return Server::get().offer(name, key, fd); }

void fd_withdraw(uint64_t key) { Server::get().withdraw(key); }

int fd_fetch(const std::string &name, uint64_t key, int timeout_ms, int *fd) {
    int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) return -1;
    sockaddr_un a;
    const socklen_t n = abstract_addr(name, &a);
    int rc = -1;
    uint8_t st = 0xFF;
    msghdr m{};
    iovec io{&st, 1};
    char ctl[CMSG_SPACE(sizeof(int))];
    m.msg_iov = &io;
    m.msg_iovlen = 1;
    m.msg_control = ctl;
    m.msg_controllen = sizeof(ctl);
    if (connect(s, reinterpret_cast<sockaddr *>(&a), n) == 0 &&
        send(s, &key, sizeof(key), MSG_NOSIGNAL) == static_cast<ssize_t>(sizeof(key)) && wait_in(s, timeout_ms) &&
        recvmsg(s, &m, MSG_CMSG_CLOEXEC) == 1) {
        if (st == kNoKey) {
            rc = 1;
        } else if (st == kOk) {
            cmsghdr *h = CMSG_FIRSTHDR(&m);
            if (h && h->cmsg_level == SOL_SOCKET && h->cmsg_type == SCM_RIGHTS) {
                std::memcpy(fd, CMSG_DATA(h), sizeof(int));
                rc = 0;
            }
        }
    }
    close(s);
    return rc;
}

}  // namespace ctrl
}  // namespace mpcomm
