#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cerrno>
#include <cstdlib>
#include <cstring>

#include "ctrl/wire.h"
#include "mpcomm_log.h"

namespace mpcomm {
namespace net {

bool send_all(int fd, const void *buf, size_t len) {
    const char *p = static_cast<const char *>(buf);
    while (len > 0) {
        ssize_t r = ::send(fd, p, len, MSG_NOSIGNAL);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        p += r;
        len -= static_cast<size_t>(r);
    }
    return true;
}

bool recv_all(int fd, void *buf, size_t len) {
    char *p = static_cast<char *>(buf);
    while (len > 0) {
        ssize_t r = ::recv(fd, p, len, MSG_WAITALL);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        p += r;
        len -= static_cast<size_t>(r);
    }
    return true;
}

void set_timeouts(int fd, int timeout_ms) {
    if (timeout_ms <= 0) return;
    struct timeval tv;
    tv.tv_sec = timeout_ms / 1000;
    tv.tv_usec = (timeout_ms % 1000) * 1000;
    setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
    setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &tv, sizeof(tv));
}

int ctrl_timeout_ms() {
    static const int v = [] {
        const char *e = std::getenv("MPCOMM_CTRL_TIMEOUT_MS");
        int ms = e ? std::atoi(e) : 30000;
        return ms < 0 ? 30000 : ms;
    }();
    return v;
}

int connect_tcp(const std::string &addr, int port, int timeout_ms) {
    struct sockaddr_in sa;
    std::memset(&sa, 0, sizeof(sa));
    sa.sin_family = AF_INET;
    sa.sin_port = htons(static_cast<uint16_t>(port));
    if (inet_pton(AF_INET, addr.c_str(), &sa.sin_addr) <= 0) {
        struct addrinfo hints, *res = nullptr;
        std::memset(&hints, 0, sizeof(hints));
        hints.ai_family = AF_INET;
        hints.ai_socktype = SOCK_STREAM;
        if (getaddrinfo(addr.c_str(), nullptr, &hints, &res) != 0 || !res) {
            MPCOMM_LOG_ERROR("MPComm: cannot resolve %s\n", addr.c_str());
            return -1;
        }
        sa.sin_addr = reinterpret_cast<struct sockaddr_in *>(res->ai_addr)->sin_addr;
        freeaddrinfo(res);
    }
    int fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) return -1;
    set_timeouts(fd, timeout_ms);
    if (::connect(fd, reinterpret_cast<struct sockaddr *>(&sa), sizeof(sa)) < 0) {
        MPCOMM_PLOG_ERROR("MPComm: connect to %s:%d failed", addr.c_str(), port);
        ::close(fd);
        return -1;
    }
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    return fd;
}

int listen_tcp(int port, int backlog, int *bound) {
    int fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) return -1;
    int one = 1;
    setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    struct sockaddr_in sa;
    std::memset(&sa, 0, sizeof(sa));
    sa.sin_family = AF_INET;
    sa.sin_addr.s_addr = htonl(INADDR_ANY);
    sa.sin_port = htons(static_cast<uint16_t>(port));
    if (::bind(fd, reinterpret_cast<struct sockaddr *>(&sa), sizeof(sa)) < 0 ||
        ::listen(fd, backlog) < 0) {
        MPCOMM_PLOG_ERROR("MPComm: cannot listen on port %d", port);
        ::close(fd);
        return -1;
    }
    socklen_t len = sizeof(sa);
    getsockname(fd, reinterpret_cast<struct sockaddr *>(&sa), &len);
    *bound = ntohs(sa.sin_port);
    return fd;
}

std::string peer_id(int fd, int *port) {
    struct sockaddr_in sa;
    socklen_t len = sizeof(sa);
    std::memset(&sa, 0, sizeof(sa));
    getpeername(fd, reinterpret_cast<struct sockaddr *>(&sa), &len);
    char ip[INET_ADDRSTRLEN] = {0};
    inet_ntop(AF_INET, &sa.sin_addr, ip, sizeof(ip));
    if (port) *port = ntohs(sa.sin_port);
    return std::string(ip) + ":" + std::to_string(ntohs(sa.sin_port));
}

}  // namespace net
}  // namespace mpcomm
