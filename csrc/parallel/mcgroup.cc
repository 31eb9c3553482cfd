#include "parallel/mcgroup.h"

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "cuda/gpu.h"
#include "mpcomm_log.h"
#include "parallel/vmm.h"

namespace mpcomm {
namespace vmm {

namespace {

using Clock = std::chrono::steady_clock;

// Abstract-namespace address (leading NUL): no file, gone with the socket.
socklen_t group_addr(const std::string &name, sockaddr_un *a) {
    std::memset(a, 0, sizeof(*a));
    a->sun_family = AF_UNIX;
    const std::string path = "mpcomm-mcg-" + std::to_string(mc_group_token(name));
    const size_t n = std::min(path.size(), sizeof(a->sun_path) - 2);
    std::memcpy(a->sun_path + 1, path.data(), n);
    return static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + n);
}

int ms_left(Clock::time_point deadline) {
    const auto d = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - Clock::now()).count();
    return d > 0 ? static_cast<int>(d) : 0;
}

bool wait_fd(int fd, short ev, Clock::time_point deadline) {
    pollfd p{fd, ev, 0};
    for (;;) {
        const int r = poll(&p, 1, ms_left(deadline));
        if (r > 0) return (p.revents & ev) != 0;
        if (r == 0 || errno != EINTR) return false;
    }
}

bool send_byte(int fd, char c) { return send(fd, &c, 1, MSG_NOSIGNAL) == 1; }

bool recv_byte(int fd, char *c, Clock::time_point deadline) {
    return wait_fd(fd, POLLIN, deadline) && recv(fd, c, 1, 0) == 1;
}

// The multicast object's descriptor and the copy size, in one message.
bool send_handle(int fd, int handle_fd, uint64_t size) {
    msghdr m{};
    iovec io{&size, sizeof(size)};
    m.msg_iov = &io;
    m.msg_iovlen = 1;
    char ctl[CMSG_SPACE(sizeof(int))];
    std::memset(ctl, 0, sizeof(ctl));
    m.msg_control = ctl;
    m.msg_controllen = sizeof(ctl);
    cmsghdr *c = CMSG_FIRSTHDR(&m);
    c->cmsg_level = SOL_SOCKET;
    c->cmsg_type = SCM_RIGHTS;
    c->cmsg_len = CMSG_LEN(sizeof(int));
    std::memcpy(CMSG_DATA(c), &handle_fd, sizeof(int));
    return sendmsg(fd, &m, MSG_NOSIGNAL) == static_cast<ssize_t>(sizeof(size));
}

bool recv_handle(int fd, int *handle_fd, uint64_t *size, Clock::time_point deadline) {
    if (!wait_fd(fd, POLLIN, deadline)) return false;
    msghdr m{};
    iovec io{size, sizeof(*size)};
    m.msg_iov = &io;
    m.msg_iovlen = 1;
    char ctl[CMSG_SPACE(sizeof(int))];
    m.msg_control = ctl;
    m.msg_controllen = sizeof(ctl);
    if (recvmsg(fd, &m, MSG_CMSG_CLOEXEC) != static_cast<ssize_t>(sizeof(*size))) return false;
    cmsghdr *c = CMSG_FIRSTHDR(&m);
    if (!c || c->cmsg_level != SOL_SOCKET || c->cmsg_type != SCM_RIGHTS) return false;
    std::memcpy(handle_fd, CMSG_DATA(c), sizeof(int));
    return true;
}

}  // namespace

const McOps &mc_driver_ops() {
    static const McOps ops{multicast_granularity, multicast_create, multicast_import, multicast_add_device,
                           multicast_bind_local, multicast_map, multicast_teardown};
    return ops;
}

uint64_t mc_group_token(const std::string &name) {
    uint64_t h = 1469598103934665603ull;  // FNV-1a
    for (unsigned char ch : name) {
        h ^= ch;
        h *= 1099511628211ull;
    }
    return h | 1ull;
}

int mc_group_create(const std::string &name, size_t bytes, int members, int timeout_ms, McGroup *out) {
    return mc_group_create_with(mc_driver_ops(), gpu::current_device(), name, bytes, members, timeout_ms, out);
}

int mc_group_join(const std::string &name, size_t bytes, int members, int timeout_ms, McGroup *out) {
    return mc_group_join_with(mc_driver_ops(), gpu::current_device(), name, bytes, members, timeout_ms, out);
}

int mc_group_create_with(const McOps &ops, int dev, const std::string &name, size_t bytes, int members,
                         int timeout_ms, McGroup *out) {
    if (members < 2 || bytes == 0) return -1;
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    McGroup g;
    g.dev = dev;
    g.members = members;
    g.token = mc_group_token(name);
    size_t gran = 0;
    int e = ops.granularity(bytes, members, &gran);
    if (e) return e;
    if (gran == 0) gran = 2u << 20;
    g.size = (bytes + gran - 1) / gran * gran;
    int hfd = -1;
    e = ops.create(g.size, members, &g.mc, &hfd);
    if (e) return e;
    int lfd = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    sockaddr_un a;
    const socklen_t alen = group_addr(name, &a);
    std::vector<int> peers;
    auto fail = [&](int rc, const char *what) {
        MPCOMM_LOG_ERROR("MPComm: multicast group '%s' (creator): %s\n", name.c_str(), what);
        for (int p : peers) {
            send_byte(p, 'X');
            close(p);
        }
        if (lfd >= 0) close(lfd);
        if (hfd >= 0) close(hfd);
        ops.teardown(g.mc, g.mem, g.uc, g.mcva, g.size, g.dev);
        return rc;
    };
    if (lfd < 0 || bind(lfd, reinterpret_cast<sockaddr *>(&a), alen) != 0 || listen(lfd, members) != 0)
        return fail(-1, "cannot listen (is another group of this name open?)");
    if ((e = ops.add_device(g.mc, g.dev))) return fail(e, "cuMulticastAddDevice");
    // Hand the object to every other member; each adds its GPU.
    while (static_cast<int>(peers.size()) < members - 1) {
        if (!wait_fd(lfd, POLLIN, deadline)) return fail(-1, "timed out waiting for members");
        int p = accept4(lfd, nullptr, nullptr, SOCK_CLOEXEC);
        if (p < 0) continue;
        peers.push_back(p);
        if (!send_handle(p, hfd, g.size)) return fail(-1, "handle hand-off");
    }
    close(lfd);
    lfd = -1;
    close(hfd);
    hfd = -1;
    char c = 0;
    for (int p : peers)
        if (!recv_byte(p, &c, deadline) || c != 'A') return fail(-1, "a member could not add its GPU");
    // Every device is added: bind, then map.
    for (int p : peers)
        if (!send_byte(p, 'B')) return fail(-1, "bind signal");
    if ((e = ops.bind(g.mc, g.size, g.dev, &g.mem, &g.uc))) return fail(e, "bind");
    for (int p : peers)
        if (!recv_byte(p, &c, deadline) || c != 'b') return fail(-1, "a member could not bind");
    for (int p : peers)
        if (!send_byte(p, 'M')) return fail(-1, "map signal");
    if ((e = ops.map(g.mc, g.size, g.dev, &g.mcva))) return fail(e, "map");
    for (int p : peers)
        if (!recv_byte(p, &c, deadline) || c != 'm') return fail(-1, "a member could not map");
    for (int p : peers) close(p);
    *out = g;
    return 0;
}

int mc_group_join_with(const McOps &ops, int dev, const std::string &name, size_t bytes, int members,
                       int timeout_ms, McGroup *out) {
    if (members < 2 || bytes == 0) return -1;
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    McGroup g;
    g.dev = dev;
    g.members = members;
    g.token = mc_group_token(name);
    sockaddr_un a;
    const socklen_t alen = group_addr(name, &a);
    int fd = -1;
    // The creator may not be listening yet.
    for (;;) {
        fd = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
        if (fd >= 0 && connect(fd, reinterpret_cast<sockaddr *>(&a), alen) == 0) break;
        if (fd >= 0) close(fd);
        fd = -1;
        if (ms_left(deadline) == 0) {
            MPCOMM_LOG_ERROR("MPComm: multicast group '%s': no creator\n", name.c_str());
            return -1;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(20));
    }
    auto fail = [&](int rc, const char *what) {
        MPCOMM_LOG_ERROR("MPComm: multicast group '%s' (member): %s\n", name.c_str(), what);
        send_byte(fd, 'E');
        close(fd);
        ops.teardown(g.mc, g.mem, g.uc, g.mcva, g.size, g.dev);
        return rc;
    };
    int hfd = -1;
    uint64_t size = 0;
    if (!recv_handle(fd, &hfd, &size, deadline)) return fail(-1, "no handle from the creator");
    g.size = size;
    int e = ops.import(hfd, &g.mc);
    close(hfd);
    if (e) return fail(e, "import");
    if (size < bytes) return fail(-1, "group smaller than requested");
    if ((e = ops.add_device(g.mc, g.dev))) return fail(e, "cuMulticastAddDevice");
    char c = 0;
    if (!send_byte(fd, 'A') || !recv_byte(fd, &c, deadline) || c != 'B') return fail(-1, "no bind signal");
    if ((e = ops.bind(g.mc, g.size, g.dev, &g.mem, &g.uc))) return fail(e, "bind");
    if (!send_byte(fd, 'b') || !recv_byte(fd, &c, deadline) || c != 'M') return fail(-1, "no map signal");
    if ((e = ops.map(g.mc, g.size, g.dev, &g.mcva))) return fail(e, "map");
    send_byte(fd, 'm');
    close(fd);
    *out = g;
    return 0;
}

int mc_group_release(McGroup *g) {
    if (!g || !g->mc) return 0;
    const int e = multicast_teardown(g->mc, g->mem, g->uc, g->mcva, g->size, g->dev);
    *g = McGroup{};
    return e;
}

}  // namespace vmm
}  // namespace mpcomm
