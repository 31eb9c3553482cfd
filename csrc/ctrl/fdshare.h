// File-descriptor hand-off between processes of one host: a process offers,
// under a 64-bit key, a provider that exports descriptors on request (e.g.
// the POSIX handles of the VMM allocations behind a registered range);
// another process of the same user fetches them by key over the owner's
// abstract Unix socket (SOCK_SEQPACKET; SCM_RIGHTS passes the descriptors
// themselves, so no path or ptrace permission is involved). Descriptors
// are created per request and closed once sent, so an offer holds none.
// The server thread starts with the first offer and ends with the process.
#ifndef MPCOMM_B200_CSRC_CTRL_FDSHARE_H_
#define MPCOMM_B200_CSRC_CTRL_FDSHARE_H_

#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace mpcomm {
namespace ctrl {

// One descriptor with the byte range it stands for in the offered object.
struct FdSegment {
    uint64_t offset = 0;
    uint64_t size = 0;
    int fd = -1;
};
// Fills the segments (new descriptors, in offset order); false on failure.
using FdProvider = std::function<bool(std::vector<FdSegment> *)>;

constexpr size_t kFdMaxSegments = 4096;

// Abstract socket name of process `pid`'s server on this host (boot-unique).
std::string fd_service_name(long pid);

// Offers `provider` under `key` on this process's server, whose abstract
// socket name is `name` (the same for every offer of the process). 0, or -1
// when the server cannot listen.
int fd_offer(const std::string &name, uint64_t key, FdProvider provider);
// Withdraws `key`.
void fd_withdraw(uint64_t key);
// Fetches the segments offered under `key` by the server `name`: 0 and new
// descriptors in *out (the caller closes them), 1 if the server has no such
// key or its provider failed, -1 if it could not be reached or answered
// within `timeout_ms`.
int fd_fetch(const std::string &name, uint64_t key, int timeout_ms, std::vector<FdSegment> *out);

}  // namespace ctrl
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_CTRL_FDSHARE_H_
