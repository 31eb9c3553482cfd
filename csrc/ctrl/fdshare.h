// File-descriptor hand-off between processes of one host: a process offers,
// under a 64-bit key, an object made of segments (e.g. the VMM allocations
// behind a registered range) and a function that exports one segment as a
// new descriptor; another process of the same user fetches them by key over
// the owner's abstract Unix socket (SOCK_SEQPACKET; SCM_RIGHTS passes the
// descriptors themselves, so no path or ptrace permission is involved).
// Descriptors are exported per request and travel 64 at a time: each side
// holds at most one message's worth open, whatever the segment count, so a
// range of thousands of allocations stays within a default descriptor limit.
// The server thread starts with the first offer and ends with the process.
#ifndef MPCOMM_B200_CSRC_CTRL_FDSHARE_H_
#define MPCOMM_B200_CSRC_CTRL_FDSHARE_H_

#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace mpcomm {
namespace ctrl {

// One segment with the byte range it stands for in the offered object.
struct FdSegment {
    uint64_t offset = 0;
    uint64_t size = 0;
    int fd = -1;
};

struct FdOffer {
    std::vector<FdSegment> segments;         // offsets and sizes (fd unused), in offset order
    std::function<int(size_t)> export_fd;    // a new descriptor of segment i, or -1
};

constexpr size_t kFdMaxSegments = 65536;

// Abstract socket name of process `pid`'s server on this host (boot-unique).
std::string fd_service_name(long pid);

// Offers `offer` under `key` on this process's server, whose abstract
// socket name is `name` (the same for every offer of the process). 0, or -1
// when the server cannot listen.
int fd_offer(const std::string &name, uint64_t key, FdOffer offer);
// Withdraws `key`.
void fd_withdraw(uint64_t key);
// Fetches the object offered under `key` by the server `name`: on_begin
// (segment count, total bytes) once, then on_segment for every segment in
// order; its descriptor is closed when on_segment returns (a callback that
// keeps it must dup it). Either callback returning false ends the fetch.
// 0 when every segment was delivered and accepted, 1 if the server has no
// such key or could not export it, -1 if it could not be reached or
// answered within `timeout_ms` (or a callback refused).
int fd_fetch(const std::string &name, uint64_t key, int timeout_ms,
             const std::function<bool(size_t count, uint64_t bytes)> &on_begin,
             const std::function<bool(const FdSegment &)> &on_segment);

}  // namespace ctrl
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_CTRL_FDSHARE_H_
