// File-descriptor hand-off between processes of one host: a process offers
// descriptors it exported (e.g. a VMM allocation's POSIX handle) under
// 64-bit keys; another process of the same user fetches one by key over
// the owner's abstract Unix socket (SCM_RIGHTS passes the descriptor
// itself, so no path or ptrace permission is involved). The server thread
// starts with the first offer and ends with the process.
#ifndef MPCOMM_B200_CSRC_CTRL_FDSHARE_H_
#define MPCOMM_B200_CSRC_CTRL_FDSHARE_H_

#include <cstdint>
#include <string>

namespace mpcomm {
namespace ctrl {

// Offers `fd` (ownership passes here) under `key` on this process's server,
// whose abstract socket name is `name` (the same for every offer of the
// process). 0, or -1 when the server cannot listen (fd is then closed).
int fd_offer(const std::string &name, uint64_t key, int fd);
// Withdraws `key` and closes its descriptor.
void fd_withdraw(uint64_t key);
// Fetches the descriptor offered under `key` by the server `name`: 0 and a
// new descriptor in *fd (the caller closes it), 1 if the server has no such
// key, -1 if it could not be reached or refused within `timeout_ms`.
int fd_fetch(const std::string &name, uint64_t key, int timeout_ms, int *fd);

}  // namespace ctrl
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_CTRL_FDSHARE_H_
