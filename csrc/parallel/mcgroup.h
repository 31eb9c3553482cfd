// NVLS multicast groups formed between processes on one box, without any
// launcher or collective library: the first member creates the multicast
// object and hands it to the others over an abstract Unix socket named after
// the group; all members then add their GPU, bind one allocation of their
// own and map the multicast address, in lock step (the driver wants every
// device added before any binds). Each step waits at most `timeout_ms`.
#ifndef MPCOMM_B200_CSRC_PARALLEL_MCGROUP_H_
#define MPCOMM_B200_CSRC_PARALLEL_MCGROUP_H_

#include <cstddef>
#include <cstdint>
#include <string>

namespace mpcomm {
namespace vmm {

struct McGroup {
    uint64_t mc = 0;       // multicast object handle
    uint64_t mem = 0;      // this member's bound physical allocation
    void *uc = nullptr;    // this member's copy (unicast mapping)
    void *mcva = nullptr;  // multicast mapping (target of multimem stores)
    size_t size = 0;       // bytes of each copy (rounded to the multicast granularity)
    int dev = -1;
    uint64_t token = 0;    // group identity shared by every member (from the name)
    int members = 0;
};

// Group identity of `name` (non-zero).
uint64_t mc_group_token(const std::string &name);
// First member (on the current device). Returns 0 once every member has
// bound its copy, else a CUresult or -1 (timeout / protocol error).
int mc_group_create(const std::string &name, size_t bytes, int members, int timeout_ms, McGroup *out);
// Any other member (on the current device), in any order with the creator.
int mc_group_join(const std::string &name, size_t bytes, int members, int timeout_ms, McGroup *out);
// Unmaps, unbinds and releases this member's part of the group.
int mc_group_release(McGroup *g);

// The driver steps a member takes, replaceable so that the hand-off and
// lock-step protocol runs (and fails) in tests without a GPU. Each returns
// 0 or an error code, like the vmm functions they default to.
struct McOps {
    int (*granularity)(size_t size, int ndev, size_t *gran);
    int (*create)(size_t size, int ndev, uint64_t *mc, int *fd);
    int (*import)(int fd, uint64_t *mc);
    int (*add_device)(uint64_t mc, int dev);
    int (*bind)(uint64_t mc, size_t size, int dev, uint64_t *mem, void **uc);
    int (*map)(uint64_t mc, size_t size, int dev, void **mcva);
    int (*teardown)(uint64_t mc, uint64_t mem, void *uc, void *mcva, size_t size, int dev);
};
const McOps &mc_driver_ops();
int mc_group_create_with(const McOps &ops, int dev, const std::string &name, size_t bytes, int members,
                         int timeout_ms, McGroup *out);
int mc_group_join_with(const McOps &ops, int dev, const std::string &name, size_t bytes, int members,
                       int timeout_ms, McGroup *out);

}  // namespace vmm
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_PARALLEL_MCGROUP_H_
