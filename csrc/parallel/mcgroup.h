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

}  // namespace vmm
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_PARALLEL_MCGROUP_H_
