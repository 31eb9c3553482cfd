// NVTX annotations through the header-only NVTX v3 API of the CUDA toolkit.
// Without a profiler that injects itself (Nsight Systems and the like) each
// call is a no-op behind one function pointer; MPCOMM_NVTX=0 skips them.
#ifndef MPCOMM_B200_CSRC_CORE_NVTX_H_
#define MPCOMM_B200_CSRC_CORE_NVTX_H_

#include <nvtx3/nvToolsExt.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>

namespace mpcomm {
namespace nvtx {

inline bool enabled() {
    static const bool on = [] {
        const char *e = std::getenv("MPCOMM_NVTX");
        return !(e && std::strcmp(e, "0") == 0);
    }();
    return on;
}

// Scoped range on the calling thread (push/pop).
class Range {
 public:
    explicit Range(const char *name) : on_(enabled()) {
        if (on_) nvtxRangePushA(name);
    }
    ~Range() {
        if (on_) nvtxRangePop();
    }
    Range(const Range &) = delete;
    Range &operator=(const Range &) = delete;

 private:
    bool on_;
};

// Process range that may end on another thread (a transfer's lifetime).
inline uint64_t start(const char *msg) { return enabled() ? nvtxRangeStartA(msg) : 0; }
inline void end(uint64_t id) {
    if (id) nvtxRangeEnd(id);
}

}  // namespace nvtx
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_CORE_NVTX_H_
