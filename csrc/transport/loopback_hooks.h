// Host-side fault hooks of the "lo" backend (tests and fault drills).
// Rails are addressed by gid (MPComm::getGid(i)).
#ifndef MPCOMM_B200_CSRC_TRANSPORT_LOOPBACK_HOOKS_H_
#define MPCOMM_B200_CSRC_TRANSPORT_LOOPBACK_HOOKS_H_

#include <cstdint>
#include <string>

namespace mpcomm {
namespace fabric {

// The next `count` WRs executed by the rail complete with kWcRemAccessErr.
int loopback_inject_wc_errors(const std::string &gid, int count);
// A down port completes every WR with kWcRetryExcErr and reports
// port_active() == false (what quarantine probing checks).
int loopback_set_port_active(const std::string &gid, bool active);
// Adds a delay before each WR (keeps WRs outstanding for flow-control tests).
int loopback_set_wr_delay_us(const std::string &gid, uint64_t us);

}  // namespace fabric
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_TRANSPORT_LOOPBACK_HOOKS_H_
