// Control-plane wire format.
//
// Byte-for-byte compatible with the reference so that peers interoperate
// (reference src/mpcomm.cpp:175-182, 215-248, 3479-3848, 3982-4896): all
// integers are host-endian, sent raw; the first u32 a client sends selects
// the session type:
//   0x4D504251 "MPBQ"  buffer query
//   0x4D505143 "MPQC"  QoS control channel
//   anything else      NIC count of a connect handshake (< 0x10000000)
// Connect handshake (A = active, P = passive):
//   A->P u32 num_nics; P->A u32 num_nics
//   A->P i32 numa_count, i32[n] nic_numa; P->A the same (P's)
//   A->P {u32 len, bytes}[n] nic names; P->A the same
//   A->P u32 qps; P->A u32 qps; both use min()
//   per (local rail, remote rail) pair x qp:
//     A->P RemoteEndpointInfo{gid, lid, qp_num, rkey=0, addr=remote_nic,
//                             length=local_nic}
//     P->A RemoteEndpointInfo (P's QP)
//     A->P u8 status (0 ok / 1 failed: both drop the pair)
// Buffer query: S->C u32 num_buffers (0 ends), u32 num_nics,
//   char gid[64] x num_nics, then per buffer: u64 addr, u64 length,
//   i32 numa_tag, i32 gpu_device_id, u32 aff_cnt (<=16), u32 aff[aff_cnt],
//   u32 rkey[num_nics].
#ifndef MPCOMM_B200_CSRC_CTRL_WIRE_H_
#define MPCOMM_B200_CSRC_CTRL_WIRE_H_

#include <cstddef>
#include <cstdint>
#include <string>

#include "core/core.h"

namespace mpcomm {

constexpr uint32_t kMsgTypeBufferQuery = 0x4D504251;
constexpr uint32_t kMsgTypeQosControlOpen = 0x4D505143;
constexpr uint32_t kQosControlFrameMagic = 0x4D505146;
constexpr uint32_t kQosControlVersion = 1;
// Values below this in the first u32 are a connect's NIC count.
constexpr uint32_t kMaxConnectNicCount = 0x10000000;

struct RemoteEndpointInfo {
    char gid[64];
    uint16_t lid;
    uint32_t qp_num;
    uint32_t rkey;
    uint64_t addr;
    uint64_t length;
};
static_assert(sizeof(RemoteEndpointInfo) == 96, "wire size of RemoteEndpointInfo");
static_assert(offsetof(RemoteEndpointInfo, lid) == 64, "lid offset");
static_assert(offsetof(RemoteEndpointInfo, qp_num) == 68, "qp_num offset");
static_assert(offsetof(RemoteEndpointInfo, rkey) == 72, "rkey offset");
static_assert(offsetof(RemoteEndpointInfo, addr) == 80, "addr offset");
static_assert(offsetof(RemoteEndpointInfo, length) == 88, "length offset");

enum class QosFrameType : uint32_t { kUpdate = 1, kClear = 2 };

struct QosControlHello {
    uint32_t version;
    char host_id[128];
};
static_assert(sizeof(QosControlHello) == 132, "wire size of QosControlHello");

struct QosControlFrame {
    uint32_t magic;
    uint32_t version;
    uint32_t type;
    int32_t target_gpu_device;
    uint32_t affinity_nic_count;
    uint32_t affinity_nic_indices[kMaxRails];
    uint64_t rate_bytes_per_sec;
    uint64_t burst_bytes;
    uint64_t generation;
};
static_assert(sizeof(QosControlFrame) == 112, "wire size of QosControlFrame");

namespace net {

// Full-length send/recv; false on error, EOF or timeout.
bool send_all(int fd, const void *buf, size_t len);
bool recv_all(int fd, void *buf, size_t len);
template <typename T>
bool send_pod(int fd, const T &v) {
    return send_all(fd, &v, sizeof(T));
}
template <typename T>
bool recv_pod(int fd, T *v) {
    return recv_all(fd, v, sizeof(T));
}
// Resolves addr (dotted quad or hostname), connects with TCP_NODELAY and
// send/recv timeouts of timeout_ms (0 = none). Returns fd or -1.
int connect_tcp(const std::string &addr, int port, int timeout_ms);
// Listens on 0.0.0.0:port (0 = ephemeral). Returns fd, *bound = port.
int listen_tcp(int port, int backlog, int *bound);
void set_timeouts(int fd, int timeout_ms);
// "ip:port" of the peer of a connected socket.
std::string peer_id(int fd, int *port);
// Control-plane socket timeout (MPCOMM_CTRL_TIMEOUT_MS, default 30000).
int ctrl_timeout_ms();

}  // namespace net
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_CTRL_WIRE_H_
