// Minimal MPComm round trip from C++ (parity: reference
// user_examples/minimal/hello_mpcomm.cpp:49-118): init -> register ->
// publish/query -> put -> get -> memcmp -> shutdown.
//
// One process plays both roles over the TCP control plane. Fabric:
// MPCOMM_FABRIC (default here: "lo", the in-process loopback, so it runs on
// any host; use "nvl" on a GPU box, "ib" with RDMA NICs).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#include "mpcomm.h"

int main() {
    setenv("MPCOMM_FABRIC", "lo", 0);
    const size_t n = 8 << 20;
    std::vector<unsigned char> src(n), remote(n, 0), back(n, 0);
    std::mt19937 rng(0);
    for (auto &b : src) b = static_cast<unsigned char>(rng());

    mpcomm::MPComm target, initiator;
    if (target.init("target") || initiator.init("initiator")) return std::fprintf(stderr, "init failed\n"), 1;
    target.registerMemory(remote.data(), n);
    target.publishBuffer(remote.data(), n);
    target.startAcceptThread();
    initiator.registerMemory(src.data(), n);
    initiator.registerMemory(back.data(), n);
    if (initiator.connect("target", "127.0.0.1", target.getTcpPort()))
        return std::fprintf(stderr, "connect failed\n"), 1;
    mpcomm::RemoteBufferEntry buf;
    if (initiator.queryRemoteBufferByNuma("target", "127.0.0.1", target.getTcpPort(), -1, buf))
        return std::fprintf(stderr, "query failed\n"), 1;

    auto h = initiator.putAsync(reinterpret_cast<uintptr_t>(src.data()), "target", buf.addr, n);
    int rc = initiator.waitTransfer(h, 10000);
    auto r = initiator.getTransferResult(h);
    initiator.releaseTransfer(h);
    std::printf("put: rc=%d bytes=%zu %.3f ms\n", rc, r.bytes_transferred, r.elapsed_ms);
    h = initiator.getAsync(reinterpret_cast<uintptr_t>(back.data()), "target", buf.addr, n);
    rc |= initiator.waitTransfer(h, 10000);
    initiator.releaseTransfer(h);
    const bool ok = rc == 0 && std::memcmp(src.data(), back.data(), n) == 0 &&
                    std::memcmp(src.data(), remote.data(), n) == 0;
    std::printf("round trip %s (fabric %s, %zu rails)\n", ok ? "OK" : "FAILED",
                initiator.getFabricName().c_str(), initiator.getNumNics());
    initiator.shutdown();
    target.shutdown();
    return ok ? 0 : 1;
}
