// Multi-threaded stress of the transfer engine on the loopback fabric, built
// twice: plain and with -fsanitize=thread (target test_engine_tsan), so data
// races in the engine, the handle/completion protocol, the staging pool and
// the control plane show up as ThreadSanitizer reports.
//
// Four caller threads submit PUT/GET/scatter/broadcast transfers (registered
// and unregistered = staged) against one target, while another thread
// publishes/queries buffers and toggles the throttle; every byte is checked.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

#include "mpcomm.h"

#define CHECK(c)                                                                  \
    do {                                                                          \
        if (!(c)) {                                                               \
            std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #c); \
            std::exit(1);                                                         \
        }                                                                         \
    } while (0)

int main() {
    setenv("MPCOMM_FABRIC", "lo", 1);
    setenv("MPCOMM_LOG_LEVEL", "1", 0);
    setenv("MPCOMM_MAX_RDMA_TRANSFER_SIZE", "65536", 1);
    setenv("MPCOMM_STAGING_SLAB_BYTES", "131072", 1);
    const size_t per = 1 << 20;
    const int threads = 4;
    const char *rs = std::getenv("MPCOMM_STRESS_ROUNDS");  // more interleavings under TSAN
    const int rounds = rs && std::atoi(rs) > 0 ? std::atoi(rs) : 12;
    mpcomm::MPComm a, b;
    CHECK(a.init("A") == 0 && b.init("B") == 0 && b.startAcceptThread() == 0);
    std::vector<unsigned char> target(per * threads, 0);
    CHECK(b.registerMemory(target.data(), target.size()) == 0);
    CHECK(b.publishBuffer(target.data(), target.size()) == 0);
    CHECK(a.connect("B", "127.0.0.1", b.getTcpPort()) == 0);
    mpcomm::RemoteBufferInfo info;
    CHECK(a.queryRemoteBuffer("B", "127.0.0.1", b.getTcpPort(), info) == 0);
    const uintptr_t raddr = info.buffers[0].addr;

    std::atomic<bool> stop{false};
    std::thread meddler([&] {
        std::vector<unsigned char> extra(4096);
        CHECK(b.registerMemory(extra.data(), extra.size()) == 0);
        int i = 0;
        while (!stop.load()) {
            b.publishBuffer(extra.data(), extra.size(), i & 3);
            mpcomm::RemoteBufferInfo tmp;
            a.queryRemoteBuffer("B", "127.0.0.1", b.getTcpPort(), tmp);
            if (i % 5 == 0) a.setNicThrottle(2, 32768);
            if (i % 5 == 2) a.clearNicThrottle();
            b.unpublishBuffer(extra.data());
            ++i;
            std::this_thread::sleep_for(std::chrono::milliseconds(2));
        }
    });
    std::vector<std::thread> ts;
    std::atomic<int> failures{0};
    for (int t = 0; t < threads; ++t) {
        ts.emplace_back([&, t] {
            std::mt19937 rng(t);
            std::vector<unsigned char> src(per), back(per);
            const bool staged = t % 2 == 1;  // odd threads use unregistered memory
            if (!staged) {
                CHECK(a.registerMemory(src.data(), per) == 0);
                CHECK(a.registerMemory(back.data(), per) == 0);
            }
            const uintptr_t r = raddr + static_cast<uintptr_t>(t) * per;
            for (int k = 0; k < rounds; ++k) {
                for (auto &x : src) x = static_cast<unsigned char>(rng());
                // k % 3: 0 PUT, 1 broadcast of the first half to both halves
                // (a fused one-to-many WRITE on loopback rails), 2 scatter.
                const bool bcast = k % 3 == 1;
                auto h = (k % 3 == 2) ? a.scatterAsync(reinterpret_cast<uintptr_t>(src.data()), {"B", "B"},
                                                       {r, r + per / 2}, {per / 2, per / 2})
                         : bcast      ? a.broadcastAsync(reinterpret_cast<uintptr_t>(src.data()), per / 2, {"B", "B"},
                                                         {r, r + per / 2})
                                      : a.putAsync(reinterpret_cast<uintptr_t>(src.data()), "B", r, per);
                if (h == mpcomm::INVALID_TRANSFER_HANDLE || a.waitTransfer(h, 30000) != 0) ++failures;
                auto res = a.getTransferResult(h);
                if (res.bytes_transferred != per) ++failures;
                a.releaseTransfer(h);
                h = a.getAsync(reinterpret_cast<uintptr_t>(back.data()), "B", r, per);
                // poll instead of wait on some rounds: exercises isTransferComplete
                if (k % 2) {
                    while (!a.isTransferComplete(h)) std::this_thread::yield();
                } else if (a.waitTransfer(h, 30000) != 0) {
                    ++failures;
                }
                a.releaseTransfer(h);
                if (bcast) {
                    if (std::memcmp(src.data(), back.data(), per / 2) != 0 ||
                        std::memcmp(src.data(), back.data() + per / 2, per / 2) != 0)
                        ++failures;
                } else if (std::memcmp(src.data(), back.data(), per) != 0) {
                    ++failures;
                }
            }
        });
    }
    for (auto &t : ts) t.join();
    stop = true;
    meddler.join();
    a.shutdown();
    b.shutdown();
    CHECK(failures.load() == 0);
    std::printf("engine stress passed (%d threads x %d rounds)\n", threads, rounds);
    return 0;
}
