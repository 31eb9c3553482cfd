// Native unit tests of the engine's building blocks (no GPU, no network).
// Run by tests/test_native.py; exits non-zero on the first failure.
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <set>
#include <algorithm>
#include <atomic>
#include <mutex>
#include <thread>
#include <vector>

#include <sys/mman.h>
#include <sys/resource.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include "core/core.h"
#include "ctrl/fdshare.h"
#include "ctrl/wire.h"
#include "parallel/mcgroup.h"
#include "topo/topology.h"

using namespace mpcomm;

static std::atomic<int> g_checks{0};  // CHECKs also run on member threads
#define CHECK(cond)                                                                    \
    do {                                                                               \
        ++g_checks;                                                                    \
        if (!(cond)) {                                                                 \
            std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #cond); \
            std::exit(1);                                                              \
        }                                                                              \
    } while (0)

static void test_wrid() {
    const uint64_t id = WrId::encode(3, 7, 0xBEEF, 0x12345678);
    CHECK(id == 0x0307BEEF12345678ull);
    CHECK(WrId::rail(id) == 3 && WrId::qp(id) == 7 && WrId::handle(id) == 0xBEEF &&
          WrId::chunk(id) == 0x12345678);
    // fields are masked, never bleed into neighbours
    const uint64_t m = WrId::encode(0x1FF, 0x1FF, 0x1FFFF, 0x1FFFFFFFFull);
    CHECK(WrId::rail(m) == 0xFF && WrId::qp(m) == 0xFF && WrId::handle(m) == 0xFFFF &&
          WrId::chunk(m) == 0xFFFFFFFF);
}

static void test_handle_pool() {
    HandlePool p;
    std::set<uint64_t> seen;
    for (int i = 0; i < 65535; ++i) {
        uint64_t h = p.allocate();
        CHECK(h >= 1 && h <= 65535);
        CHECK(seen.insert(h).second);
    }
    CHECK(p.allocate() == 0);  // exhausted -> INVALID_TRANSFER_HANDLE
    p.release(42);
    CHECK(p.allocate() == 42);  // recycled
    p.release(0);               // ignored
    CHECK(p.allocate() == 0);
}

static void test_mpsc_ring() {
    MpscRing r(1024);
    const int producers = 4, per = 20000;
    std::vector<std::thread> ts;
    for (int t = 0; t < producers; ++t)
        ts.emplace_back([&r, t] {
            for (int i = 0; i < per; ++i)
                while (!r.try_push(static_cast<uint64_t>(t) * per + i + 1)) cpu_relax();
        });
    std::vector<int> last(producers, -1);
    size_t got = 0;
    while (got < static_cast<size_t>(producers * per)) {
        uint64_t v;
        if (!r.try_pop(&v)) continue;
        ++got;
        int t = static_cast<int>((v - 1) / per), i = static_cast<int>((v - 1) % per);
        CHECK(i > last[t]);  // FIFO per producer
        last[t] = i;
    }
    for (auto &t : ts) t.join();
    uint64_t v;
    CHECK(!r.try_pop(&v));
}

static void test_chunk_plan() {
    ChunkPlan p;
    p.build(0x1000, {0x100000, 0x200000, 0x300000}, {300, 0, 250}, 128, false);
    CHECK(p.total() == 3 + 0 + 2);
    Chunk c = p.get(0);
    CHECK(c.host_idx == 0 && c.local_addr == 0x1000 && c.remote_addr == 0x100000 && c.length == 128);
    c = p.get(2);
    CHECK(c.host_idx == 0 && c.length == 300 - 256 && c.remote_addr == 0x100000 + 256);
    c = p.get(3);  // skips the empty host
    CHECK(c.host_idx == 2 && c.local_addr == 0x1000 + 300 && c.remote_addr == 0x300000 && c.length == 128);
    c = p.get(4);
    CHECK(c.length == 250 - 128);
    // broadcast: every host reads from local offset 0
    ChunkPlan b;
    b.build(0x5000, {0x10, 0x20}, {100, 100}, 64, true);
    CHECK(b.total() == 4);
    CHECK(b.get(2).local_addr == 0x5000 && b.get(2).host_idx == 1 && b.get(3).local_addr == 0x5000 + 64);
}

static void test_token_bucket() {
    TokenBucket tb;
    tb.configure(0, 0);
    CHECK(!tb.consume(1));  // rate 0 pauses
    tb.configure(1000000000ull, 1 << 20);  // 1 GB/s
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
    CHECK(tb.consume(1 << 20));    // ~2 MB accrued, capped at the 1 MiB burst
    CHECK(!tb.consume(1 << 20));   // drained
    CHECK(default_qos_burst(0) == 0);
    CHECK(default_qos_burst(1000) == 4096);
    CHECK(default_qos_burst(1ull << 40) == 65536);
    CHECK(default_qos_burst(200000000) == 20000);
}

static void test_topology_parsers() {
    auto v = topo::parse_cpulist("0-3,8,10-11");
    CHECK(v.size() == 7 && v[0] == 0 && v[3] == 3 && v[4] == 8 && v[6] == 11);
    CHECK(topo::parse_cpulist("").empty());
    CHECK(topo::name_suffix("mlx5_3") == 3 && topo::name_suffix("mlx5_bond_12") == 12 &&
          topo::name_suffix("eth") == -1 && topo::name_suffix("nvl_0") == 0);
    CHECK(topo::common_path_components("/sys/devices/pci0000:10/0000:10:01.0/0000:11:00.0",
                                       "/sys/devices/pci0000:10/0000:10:01.0/0000:12:00.0") == 4);
    auto aff = topo::best_affinity("/sys/devices/pci0000:10/0000:10:01.0/0000:11:00.0",
                                   {"/sys/devices/pci0000:20/0000:20:01.0/0000:21:00.0",
                                    "/sys/devices/pci0000:10/0000:10:01.0/0000:13:00.0",
                                    "/sys/devices/pci0000:10/0000:10:02.0/0000:14:00.0"});
    CHECK(aff.size() == 1 && aff[0] == 1);
    // sharing only the root complex is not affinity
    CHECK(topo::best_affinity("/sys/devices/pci0000:10/a", {"/sys/devices/pci0000:10/b"}).empty());
}

static void test_wire_layout() {
    RemoteEndpointInfo e;
    std::memset(&e, 0, sizeof(e));
    std::strcpy(e.gid, "fe:80");
    e.lid = 0x1234;
    e.qp_num = 0xA1B2C3D4;
    e.rkey = 0x55;
    e.addr = 7;
    e.length = 9;
    const unsigned char *b = reinterpret_cast<const unsigned char *>(&e);
    CHECK(sizeof(e) == 96);
    CHECK(b[64] == 0x34 && b[65] == 0x12);                 // lid, host-endian (LE)
    CHECK(b[68] == 0xD4 && b[71] == 0xA1);                 // qp_num
    CHECK(b[72] == 0x55 && b[80] == 7 && b[88] == 9);
    CHECK(kMsgTypeBufferQuery == 0x4D504251 && kMsgTypeQosControlOpen == 0x4D505143 &&
          kQosControlFrameMagic == 0x4D505146);
}

// Descriptor hand-off (VMM handles between processes): an offer exports its
// segments per request and they arrive, in order and with their offsets, as
// new descriptors of the same files, 64 per message; unknown and withdrawn
// keys and a failing export answer 1, a missing server -1. 300 segments go
// through under a descriptor limit far below 2 x 300, since each side holds
// at most one message's worth open.
static void test_fd_share() {
    const std::string name = "mpcomm-test-fd." + std::to_string(getpid());
    int f = memfd_create("fdshare", 0);
    CHECK(f >= 0 && ftruncate(f, 4096) == 0);
    CHECK(pwrite(f, "B200", 4, 0) == 4);
    const size_t nseg = 300;
    std::atomic<int> exports{0};
    ctrl::FdOffer o;
    for (size_t i = 0; i < nseg; ++i) o.segments.push_back(ctrl::FdSegment{i * 4096, 4096, -1});
    o.export_fd = [f, &exports](size_t) {
        ++exports;
        return dup(f);
    };
    CHECK(ctrl::fd_offer(name, 7, o) == 0);
    ctrl::FdOffer bad = o;
    bad.export_fd = [f](size_t i) { return i < 100 ? dup(f) : -1; };  // fails in the second message
    CHECK(ctrl::fd_offer(name, 9, bad) == 0);
    rlimit old{};
    CHECK(getrlimit(RLIMIT_NOFILE, &old) == 0);
    rlimit low = old;
    low.rlim_cur = std::min<rlim_t>(old.rlim_cur, 256);
    CHECK(setrlimit(RLIMIT_NOFILE, &low) == 0);
    size_t count = 0, seen = 0;
    uint64_t bytes = 0;
    bool ordered = true, same_file = true;
    const int rc = ctrl::fd_fetch(
        name, 7, 5000, [&](size_t c, uint64_t b) { count = c; bytes = b; return true; },
        [&](const ctrl::FdSegment &g) {
            char buf[4] = {0};
            ordered &= g.offset == seen * 4096 && g.size == 4096 && g.fd != f;
            same_file &= pread(g.fd, buf, 4, 0) == 4 && std::memcmp(buf, "B200", 4) == 0;
            ++seen;
            return true;
        });
    CHECK(setrlimit(RLIMIT_NOFILE, &old) == 0);
    CHECK(rc == 0 && count == nseg && bytes == nseg * 4096 && seen == nseg && ordered && same_file);
    CHECK(exports.load() == static_cast<int>(nseg));
    auto none = [](size_t, uint64_t) { return true; };
    auto any = [](const ctrl::FdSegment &) { return true; };
    CHECK(ctrl::fd_fetch(name, 8, 2000, none, any) == 1);
    CHECK(ctrl::fd_fetch(name, 9, 2000, none, any) == 1);
    // A receiver that stops early ends the fetch with -1 and leaks nothing.
    size_t taken = 0;
    CHECK(ctrl::fd_fetch(name, 7, 2000, none, [&](const ctrl::FdSegment &) { return ++taken < 10; }) == -1);
    CHECK(taken == 10);
    ctrl::fd_withdraw(7);
    CHECK(ctrl::fd_fetch(name, 7, 2000, none, any) == 1);
    CHECK(ctrl::fd_fetch(name + ".absent", 7, 200, none, any) == -1);
    // A server that accepts and never answers: the fetch gives up at its timeout.
    {
        const std::string mute = name + ".mute";
        int l = socket(AF_UNIX, SOCK_SEQPACKET, 0);
        sockaddr_un a{};
        a.sun_family = AF_UNIX;
        std::memcpy(a.sun_path + 1, mute.data(), mute.size());
        const socklen_t alen = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + mute.size());
        CHECK(l >= 0 && bind(l, reinterpret_cast<sockaddr *>(&a), alen) == 0 && listen(l, 4) == 0);
        const auto t0 = std::chrono::steady_clock::now();
        CHECK(ctrl::fd_fetch(mute, 7, 300, none, any) == -1);
        const auto dt = std::chrono::steady_clock::now() - t0;
        CHECK(dt >= std::chrono::milliseconds(250) && dt < std::chrono::seconds(3));
        close(l);
    }
    close(f);
    // Multicast group names map to one non-zero identity in every process.
    CHECK(vmm::mc_group_token("grp") == vmm::mc_group_token("grp"));
    CHECK(vmm::mc_group_token("grp") != vmm::mc_group_token("grp2") && vmm::mc_group_token("") != 0);
}

// NVLS group formation without a GPU: fake driver steps record what each
// member did, so the hand-off (the creator's object arrives over the socket),
// the lock step (every device added before any bind, every bind before any
// map) and failure propagation (a member that fails, or never comes, ends
// every call with an error within the timeout) are checked on the host.
namespace fake_mc {
std::mutex mu;
std::vector<std::string> log;
int members = 0, fail_dev = -1;
std::string fail_step;
std::atomic<int> teardowns{0};
int step(const char *what, int dev) {
    std::lock_guard<std::mutex> g(mu);
    log.push_back(std::string(what) + std::to_string(dev));
    return (fail_dev == dev && fail_step == what) ? 999 : 0;
}
int count(const char *what) {
    int n = 0;
    for (auto &e : log) n += e.rfind(what, 0) == 0;
    return n;
}
int gran(size_t, int, size_t *g) { *g = 4096; return 0; }
int create(size_t, int, uint64_t *mc, int *fd) {
    *fd = memfd_create("mcg", 0);
    if (*fd < 0 || pwrite(*fd, "MCOBJ", 5, 0) != 5) return 1;
    *mc = 0xC0FFEE;
    return 0;
}
int import(int fd, uint64_t *mc) {
    char b[5] = {0};
    if (pread(fd, b, 5, 0) != 5 || std::memcmp(b, "MCOBJ", 5) != 0) return 2;  // not the creator's object
    *mc = 0xC0FFEE;
    return 0;
}
int add(uint64_t, int dev) { return step("add", dev); }
int bind(uint64_t, size_t, int dev, uint64_t *mem, void **uc) {
    std::lock_guard<std::mutex> g(mu);  // the lock step: all adds happen before any bind
    if (count("add") != members) log.push_back("EARLY-BIND");
    log.push_back("bind" + std::to_string(dev));
    *mem = 1;
    *uc = reinterpret_cast<void *>(0x1000);
    return (fail_dev == dev && fail_step == "bind") ? 999 : 0;
}
int map(uint64_t, size_t, int dev, void **va) {
    std::lock_guard<std::mutex> g(mu);
    if (count("bind") != members) log.push_back("EARLY-MAP");
    log.push_back("map" + std::to_string(dev));
    *va = reinterpret_cast<void *>(0x2000);
    return 0;
}
int teardown(uint64_t, uint64_t, void *, void *, size_t, int) { ++teardowns; return 0; }
const vmm::McOps ops{gran, create, import, add, bind, map, teardown};

// Runs a group of `n` members (dev 0 creates); `absent` members never come.
std::vector<int> run(const std::string &name, int n, int absent, int timeout_ms) {
    log.clear();
    teardowns = 0;
    members = n;
    std::vector<int> rc(n - absent, 123);
    std::vector<std::thread> ts;
    for (int d = 0; d < n - absent; ++d)
        ts.emplace_back([&, d] {
            vmm::McGroup g;
            rc[d] = d == 0 ? vmm::mc_group_create_with(ops, d, name, 10000, n, timeout_ms, &g)
                           : vmm::mc_group_join_with(ops, d, name, 10000, n, timeout_ms, &g);
            if (rc[d] == 0) CHECK(g.size == 12288 && g.mc == 0xC0FFEE && g.uc && g.mcva && g.members == n);
        });
    for (auto &t : ts) t.join();
    return rc;
}
}  // namespace fake_mc

static void test_mc_group_protocol() {
    const std::string base = "mpcomm-test-mcg." + std::to_string(getpid());
    auto rc = fake_mc::run(base + ".ok", 4, 0, 5000);
    for (int r : rc) CHECK(r == 0);
    CHECK(fake_mc::count("add") == 4 && fake_mc::count("bind") == 4 && fake_mc::count("map") == 4);
    CHECK(fake_mc::count("EARLY") == 0 && fake_mc::teardowns == 0);
    // A member whose bind fails: every call fails, each member tears down.
    fake_mc::fail_dev = 2;
    fake_mc::fail_step = "bind";
    auto t0 = std::chrono::steady_clock::now();
    rc = fake_mc::run(base + ".bindfail", 4, 0, 3000);
    for (int r : rc) CHECK(r != 0);
    CHECK(fake_mc::teardowns == 4 && fake_mc::count("map") == 0);
    CHECK(std::chrono::steady_clock::now() - t0 < std::chrono::seconds(3));
    fake_mc::fail_dev = -1;
    // A member that never comes: the creator gives up at its timeout and
    // releases the members that did come.
    t0 = std::chrono::steady_clock::now();
    rc = fake_mc::run(base + ".absent", 3, 1, 400);
    for (int r : rc) CHECK(r == -1);
    CHECK(fake_mc::count("bind") == 0 && fake_mc::teardowns == 2);
    CHECK(std::chrono::steady_clock::now() - t0 < std::chrono::seconds(3));
    // A creator that accepts and then stalls: the joiner gives up at its timeout.
    {
        const std::string name = base + ".stall";
        const std::string path = "mpcomm-mcg-" + std::to_string(vmm::mc_group_token(name));
        int l = socket(AF_UNIX, SOCK_STREAM, 0);
        sockaddr_un a{};
        a.sun_family = AF_UNIX;
        std::memcpy(a.sun_path + 1, path.data(), path.size());
        const socklen_t alen = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + path.size());
        CHECK(l >= 0 && bind(l, reinterpret_cast<sockaddr *>(&a), alen) == 0 && listen(l, 4) == 0);
        vmm::McGroup g;
        t0 = std::chrono::steady_clock::now();
        CHECK(vmm::mc_group_join_with(fake_mc::ops, 1, name, 4096, 2, 300, &g) == -1);
        const auto dt = std::chrono::steady_clock::now() - t0;
        CHECK(dt >= std::chrono::milliseconds(250) && dt < std::chrono::seconds(3) && g.mc == 0);
        close(l);
    }
}

int main() {
    test_wrid();
    test_handle_pool();
    test_mpsc_ring();
    test_chunk_plan();
    test_token_bucket();
    test_topology_parsers();
    test_wire_layout();
    test_fd_share();
    test_mc_group_protocol();
    std::printf("native core tests passed (%d checks)\n", g_checks.load());
    return 0;
}
