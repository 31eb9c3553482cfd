#include "topo/topology.h"

#include <dirent.h>
#include <limits.h>
#include <pthread.h>
#include <sched.h>
#include <stdlib.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <thread>
#include <cstdint>
#include <cctype>
#include <cstring>
#include <fstream>
#include <sstream>

namespace mpcomm {
namespace topo {

namespace {

std::string read_line(const std::string &path) {
    std::ifstream f(path);
    std::string s;
    if (f) std::getline(f, s);
    while (!s.empty() && std::isspace(static_cast<unsigned char>(s.back()))) s.pop_back();
    return s;
}

int read_int(const std::string &path, int dflt) {
    std::string s = read_line(path);
    if (s.empty()) return dflt;
    char *end = nullptr;
    long v = std::strtol(s.c_str(), &end, 10);
    return (end && *end == '\0') ? static_cast<int>(v) : dflt;
}

std::string realpath_str(const std::string &p) {
    char buf[PATH_MAX];
    if (!::realpath(p.c_str(), buf)) return std::string();
    return std::string(buf);
}

std::vector<std::string> split_path(const std::string &p) {
    std::vector<std::string> out;
    std::string cur;
    for (char c : p) {
        if (c == '/') {
            if (!cur.empty()) out.push_back(cur);
            cur.clear();
        } else {
            cur.push_back(c);
        }
    }
    if (!cur.empty()) out.push_back(cur);
    return out;
}

}  // namespace

const std::string &sysfs_root() {
    static const std::string root = [] {
        const char *e = std::getenv("MPCOMM_SYSFS_ROOT");
        return std::string(e && *e ? e : "/sys");
    }();
    return root;
}

std::vector<int> parse_cpulist(const std::string &s) {
    std::vector<int> cpus;
    std::stringstream ss(s);
    std::string part;
    while (std::getline(ss, part, ',')) {
        if (part.empty()) continue;
        size_t dash = part.find('-');
        char *end = nullptr;
        if (dash == std::string::npos) {
            long v = std::strtol(part.c_str(), &end, 10);
            if (end && *end == '\0') cpus.push_back(static_cast<int>(v));
        } else {
            long a = std::strtol(part.substr(0, dash).c_str(), nullptr, 10);
            long b = std::strtol(part.substr(dash + 1).c_str(), nullptr, 10);
            for (long v = a; v <= b && v - a < 65536; ++v) cpus.push_back(static_cast<int>(v));
        }
    }
    return cpus;
}

int numa_node_count() {
    DIR *d = opendir((sysfs_root() + "/devices/system/node").c_str());
    if (!d) return 1;
    int n = 0;
    while (struct dirent *e = readdir(d)) {
        if (!std::strncmp(e->d_name, "node", 4) && std::isdigit(static_cast<unsigned char>(e->d_name[4])))
            ++n;
    }
    closedir(d);
    return n > 0 ? n : 1;
}

std::vector<int> numa_cpus(int node) {
    return parse_cpulist(read_line(sysfs_root() + "/devices/system/node/node" + std::to_string(node) +
                                   "/cpulist"));
}

int pci_numa_node(const std::string &bdf) {
    if (bdf.empty()) return -1;
    return read_int(sysfs_root() + "/bus/pci/devices/" + bdf + "/numa_node", -1);
}

std::string pci_realpath(const std::string &bdf) {
    if (bdf.empty()) return std::string();
    return realpath_str(sysfs_root() + "/bus/pci/devices/" + bdf);
}

int ib_numa_node(const std::string &nic) {
    return read_int(sysfs_root() + "/class/infiniband/" + nic + "/device/numa_node", -1);
}

std::string ib_realpath(const std::string &nic) {
    return realpath_str(sysfs_root() + "/class/infiniband/" + nic + "/device");
}

std::vector<std::string> ib_device_names() {
    std::vector<std::string> out;
    DIR *d = opendir((sysfs_root() + "/class/infiniband").c_str());
    if (!d) return out;
    while (struct dirent *e = readdir(d))
        if (e->d_name[0] != '.') out.emplace_back(e->d_name);
    closedir(d);
    std::sort(out.begin(), out.end());
    return out;
}

size_t common_path_components(const std::string &a, const std::string &b) {
    auto pa = split_path(a), pb = split_path(b);
    size_t n = 0;
    while (n < pa.size() && n < pb.size() && pa[n] == pb[n]) ++n;
    return n;
}

std::vector<size_t> best_affinity(const std::string &target, const std::vector<std::string> &paths) {
    std::vector<size_t> out;
    if (target.empty()) return out;
    size_t best = 0;
    std::vector<size_t> score(paths.size(), 0);
    for (size_t i = 0; i < paths.size(); ++i) {
        score[i] = paths[i].empty() ? 0 : common_path_components(target, paths[i]);
        best = std::max(best, score[i]);
    }
    // "/sys/devices/pci0000:xx" is 3 components: sharing only the root
    // complex is not affinity.
    if (best <= 3) return out;
    for (size_t i = 0; i < paths.size(); ++i)
        if (score[i] == best) out.push_back(i);
    return out;
}

int name_suffix(const std::string &name) {
    size_t i = name.size();
    while (i > 0 && std::isdigit(static_cast<unsigned char>(name[i - 1]))) --i;
    if (i == name.size()) return -1;
    return static_cast<int>(std::strtol(name.c_str() + i, nullptr, 10));
}

int numa_node_of_addr(const void *addr) {
    if (!addr) return -1;
    void *page = reinterpret_cast<void *>(reinterpret_cast<uintptr_t>(addr) &
                                          ~static_cast<uintptr_t>(sysconf(_SC_PAGESIZE) - 1));
    int status = -1;
    // move_pages(pid=0, count=1, pages, nodes=NULL, status, flags=0) only
    // reports the node of each page.
    long r = syscall(SYS_move_pages, 0, 1UL, &page, nullptr, &status, 0);
    if (r != 0 || status < 0) return -1;
    return status;
}

void *numa_alloc(size_t bytes, int node) {
    void *p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    if (p == MAP_FAILED) return nullptr;
    if (node >= 0 && node < 64) {
        unsigned long mask = 1UL << node;
        // MPOL_PREFERRED = 1: falls back to other nodes instead of failing.
        syscall(SYS_mbind, p, bytes, 1, &mask, 64UL, 0U);
    }
    // First touch places the pages under the policy.
    long pg = sysconf(_SC_PAGESIZE);
    for (size_t off = 0; off < bytes; off += static_cast<size_t>(pg)) static_cast<char *>(p)[off] = 0;
    return p;
}

void numa_free(void *p, size_t bytes) {
    if (p) munmap(p, bytes);
}

bool bind_thread_to_cpus(const std::vector<int> &cpus) {
    if (cpus.empty()) return false;
    cpu_set_t cur, want;
    CPU_ZERO(&want);
    if (sched_getaffinity(0, sizeof(cur), &cur) != 0) return false;
    int n = 0;
    for (int c : cpus) {
        if (c >= 0 && c < CPU_SETSIZE && CPU_ISSET(c, &cur)) {
            CPU_SET(c, &want);
            ++n;
        }
    }
    if (n == 0) return false;
    return pthread_setaffinity_np(pthread_self(), sizeof(want), &want) == 0;
}

namespace {

// Sums the words of [p, p + n) (n a multiple of 64); the result only keeps
// the loads from being dropped.
uint64_t sum_words(const uint64_t *p, size_t n) {
    uint64_t a = 0, b = 0, c = 0, d = 0;
    for (size_t i = 0; i < n; i += 4) {
        a += p[i];
        b += p[i + 1];
        c += p[i + 2];
        d += p[i + 3];
    }
    return a ^ b ^ c ^ d;
}

}  // namespace

bool host_bandwidth(size_t bytes, int threads, int node, int reps, HostBandwidth *out) {
    std::vector<int> cpus;
    cpu_set_t cur;
    if (sched_getaffinity(0, sizeof(cur), &cur) == 0)
        for (int c = 0; c < CPU_SETSIZE; ++c)
            if (CPU_ISSET(c, &cur)) cpus.push_back(c);
    if (threads <= 0) threads = cpus.empty() ? 1 : static_cast<int>(cpus.size());
    bytes &= ~static_cast<size_t>(4095);
    const size_t slice = (bytes / static_cast<size_t>(threads)) & ~static_cast<size_t>(4095);
    if (slice == 0) return false;
    char *buf = static_cast<char *>(numa_alloc(slice * static_cast<size_t>(threads), node));
    if (!buf) return false;
    std::atomic<uint64_t> sink{0};
    auto pass = [&](bool write) {
        std::vector<std::thread> ts;
        std::atomic<int> ready{0};
        std::atomic<bool> go{false};
        for (int t = 0; t < threads; ++t) {
            ts.emplace_back([&, t] {
                if (!cpus.empty()) bind_thread_to_cpus({cpus[static_cast<size_t>(t) % cpus.size()]});
                char *p = buf + static_cast<size_t>(t) * slice;
                ready.fetch_add(1);
                while (!go.load(std::memory_order_acquire)) std::this_thread::yield();
                if (write)
                    std::memset(p, t & 0xFF, slice);
                else
                    sink.fetch_xor(sum_words(reinterpret_cast<const uint64_t *>(p), slice / 8));
            });
        }
        while (ready.load() < threads) std::this_thread::yield();
        const auto t0 = std::chrono::steady_clock::now();
        go.store(true, std::memory_order_release);
        for (auto &th : ts) th.join();
        const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        return static_cast<double>(slice) * threads / s / 1e9;
    };
    HostBandwidth r;
    r.threads = threads;
    for (int i = 0; i < std::max(1, reps); ++i) {
        r.write_gbs = std::max(r.write_gbs, pass(true));
        r.read_gbs = std::max(r.read_gbs, pass(false));
    }
    numa_free(buf, slice * static_cast<size_t>(threads));
    *out = r;
    return true;
}

}  // namespace topo
}  // namespace mpcomm
