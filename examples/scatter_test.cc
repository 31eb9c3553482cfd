// scatter_test — PUT/GET/scatter/gather/broadcast bandwidth tool over the
// MPComm C++ API (parity: reference user_examples/scatter_test.cpp, the tool
// behind its README numbers; option names kept where they overlap).
//
//   target:     scatter_test --mode target --host-id T --tcp-port 5000 --buffer-size 4G [--gpu 0]
//   initiator:  scatter_test --target T:10.0.0.2:5000 --size 1G --batch-size 4
//                            --test-type put,get --iterations 10 --warmup 3 [--gpu 0]
//   both:       scatter_test --mode both --buffer-size 4G --size 1G ...  (serves its own
//               buffer and targets itself: the single-box memory-pool setup; with
//               --target options it serves AND initiates to those targets, the
//               multi-initiator setup where every host runs one process)
// Orchestration: --ready-file P is written once the buffer is served,
// --wait-go-file P delays the tests until P exists, --hold-file P keeps a
// "both" process serving after its tests until P exists (at most
// --hold-timeout s), --done-file P is written when its tests are finished,
// --json prints one JSON line per test.
// GB/s = bytes / 1e9 / wall seconds of the timed iterations (as the reference).
// --gpu N puts the local (and served) buffers in HBM of GPU N (cudaMalloc).
// --verify fills the local buffer with seeded bytes and, after the tests,
// reads every target slot the last put/scatter/broadcast test wrote back
// with GETs and compares it byte for byte (the reference harness verifies
// by read-back the same way).
// --nvls NAME:MEMBERS (with --gpu) makes this process one member of an NVLS
// multicast group of MEMBERS GPUs (exactly one process also passes
// --nvls-create): a target serves its copy of the group buffer, an
// initiator registers its own copy, and a broadcast to all the other
// members then goes out as multicast stores through the NVSwitch (one
// launch per chunk; --verify also checks the initiator's own copy). Every
// process needs the same --buffer-size (default --size x --batch-size).
// A target leaves cleanly on SIGTERM/SIGINT (unregisters, releases its copy).
// With MPCOMM_KERNEL_TRACE set, --json adds the timed launches by kind.
#include <cuda_runtime.h>
#include <unistd.h>

#include <csignal>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <random>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "mpcomm.h"

namespace {

volatile std::sig_atomic_t g_stop = 0;
void on_signal(int) { g_stop = 1; }

struct Target {
    std::string id, addr;
    int port = 0;
};

size_t parse_size(const std::string &s) {
    char *end = nullptr;
    double v = std::strtod(s.c_str(), &end);
    size_t mul = 1;
    if (end && *end) {
        switch (*end) {
            case 'K': case 'k': mul = 1ull << 10; break;
            case 'M': case 'm': mul = 1ull << 20; break;
            case 'G': case 'g': mul = 1ull << 30; break;
            case 'T': case 't': mul = 1ull << 40; break;
            default: break;
        }
    }
    return static_cast<size_t>(v * static_cast<double>(mul));
}

std::vector<std::string> split(const std::string &s, char d) {
    std::vector<std::string> out;
    std::stringstream ss(s);
    std::string p;
    while (std::getline(ss, p, d))
        if (!p.empty()) out.push_back(p);
    return out;
}

void *alloc_buf(size_t n, int gpu) {
    if (gpu >= 0) {
        void *p = nullptr;
        cudaSetDevice(gpu);
        if (cudaMalloc(&p, n) != cudaSuccess) return nullptr;
        cudaMemset(p, 0x5A, n);
        cudaDeviceSynchronize();
        return p;
    }
    void *p = nullptr;
    if (posix_memalign(&p, 1 << 21, n)) return nullptr;
    std::memset(p, 0x5A, n);
    return p;
}

void usage(const char *prog) {
    std::printf(
        "Usage: %s [--mode initiator|target|both] [--host-id ID] [--device DEVS] [--tcp-port P]\n"
        "          [--target ID:ADDR:PORT]... [--size S] [--buffer-size S] [--batch-size B]\n"
        "          [--iterations N] [--warmup W] [--test-type put,get,scatter,gather,broadcast]\n"
        "          [--gpu N] [--wait-go-file PATH] [--ready-file PATH] [--hold-file PATH]\n"
        "          [--hold-timeout S] [--done-file PATH] [--json] [--verify] [--verbose]\n"
        "          [--nvls NAME:MEMBERS [--nvls-create]]\n"
        "Sizes take K/M/G/T suffixes. Fabric: MPCOMM_FABRIC (auto|nvl|ib|sock|lo).\n",
        prog);
}

}  // namespace

int main(int argc, char **argv) {
    std::string mode = "initiator", host_id = "test:0", devices, tests = "put,get", go_file, ready_file, hold_file, done_file;
    int tcp_port = 0, iters = 10, warmup = 3, gpu = -1, hold_timeout = 600;
    size_t size = 1ull << 30, buf_size = 0, batch = 4;
    bool verbose = false, json = false, verify = false, nvls_create = false;
    std::string nvls_name;
    int nvls_members = 0;
    std::vector<Target> targets;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        auto next = [&]() -> std::string { return i + 1 < argc ? argv[++i] : std::string(); };
        if (a == "--mode") mode = next();
        else if (a == "--host-id") host_id = next();
        else if (a == "--device") devices = next();
        else if (a == "--tcp-port") tcp_port = std::atoi(next().c_str());
        else if (a == "--target") {
            auto f = split(next(), ':');
            if (f.size() < 3) return usage(argv[0]), 2;
            targets.push_back(Target{f[0], f[1], std::atoi(f[2].c_str())});
        } else if (a == "--size") size = parse_size(next());
        else if (a == "--buffer-size") buf_size = parse_size(next());
        else if (a == "--batch-size") batch = std::strtoul(next().c_str(), nullptr, 10);
        else if (a == "--iterations") iters = std::atoi(next().c_str());
        else if (a == "--warmup") warmup = std::atoi(next().c_str());
        else if (a == "--test-type") tests = next();
        else if (a == "--gpu") gpu = std::atoi(next().c_str());
        else if (a == "--wait-go-file") go_file = next();
        else if (a == "--ready-file") ready_file = next();
        else if (a == "--hold-file") hold_file = next();
        else if (a == "--done-file") done_file = next();
        else if (a == "--hold-timeout") hold_timeout = std::atoi(next().c_str());
        else if (a == "--json") json = true;
        else if (a == "--verify") verify = true;
        else if (a == "--nvls") {
            auto f = split(next(), ':');
            if (f.size() != 2) return usage(argv[0]), 2;
            nvls_name = f[0];
            nvls_members = std::atoi(f[1].c_str());
        } else if (a == "--nvls-create") nvls_create = true;
        else if (a == "--verbose" || a == "-v") verbose = true;
        else if (a == "--help" || a == "-h") return usage(argv[0]), 0;
        else return usage(argv[0]), 2;
    }
    if (batch == 0) batch = 1;
    if (gpu >= 0) cudaSetDevice(gpu);
    mpcomm::MPComm comm;
    if (comm.init(host_id, devices, tcp_port) != 0) return std::fprintf(stderr, "init failed\n"), 1;
    std::printf("[scatter_test] host %s fabric %s rails %zu tcp %d\n", host_id.c_str(),
                comm.getFabricName().c_str(), comm.getNumNics(), comm.getTcpPort());
    std::signal(SIGTERM, on_signal);
    std::signal(SIGINT, on_signal);

    // NVLS group membership: this process's copy of the group buffer.
    mpcomm::MulticastGroup grp;
    if (!nvls_name.empty()) {
        if (gpu < 0 || nvls_members < 2) return std::fprintf(stderr, "--nvls needs --gpu and MEMBERS >= 2\n"), 2;
        const size_t want = buf_size ? buf_size : size * batch;
        const int rc = nvls_create ? mpcomm::createMulticastGroup(nvls_name, want, nvls_members, &grp)
                                   : mpcomm::joinMulticastGroup(nvls_name, want, nvls_members, &grp);
        if (rc) return std::fprintf(stderr, "NVLS group %s: %d\n", nvls_name.c_str(), rc), 1;
        cudaMemset(grp.uc_addr, 0x5A, grp.length);
        cudaDeviceSynchronize();
        if (comm.registerMulticastGroup(grp))
            return std::fprintf(stderr, "registerMulticastGroup failed\n"), mpcomm::releaseMulticastGroup(&grp), 1;
        std::printf("[scatter_test] NVLS group %s: copy %p (%zu bytes), %d members\n", nvls_name.c_str(),
                    grp.uc_addr, grp.length, grp.members);
    }
    auto finish = [&](int rc) {
        if (grp.uc_addr) {
            comm.unpublishBuffer(grp.uc_addr);
            comm.unregisterMemory(grp.uc_addr);
        }
        comm.shutdown();
        mpcomm::releaseMulticastGroup(&grp);
        return rc;
    };

    void *served = nullptr;
    if (mode == "target" || mode == "both") {
        if (!buf_size) buf_size = size * batch;
        served = grp.uc_addr ? grp.uc_addr : alloc_buf(buf_size, gpu);
        if (!served || (!grp.uc_addr && comm.registerMemory(served, buf_size)) || comm.publishBuffer(served, buf_size))
            return std::fprintf(stderr, "serving buffer failed\n"), finish(1);
        comm.startAcceptThread();
        std::printf("[scatter_test] serving %zu bytes at %p (ready)\n", buf_size, served);
        std::fflush(stdout);
        if (!ready_file.empty()) {
            const std::string tmp = ready_file + ".tmp";
            if (FILE *f = std::fopen(tmp.c_str(), "w")) {
                std::fprintf(f, "%d\n", comm.getTcpPort());
                std::fclose(f);
                std::rename(tmp.c_str(), ready_file.c_str());
            }
        }
        if (mode == "target") {
            for (int tick = 1; !g_stop; ++tick) {
                std::this_thread::sleep_for(std::chrono::milliseconds(50));
                if (verbose && tick % 100 == 0)
                    std::printf("[scatter_test] published=%zu\n", comm.getPublishedBufferCount());
            }
            std::printf("[scatter_test] target %s stopping\n", host_id.c_str());
            return finish(0);
        }
        if (targets.empty()) targets.push_back(Target{"self", "127.0.0.1", comm.getTcpPort()});
    }
    if (targets.empty()) return usage(argv[0]), finish(2);
    if (!go_file.empty()) {
        const auto until = std::chrono::steady_clock::now() + std::chrono::seconds(hold_timeout);
        while (access(go_file.c_str(), F_OK) != 0) {
            if (std::chrono::steady_clock::now() >= until)
                return std::fprintf(stderr, "no go file %s after %d s\n", go_file.c_str(), hold_timeout), finish(1);
            std::this_thread::sleep_for(std::chrono::milliseconds(50));
        }
    }

    std::vector<uintptr_t> remote;
    // Connect retries while targets come up (MPCOMM_CONNECT_RETRIES,
    // MPCOMM_CONNECT_RETRY_INTERVAL_MS; the reference tool's variables).
    auto env_int = [](const char *name, int def) {
        const char *v = std::getenv(name);
        return v && *v ? std::atoi(v) : def;
    };
    const int retries = std::max(1, env_int("MPCOMM_CONNECT_RETRIES", 30));
    const int retry_ms = std::max(1, env_int("MPCOMM_CONNECT_RETRY_INTERVAL_MS", 500));
    for (auto &t : targets) {
        int rc = -1;
        for (int attempt = 0; attempt < retries && rc != 0; ++attempt) {
            rc = comm.connect(t.id, t.addr, t.port);
            if (rc) std::this_thread::sleep_for(std::chrono::milliseconds(retry_ms));
        }
        mpcomm::RemoteBufferEntry e;
        if (rc || comm.queryRemoteBufferByNuma(t.id, t.addr, t.port, -1, e))
            return std::fprintf(stderr, "connect/query %s failed\n", t.id.c_str()), finish(1);
        if (e.length < size * batch) return std::fprintf(stderr, "remote buffer too small\n"), finish(1);
        remote.push_back(e.addr);
    }
    const size_t local_bytes = size * batch * targets.size();
    void *local = alloc_buf(local_bytes, gpu);
    if (!local || comm.registerMemory(local, local_bytes)) return std::fprintf(stderr, "local buffer failed\n"), finish(1);
    const uintptr_t lp = reinterpret_cast<uintptr_t>(local);
    std::vector<unsigned char> pattern;
    if (verify) {
        pattern.resize(local_bytes);
        std::mt19937_64 rng(0x5CA77E5ull);
        for (size_t i = 0; i + 8 <= local_bytes; i += 8) {
            const uint64_t v = rng();
            std::memcpy(&pattern[i], &v, 8);
        }
        if (gpu >= 0) cudaMemcpy(local, pattern.data(), local_bytes, cudaMemcpyHostToDevice);
        else std::memcpy(local, pattern.data(), local_bytes);
    }
    std::string last_write;

    for (const std::string &tt : split(tests, ',')) {
        auto one_round = [&]() -> int {
            std::vector<mpcomm::TransferHandle> hs;
            if (tt == "broadcast") {
                // One request per batch slot to every target at once (one
                // length, the same local bytes; on the GPU fabric the engine
                // writes all targets in one launch per chunk).
                std::vector<std::string> ids;
                for (auto &t : targets) ids.push_back(t.id);
                for (size_t b = 0; b < batch; ++b) {
                    std::vector<uintptr_t> rs;
                    for (size_t t = 0; t < targets.size(); ++t) rs.push_back(remote[t] + b * size);
                    mpcomm::TransferHandle h = comm.broadcastAsync(lp + b * size, size, ids, rs);
                    if (h == mpcomm::INVALID_TRANSFER_HANDLE) return -1;
                    hs.push_back(h);
                }
            }
            for (size_t b = 0; b < batch && tt != "broadcast"; ++b) {
                for (size_t t = 0; t < targets.size(); ++t) {
                    const uintptr_t l = lp + (t * batch + b) * size;
                    const uintptr_t r = remote[t] + b * size;
                    mpcomm::TransferHandle h = mpcomm::INVALID_TRANSFER_HANDLE;
                    if (tt == "put") h = comm.putAsync(l, targets[t].id, r, size);
                    else if (tt == "get") h = comm.getAsync(l, targets[t].id, r, size);
                    else if (tt == "scatter") h = comm.scatterAsync(l, {targets[t].id}, {r}, {size});
                    else if (tt == "gather") h = comm.gatherAsync(l, {targets[t].id}, {r}, {size});
                    if (h == mpcomm::INVALID_TRANSFER_HANDLE) return -1;
                    hs.push_back(h);
                }
            }
            int rc = 0;
            for (auto h : hs) {
                rc |= comm.waitTransfer(h, 600000);
                comm.releaseTransfer(h);
            }
            return rc;
        };
        for (int w = 0; w < warmup; ++w)
            if (one_round()) return std::fprintf(stderr, "%s warm-up failed\n", tt.c_str()), finish(1);
        // Kernel trace (MPCOMM_KERNEL_TRACE): launches of the timed rounds by kind.
        const bool traced = std::getenv("MPCOMM_KERNEL_TRACE") != nullptr;
        uint64_t seq0 = 0;
        if (traced)
            for (const auto &r : mpcomm::MPComm::getKernelTrace()) seq0 = std::max(seq0, r.seq);
        const uint64_t launches0 = mpcomm::MPComm::getKernelLaunchCount();
        auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < iters; ++i)
            if (one_round()) return std::fprintf(stderr, "%s failed\n", tt.c_str()), finish(1);
        const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        const double bytes = static_cast<double>(size) * batch * targets.size() * iters;
        std::printf("--- %s Summary: size=%zu batch=%zu targets=%zu iters=%d  %.3f GB/s  (%.3f ms/round)\n",
                    tt.c_str(), size, batch, targets.size(), iters, bytes / 1e9 / s, s * 1e3 / iters);
        const uint64_t launches = mpcomm::MPComm::getKernelLaunchCount() - launches0;
        std::string kinds;
        if (traced) {
            std::map<std::string, int> by_kind;
            for (const auto &r : mpcomm::MPComm::getKernelTrace())
                if (r.seq > seq0) ++by_kind[r.kind];
            for (const auto &kv : by_kind)
                kinds += (kinds.empty() ? "" : ", ") + ("\"" + kv.first + "\": ") + std::to_string(kv.second);
            kinds = ", \"kernel_kinds\": {" + kinds + "}";
        }
        if (json)
            std::printf("{\"tool\": \"scatter_test\", \"host\": \"%s\", \"test\": \"%s\", \"size\": %zu, "
                        "\"batch\": %zu, \"targets\": %zu, \"iters\": %d, \"gbps\": %.4f, \"ms_per_round\": %.4f, "
                        "\"kernel_launches\": %llu, \"nvls_member\": %s%s}\n",
                        host_id.c_str(), tt.c_str(), size, batch, targets.size(), iters, bytes / 1e9 / s,
                        s * 1e3 / iters, static_cast<unsigned long long>(launches), grp.uc_addr ? "true" : "false",
                        kinds.c_str());
        std::fflush(stdout);
        if (tt == "put" || tt == "scatter" || tt == "broadcast") last_write = tt;
    }
    if (verify && !last_write.empty()) {
        // Read every written slot back and compare with what was sent.
        void *scratch = alloc_buf(size, gpu);
        if (!scratch || comm.registerMemory(scratch, size)) return std::fprintf(stderr, "verify buffer failed\n"), finish(1);
        std::vector<unsigned char> got(size);
        size_t bad = 0;
        for (size_t t = 0; t < targets.size(); ++t) {
            for (size_t b = 0; b < batch; ++b) {
                const size_t src_off = last_write == "broadcast" ? b * size : (t * batch + b) * size;
                mpcomm::TransferHandle h =
                    comm.getAsync(reinterpret_cast<uintptr_t>(scratch), targets[t].id, remote[t] + b * size, size);
                if (h == mpcomm::INVALID_TRANSFER_HANDLE || comm.waitTransfer(h, 600000))
                    return std::fprintf(stderr, "verify read-back failed\n"), finish(1);
                comm.releaseTransfer(h);
                if (gpu >= 0) cudaMemcpy(got.data(), scratch, size, cudaMemcpyDeviceToHost);
                else std::memcpy(got.data(), scratch, size);
                if (std::memcmp(got.data(), &pattern[src_off], size) != 0) ++bad;
            }
        }
        size_t slots = targets.size() * batch;
        if (last_write == "broadcast" && grp.uc_addr && !served) {
            // An NVLS member's own copy receives every multicast broadcast too.
            for (size_t b = 0; b < batch; ++b, ++slots) {
                cudaMemcpy(got.data(), static_cast<char *>(grp.uc_addr) + b * size, size, cudaMemcpyDeviceToHost);
                if (std::memcmp(got.data(), &pattern[b * size], size) != 0) ++bad;
            }
        }
        std::printf("[scatter_test] verify %s: %zu of %zu slots differ\n", last_write.c_str(), bad, slots);
        if (json)
            std::printf("{\"tool\": \"scatter_test\", \"verify\": \"%s\", \"slots\": %zu, \"bad\": %zu}\n",
                        last_write.c_str(), slots, bad);
        std::fflush(stdout);
        if (bad) return finish(1);
    }
    if (!done_file.empty())
        if (FILE *f = std::fopen(done_file.c_str(), "w")) std::fclose(f);
    if (!hold_file.empty() && served) {
        // Keep serving for the other initiators until released (bounded).
        const auto until = std::chrono::steady_clock::now() + std::chrono::seconds(hold_timeout);
        while (access(hold_file.c_str(), F_OK) != 0 && std::chrono::steady_clock::now() < until)
            std::this_thread::sleep_for(std::chrono::milliseconds(50));
    }
    return finish(0);
}
