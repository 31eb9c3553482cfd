// scatter_test — PUT/GET/scatter/gather/broadcast bandwidth tool over the
// MPComm C++ API (parity: reference user_examples/scatter_test.cpp, the tool
// behind its README numbers; option names kept where they overlap).
//
//   target:     scatter_test --mode target --host-id T --tcp-port 5000 --buffer-size 4G [--gpu 0]
//   initiator:  scatter_test --target T:10.0.0.2:5000 --size 1G --batch-size 4 \
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
#include <cuda_runtime.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <random>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "mpcomm.h"

namespace {

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
        "Sizes take K/M/G/T suffixes. Fabric: MPCOMM_FABRIC (auto|nvl|ib|sock|lo).\n",
        prog);
}

}  // namespace

int main(int argc, char **argv) {
    std::string mode = "initiator", host_id = "test:0", devices, tests = "put,get", go_file, ready_file, hold_file, done_file;
    int tcp_port = 0, iters = 10, warmup = 3, gpu = -1, hold_timeout = 600;
    size_t size = 1ull << 30, buf_size = 0, batch = 4;
    bool verbose = false, json = false, verify = false;
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

    void *served = nullptr;
    if (mode == "target" || mode == "both") {
        if (!buf_size) buf_size = size * batch;
        served = alloc_buf(buf_size, gpu);
        if (!served || comm.registerMemory(served, buf_size) || comm.publishBuffer(served, buf_size))
            return std::fprintf(stderr, "serving buffer failed\n"), 1;
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
            for (;;) {
                std::this_thread::sleep_for(std::chrono::seconds(verbose ? 5 : 60));
                if (verbose) std::printf("[scatter_test] published=%zu\n", comm.getPublishedBufferCount());
            }
        }
        if (targets.empty()) targets.push_back(Target{"self", "127.0.0.1", comm.getTcpPort()});
    }
    if (targets.empty()) return usage(argv[0]), 2;
    if (!go_file.empty()) {
        const auto until = std::chrono::steady_clock::now() + std::chrono::seconds(hold_timeout);
        while (access(go_file.c_str(), F_OK) != 0) {
            if (std::chrono::steady_clock::now() >= until)
                return std::fprintf(stderr, "no go file %s after %d s\n", go_file.c_str(), hold_timeout), 1;
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
            return std::fprintf(stderr, "connect/query %s failed\n", t.id.c_str()), 1;
        if (e.length < size * batch) return std::fprintf(stderr, "remote buffer too small\n"), 1;
        remote.push_back(e.addr);
    }
    const size_t local_bytes = size * batch * targets.size();
    void *local = alloc_buf(local_bytes, gpu);
    if (!local || comm.registerMemory(local, local_bytes)) return std::fprintf(stderr, "local buffer failed\n"), 1;
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
            if (one_round()) return std::fprintf(stderr, "%s warm-up failed\n", tt.c_str()), 1;
        const uint64_t launches0 = mpcomm::MPComm::getKernelLaunchCount();
        auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < iters; ++i)
            if (one_round()) return std::fprintf(stderr, "%s failed\n", tt.c_str()), 1;
        const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        const double bytes = static_cast<double>(size) * batch * targets.size() * iters;
        std::printf("--- %s Summary: size=%zu batch=%zu targets=%zu iters=%d  %.3f GB/s  (%.3f ms/round)\n",
                    tt.c_str(), size, batch, targets.size(), iters, bytes / 1e9 / s, s * 1e3 / iters);
        const uint64_t launches = mpcomm::MPComm::getKernelLaunchCount() - launches0;
        if (json)
            std::printf("{\"tool\": \"scatter_test\", \"host\": \"%s\", \"test\": \"%s\", \"size\": %zu, "
                        "\"batch\": %zu, \"targets\": %zu, \"iters\": %d, \"gbps\": %.4f, \"ms_per_round\": %.4f, "
                        "\"kernel_launches\": %llu}\n",
                        host_id.c_str(), tt.c_str(), size, batch, targets.size(), iters, bytes / 1e9 / s,
                        s * 1e3 / iters, static_cast<unsigned long long>(launches));
        std::fflush(stdout);
        if (tt == "put" || tt == "scatter" || tt == "broadcast") last_write = tt;
    }
    if (verify && !last_write.empty()) {
        // Read every written slot back and compare with what was sent.
        void *scratch = alloc_buf(size, gpu);
        if (!scratch || comm.registerMemory(scratch, size)) return std::fprintf(stderr, "verify buffer failed\n"), 1;
        std::vector<unsigned char> got(size);
        size_t bad = 0;
        for (size_t t = 0; t < targets.size(); ++t) {
            for (size_t b = 0; b < batch; ++b) {
                const size_t src_off = last_write == "broadcast" ? b * size : (t * batch + b) * size;
                mpcomm::TransferHandle h =
                    comm.getAsync(reinterpret_cast<uintptr_t>(scratch), targets[t].id, remote[t] + b * size, size);
                if (h == mpcomm::INVALID_TRANSFER_HANDLE || comm.waitTransfer(h, 600000))
                    return std::fprintf(stderr, "verify read-back failed\n"), 1;
                comm.releaseTransfer(h);
                if (gpu >= 0) cudaMemcpy(got.data(), scratch, size, cudaMemcpyDeviceToHost);
                else std::memcpy(got.data(), scratch, size);
                if (std::memcmp(got.data(), &pattern[src_off], size) != 0) ++bad;
            }
        }
        std::printf("[scatter_test] verify %s: %zu of %zu slots differ\n", last_write.c_str(), bad,
                    targets.size() * batch);
        if (json)
            std::printf("{\"tool\": \"scatter_test\", \"verify\": \"%s\", \"slots\": %zu, \"bad\": %zu}\n",
                        last_write.c_str(), targets.size() * batch, bad);
        std::fflush(stdout);
        if (bad) return 1;
    }
    if (!done_file.empty())
        if (FILE *f = std::fopen(done_file.c_str(), "w")) std::fclose(f);
    if (!hold_file.empty() && served) {
        // Keep serving for the other initiators until released (bounded).
        const auto until = std::chrono::steady_clock::now() + std::chrono::seconds(hold_timeout);
        while (access(hold_file.c_str(), F_OK) != 0 && std::chrono::steady_clock::now() < until)
            std::this_thread::sleep_for(std::chrono::milliseconds(50));
    }
    comm.shutdown();
    return 0;
}
