// Small lock-light building blocks of the transfer engine.
//
//  * WrId         — 64-bit work-request id: rail[63:56] | qp[55:48] |
//                   handle[47:32] | chunk[31:0]. Same field layout as the
//                   reference's WrIdEncoding (src/mpcomm.cpp:140-172) because
//                   the 16-bit handle space is part of the public contract
//                   (handles 1..65535, INVALID_TRANSFER_HANDLE = 0).
//  * HandlePool   — recyclable 16-bit handles (reference :939-968).
//  * MpscRing     — bounded multi-producer/single-consumer queue of handles
//                   with per-slot sequence numbers (reference used a CAS'd
//                   head over atomic slots, :616-664).
//  * TokenBucket  — byte token bucket; rate 0 means "paused".
//  * ChunkPlan    — lazy chunk metadata: per-host start index + binary
//                   search, so a 1 GiB x N-host transfer stores O(hosts).
#ifndef MPCOMM_B200_CSRC_CORE_CORE_H_
#define MPCOMM_B200_CSRC_CORE_CORE_H_

#include <time.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <mutex>
#include <vector>

namespace mpcomm {

constexpr size_t kMaxRails = 16;         // "kMaxNics" in the reference
constexpr size_t kMaxQpsPerRail = 16;    // "kMaxQPsPerNic"
constexpr size_t kMaxNumaNodes = 8;
constexpr size_t kMaxGpuDomains = 16;

inline uint64_t monotonic_raw_ns() {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC_RAW, &ts);
    return static_cast<uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<uint64_t>(ts.tv_nsec);
}

inline void cpu_relax() {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#elif defined(__aarch64__)
    asm volatile("yield" ::: "memory");
#endif
}

struct WrId {
    static constexpr unsigned kRailShift = 56, kQpShift = 48, kHandleShift = 32;
    static constexpr uint64_t kByte = 0xFF, kHandleMask = 0xFFFF, kChunkMask = 0xFFFFFFFFull;

    static constexpr uint64_t encode(uint64_t rail, uint64_t qp, uint64_t handle, uint64_t chunk) {
        return ((rail & kByte) << kRailShift) | ((qp & kByte) << kQpShift) |
               ((handle & kHandleMask) << kHandleShift) | (chunk & kChunkMask);
    }
    static constexpr size_t rail(uint64_t id) { return (id >> kRailShift) & kByte; }
    static constexpr size_t qp(uint64_t id) { return (id >> kQpShift) & kByte; }
    static constexpr uint64_t handle(uint64_t id) { return (id >> kHandleShift) & kHandleMask; }
    static constexpr size_t chunk(uint64_t id) { return id & kChunkMask; }
};

class HandlePool {
 public:
    static constexpr uint64_t kMin = 1, kMax = 0xFFFF;
    // Returns 0 (INVALID_TRANSFER_HANDLE) when all 65535 handles are live.
    uint64_t allocate() {
        std::lock_guard<std::mutex> g(mu_);
        if (!free_.empty()) {
            uint64_t h = free_.back();
            free_.pop_back();
            return h;
        }
        return next_ <= kMax ? next_++ : 0;
    }
    void release(uint64_t h) {
        if (h == 0 || h > kMax) return;
        std::lock_guard<std::mutex> g(mu_);
        free_.push_back(h);
    }
    size_t live() const {
        std::lock_guard<std::mutex> g(mu_);
        return static_cast<size_t>(next_ - kMin) - free_.size();
    }

 private:
    mutable std::mutex mu_;
    std::vector<uint64_t> free_;
    uint64_t next_ = kMin;
};

// Bounded MPSC ring (capacity power of two). Producers claim a ticket with
// fetch_add-free CAS on tail and publish through the slot's sequence word;
// the single consumer reads slots in order.
class MpscRing {
 public:
    explicit MpscRing(size_t capacity_pow2 = 4096)
        : mask_(capacity_pow2 - 1), slots_(new Slot[capacity_pow2]) {
        for (size_t i = 0; i <= mask_; ++i) slots_[i].seq.store(i, std::memory_order_relaxed);
    }
    bool try_push(uint64_t v) {
        size_t pos = tail_.load(std::memory_order_relaxed);
        for (;;) {
            Slot &s = slots_[pos & mask_];
            size_t seq = s.seq.load(std::memory_order_acquire);
            intptr_t dif = static_cast<intptr_t>(seq) - static_cast<intptr_t>(pos);
            if (dif == 0) {
                if (tail_.compare_exchange_weak(pos, pos + 1, std::memory_order_relaxed)) {
                    s.value = v;
                    s.seq.store(pos + 1, std::memory_order_release);
                    return true;
                }
            } else if (dif < 0) {
                return false;  // full
            } else {
                pos = tail_.load(std::memory_order_relaxed);
            }
        }
    }
    bool try_pop(uint64_t *out) {
        Slot &s = slots_[head_ & mask_];
        size_t seq = s.seq.load(std::memory_order_acquire);
        if (static_cast<intptr_t>(seq) - static_cast<intptr_t>(head_ + 1) < 0) return false;
        *out = s.value;
        s.seq.store(head_ + mask_ + 1, std::memory_order_release);
        ++head_;
        return true;
    }
    size_t capacity() const { return mask_ + 1; }

 private:
    struct alignas(64) Slot {
        std::atomic<size_t> seq;
        uint64_t value;
    };
    size_t mask_;
    std::unique_ptr<Slot[]> slots_;
    alignas(64) std::atomic<size_t> tail_{0};
    alignas(64) size_t head_ = 0;
};

// Byte token bucket. rate == 0 => every consume() fails (explicit pause).
// Capacity is max(burst, request) so a chunk larger than the burst can
// still pass once enough time has accrued.
class TokenBucket {
 public:
    void configure(uint64_t rate_bps, uint64_t burst) {
        std::lock_guard<std::mutex> g(mu_);
        rate_ = rate_bps;
        burst_ = burst;
        tokens_ = 0.0;
        last_ = std::chrono::steady_clock::now();
    }
    bool consume(uint64_t bytes) {
        std::lock_guard<std::mutex> g(mu_);
        if (rate_ == 0) return false;
        auto now = std::chrono::steady_clock::now();
        double dt = std::chrono::duration<double>(now - last_).count();
        last_ = now;
        double cap = static_cast<double>(std::max(burst_, bytes));
        tokens_ = std::min(cap, tokens_ + dt * static_cast<double>(rate_));
        if (tokens_ < static_cast<double>(bytes)) return false;
        tokens_ -= static_cast<double>(bytes);
        return true;
    }
    uint64_t rate() const {
        std::lock_guard<std::mutex> g(mu_);
        return rate_;
    }
    uint64_t burst() const {
        std::lock_guard<std::mutex> g(mu_);
        return burst_;
    }

 private:
    mutable std::mutex mu_;
    uint64_t rate_ = 0, burst_ = 0;
    double tokens_ = 0.0;
    std::chrono::steady_clock::time_point last_{};
};

// Default burst for a pacing rate: rate/10000 clamped to [4 KiB, 64 KiB]
// (the reference's defaultQosBurstBytes, src/mpcomm.cpp:2405-2413).
inline uint64_t default_qos_burst(uint64_t rate_bps) {
    if (rate_bps == 0) return 0;
    return std::min<uint64_t>(64 << 10, std::max<uint64_t>(4 << 10, rate_bps / 10000));
}

struct Chunk {
    size_t host_idx;
    uintptr_t local_addr;
    uintptr_t remote_addr;
    size_t length;
};

// Chunk layout of one transfer. Host i's bytes are split into
// ceil(len_i / chunk) chunks numbered after host i-1's; broadcast keeps the
// local offset at 0 for every host.
class ChunkPlan {
 public:
    void build(uintptr_t local, const std::vector<uintptr_t> &remote,
               const std::vector<size_t> &lengths, size_t chunk, bool broadcast) {
        local_ = local;
        remote_ = remote;
        lengths_ = lengths;
        chunk_ = chunk;
        starts_.resize(lengths.size());
        offsets_.resize(lengths.size());
        size_t total = 0, off = 0;
        for (size_t i = 0; i < lengths.size(); ++i) {
            starts_[i] = total;
            offsets_[i] = off;
            total += (lengths[i] + chunk - 1) / chunk;
            if (!broadcast) off += lengths[i];
        }
        total_ = total;
    }
    size_t total() const { return total_; }
    size_t chunk_size() const { return chunk_; }
    Chunk get(size_t idx) const {
        size_t h = static_cast<size_t>(
            std::upper_bound(starts_.begin(), starts_.end(), idx) - starts_.begin()) - 1;
        // Hosts with zero length share a start index; upper_bound lands on the
        // last of them, which is never a zero-length host for a valid idx.
        size_t off = (idx - starts_[h]) * chunk_;
        size_t len = std::min(chunk_, lengths_[h] - off);
        return Chunk{h, local_ + offsets_[h] + off, remote_[h] + off, len};
    }

 private:
    uintptr_t local_ = 0;
    std::vector<uintptr_t> remote_;
    std::vector<size_t> lengths_, starts_, offsets_;
    size_t chunk_ = 1, total_ = 0;
};

}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_CORE_CORE_H_
