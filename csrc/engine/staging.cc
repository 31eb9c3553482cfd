#include "engine/staging.h"

#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstring>

#include "cuda/gpu.h"
#include "kernels/launch.h"
#include "mpcomm_log.h"
#include "topo/topology.h"

namespace mpcomm {

enum PieceState { kWaitSlab = 0, kCopyIn, kXfer, kCopyOut, kDone };

struct StagingEngine::DevicePool {
    int dev = -1;
    char *base = nullptr;
    size_t slab_bytes = 0, nslabs = 0;
    bool registered = false;
    std::vector<int> free;        // orchestrator thread only
    void *stream = nullptr;       // pool stream (used when no fabric stream is set)
    uint64_t *done = nullptr;     // host-mapped completion word per slab
    uint32_t *ctr = nullptr;      // device: last-CTA counter per slab (a launch per slab at a time)
    uint32_t *status = nullptr;   // device: bounded-wait status of the copies
    uint64_t seq = 0;             // orchestrator thread only
};

struct StagingEngine::Piece {
    size_t host;
    uintptr_t local;
    uintptr_t remote;
    size_t len;
    DevicePool *pool = nullptr;  // device piece (slab in that GPU's HBM)
    int state = kWaitSlab;
    int slab = -1;
    uint64_t wait_value = 0;  // device piece: completion word value of its copy
    std::chrono::steady_clock::time_point launched;
    TransferHandle sub = INVALID_TRANSFER_HANDLE;
    std::atomic<bool> copied{false};
};

struct StagingEngine::Staged {
    std::shared_ptr<Transfer> t;
    Direction dir;
    std::vector<std::unique_ptr<Piece>> pieces;
    size_t done = 0;
    int error = 0;
};

namespace {

// True when every page of [addr, addr + len) is mapped in this process.
bool host_range_mapped(uintptr_t addr, size_t len) {
    if (len == 0) return true;
    const uintptr_t pg = static_cast<uintptr_t>(sysconf(_SC_PAGESIZE));
    const uintptr_t lo = addr & ~(pg - 1), hi = (addr + len + pg - 1) & ~(pg - 1);
    // mincore fails with ENOMEM when the range holds an unmapped page; the
    // residency vector itself is not needed, so it is filled in pieces.
    unsigned char vec[256];
    for (uintptr_t p = lo; p < hi; p += 256 * pg) {
        const size_t n = std::min<uintptr_t>(hi - p, 256 * pg);
        if (mincore(reinterpret_cast<void *>(p), n, vec) != 0 && errno == ENOMEM) return false;
    }
    return true;
}

// A device copy that has not published its completion word after this long
// is checked for a launch or context error.
constexpr auto kDeviceCopyCheckAfter = std::chrono::seconds(5);

}  // namespace

StagingEngine::StagingEngine(MPComm::Impl *impl)
    : impl_(impl),
      slab_bytes_(impl->config().staging_slab_bytes),
      nslabs_(impl->config().staging_slabs),
      nthreads_(impl->config().staging_threads),
      dev_slab_bytes_(impl->config().staging_device_slab_bytes) {
    dev_pools_.resize(kMaxGpuDomains);
}

StagingEngine::~StagingEngine() {
    running_ = false;
    cv_.notify_all();
    if (orchestrator_.joinable()) orchestrator_.join();
    {
        std::lock_guard<std::mutex> g(cmu_);
        copies_.clear();
    }
    ccv_.notify_all();
    for (auto &t : copiers_)
        if (t.joinable()) t.join();
    for (auto &s : active_) {
        s->t->error.store(MPCOMM_ERR_TRANSFER);
        impl_->finishTransfer(s->t.get());
    }
    if (slab_base_) {
        if (slabs_registered_) impl_->unregisterMemory(slab_base_);
        topo::numa_free(slab_base_, slab_total_);
    }
    for (auto &dp : dev_pools_) {
        if (!dp) continue;
        gpu::set_device(dp->dev);
        if (dp->stream) gpu::stream_sync(dp->stream);
        if (impl_->fabricStream()) gpu::stream_sync(impl_->fabricStream());
        if (dp->registered) impl_->unregisterMemory(dp->base);
        gpu::device_free(dp->base);
        gpu::device_free(dp->ctr);
        gpu::device_free(dp->status);
        gpu::host_free(dp->done);
        gpu::stream_destroy(dp->stream);
    }
}

void StagingEngine::start_threads() {
    if (threads_started_) return;
    threads_started_ = true;
    for (size_t i = 0; i < nthreads_; ++i) copiers_.emplace_back([this] { copy_worker(); });
    orchestrator_ = std::thread([this] { orchestrate(); });
}

bool StagingEngine::ensure_slabs() {
    if (slab_base_) return slabs_registered_;
    slab_total_ = slab_bytes_ * nslabs_;
    slab_base_ = topo::numa_alloc(slab_total_, -1);
    if (!slab_base_) return false;
    slabs_registered_ = impl_->registerMemory(slab_base_, slab_total_) == MPCOMM_SUCCESS;
    if (!slabs_registered_) {
        MPCOMM_LOG_ERROR("MPComm: staging slabs could not be registered\n");
        return false;
    }
    for (size_t i = 0; i < nslabs_; ++i) free_slabs_.push_back(static_cast<int>(nslabs_ - 1 - i));
    start_threads();
    MPCOMM_LOG_INFO("MPComm: staging pool ready (%zu slabs x %zu B, %zu copy threads)\n", nslabs_,
                    slab_bytes_, nthreads_);
    return true;
}

StagingEngine::DevicePool *StagingEngine::ensure_device_pool(int dev) {
    if (dev < 0 || dev >= static_cast<int>(dev_pools_.size())) return nullptr;
    if (dev_pools_[dev]) return dev_pools_[dev]->registered ? dev_pools_[dev].get() : nullptr;
    auto dp = std::make_unique<DevicePool>();
    dp->dev = dev;
    dp->slab_bytes = (dev_slab_bytes_ + 255) & ~static_cast<size_t>(255);
    dp->nslabs = nslabs_;
    const int prev = gpu::current_device();
    gpu::set_device(dev);
    dp->base = static_cast<char *>(gpu::device_alloc(dp->slab_bytes * dp->nslabs));
    dp->ctr = static_cast<uint32_t *>(gpu::device_alloc(dp->nslabs * sizeof(uint32_t)));
    dp->status = static_cast<uint32_t *>(gpu::device_alloc(64));
    dp->done = static_cast<uint64_t *>(gpu::host_alloc_mapped(dp->nslabs * sizeof(uint64_t)));
    dp->stream = gpu::stream_create(dev);
    bool ok = dp->base && dp->ctr && dp->status && dp->done && dp->stream;
    if (ok) {
        ok = gpu::memset_device(dp->ctr, 0, dp->nslabs * sizeof(uint32_t)) == 0 &&
             gpu::memset_device(dp->status, 0, 64) == 0;
        std::memset(dp->done, 0, dp->nslabs * sizeof(uint64_t));
    }
    if (ok) dp->registered = impl_->registerMemory(dp->base, dp->slab_bytes * dp->nslabs) == MPCOMM_SUCCESS;
    if (prev >= 0) gpu::set_device(prev);
    if (!dp->registered) {
        MPCOMM_LOG_ERROR("MPComm: device staging slabs on GPU %d could not be %s\n", dev,
                         ok ? "registered" : "allocated");
        gpu::device_free(dp->base);
        gpu::device_free(dp->ctr);
        gpu::device_free(dp->status);
        gpu::host_free(dp->done);
        gpu::stream_destroy(dp->stream);
        dp->base = nullptr;
        dp->ctr = dp->status = nullptr;
        dp->done = nullptr;
        dp->stream = nullptr;
        dev_pools_[dev] = std::move(dp);
        return nullptr;
    }
    for (size_t i = 0; i < dp->nslabs; ++i) dp->free.push_back(static_cast<int>(dp->nslabs - 1 - i));
    MPCOMM_LOG_INFO("MPComm: device staging pool ready on GPU %d (%zu slabs x %zu B of HBM)\n", dev, dp->nslabs,
                    dp->slab_bytes);
    dev_pools_[dev] = std::move(dp);
    start_threads();
    return dev_pools_[dev].get();
}

TransferHandle StagingEngine::submit(uintptr_t local, const std::vector<std::string> &hosts,
                                     const std::vector<uintptr_t> &raddrs,
                                     const std::vector<size_t> &lens, Direction dir) {
    size_t span = 0;
    for (size_t l : lens) span = dir == Direction::kBroadcast ? std::max(span, l) : span + l;
    gpu::PtrInfo info;
    const bool device = gpu::query_pointer(reinterpret_cast<const void *>(local), &info) && info.is_device;
    if (device && info.base && local + span > info.base + info.size) {
        MPCOMM_LOG_ERROR("MPComm: staged transfer 0x%lx+%zu runs past its device allocation\n",
                         static_cast<unsigned long>(local), span);
        return INVALID_TRANSFER_HANDLE;
    }
    if (!device && !host_range_mapped(local, span)) {
        MPCOMM_LOG_ERROR("MPComm: staged transfer 0x%lx+%zu: the range is neither device memory nor mapped "
                         "host memory\n", static_cast<unsigned long>(local), span);
        return INVALID_TRANSFER_HANDLE;
    }
    DevicePool *pool = nullptr;
    size_t piece_bytes = slab_bytes_;
    {
        std::lock_guard<std::mutex> g(mu_);
        if (device) {
            pool = ensure_device_pool(info.device);
            if (!pool) return INVALID_TRANSFER_HANDLE;
            piece_bytes = pool->slab_bytes;
        } else if (!ensure_slabs()) {
            return INVALID_TRANSFER_HANDLE;
        }
    }
    auto s = std::make_shared<Staged>();
    s->dir = dir;
    s->t = impl_->newCompositeTransfer(dir, local, hosts, raddrs, lens);
    if (!s->t) return INVALID_TRANSFER_HANDLE;
    s->t->local_gpu = device ? info.device : -1;
    size_t off = 0;
    for (size_t h = 0; h < hosts.size(); ++h) {
        const size_t base = dir == Direction::kBroadcast ? 0 : off;
        for (size_t p = 0; p < lens[h]; p += piece_bytes) {
            auto pc = std::make_unique<Piece>();
            pc->host = h;
            pc->local = local + base + p;
            pc->remote = raddrs[h] + p;
            pc->len = std::min(piece_bytes, lens[h] - p);
            pc->pool = pool;
            s->pieces.push_back(std::move(pc));
        }
        off += lens[h];
    }
    const TransferHandle handle = s->t->handle;
    if (s->pieces.empty()) {
        impl_->finishTransfer(s->t.get());
        return handle;
    }
    {
        std::lock_guard<std::mutex> g(mu_);
        incoming_.push_back(std::move(s));
    }
    cv_.notify_all();
    return handle;
}

void StagingEngine::enqueue_copy(std::function<void()> job) {
    {
        std::lock_guard<std::mutex> g(cmu_);
        copies_.push_back(std::move(job));
    }
    ccv_.notify_one();
}

void StagingEngine::copy_worker() {
    for (;;) {
        std::function<void()> job;
        {
            std::unique_lock<std::mutex> g(cmu_);
            ccv_.wait(g, [&] { return !running_ || !copies_.empty(); });
            if (copies_.empty()) return;
            job = std::move(copies_.front());
            copies_.pop_front();
        }
        job();
        copies_done_.fetch_add(1, std::memory_order_release);
        cv_.notify_all();
    }
}

bool StagingEngine::launch_device_copy(Piece *p, bool to_slab) {
    DevicePool *dp = p->pool;
    char *slab = dp->base + static_cast<size_t>(p->slab) * dp->slab_bytes;
    kern::CopyDesc d;
    d.src = to_slab ? reinterpret_cast<const void *>(p->local) : slab;
    d.dst = to_slab ? static_cast<void *>(slab) : reinterpret_cast<void *>(p->local);
    d.bytes = p->len;
    // The fabric stream, when it belongs to this device, keeps the stage
    // copies in the same stream as the caller's other fabric kernels.
    void *fs = impl_->fabricStream();
    void *stream = (fs && gpu::stream_device(fs) == dp->dev) ? fs : dp->stream;
    p->wait_value = ++dp->seq;
    gpu::set_device(dp->dev);
    const int e = kern::copy_batch(&d, 1, 0, stream, dp->status, nullptr, kern::kModeAuto, nullptr, 0,
                                   &dp->done[p->slab], p->wait_value, &dp->ctr[p->slab]);
    if (e != 0) {
        MPCOMM_LOG_ERROR("MPComm: device staging copy on GPU %d failed to launch: %s\n", dp->dev,
                         gpu::error_string(e));
        return false;
    }
    p->launched = std::chrono::steady_clock::now();
    return true;
}

int StagingEngine::poll_device_copy(Piece *p) {
    DevicePool *dp = p->pool;
    if (__atomic_load_n(&dp->done[p->slab], __ATOMIC_ACQUIRE) >= p->wait_value) return 1;
    if (std::chrono::steady_clock::now() - p->launched < kDeviceCopyCheckAfter) return 0;
    // Long overdue: a sticky device error stops every later launch too.
    gpu::set_device(dp->dev);
    const int e = gpu::last_error_clear();
    if (e != 0) {
        MPCOMM_LOG_ERROR("MPComm: device staging copy on GPU %d failed: %s\n", dp->dev, gpu::error_string(e));
        return -1;
    }
    p->launched = std::chrono::steady_clock::now();
    return 0;
}

// Advances every piece of `s` by at most one state. True when it progressed.
bool StagingEngine::step(Staged *s) {
    bool progress = false;
    char *slabs = static_cast<char *>(slab_base_);
    const bool outbound = s->dir != Direction::kGather;
    auto fail = [&](Piece *p) {
        s->error = MPCOMM_ERR_TRANSFER;
        if (p->pool) p->pool->free.push_back(p->slab);
        else free_slabs_.push_back(p->slab);
        p->state = kDone;
        ++s->done;
        progress = true;
    };
    for (auto &up : s->pieces) {
        Piece *p = up.get();
        DevicePool *dp = p->pool;
        char *slab = dp ? nullptr : slabs + static_cast<size_t>(std::max(p->slab, 0)) * slab_bytes_;
        switch (p->state) {
            case kWaitSlab: {
                std::vector<int> &fl = dp ? dp->free : free_slabs_;
                if (fl.empty()) break;
                p->slab = fl.back();
                fl.pop_back();
                const uintptr_t slab_addr =
                    dp ? reinterpret_cast<uintptr_t>(dp->base) + static_cast<size_t>(p->slab) * dp->slab_bytes
                       : reinterpret_cast<uintptr_t>(slabs + static_cast<size_t>(p->slab) * slab_bytes_);
                if (outbound) {
                    p->state = kCopyIn;
                    if (dp) {
                        if (!launch_device_copy(p, true)) {
                            fail(p);
                            break;
                        }
                    } else {
                        char *hs = reinterpret_cast<char *>(slab_addr);
                        enqueue_copy([p, hs] {
                            std::memcpy(hs, reinterpret_cast<const void *>(p->local), p->len);
                            p->copied.store(true, std::memory_order_release);
                        });
                    }
                } else {
                    p->sub = impl_->submit(slab_addr, {s->t->hosts[p->host]}, {p->remote}, {p->len},
                                           Direction::kGather);
                    if (!p->sub) {
                        fail(p);
                        break;
                    }
                    p->state = kXfer;
                }
                progress = true;
                break;
            }
            case kCopyIn: {
                int st = 0;
                if (dp) st = poll_device_copy(p);
                else st = p->copied.load(std::memory_order_acquire) ? 1 : 0;
                if (st < 0) {
                    fail(p);
                    break;
                }
                if (st == 0) break;
                p->copied.store(false);
                const uintptr_t slab_addr =
                    dp ? reinterpret_cast<uintptr_t>(dp->base) + static_cast<size_t>(p->slab) * dp->slab_bytes
                       : reinterpret_cast<uintptr_t>(slab);
                p->sub = impl_->submit(slab_addr, {s->t->hosts[p->host]}, {p->remote}, {p->len},
                                       Direction::kScatter);
                if (!p->sub) {
                    fail(p);
                    break;
                }
                p->state = kXfer;
                progress = true;
                break;
            }
            case kXfer:
                if (impl_->isTransferComplete(p->sub)) {
                    TransferResult r = impl_->getTransferResult(p->sub);
                    impl_->releaseTransfer(p->sub);
                    if (r.error_code != MPCOMM_SUCCESS) s->error = r.error_code;
                    else s->t->bytes.fetch_add(p->len, std::memory_order_relaxed);
                    if (!outbound && r.error_code == MPCOMM_SUCCESS) {
                        p->state = kCopyOut;
                        if (dp) {
                            if (!launch_device_copy(p, false)) {
                                fail(p);
                                break;
                            }
                        } else {
                            enqueue_copy([p, slab] {
                                std::memcpy(reinterpret_cast<void *>(p->local), slab, p->len);
                                p->copied.store(true, std::memory_order_release);
                            });
                        }
                    } else {
                        if (dp) dp->free.push_back(p->slab);
                        else free_slabs_.push_back(p->slab);
                        p->state = kDone;
                        ++s->done;
                    }
                    progress = true;
                }
                break;
            case kCopyOut: {
                int st = 0;
                if (dp) st = poll_device_copy(p);
                else st = p->copied.load(std::memory_order_acquire) ? 1 : 0;
                if (st < 0) {
                    fail(p);
                    break;
                }
                if (st == 0) break;
                if (dp) dp->free.push_back(p->slab);
                else free_slabs_.push_back(p->slab);
                p->state = kDone;
                ++s->done;
                progress = true;
                break;
            }
            default:
                break;
        }
    }
    return progress;
}

void StagingEngine::orchestrate() {
    while (running_) {
        bool progress = false;
        {
            std::lock_guard<std::mutex> g(mu_);
            while (!incoming_.empty()) {
                active_.push_back(std::move(incoming_.front()));
                incoming_.pop_front();
                progress = true;
            }
        }
        for (size_t i = 0; i < active_.size();) {
            Staged *s = active_[i].get();
            progress |= step(s);
            if (s->done == s->pieces.size()) {
                s->t->error.store(s->error);
                impl_->finishTransfer(s->t.get());
                active_[i] = std::move(active_.back());
                active_.pop_back();
                progress = true;
            } else {
                ++i;
            }
        }
        if (!progress) {
            std::unique_lock<std::mutex> g(mu_);
            cv_.wait_for(g, std::chrono::microseconds(active_.empty() ? 2000 : 20));
        }
    }
}

}  // namespace mpcomm
