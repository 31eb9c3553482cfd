#include "engine/staging.h"

#include <algorithm>
#include <cstring>

#include "mpcomm_log.h"
#include "topo/topology.h"

namespace mpcomm {

enum PieceState { kWaitSlab = 0, kCopyIn, kXfer, kCopyOut, kDone };

struct StagingEngine::Piece {
    size_t host;
    uintptr_t local;
    uintptr_t remote;
    size_t len;
    int state = kWaitSlab;
    int slab = -1;
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

StagingEngine::StagingEngine(MPComm::Impl *impl)
    : impl_(impl),
      slab_bytes_(impl->config().staging_slab_bytes),
      nslabs_(impl->config().staging_slabs),
      nthreads_(impl->config().staging_threads) {}

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
    for (size_t i = 0; i < nthreads_; ++i) copiers_.emplace_back([this] { copy_worker(); });
    orchestrator_ = std::thread([this] { orchestrate(); });
    MPCOMM_LOG_INFO("MPComm: staging pool ready (%zu slabs x %zu B, %zu copy threads)\n", nslabs_,
                    slab_bytes_, nthreads_);
    return true;
}

TransferHandle StagingEngine::submit(uintptr_t local, const std::vector<std::string> &hosts,
                                     const std::vector<uintptr_t> &raddrs,
                                     const std::vector<size_t> &lens, Direction dir) {
    {
        std::lock_guard<std::mutex> g(mu_);
        if (!ensure_slabs()) return INVALID_TRANSFER_HANDLE;
    }
    auto s = std::make_shared<Staged>();
    s->dir = dir;
    s->t = impl_->newCompositeTransfer(dir, local, hosts, raddrs, lens);
    if (!s->t) return INVALID_TRANSFER_HANDLE;
    size_t off = 0;
    for (size_t h = 0; h < hosts.size(); ++h) {
        const size_t base = dir == Direction::kBroadcast ? 0 : off;
        for (size_t p = 0; p < lens[h]; p += slab_bytes_) {
            auto pc = std::make_unique<Piece>();
            pc->host = h;
            pc->local = local + base + p;
            pc->remote = raddrs[h] + p;
            pc->len = std::min(slab_bytes_, lens[h] - p);
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

// Advances every piece of `s` by at most one state. True when it progressed.
bool StagingEngine::step(Staged *s) {
    bool progress = false;
    char *slabs = static_cast<char *>(slab_base_);
    const bool outbound = s->dir != Direction::kGather;
    for (auto &up : s->pieces) {
        Piece *p = up.get();
        switch (p->state) {
            case kWaitSlab: {
                if (free_slabs_.empty()) break;
                p->slab = free_slabs_.back();
                free_slabs_.pop_back();
                char *slab = slabs + static_cast<size_t>(p->slab) * slab_bytes_;
                if (outbound) {
                    p->state = kCopyIn;
                    enqueue_copy([p, slab] {
                        std::memcpy(slab, reinterpret_cast<const void *>(p->local), p->len);
                        p->copied.store(true, std::memory_order_release);
                    });
                } else {
                    p->sub = impl_->submit(reinterpret_cast<uintptr_t>(slab), {s->t->hosts[p->host]},
                                           {p->remote}, {p->len}, Direction::kGather);
                    p->state = p->sub ? kXfer : kDone;
                    if (!p->sub) {
                        s->error = MPCOMM_ERR_TRANSFER;
                        free_slabs_.push_back(p->slab);
                        ++s->done;
                    }
                }
                progress = true;
                break;
            }
            case kCopyIn:
                if (p->copied.load(std::memory_order_acquire)) {
                    p->copied.store(false);
                    char *slab = slabs + static_cast<size_t>(p->slab) * slab_bytes_;
                    p->sub = impl_->submit(reinterpret_cast<uintptr_t>(slab), {s->t->hosts[p->host]},
                                           {p->remote}, {p->len}, Direction::kScatter);
                    if (p->sub) {
                        p->state = kXfer;
                    } else {
                        s->error = MPCOMM_ERR_TRANSFER;
                        free_slabs_.push_back(p->slab);
                        p->state = kDone;
                        ++s->done;
                    }
                    progress = true;
                }
                break;
            case kXfer:
                if (impl_->isTransferComplete(p->sub)) {
                    TransferResult r = impl_->getTransferResult(p->sub);
                    impl_->releaseTransfer(p->sub);
                    if (r.error_code != MPCOMM_SUCCESS) s->error = r.error_code;
                    else s->t->bytes.fetch_add(p->len, std::memory_order_relaxed);
                    if (!outbound && r.error_code == MPCOMM_SUCCESS) {
                        char *slab = slabs + static_cast<size_t>(p->slab) * slab_bytes_;
                        p->state = kCopyOut;
                        enqueue_copy([p, slab] {
                            std::memcpy(reinterpret_cast<void *>(p->local), slab, p->len);
                            p->copied.store(true, std::memory_order_release);
                        });
                    } else {
                        free_slabs_.push_back(p->slab);
                        p->state = kDone;
                        ++s->done;
                    }
                    progress = true;
                }
                break;
            case kCopyOut:
                if (p->copied.load(std::memory_order_acquire)) {
                    free_slabs_.push_back(p->slab);
                    p->state = kDone;
                    ++s->done;
                    progress = true;
                }
                break;
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
