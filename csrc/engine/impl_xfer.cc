// Transfer submission, the worker hot loop and the completion API.
// Parity: reference src/mpcomm.cpp:4929-5479 (submit), :5969-7061 (worker),
// :7213-7357 (completion routing), :5563-5740 (completion API),
// :7068-7155 (quarantine probe), :5802-5929 (fault injection).
#include <sys/prctl.h>

#include <algorithm>
#include <cstring>
#include <limits>
#include <thread>

#include "core/nvtx.h"
#include "cuda/gpu.h"
#include "engine/impl.h"
#include "engine/staging.h"
#include "mpcomm_log.h"
#include "topo/topology.h"

namespace mpcomm {

namespace {
constexpr size_t kMaxChunk = 1ull << 30;  // WR length is 32-bit
const char *dir_name(Direction d) {
    return d == Direction::kScatter ? "Scatter" : d == Direction::kGather ? "Gather" : "Broadcast";
}
}  // namespace

size_t MPComm::Impl::effectiveChunk(const std::vector<size_t> &cand) const {
    size_t c = throttle_chunk_.load(std::memory_order_relaxed);
    if (c == 0) {
        c = std::numeric_limits<size_t>::max();
        for (size_t r : cand) c = std::min(c, rails_[r]->rail->preferred_chunk(cfg_));
        if (c == std::numeric_limits<size_t>::max()) c = cfg_.max_rdma_transfer_size;
    }
    return std::max<size_t>(1, std::min(c, kMaxChunk));
}

std::shared_ptr<Transfer> MPComm::Impl::findTransfer(TransferHandle h) const {
    std::lock_guard<std::mutex> g(xfer_mu_);
    auto it = transfers_.find(h);
    return it == transfers_.end() ? nullptr : it->second;
}

TransferHandle MPComm::Impl::submit(uintptr_t local, const std::vector<std::string> &hosts,
                                    const std::vector<uintptr_t> &raddrs,
                                    const std::vector<size_t> &lens, Direction dir) {
    const char *op = dir_name(dir);
    if (!initialized_) {
        MPCOMM_LOG_ERROR("MPComm: %sAsync failed - not initialized\n", op);
        return INVALID_TRANSFER_HANDLE;
    }
    if (hosts.empty() || raddrs.size() != hosts.size() || lens.size() != hosts.size()) {
        MPCOMM_LOG_ERROR("MPComm: %sAsync failed - invalid arguments\n", op);
        return INVALID_TRANSFER_HANDLE;
    }
    if (rails_.empty()) {
        MPCOMM_LOG_ERROR("MPComm: %sAsync failed - no rails available\n", op);
        return INVALID_TRANSFER_HANDLE;
    }
    size_t span = 0;
    for (size_t l : lens) span = dir == Direction::kBroadcast ? std::max(span, l) : span + l;
    Region region;
    const bool registered = span == 0 || lookupRegion(local, span, &region);
    if (!registered) {
        if (cfg_.staging_enable && staging_) return staging_->submit(local, hosts, raddrs, lens, dir);
        MPCOMM_LOG_ERROR("MPComm: %sAsync failed - local buffer 0x%lx+%zu not registered\n", op,
                         static_cast<unsigned long>(local), span);
        return INVALID_TRANSFER_HANDLE;
    }
    auto t = std::make_shared<Transfer>();
    t->t_start = Clock::now();
    t->dir = dir;
    t->op = dir == Direction::kGather ? fabric::Opcode::kRead : fabric::Opcode::kWrite;
    t->local_addr = local;
    t->hosts = hosts;
    t->remote_addrs = raddrs;
    t->lengths = lens;
    for (auto &h : hosts) {
        auto c = connection(h);
        if (!c) {
            MPCOMM_LOG_ERROR("MPComm: %sAsync failed - not connected to %s\n", op, h.c_str());
            return INVALID_TRANSFER_HANDLE;
        }
        t->conns.push_back(c);
    }
    t->handle = handles_.allocate();
    if (t->handle == INVALID_TRANSFER_HANDLE) {
        MPCOMM_LOG_ERROR("MPComm: %sAsync failed - handle pool exhausted (65535 live handles; "
                         "release finished transfers)\n", op);
        return INVALID_TRANSFER_HANDLE;
    }
    t->local_gpu = region.gpu;
    if (nvtx::enabled()) {
        size_t total = 0;
        for (size_t l : lens) total += l;
        char msg[96];
        std::snprintf(msg, sizeof(msg), "mpcomm %s %zu B x%zu #%lu", op, total, hosts.size(),
                      static_cast<unsigned long>(t->handle));
        t->nvtx = nvtx::start(msg);
    }
    if (cfg_.pcie_stat_enable && dir != Direction::kGather) {
        t->remote_gpu.resize(hosts.size(), -1);
        for (size_t i = 0; i < hosts.size(); ++i) t->remote_gpu[i] = t->conns[i]->remote_gpu_for(raddrs[i]);
    }
    // Candidate rails: PCIe-affine to the local GPU buffer, else NUMA-local,
    // else all; quarantined rails dropped unless that empties the set.
    std::vector<size_t> cand = region.affine_rails;
    // PXN (NVLink proxy rails): a GPU buffer moving to or from host memory
    // is striped over every GPU's rail — peers read/write the buffer over
    // NVLink and cross their own PCIe links — instead of only its own link
    // (the reference routes SCATTERs through a proxy GPU's NIC the same way,
    // src/mpcomm.cpp:5135-5403).
    if (cfg_.pxn_enable && region.gpu >= 0 && !cand.empty()) {
        bool host_side = true;
        for (size_t i = 0; i < hosts.size(); ++i) host_side &= t->conns[i]->remote_gpu_for(raddrs[i]) < 0;
        if (host_side) {
            cand.clear();
            for (size_t i = 0; i < rails_.size(); ++i)
                if (rails_[i]->gpu >= 0) cand.push_back(i);
        }
    }
    if (cand.empty()) cand = localNicsForNuma(region.numa);
    if (cand.empty())
        for (size_t i = 0; i < rails_.size(); ++i) cand.push_back(i);
    std::vector<size_t> healthy;
    for (size_t r : cand)
        if (!rails_[r]->quarantined.load(std::memory_order_relaxed)) healthy.push_back(r);
    if (!healthy.empty()) cand.swap(healthy);
    t->candidates = cand;
    size_t chunk = effectiveChunk(cand);
    // Fused broadcast: when one candidate rail reaches every destination and
    // can write them all in one device operation (GPU fabric: a gather_bcast
    // launch per chunk that reads each source tile once; NVLS multicast
    // stores when the destinations form one multicast group), each chunk is
    // posted once as a one-to-many WRITE instead of once per destination
    // (the reference posts one RDMA WRITE per host, src/mpcomm.cpp:4937-4954).
    if (dir == Direction::kBroadcast && cfg_.fused_broadcast) {
        for (size_t r : cand) {
            fabric::Rail *rl = rails_[r]->rail.get();
            const size_t al = std::max<size_t>(1, rl->fanout_alignment());
            if (hosts.size() > rl->max_fanout() || chunk < al) continue;
            bool ok = local % al == 0 && lens[0] % al == 0;
            for (size_t i = 0; ok && i < hosts.size(); ++i)
                ok = lens[i] == lens[0] && raddrs[i] % al == 0 && t->conns[i]->group_for(r) != nullptr;
            if (!ok) continue;
            t->fanout = true;
            t->fanout_rail = r;
            t->host_source = region.gpu < 0;
            chunk -= chunk % al;
            break;
        }
    }
    if (t->fanout)
        t->plan.build(local, {raddrs[0]}, {lens[0]}, chunk, true);
    else
        t->plan.build(local, raddrs, lens, chunk, dir == Direction::kBroadcast);
    size_t ol = throttle_outstanding_.load(std::memory_order_relaxed);
    if (ol == 0) ol = rails_[cand[0]]->rail->preferred_outstanding(cfg_);
    t->outstanding_limit = std::max<size_t>(1, ol);
    t->repost_budget = t->plan.total() + 16;
    t->owner = numaForAddr(local) % static_cast<int>(std::max<size_t>(1, workers_.size()));
    t->numa = t->owner;
    t->t_queued = Clock::now();
    const uint64_t h = t->handle;
    {
        std::lock_guard<std::mutex> g(xfer_mu_);
        transfers_[h] = t;
    }
    handle_table_[h].store(t.get(), std::memory_order_release);
    if (t->plan.total() == 0) {
        t->t_worker = t->t_first_post = t->t_all_posted = Clock::now();
        finishTransfer(t.get());
        return h;
    }
    {
        std::lock_guard<std::mutex> g(admit_mu_);
        admit_[h] = t;
    }
    Worker *w = workers_[t->owner].get();
    while (!w->queue.try_push(h)) cpu_relax();
    wakeWorker(w);
    return h;
}

// Paged PUT (the fused PXN gather + forward as a transfer): the GPU that
// holds `indices` gathers the pages from the pool and stores them into the
// remote range, one launch per chunk of pages, on its own rail.
TransferHandle MPComm::Impl::submitPaged(uintptr_t pool, const int64_t *indices, int n, int bs,
                                         const std::string &host, uintptr_t raddr) {
    if (!initialized_ || !pool || !indices || n <= 0 || bs <= 0) {
        MPCOMM_LOG_ERROR("MPComm: putPagesAsync failed - invalid arguments\n");
        return INVALID_TRANSFER_HANDLE;
    }
    auto conn = connection(host);
    if (!conn) {
        MPCOMM_LOG_ERROR("MPComm: putPagesAsync failed - not connected to %s\n", host.c_str());
        return INVALID_TRANSFER_HANDLE;
    }
    const int gpu = gpu::device_of(indices);
    size_t rail = SIZE_MAX;
    for (size_t r = 0; r < rails_.size(); ++r)
        if (rails_[r]->gpu == gpu && gpu >= 0 && rails_[r]->rail->supports_paged() && conn->group_for(r)) rail = r;
    if (rail == SIZE_MAX) {
        MPCOMM_LOG_ERROR("MPComm: putPagesAsync failed - the indices must be device memory of a GPU whose "
                         "fabric rail is connected to %s (GPU fabric; MPCOMM_PXN_ENABLE=1 opens a rail per GPU)\n",
                         host.c_str());
        return INVALID_TRANSFER_HANDLE;
    }
    auto t = std::make_shared<Transfer>();
    t->t_start = Clock::now();
    t->dir = Direction::kScatter;
    t->op = fabric::Opcode::kWrite;
    t->paged = true;
    t->paged_rail = rail;
    t->pool = pool;
    t->indices = indices;
    t->page_bytes = static_cast<uint32_t>(bs);
    {
        // Index bound from the DRAM mapping that holds the pool, if known.
        std::lock_guard<std::mutex> g(map_mu_);
        for (auto &kv : mappings_) {
            const uintptr_t d0 = kv.second.dev_ptr, d1 = d0 + kv.second.len;
            if (pool >= d0 && pool < d1) t->pool_pages = (d1 - pool) / static_cast<uintptr_t>(bs);
        }
    }
    const size_t total = static_cast<size_t>(n) * static_cast<size_t>(bs);
    t->local_addr = 0;
    t->hosts = {host};
    t->remote_addrs = {raddr};
    t->lengths = {total};
    t->conns = {conn};
    t->candidates = {rail};
    t->local_gpu = gpu;
    t->host_source = gpu::device_of(reinterpret_cast<const void *>(pool)) < 0;
    // Pages per launch: MPCOMM_PAGED_CHUNK_SIZE bytes (default the 1 GiB WR
    // limit). Launches of one stream run one after another anyway, so fewer,
    // larger ones only save launch and completion latency.
    t->pages_per_chunk =
        std::max<size_t>(1, std::min(cfg_.paged_chunk_size, kMaxChunk) / static_cast<size_t>(bs));
    t->plan.build(0, {raddr}, {total}, t->pages_per_chunk * static_cast<size_t>(bs), false);
    size_t ol = throttle_outstanding_.load(std::memory_order_relaxed);
    if (ol == 0) ol = rails_[rail]->rail->preferred_outstanding(cfg_);
    t->outstanding_limit = std::max<size_t>(1, ol);
    t->repost_budget = t->plan.total() + 16;
    t->handle = handles_.allocate();
    if (t->handle == INVALID_TRANSFER_HANDLE) {
        MPCOMM_LOG_ERROR("MPComm: putPagesAsync failed - handle pool exhausted\n");
        return INVALID_TRANSFER_HANDLE;
    }
    t->owner = rails_[rail]->numa % static_cast<int>(std::max<size_t>(1, workers_.size()));
    t->numa = t->owner;
    t->t_queued = Clock::now();
    const uint64_t h = t->handle;
    {
        std::lock_guard<std::mutex> g(xfer_mu_);
        transfers_[h] = t;
    }
    handle_table_[h].store(t.get(), std::memory_order_release);
    {
        std::lock_guard<std::mutex> g(admit_mu_);
        admit_[h] = t;
    }
    Worker *w = workers_[t->owner].get();
    while (!w->queue.try_push(h)) cpu_relax();
    wakeWorker(w);
    return h;
}

void MPComm::Impl::wakeWorker(Worker *w) {
    w->doorbell.fetch_add(1);  // seq_cst: ordered against the worker's `sleeping` store
    if (w->sleeping.load()) {
        std::lock_guard<std::mutex> g(w->wake_mu);
        w->wake_cv.notify_one();
    }
}

std::shared_ptr<Transfer> MPComm::Impl::newCompositeTransfer(Direction dir, uintptr_t local,
                                                             const std::vector<std::string> &hosts,
                                                             const std::vector<uintptr_t> &raddrs,
                                                             const std::vector<size_t> &lens) {
    auto t = std::make_shared<Transfer>();
    t->t_start = Clock::now();
    t->dir = dir;
    t->composite = true;
    t->local_addr = local;
    t->hosts = hosts;
    t->remote_addrs = raddrs;
    t->lengths = lens;
    t->handle = handles_.allocate();
    if (t->handle == INVALID_TRANSFER_HANDLE) return nullptr;
    std::lock_guard<std::mutex> g(xfer_mu_);
    transfers_[t->handle] = t;
    handle_table_[t->handle].store(t.get(), std::memory_order_release);
    return t;
}

// ---------------------------------------------------------------------------
// Worker
// ---------------------------------------------------------------------------
void MPComm::Impl::workerLoop(Worker *w) {
    topo::bind_thread_to_cpus(topo::numa_cpus(w->numa));
    // Short sleeps of this thread should be short: the default 50 us timer
    // slack would stretch the 20 us poll sleep to ~70 us.
    prctl(PR_SET_TIMERSLACK, 1000UL, 0, 0, 0);
    std::vector<fabric::WorkCompletion> wcs(std::max<size_t>(cfg_.poll_batch_size, 1));
    std::vector<fabric::QueuePair *> touched;
    std::vector<fabric::WorkCompletion> inbox;
    size_t idle = 0;
    while (running_.load(std::memory_order_acquire)) {
        bool progress = false;
        ++w->loops;

        // Phase 1: admit newly submitted transfers.
        uint64_t h;
        while (w->queue.try_pop(&h)) {
            std::shared_ptr<Transfer> sp;
            {
                std::lock_guard<std::mutex> g(admit_mu_);
                auto it = admit_.find(h);
                if (it == admit_.end()) continue;
                sp = std::move(it->second);
                admit_.erase(it);
            }
            sp->t_worker = Clock::now();
            w->active.push_back(std::move(sp));
            progress = true;
        }

        // Throttle epoch: record when this worker observed a new policy and
        // the WQE watermark that must drain (reference :6454-6508).
        const uint64_t ep = throttle_epoch_.load(std::memory_order_acquire);
        if (ep != w->seen_epoch) {
            w->seen_epoch = ep;
            if (throttle_drain_pending_.load(std::memory_order_relaxed)) {
                size_t outstanding = 0;
                for (size_t r = 0; r < rails_.size(); ++r) {
                    outstanding += w->rail_posted[r] - w->rail_completed[r];
                    w->drain_mark[r] = w->rail_posted[r];
                }
                uint64_t zero = 0;
                throttle_seen_ns_.compare_exchange_strong(zero, monotonic_raw_ns());
                throttle_snapshot_.store(outstanding, std::memory_order_relaxed);
                w->drain_armed = true;
            }
        }

        // Phase 2: post chunks under flow control, one doorbell per QP.
        touched.clear();
        for (auto &sp : w->active) postChunks(w, sp.get(), &touched);
        for (auto *qp : touched) qp->flush();
        if (!touched.empty()) progress = true;

        // Phase 3: completions (own rails' CQs + forwarded ones).
        for (auto &slot : rails_) {
            int n = slot->rail->poll(wcs.data(), static_cast<int>(wcs.size()));
            for (int i = 0; i < n; ++i) handleCompletion(w, wcs[i]);
            if (n > 0) progress = true;
        }
        if (w->inbox_nonempty.load(std::memory_order_acquire)) {
            {
                std::lock_guard<std::mutex> g(w->inbox_mu);
                inbox.swap(w->inbox);
                w->inbox_nonempty.store(false, std::memory_order_release);
            }
            for (auto &wc : inbox) handleCompletion(w, wc);
            inbox.clear();
            progress = true;
        }
        if (w->drain_armed) {
            bool drained = true;
            for (size_t r = 0; r < rails_.size(); ++r)
                if (w->rail_completed[r] < w->drain_mark[r]) drained = false;
            if (drained) {
                w->drain_armed = false;
                uint64_t zero = 0;
                throttle_drained_ns_.compare_exchange_strong(zero, monotonic_raw_ns());
                throttle_drain_pending_.store(false, std::memory_order_relaxed);
            }
        }

        // Phase 4: retire finished transfers.
        retire(w);

        // Phase 5: maintenance on worker 0.
        if (w->id == 0) {
            if (w->loops % cfg_.nic_probe_interval == 0) probeQuarantine();
            maybeInjectFault();
        }

        if (progress) {
            idle = 0;
        } else if (++idle > cfg_.max_idle_spins) {
            if (w->active.empty()) {
                // Nothing in flight: sleep until a submission or a forwarded
                // completion rings the doorbell (1 ms cap for maintenance).
                const uint64_t seen = w->doorbell.load();
                w->sleeping.store(true);
                {
                    std::unique_lock<std::mutex> lk(w->wake_mu);
                    w->wake_cv.wait_for(lk, std::chrono::milliseconds(1), [&] {
                        return w->doorbell.load() != seen || !running_.load(std::memory_order_acquire);
                    });
                }
                w->sleeping.store(false);
            } else {
                // Waiting on completions: poll every ~20 us.
                std::this_thread::sleep_for(std::chrono::microseconds(20));
            }
        } else {
            cpu_relax();
        }
    }
    // Shutdown: whatever is still active fails.
    for (auto &sp : w->active) {
        if (!sp->finished.load()) {
            int expect = 0;
            sp->error.compare_exchange_strong(expect, MPCOMM_ERR_TRANSFER);
            finishTransfer(sp.get());
        }
    }
    w->active.clear();
}

void MPComm::Impl::postFanoutChunks(Worker *w, Transfer *t, std::vector<fabric::QueuePair *> *touched) {
    const size_t total = t->plan.total();
    const size_t nh = t->hosts.size();
    std::vector<fabric::FanoutTarget> targets(nh);
    while (true) {
        size_t chunk;
        bool from_retry = false;
        if (!t->retry.empty()) {
            chunk = t->retry.front();
            from_retry = true;
        } else if (t->next_chunk < total) {
            chunk = t->next_chunk;
        } else {
            break;
        }
        const size_t r = t->fanout_rail;
        if (rails_[r]->quarantined.load(std::memory_order_relaxed)) {
            // Move the rest of the broadcast to another healthy rail that
            // reaches every destination in one operation (the re-post rule
            // of plain WRs); fail only when there is none.
            size_t alt = SIZE_MAX;
            for (size_t c2 : t->candidates) {
                if (c2 == r || rails_[c2]->quarantined.load(std::memory_order_relaxed) ||
                    rails_[c2]->rail->max_fanout() < nh)
                    continue;
                bool all = true;
                for (size_t i = 0; all && i < nh; ++i) all = t->conns[i]->group_for(c2) != nullptr;
                if (all) {
                    alt = c2;
                    break;
                }
            }
            if (alt == SIZE_MAX) {
                t->error.store(MPCOMM_ERR_TRANSFER);
                t->aborted = true;
                break;
            }
            MPCOMM_LOG_WARN("MPComm: fused broadcast #%lu moves from %s to %s\n",
                            static_cast<unsigned long>(t->handle), rails_[r]->name.c_str(),
                            rails_[alt]->name.c_str());
            t->fanout_rail = alt;
            continue;
        }
        const Chunk c = t->plan.get(chunk);
        QpGroup *g0 = t->conns[0]->group_for(r);
        if (!g0 || g0->qps.empty()) {
            t->error.store(MPCOMM_ERR_CONNECTION);
            t->aborted = true;
            break;
        }
        const size_t rail_out = w->rail_posted[r] - w->rail_completed[r];
        if (rail_out >= t->outstanding_limit * std::min(cfg_.qps_per_connection, g0->qps.size())) break;
        size_t q = SIZE_MAX, q_out = SIZE_MAX;
        const size_t nq = std::min(g0->qps.size(), kMaxQpsPerRail);
        for (size_t i = 0; i < nq; ++i) {
            const size_t out = w->qp_posted[r][i] - w->qp_completed[r][i];
            if (out < t->outstanding_limit && out < q_out) {
                q = i;
                q_out = out;
            }
        }
        if (q == SIZE_MAX) break;
        const size_t off = c.remote_addr - t->remote_addrs[0];
        bool deferred = false, missing = false;
        for (size_t i = 0; i < nh; ++i) {
            QpGroup *g = t->conns[i]->group_for(r);
            const uintptr_t ra = t->remote_addrs[i] + off;
            if (!g || g->qps.empty()) {
                missing = true;
                break;
            }
            if (!qosAllowRemoteWrite(*t->conns[i], ra, c.length)) {
                deferred = true;
                break;
            }
            targets[i].qp = g->qps[std::min(q, g->qps.size() - 1)].get();
            targets[i].remote_addr = ra;
            targets[i].rkey = t->conns[i]->rkey_for(ra, g->remote_rail);
            if (targets[i].rkey == 0) missing = true;
        }
        if (deferred) break;
        if (missing) {
            MPCOMM_LOG_ERROR("MPComm: fused broadcast: no connection or rkey for a destination (query the peers' "
                             "buffers first)\n");
            t->error.store(MPCOMM_ERR_MEMORY);
            t->aborted = true;
            break;
        }
        if (!t->lkey_ok[r]) {
            Region reg;
            if (!lookupRegion(c.local_addr, c.length, &reg) || r >= reg.keys.size()) {
                t->error.store(MPCOMM_ERR_MEMORY);
                t->aborted = true;
                break;
            }
            t->lkeys[r] = reg.keys[r];
            t->lkey_ok[r] = true;
        }
        fabric::WorkRequest wr;
        wr.wr_id = WrId::encode(r, q, t->handle, chunk);
        wr.op = fabric::Opcode::kWrite;
        wr.local_addr = c.local_addr;
        wr.lkey = t->lkeys[r].lkey;
        wr.remote_addr = 0;
        wr.rkey = 0;
        wr.length = static_cast<uint32_t>(c.length);
        // A host-memory source is an H2D read on the rail's GPU: it gets a QoS
        // window like tmaGather, so READ posts on that GPU's rails yield.
        kern::H2DWindow *win = nullptr;
        uint32_t *wctr = nullptr;
        if (t->host_source) acquireH2DWindow(rails_[r]->gpu, &win, &wctr);
        fabric::QueuePair *qp = g0->qps[q].get();
        if (qp->post_fanout(wr, targets.data(), nh, win) != 0) {
            if (win) __atomic_store_n(&win->armed, 0u, __ATOMIC_RELEASE);
            MPCOMM_LOG_ERROR("MPComm: fused broadcast post failed on %s\n", rails_[r]->name.c_str());
            t->error.store(MPCOMM_ERR_TRANSFER);
            t->aborted = true;
            break;
        }
        ++w->rail_posted[r];
        ++w->qp_posted[r][q];
        ++t->in_flight;
        if (from_retry) t->retry.pop_front();
        else ++t->next_chunk;
        if (std::find(touched->begin(), touched->end(), qp) == touched->end()) touched->push_back(qp);
        if (!t->first_posted) {
            t->first_posted = true;
            t->t_first_post = Clock::now();
        }
        if (t->next_chunk == total && t->retry.empty()) t->t_all_posted = Clock::now();
    }
}

void MPComm::Impl::postPagedChunks(Worker *w, Transfer *t, std::vector<fabric::QueuePair *> *touched) {
    const size_t total = t->plan.total();
    const size_t r = t->paged_rail;
    while (true) {
        size_t chunk;
        bool from_retry = false;
        if (!t->retry.empty()) {
            chunk = t->retry.front();
            from_retry = true;
        } else if (t->next_chunk < total) {
            chunk = t->next_chunk;
        } else {
            break;
        }
        if (rails_[r]->quarantined.load(std::memory_order_relaxed)) {
            // Only the GPU holding the indices can run the gather.
            t->error.store(MPCOMM_ERR_TRANSFER);
            t->aborted = true;
            break;
        }
        const Chunk c = t->plan.get(chunk);
        QpGroup *g = t->conns[0]->group_for(r);
        if (!g || g->qps.empty()) {
            t->error.store(MPCOMM_ERR_CONNECTION);
            t->aborted = true;
            break;
        }
        const size_t rail_out = w->rail_posted[r] - w->rail_completed[r];
        if (rail_out >= t->outstanding_limit * std::min(cfg_.qps_per_connection, g->qps.size())) break;
        size_t q = SIZE_MAX, q_out = SIZE_MAX;
        const size_t nq = std::min(g->qps.size(), kMaxQpsPerRail);
        for (size_t i = 0; i < nq; ++i) {
            const size_t out = w->qp_posted[r][i] - w->qp_completed[r][i];
            if (out < t->outstanding_limit && out < q_out) {
                q = i;
                q_out = out;
            }
        }
        if (q == SIZE_MAX) break;
        if (!qosAllowRemoteWrite(*t->conns[0], c.remote_addr, c.length)) break;
        fabric::PagedWrite pw;
        pw.wr_id = WrId::encode(r, q, t->handle, chunk);
        pw.pool = t->pool;
        pw.pool_pages = t->pool_pages;
        pw.indices = t->indices + chunk * t->pages_per_chunk;
        pw.count = static_cast<uint32_t>(c.length / t->page_bytes);
        pw.page_bytes = t->page_bytes;
        pw.remote_addr = c.remote_addr;
        pw.rkey = t->conns[0]->rkey_for(c.remote_addr, g->remote_rail);
        if (pw.rkey == 0) {
            MPCOMM_LOG_ERROR("MPComm: no rkey for remote 0x%lx on %s (query the peer's buffers first)\n",
                             static_cast<unsigned long>(c.remote_addr), t->conns[0]->host_id.c_str());
            t->error.store(MPCOMM_ERR_MEMORY);
            t->aborted = true;
            break;
        }
        kern::H2DWindow *win = nullptr;
        uint32_t *wctr = nullptr;
        if (t->host_source) acquireH2DWindow(rails_[r]->gpu, &win, &wctr);
        pw.h2d_window = win;
        fabric::QueuePair *qp = g->qps[q].get();
        if (qp->post_paged(pw) != 0) {
            if (win) __atomic_store_n(&win->armed, 0u, __ATOMIC_RELEASE);
            t->error.store(MPCOMM_ERR_TRANSFER);
            t->aborted = true;
            break;
        }
        ++w->rail_posted[r];
        ++w->qp_posted[r][q];
        ++t->in_flight;
        if (from_retry) t->retry.pop_front();
        else ++t->next_chunk;
        if (std::find(touched->begin(), touched->end(), qp) == touched->end()) touched->push_back(qp);
        if (!t->first_posted) {
            t->first_posted = true;
            t->t_first_post = Clock::now();
        }
        if (t->next_chunk == total && t->retry.empty()) t->t_all_posted = Clock::now();
    }
}

void MPComm::Impl::postChunks(Worker *w, Transfer *t, std::vector<fabric::QueuePair *> *touched) {
    if (t->finished.load(std::memory_order_relaxed) || t->aborted) return;
    if (t->fanout) {
        postFanoutChunks(w, t, touched);
        return;
    }
    if (t->paged) {
        postPagedChunks(w, t, touched);
        return;
    }
    const size_t total = t->plan.total();
    const size_t qps_cap = cfg_.qps_per_connection;
    while (true) {
        size_t chunk;
        bool from_retry = false;
        if (!t->retry.empty()) {
            chunk = t->retry.front();
            from_retry = true;
        } else if (t->next_chunk < total) {
            chunk = t->next_chunk;
        } else {
            break;
        }
        const Chunk c = t->plan.get(chunk);
        const auto &conn = t->conns[c.host_idx];

        // Rail: least outstanding healthy candidate with a connected group.
        size_t best = SIZE_MAX, best_out = SIZE_MAX;
        QpGroup *best_group = nullptr;
        bool all_quarantined = true;
        for (size_t r : t->candidates)
            if (!rails_[r]->quarantined.load(std::memory_order_relaxed)) all_quarantined = false;
        for (size_t r : t->candidates) {
            if (!all_quarantined && rails_[r]->quarantined.load(std::memory_order_relaxed)) continue;
            QpGroup *g = conn->group_for(r);
            if (!g || g->qps.empty()) continue;
            const size_t out = w->rail_posted[r] - w->rail_completed[r];
            const size_t cap = t->outstanding_limit * std::min(qps_cap, g->qps.size());
            if (out < cap && out < best_out) {
                best = r;
                best_out = out;
                best_group = g;
            }
        }
        if (best == SIZE_MAX) {
            bool any_group = false;
            for (size_t r : t->candidates) any_group |= conn->group_for(r) != nullptr;
            if (!any_group) {
                MPCOMM_LOG_ERROR("MPComm: no connected rail to %s among the transfer's candidates\n",
                                 conn->host_id.c_str());
                t->error.store(MPCOMM_ERR_CONNECTION);
                t->aborted = true;
            }
            break;
        }
        // QP: least outstanding below the per-QP limit.
        size_t q = SIZE_MAX, q_out = SIZE_MAX;
        const size_t nq = std::min(best_group->qps.size(), kMaxQpsPerRail);
        for (size_t i = 0; i < nq; ++i) {
            const size_t out = w->qp_posted[best][i] - w->qp_completed[best][i];
            if (out < t->outstanding_limit && out < q_out) {
                q = i;
                q_out = out;
            }
        }
        if (q == SIZE_MAX) break;
        if (t->op == fabric::Opcode::kWrite && !qosAllowRemoteWrite(*conn, c.remote_addr, c.length)) break;
        if (!qosAllowPost(*t, best, c.length)) {
            const int dom = t->local_gpu;
            if (cfg_.pcie_stat_enable && dom >= 0 && dom < static_cast<int>(kMaxGpuDomains))
                pcie_[dom].defer_count.fetch_add(1, std::memory_order_relaxed);
            break;
        }
        if (!t->lkey_ok[best]) {
            Region reg;
            if (!lookupRegion(c.local_addr, c.length, &reg) || best >= reg.keys.size()) {
                MPCOMM_LOG_ERROR("MPComm: lkey lookup failed for 0x%lx on %s\n",
                                 static_cast<unsigned long>(c.local_addr), rails_[best]->name.c_str());
                t->error.store(MPCOMM_ERR_MEMORY);
                t->aborted = true;
                break;
            }
            t->lkeys[best] = reg.keys[best];
            t->lkey_ok[best] = true;
        }
        const uint32_t rkey = conn->rkey_for(c.remote_addr, best_group->remote_rail);
        if (rkey == 0) {
            MPCOMM_LOG_ERROR("MPComm: no rkey for remote 0x%lx on %s (query the peer's buffers or "
                             "call updateRemoteMemoryInfo)\n",
                             static_cast<unsigned long>(c.remote_addr), conn->host_id.c_str());
            t->error.store(MPCOMM_ERR_MEMORY);
            t->aborted = true;
            break;
        }
        fabric::WorkRequest wr;
        wr.wr_id = WrId::encode(best, q, t->handle, chunk);
        wr.op = t->op;
        wr.local_addr = c.local_addr;
        wr.lkey = t->lkeys[best].lkey;
        wr.remote_addr = c.remote_addr;
        wr.rkey = rkey;
        wr.length = static_cast<uint32_t>(c.length);
        fabric::QueuePair *qp = best_group->qps[q].get();
        const int dom = t->op == fabric::Opcode::kRead
                            ? t->local_gpu
                            : (t->remote_gpu.empty() ? -1 : t->remote_gpu[c.host_idx]);
        if (cfg_.pcie_stat_enable) pcieOnPosted(dom, c.length);
        if (qp->post(&wr, 1) != 0) {
            if (cfg_.pcie_stat_enable) pcieOnCompleted(dom, c.length);
            quarantine(best, fabric::kWcGeneralErr);
            if (!cfg_.repost_on_failure || t->repost_budget == 0) {
                t->error.store(MPCOMM_ERR_TRANSFER);
                t->aborted = true;
                break;
            }
            --t->repost_budget;
            continue;  // the rail is quarantined now; retry picks another
        }
        ++w->rail_posted[best];
        ++w->qp_posted[best][q];
        ++t->in_flight;
        if (from_retry) t->retry.pop_front();
        else ++t->next_chunk;
        if (std::find(touched->begin(), touched->end(), qp) == touched->end()) touched->push_back(qp);
        if (!t->first_posted) {
            t->first_posted = true;
            t->t_first_post = Clock::now();
        }
        if (t->next_chunk == total && t->retry.empty()) t->t_all_posted = Clock::now();
    }
}

void MPComm::Impl::handleCompletion(Worker *w, const fabric::WorkCompletion &wc) {
    const uint64_t h = WrId::handle(wc.wr_id);
    const size_t rail = WrId::rail(wc.wr_id), q = WrId::qp(wc.wr_id), chunk = WrId::chunk(wc.wr_id);
    Transfer *t = handle_table_[h].load(std::memory_order_acquire);
    if (!t || t->composite || rail >= rails_.size() || q >= kMaxQpsPerRail) return;  // orphan
    if (t->owner != w->id) {
        Worker *o = workers_[t->owner].get();
        {
            std::lock_guard<std::mutex> g(o->inbox_mu);
            o->inbox.push_back(wc);
            o->inbox_nonempty.store(true, std::memory_order_release);
        }
        wakeWorker(o);
        return;
    }
    ++w->rail_completed[rail];
    ++w->qp_completed[rail][q];
    if (t->in_flight) --t->in_flight;
    const Chunk c = t->plan.get(chunk);
    const int dom = t->op == fabric::Opcode::kRead
                        ? t->local_gpu
                        : (t->remote_gpu.empty() ? -1 : t->remote_gpu[c.host_idx]);
    if (cfg_.pcie_stat_enable && !t->fanout && !t->paged) pcieOnCompleted(dom, c.length);
    if (wc.status == fabric::kWcSuccess || cfg_.fault_tolerate) {
        // A fused broadcast chunk wrote its bytes to every destination.
        const uint64_t moved = t->fanout ? c.length * t->hosts.size() : c.length;
        t->bytes.fetch_add(moved, std::memory_order_relaxed);
        t->rail_bytes[rail].fetch_add(moved, std::memory_order_relaxed);
        t->done_chunks.fetch_add(1, std::memory_order_relaxed);
        nic_completed_bytes_.fetch_add(moved, std::memory_order_relaxed);
        rails_[rail]->completed_bytes.fetch_add(moved, std::memory_order_relaxed);
        return;
    }
    MPCOMM_LOG_WARN("MPComm: WC error %d on %s (handle %lu chunk %zu)\n", wc.status,
                    rails_[rail]->name.c_str(), static_cast<unsigned long>(h), chunk);
    quarantine(rail, wc.status);
    // Re-post on a healthy rail instead of failing the transfer (the
    // reference fails it, src/mpcomm.cpp:7320-7327).
    bool alt = false;
    for (size_t r : t->candidates)
        alt |= !rails_[r]->quarantined.load(std::memory_order_relaxed) && t->conns[c.host_idx]->group_for(r);
    if (cfg_.repost_on_failure && alt && t->repost_budget > 0 && !t->aborted) {
        --t->repost_budget;
        t->retry.push_back(chunk);
        return;
    }
    t->error.store(MPCOMM_ERR_TRANSFER);
    t->aborted = true;
    t->done_chunks.fetch_add(1, std::memory_order_relaxed);
}

void MPComm::Impl::retire(Worker *w) {
    auto &act = w->active;
    for (size_t i = 0; i < act.size();) {
        Transfer *t = act[i].get();
        const bool posted_all = t->next_chunk >= t->plan.total() && t->retry.empty();
        if ((t->aborted || posted_all) && t->in_flight == 0) {
            if (t->aborted && t->error.load() == 0) t->error.store(MPCOMM_ERR_TRANSFER);
            finishTransfer(t);
            act[i] = std::move(act.back());
            act.pop_back();
        } else {
            ++i;
        }
    }
}

void MPComm::Impl::quarantine(size_t rail, int status) {
    if (rail >= rails_.size()) return;
    if (!rails_[rail]->quarantined.exchange(true)) {
        rails_[rail]->quarantine_since_ns.store(monotonic_raw_ns());
        MPCOMM_LOG_WARN("MPComm: rail %s quarantined (status %d)\n", rails_[rail]->name.c_str(), status);
    }
}

void MPComm::Impl::probeQuarantine() {
    const uint64_t now = monotonic_raw_ns();
    for (size_t r = 0; r < rails_.size(); ++r) {
        RailSlot *s = rails_[r].get();
        if (!s->quarantined.load()) continue;
        const double held = static_cast<double>(now - s->quarantine_since_ns.load()) * 1e-9;
        if (held < cfg_.nic_quarantine_sec || !s->rail->port_active()) continue;
        bool ok = true;
        std::lock_guard<std::mutex> g(conn_mu_);
        for (auto &kv : connections_)
            for (auto &gp : kv.second->groups)
                if (gp.first.first == r)
                    for (auto &qp : gp.second->qps)
                        if (qp->state() != fabric::QpState::kRts && qp->recover() != 0) ok = false;
        if (ok) {
            s->quarantined.store(false);
            MPCOMM_LOG_INFO("MPComm: rail %s re-admitted after %.1f s\n", s->name.c_str(), held);
        } else {
            s->quarantine_since_ns.store(now);
        }
    }
}

void MPComm::Impl::maybeInjectFault() {
    if (cfg_.fault_after_sec < 0) return;
    const double t = std::chrono::duration<double>(Clock::now() - init_time_).count();
    if (!fault_injected_ && t >= cfg_.fault_after_sec) {
        std::lock_guard<std::mutex> g(conn_mu_);
        if (connections_.empty()) return;  // fire once there is something to break
        fault_injected_ = true;
        for (auto &kv : connections_)
            for (auto &gp : kv.second->groups) {
                const bool rail_hit = cfg_.fault_mode == "all_nic" ||
                                      gp.first.first == static_cast<size_t>(cfg_.fault_nic);
                if (!rail_hit) continue;
                for (size_t i = 0; i < gp.second->qps.size(); ++i) {
                    if (cfg_.fault_mode == "single_qp" && i > 0) break;
                    gp.second->qps[i]->to_err();
                    fault_qps_.push_back(gp.second->qps[i].get());
                }
            }
        MPCOMM_LOG_WARN("MPComm: fault injection (%s) moved %zu QPs to ERR\n", cfg_.fault_mode.c_str(),
                        fault_qps_.size());
    }
    if (fault_injected_ && !fault_recovered_ && cfg_.fault_recover_after_sec >= 0 &&
        t >= cfg_.fault_recover_after_sec) {
        fault_recovered_ = true;
        std::lock_guard<std::mutex> g(conn_mu_);
        for (auto *qp : fault_qps_) qp->recover();
        MPCOMM_LOG_WARN("MPComm: fault injection recovered %zu QPs\n", fault_qps_.size());
    }
}

// ---------------------------------------------------------------------------
// Completion API
// ---------------------------------------------------------------------------
bool MPComm::Impl::isTransferComplete(TransferHandle h) {
    auto t = findTransfer(h);
    return !t || t->finished.load(std::memory_order_acquire);
}

int MPComm::Impl::waitTransfer(TransferHandle h, int timeout_ms) {
    auto t = findTransfer(h);
    if (!t) return MPCOMM_ERR_INVALID_HANDLE;
    const auto t0 = Clock::now();
    // Spin briefly (short transfers finish within it), then block on the
    // completion condition variable, which finishTransfer notifies.
    for (size_t spins = 0; spins < 4096; ++spins) {
        if (t->finished.load(std::memory_order_acquire)) return t->error.load(std::memory_order_acquire);
        cpu_relax();
    }
    done_waiters_.fetch_add(1);
    {
        std::unique_lock<std::mutex> lk(done_mu_);
        while (!t->finished.load(std::memory_order_acquire)) {
            auto step = std::chrono::milliseconds(10);
            if (timeout_ms >= 0) {
                const auto left = std::chrono::milliseconds(timeout_ms) -
                                  std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0);
                if (left.count() <= 0) {
                    done_waiters_.fetch_sub(1);
                    return MPCOMM_ERR_TIMEOUT;
                }
                if (left < step) step = left;
            }
            done_cv_.wait_for(lk, step);
        }
    }
    done_waiters_.fetch_sub(1);
    return t->error.load(std::memory_order_acquire);
}

TransferResult MPComm::Impl::getTransferResult(TransferHandle h) {
    TransferResult r{MPCOMM_ERR_INVALID_HANDLE, 0, 0.0};
    auto t = findTransfer(h);
    if (!t) return r;
    const bool fin = t->finished.load(std::memory_order_acquire);
    r.error_code = fin ? t->error.load() : MPCOMM_ERR_PENDING;
    if (fin && r.error_code == MPCOMM_SUCCESS) r.error_code = MPCOMM_SUCCESS;
    r.bytes_transferred = t->bytes.load();
    auto end = fin ? t->t_end : Clock::now();
    r.elapsed_ms = std::chrono::duration<double, std::milli>(end - t->t_start).count();
    return r;
}

void MPComm::Impl::releaseTransfer(TransferHandle h) {
    std::shared_ptr<Transfer> t;
    {
        std::lock_guard<std::mutex> g(xfer_mu_);
        auto it = transfers_.find(h);
        if (it == transfers_.end()) return;
        t = it->second;
        transfers_.erase(it);
    }
    const uint64_t n = stats_counter_.fetch_add(1) + 1;
    if (mpcomm_get_log_level() >= MPCOMM_LOG_LEVEL_DEBUG && t->finished.load() &&
        (cfg_.transfer_stats_interval == 0 || n % cfg_.transfer_stats_interval == 0)) {
        auto ms = [](Clock::time_point a, Clock::time_point b) {
            return std::chrono::duration<double, std::milli>(b - a).count();
        };
        const double total = ms(t->t_start, t->t_end);
        MPCOMM_LOG_DEBUG("MPComm: %sAsync h=%lu %lu B in %.3f ms (%.2f GB/s) | prep %.3f queue %.3f "
                         "first-post %.3f posting %.3f completion %.3f ms\n",
                         dir_name(t->dir), static_cast<unsigned long>(h),
                         static_cast<unsigned long>(t->bytes.load()), total,
                         total > 0 ? t->bytes.load() / total / 1e6 : 0.0, ms(t->t_start, t->t_queued),
                         ms(t->t_queued, t->t_worker), ms(t->t_worker, t->t_first_post),
                         ms(t->t_first_post, t->t_all_posted), ms(t->t_all_posted, t->t_end));
        for (size_t r = 0; r < rails_.size(); ++r) {
            const uint64_t b = t->rail_bytes[r].load();
            if (!b) continue;
            MPCOMM_LOG_DEBUG("MPComm:   rail %-10s %12lu B  share %5.1f%%  %.2f Gbps\n",
                             rails_[r]->name.c_str(), static_cast<unsigned long>(b),
                             100.0 * b / std::max<uint64_t>(1, t->bytes.load()),
                             total > 0 ? b * 8.0 / (total * 1e6) : 0.0);
        }
    }
    if (t->life.fetch_or(2) & 1) {
        handle_table_[h].store(nullptr, std::memory_order_release);
        handles_.release(h);
    }
}

void MPComm::Impl::finishTransfer(Transfer *t) {
    t->t_end = Clock::now();
    nvtx::end(t->nvtx);
    t->finished.store(true);  // seq_cst: ordered against done_waiters_ below
    if (done_waiters_.load() > 0) {
        std::lock_guard<std::mutex> g(done_mu_);  // a waiter is either before its check or in wait
        done_cv_.notify_all();
    }
    if (t->life.fetch_or(1) & 2) {
        handle_table_[t->handle].store(nullptr, std::memory_order_release);
        handles_.release(t->handle);
    }
}

}  // namespace mpcomm
