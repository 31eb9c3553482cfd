// Two-stage staging pool: the non-zero-copy PUT/GET path for local buffers
// that are not registered.
//
// The reference advertises this path and publishes its numbers
// (README.md:47,105-106,115-116) but ships no code for it, so this design
// follows the README's description: a multi-threaded, two-stage pipeline
// over pre-registered slabs.
//   SCATTER/PUT/BROADCAST: stage 1 copies a piece of the user buffer into a
//     free slab, stage 2 posts it through the zero-copy engine from the slab;
//     the slab returns to the pool on completion.
//   GATHER/GET: stage 1 reads the remote piece into a slab through the
//     zero-copy engine, stage 2 copies it out to the user buffer.
// Pieces of one transfer (and of concurrent transfers) overlap: while one
// slab is on the wire, others are being filled or drained.
//
// Where the slabs live follows the user buffer:
//   * host memory: slabs in host DRAM, stage copies by a pool of CPU threads;
//   * device memory (HBM of GPU g, not registered): slabs in g's own HBM,
//     registered once, and the stage copies are launches of the sm_100a
//     bulk-copy kernel on g (the fabric stream when the caller set one, else
//     a stream of the pool), each publishing a host-mapped completion word
//     that the orchestrator polls. The bytes never cross PCIe for staging:
//     a device-to-device copy runs at HBM rate, far above any link the
//     second stage then uses.
// A range that is neither device memory nor mapped host memory is refused.
#ifndef MPCOMM_B200_CSRC_ENGINE_STAGING_H_
#define MPCOMM_B200_CSRC_ENGINE_STAGING_H_

#include <atomic>
#include <condition_variable>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "engine/impl.h"

namespace mpcomm {

class StagingEngine {
 public:
    explicit StagingEngine(MPComm::Impl *impl);
    ~StagingEngine();
    TransferHandle submit(uintptr_t local, const std::vector<std::string> &hosts,
                          const std::vector<uintptr_t> &raddrs, const std::vector<size_t> &lens,
                          Direction dir);
    size_t slab_bytes() const { return slab_bytes_; }
    size_t slab_count() const { return nslabs_; }

 private:
    struct Piece;
    struct Staged;
    struct DevicePool;
    bool ensure_slabs();
    DevicePool *ensure_device_pool(int dev);
    void start_threads();
    void orchestrate();
    void copy_worker();
    void enqueue_copy(std::function<void()> job);
    bool step(Staged *s);
    // Stage copy of a device piece between the user buffer and its slab.
    bool launch_device_copy(Piece *p, bool to_slab);
    // 1 = the piece's device copy finished, 0 = pending, -1 = failed.
    int poll_device_copy(Piece *p);

    MPComm::Impl *impl_;
    size_t slab_bytes_, nslabs_, nthreads_, dev_slab_bytes_;
    void *slab_base_ = nullptr;
    size_t slab_total_ = 0;
    bool slabs_registered_ = false;
    std::vector<int> free_slabs_;
    std::vector<std::unique_ptr<DevicePool>> dev_pools_;  // by device ordinal
    bool threads_started_ = false;

    std::mutex mu_;
    std::condition_variable cv_;
    std::deque<std::shared_ptr<Staged>> incoming_;
    std::vector<std::shared_ptr<Staged>> active_;
    std::atomic<bool> running_{true};
    std::thread orchestrator_;

    std::mutex cmu_;
    std::condition_variable ccv_;
    std::deque<std::function<void()>> copies_;
    std::vector<std::thread> copiers_;
    std::atomic<int> copies_done_{0};
};

}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_ENGINE_STAGING_H_
