// Host-side entry points of the sm_100a kernels. Streams are passed as
// void* (a cudaStream_t) so callers need no CUDA headers. Every launcher
// returns 0 or a cudaError_t value and never synchronises.
#ifndef MPCOMM_B200_CSRC_KERNELS_LAUNCH_H_
#define MPCOMM_B200_CSRC_KERNELS_LAUNCH_H_

#include <cstddef>
#include <cstdint>
#include <vector>

namespace mpcomm {
namespace kern {

// One H2D QoS window record in pinned, device-mapped host memory. The
// kernel writes begin_ns when its first CTA starts and end_ns (release,
// system scope) when its last CTA has finished all stores. The host QoS
// engine treats begin != 0 && end == 0 as "window open".
// `gate` (device memory of the same GPU, may be null) counts the open
// windows of that GPU on the device: the first CTA adds 1, the last CTA
// subtracts 1. GPU-fabric copies given the same gate pause their next tile
// while it is non-zero (bounded), so background traffic yields within one
// tile instead of after its launched chunks drain.
struct H2DWindow {
    uint64_t begin_ns;
    uint64_t end_ns;
    int32_t gpu;
    uint32_t armed;
    uint32_t *gate;
};

struct LaunchInfo {
    int ctas = 0;
    int threads = 0;
    size_t smem = 0;
    int path = 0;  // 1 = bulk (TMA) pipeline, 2 = vector SM kernel
};

enum MoverMode { kModeAuto = 0, kModeSm = 1, kModeTma = 2 };

// dst[i*bs .. +bs) = pool[idx[i]*bs .. +bs) for i in [0, n).
// pool_blocks > 0 enables the index bound check (out-of-range indices are
// skipped and flagged in *status). `window`/`window_ctr` may be null.
int h2d_gather(const void *pool, int64_t pool_blocks, const int64_t *idx, void *out, int64_t n,
               int64_t bs, int mode, int max_ctas, void *stream, uint32_t *status,
               H2DWindow *window, uint32_t *window_ctr, LaunchInfo *info);
// pool[idx[i]*bs ..] = src[i*bs ..].
int h2d_scatter(const void *src, const int64_t *idx, void *pool, int64_t pool_blocks, int64_t n,
                int64_t bs, int mode, int max_ctas, void *stream, uint32_t *status,
                H2DWindow *window, uint32_t *window_ctr, LaunchInfo *info);

// One GPU-fabric work request: a contiguous copy between any two addresses
// the device can reach (local HBM, IPC-mapped peer HBM, mapped host DRAM).
struct CopyDesc {
    const void *src;
    void *dst;
    uint64_t bytes;
};
constexpr int kMaxCopyDescs = 64;
// Copies up to kMaxCopyDescs spans in one launch (descriptors travel in the
// kernel's parameter block, no staging buffer).
// mode: kModeAuto/kModeTma = bulk pipeline, kModeSm = vector SM kernel.
// gate (device memory, may be null): while *gate != 0 every pipeline waits
// before issuing its next tile, for at most gate_budget_ns in total per
// pipeline (then it runs ungated: fail-open, never a hang).
// done_flag (may be host-mapped memory): after every store of the launch has
// completed, the last CTA stores done_value there (system-scope release);
// done_ctr is its last-CTA counter (device memory, zero, self-resetting;
// launches sharing one must be stream-ordered).
int copy_batch(const CopyDesc *descs, int n, int max_ctas, void *stream, uint32_t *status,
               LaunchInfo *info, int mode = kModeAuto, const uint32_t *gate = nullptr,
               uint64_t gate_budget_ns = 0, uint64_t *done_flag = nullptr, uint64_t done_value = 0,
               uint32_t *done_ctr = nullptr);

// CRC-32 (IEEE 802.3, reflected polynomial 0xEDB88320, init/xorout
// 0xFFFFFFFF — the zlib/PNG variant) of n blocks of bs bytes each.
// Uses a per-device scratch buffer owned by the library (grown on demand).
int crc32_blocks(const void *data, int64_t n, int64_t bs, uint32_t *out, void *stream);
// Same, with caller-provided scratch of crc32_scratch_words(n, bs) words.
int crc32_blocks_scratch(const void *data, int64_t n, int64_t bs, uint32_t *out, uint32_t *scratch,
                         size_t scratch_words, void *stream);
size_t crc32_scratch_words(int64_t n, int64_t bs);
// Host reference (table-driven, byte at a time); `crc` chains calls (0 to start).
uint32_t crc32_host(const void *data, size_t len, uint32_t crc);

// Fused PXN gather + forward: for each i, copies pool[idx[i]*bs ..] (host
// DRAM mapped on this GPU) into dst[i*bs ..], where dst may be a peer GPU's
// HBM (IPC-mapped). After every store of the launch has completed, the last
// CTA publishes `flag_value` to *done_flag (system-scope release; the flag
// may live in the peer's memory). `window` (optional, needs `ctr`): H2D QoS
// window of the host pool read, opened by the first CTA, closed by the last.
int pxn_gather_forward(const void *pool, int64_t pool_blocks, const int64_t *idx, void *dst,
                       int64_t n, int64_t bs, int max_ctas, void *stream, uint32_t *status,
                       uint64_t *done_flag, uint64_t flag_value, uint32_t *ctr, LaunchInfo *info,
                       H2DWindow *window = nullptr);

// NVLS broadcast: multimem stores of src[0..bytes) into a multicast address
// (every GPU bound to the multicast object receives the bytes).
int nvls_broadcast(const void *src, void *mc_dst, uint64_t bytes, int max_ctas, void *stream,
                   LaunchInfo *info);
// Tuning knob of nvls_broadcast's store flavour and depth (0..3; see bcast.cu).
void set_nvls_variant(int v);
// Fallback fan-out: the same bytes stored to up to 8 peer pointers.
int p2p_fanout(const void *src, void *const *dsts, int ndst, uint64_t bytes, int max_ctas,
               void *stream, LaunchInfo *info);
// Fused H2D gather + broadcast of a batch of host pages to several GPUs in
// one launch (no staging of the batch in local HBM): tile k of page i,
// read from pool[idx[i]*bs ..] (mapped host DRAM) into shared memory, is
// delivered to offset i*bs of every consumer's buffer, either by multimem
// stores to `mc_dst` (an NVLS multicast address: every bound GPU receives
// it) or, when mc_dst is null, by bulk stores to each of the `ndst` (<= 8)
// device pointers in `dsts` (IPC-mapped peer HBM and/or local HBM).
// `idx` may be null: page i is then pool page i (a contiguous source).
// Completion (optional; `ctr` is a zeroed device word, self-resetting,
// launches sharing it must be stream-ordered): with mc_dst and `mc_flag`,
// the last CTA adds 1 to the 64-bit flag at multicast address `mc_flag`
// (release, system scope), so every bound GPU's copy of the flag counts
// broadcasts; in either mode it then stores `flag_value` (release, system
// scope) to each of the `nflag` (<= 8) flag pointers, which may be
// host-mapped words.
// `window` (optional, needs `ctr`): H2D QoS window of a host-memory pool,
// opened by the first CTA and closed by the last, as the H2D movers do.
// Requires 16-byte aligned pool/destinations and bs % 16 == 0.
constexpr int kMaxFanoutDsts = 8;  // P2P sink destinations per gather_bcast launch
int gather_bcast(const void *pool, int64_t pool_blocks, const int64_t *idx, int64_t n, int64_t bs, void *mc_dst,
                 void *const *dsts, int ndst, uint64_t *mc_flag, uint64_t *const *flags, int nflag,
                 uint64_t flag_value, uint32_t *ctr, int max_ctas, void *stream, uint32_t *status,
                 LaunchInfo *info, H2DWindow *window = nullptr);
// Bounded wait on a 64-bit flag written by another GPU or the host: waits
// until *flag >= value or budget_ns elapses (then sets kStatusFlagTimeout).
int wait_flag(const uint64_t *flag, uint64_t value, uint64_t budget_ns, void *stream,
              uint32_t *status);

// Kernel trace (MPCOMM_KERNEL_TRACE=<slots per device>; 0/unset = off). The
// data movers (gather, scatter, fabric batches, PXN forward) stamp their
// device start (CTA 0) and end (last CTA to exit) with %globaltimer into a
// device-memory ring; kernel_trace() reads the rings back (synchronous
// copies: not for hot paths) and returns the launches still in them.
struct KernelStamp {
    uint64_t begin_ns;
    uint64_t end_ns;
};
struct TraceRecord {
    uint64_t seq;      // launch order across devices
    int dev;
    const char *kind;  // "h2d_gather", "h2d_scatter", "copy_batch", "pxn_gather_forward", ...
    uint64_t bytes;
    uint64_t begin_ns, end_ns;
};
// Slot for the next launch on the current device (nullptr when off).
KernelStamp *trace_acquire(const char *kind, uint64_t bytes);
int kernel_trace(std::vector<TraceRecord> *out);
void kernel_trace_reset();
size_t kernel_trace_slots();

// Kernels launched by this library since load (all devices).
uint64_t launch_count();
// SM count of device `dev` (cached per device).
int sm_count(int dev);
// Device-time budget of every bounded wait, ns (MPCOMM_KERNEL_WAIT_BUDGET_MS).
uint64_t wait_budget_ns();

}  // namespace kern
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_KERNELS_LAUNCH_H_
