// Shared host/device helpers of the kernel translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "kernels/launch.h"
#include "kernels/ptx.cuh"

namespace mpcomm {
namespace kern {

// Counts one launch of this library's kernels (launch_count()).
void note_launch();
// A zeroed device word per device for kernels whose caller passed no status
// pointer (allocated on first use, lives until process exit).
uint32_t *default_status_word(int dev);

enum TileKind : uint32_t { kSkip = 0, kBulk = 1, kInline = 2, kBad = 3 };

struct Tile {
    const char *src;
    char *dst;
    uint32_t bytes;
    uint32_t kind;
};

__device__ __forceinline__ uint32_t tile_kind(const void *s, const void *d, uint32_t bytes) {
    return ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d) | bytes) & 15u) == 0
               ? kBulk
               : kInline;
}

// Warp-cooperative copy of an arbitrary span. 16-byte vectors when source
// and destination share their offset mod 16 (4 loads in flight per lane),
// 4-byte words when both are word aligned, bytes otherwise.
__device__ __forceinline__ void warp_copy_any(char *d, const char *s, uint64_t bytes) {
    const int lane = threadIdx.x & 31;
    const uintptr_t ms = reinterpret_cast<uintptr_t>(s) & 15u;
    const uintptr_t md = reinterpret_cast<uintptr_t>(d) & 15u;
    if (ms == md) {
        uint64_t head = (16u - ms) & 15u;
        if (head > bytes) head = bytes;
        for (uint64_t i = lane; i < head; i += 32) d[i] = s[i];
        const uint64_t body = (bytes - head) >> 4;
        const int4 *s4 = reinterpret_cast<const int4 *>(s + head);
        int4 *d4 = reinterpret_cast<int4 *>(d + head);
        uint64_t i = lane;
        for (; i + 96 < body; i += 128) {
            int4 a = ld_v4(s4 + i), b = ld_v4(s4 + i + 32), c = ld_v4(s4 + i + 64),
                 e = ld_v4(s4 + i + 96);
            st_v4(d4 + i, a);
            st_v4(d4 + i + 32, b);
            st_v4(d4 + i + 64, c);
            st_v4(d4 + i + 96, e);
        }
        for (; i < body; i += 32) st_v4(d4 + i, ld_v4(s4 + i));
        const uint64_t done = head + (body << 4);
        for (uint64_t k = done + lane; k < bytes; k += 32) d[k] = s[k];
        return;
    }
    if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 3u) == 0) {
        const uint64_t w = bytes >> 2;
        const uint32_t *s32 = reinterpret_cast<const uint32_t *>(s);
        uint32_t *d32 = reinterpret_cast<uint32_t *>(d);
        for (uint64_t i = lane; i < w; i += 32) d32[i] = s32[i];
        for (uint64_t k = (w << 2) + lane; k < bytes; k += 32) d[k] = s[k];
        return;
    }
    for (uint64_t i = lane; i < bytes; i += 32) d[i] = s[i];
}

// Trace stamps: CTA 0 writes the start time; every CTA raises the end time
// to its own exit time (atomicMax), so a reused slot needs no reset.
__device__ __forceinline__ void trace_begin(KernelStamp *st) {
    if (st && blockIdx.x == 0 && threadIdx.x == 0)
        *reinterpret_cast<volatile unsigned long long *>(&st->begin_ns) = globaltimer_ns();
}
__device__ __forceinline__ void trace_end(KernelStamp *st) {
    if (!st) return;
    __syncthreads();
    if (threadIdx.x == 0)
        atomicMax(reinterpret_cast<unsigned long long *>(&st->end_ns),
                  static_cast<unsigned long long>(globaltimer_ns()));
}

// H2D QoS window helpers (see H2DWindow in launch.h).
__device__ __forceinline__ void window_open(H2DWindow *win) {
    if (win && blockIdx.x == 0 && threadIdx.x == 0) {
        st_release_sys_u64(&win->begin_ns, globaltimer_ns() | 1ull);
        uint32_t *gate = *reinterpret_cast<uint32_t *volatile *>(&win->gate);
        if (gate) atomicAdd(gate, 1u);
    }
}

// Device QoS gate of a background copy: returns at once when the gate is
// closed (0) or this pipeline's pause budget is spent; otherwise sleeps
// until the gate closes or the budget runs out. `paused` accumulates the
// time spent here across calls (one per tile).
__device__ __forceinline__ void qos_gate_wait(const uint32_t *gate, uint64_t &paused, uint64_t budget) {
    if (!gate || paused >= budget || ld_acquire_gpu_u32(gate) == 0) return;
    const uint64_t t0 = globaltimer_ns();
    uint64_t now = t0;
    while (ld_acquire_gpu_u32(gate) != 0 && paused + (now - t0) < budget) {
        __nanosleep(256);
        now = globaltimer_ns();
    }
    paused += now - t0;
}

}  // namespace kern
}  // namespace mpcomm
