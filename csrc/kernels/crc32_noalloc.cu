// Allocation-free CRC-32 (see crc32_noalloc.h for who needs it and the
// limits). Same method as crc32.cu — per-thread slicing-by-4 over 2 KiB
// segments, GF(2) shift-and-xor folding of segments into 512 KiB pieces, then
// of pieces into blocks — but the per-piece partial CRCs live in a fixed
// file-scope __device__ array instead of cudaMalloc'd memory.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "cuda/gpu.h"
#include "kernels/common.cuh"
#include "kernels/crc32_noalloc.h"

namespace {

constexpr uint32_t kPoly = 0xEDB88320u;
constexpr int kThreads = 256;
constexpr uint32_t kSegBytes = 2048;
constexpr int64_t kPieceBytes = static_cast<int64_t>(kThreads) * kSegBytes;
constexpr int kMaxDevices = 64;

// The scratch: one partial CRC per 512 KiB piece. In host code this name is
// only a stand-in for the symbol; its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) uint32_t g_crc_scratch[MPCOMM_CRC32_NOALLOC_MAX_WORDS];

struct Powers {
    uint32_t x[41];  // x^(8 * 2^k) mod P, reflected
};

__host__ __device__ __forceinline__ uint32_t mul_mod_p(uint32_t a, uint32_t b) {
    uint32_t r = 0;
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
        if (a & (0x80000000u >> i)) r ^= b;
        b = (b & 1u) ? (b >> 1) ^ kPoly : (b >> 1);
    }
    return r;
}

__host__ __device__ __forceinline__ uint32_t shift_bytes(uint32_t c, uint64_t len, const uint32_t *x) {
    for (int k = 0; len && k < 41; ++k, len >>= 1)
        if (len & 1) c = mul_mod_p(c, x[k]);
    return c;
}

Powers powers_table() {
    Powers p;
    uint32_t v = 0x00800000u;  // x^8
    for (int k = 0; k < 41; ++k) {
        p.x[k] = v;
        v = mul_mod_p(v, v);
    }
    return p;
}

__global__ void __launch_bounds__(kThreads)
    noalloc_crc_pieces(const unsigned char *__restrict__ data, int64_t bs, int64_t ppb,
                       uint32_t *__restrict__ scratch, const __grid_constant__ Powers pw) {
    __shared__ uint32_t tab[4][256];
    __shared__ uint32_t wcrc[kThreads / 32], wlen[kThreads / 32];
    const int tid = threadIdx.x;
    uint32_t t0 = static_cast<uint32_t>(tid);
    for (int k = 0; k < 8; ++k) t0 = (t0 & 1u) ? (t0 >> 1) ^ kPoly : (t0 >> 1);
    tab[0][tid] = t0;
    __syncthreads();
    uint32_t tv = tab[0][tid];
    for (int s = 1; s < 4; ++s) {
        tv = (tv >> 8) ^ tab[0][tv & 0xFFu];
        tab[s][tid] = tv;
    }
    __syncthreads();

    // One CTA per (block, piece), flattened onto x: a grid's y extent stops
    // at 65535, below the 65536 pieces the scratch holds.
    const int64_t block = static_cast<int64_t>(blockIdx.x) / ppb;
    const int64_t piece = static_cast<int64_t>(blockIdx.x) - block * ppb;
    int64_t plen = bs - piece * kPieceBytes;
    if (plen > kPieceBytes) plen = kPieceBytes;
    const unsigned char *p = data + block * bs + piece * kPieceBytes + static_cast<int64_t>(tid) * kSegBytes;
    int64_t slen = plen - static_cast<int64_t>(tid) * kSegBytes;
    slen = slen < 0 ? 0 : (slen > kSegBytes ? kSegBytes : slen);
    uint32_t c = 0;
    int64_t i = 0;
    if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
        for (; i + 16 <= slen; i += 16) {
            const int4 v = *reinterpret_cast<const int4 *>(p + i);
            const uint32_t w[4] = {static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y),
                                   static_cast<uint32_t>(v.z), static_cast<uint32_t>(v.w)};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                c ^= w[q];
                c = tab[3][c & 0xFFu] ^ tab[2][(c >> 8) & 0xFFu] ^ tab[1][(c >> 16) & 0xFFu] ^ tab[0][c >> 24];
            }
        }
    }
    for (; i < slen; ++i) c = (c >> 8) ^ tab[0][(c ^ p[i]) & 0xFFu];

    uint32_t len = static_cast<uint32_t>(slen);
    const int lane = tid & 31;
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const uint32_t oc = __shfl_down_sync(0xffffffffu, c, 1 << k);
        const uint32_t ol = __shfl_down_sync(0xffffffffu, len, 1 << k);
        if ((lane & ((2 << k) - 1)) == 0) {
            c = shift_bytes(c, ol, pw.x) ^ oc;
            len += ol;
        }
    }
    if (lane == 0) {
        wcrc[tid >> 5] = c;
        wlen[tid >> 5] = len;
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0;
        for (int w = 0; w < kThreads / 32; ++w) acc = shift_bytes(acc, wlen[w], pw.x) ^ wcrc[w];
        scratch[block * ppb + piece] = acc;
    }
}

__global__ void noalloc_crc_finalize(const uint32_t *__restrict__ scratch, int64_t n, int64_t bs, int64_t ppb,
                                     uint32_t *__restrict__ out, const __grid_constant__ Powers pw) {
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= n) return;
    uint32_t acc = 0;
    for (int64_t p = 0; p < ppb; ++p) {
        int64_t len = bs - p * kPieceBytes;
        if (len > kPieceBytes) len = kPieceBytes;
        acc = shift_bytes(acc, static_cast<uint64_t>(len), pw.x) ^ scratch[b * ppb + p];
    }
    out[b] = shift_bytes(0xFFFFFFFFu, static_cast<uint64_t>(bs), pw.x) ^ acc ^ 0xFFFFFFFFu;
}

// Device address of g_crc_scratch in the current device's current context.
// The lookup is cached per (device, context): a context that is torn down and
// created again (cudaDeviceReset, primary-context release) may load the
// module at another address, so a new context gets a new lookup. Returns a
// CUDA error code.
int scratch_for_current_device(uint32_t **out) {
    using CtxGetCurrent = int (*)(void **);
    static const CtxGetCurrent ctx_get_current =
        reinterpret_cast<CtxGetCurrent>(mpcomm::gpu::driver_symbol("cuCtxGetCurrent"));
    static std::mutex mu;
    static uint32_t *addr[kMaxDevices] = {nullptr};
    static void *addr_ctx[kMaxDevices] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    void *ctx = nullptr;
    if (!ctx_get_current || ctx_get_current(&ctx) != 0) ctx = nullptr;
    std::lock_guard<std::mutex> g(mu);
    if (!addr[dev] || !ctx || addr_ctx[dev] != ctx) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_crc_scratch);
        if (e != cudaSuccess) {
            std::fprintf(stderr, "mpcomm_crc32_blocks_noalloc: cudaGetSymbolAddress failed on device %d: %s\n",
                         dev, cudaGetErrorString(e));
            return e;
        }
        // The lookup makes the primary context current if nothing was yet.
        if (!ctx && ctx_get_current && ctx_get_current(&ctx) != 0) ctx = nullptr;
        addr[dev] = static_cast<uint32_t *>(p);
        addr_ctx[dev] = ctx;
    }
    *out = addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int mpcomm_crc32_blocks_noalloc(const void *data, int64_t num_blocks, int64_t block_size,
                                           uint32_t *out, void *stream) {
    if (!data || !out || num_blocks <= 0 || block_size <= 0) return cudaErrorInvalidValue;
    const int64_t ppb = (block_size + kPieceBytes - 1) / kPieceBytes;
    if (num_blocks > MPCOMM_CRC32_NOALLOC_MAX_WORDS || ppb > MPCOMM_CRC32_NOALLOC_MAX_WORDS ||
        num_blocks * ppb > MPCOMM_CRC32_NOALLOC_MAX_WORDS) {
        std::fprintf(stderr,
                     "mpcomm_crc32_blocks_noalloc: %lld blocks x %lld bytes need %lld scratch words; the "
                     "fixed scratch holds %d (one word per 512 KiB piece). Use the allocating entry point "
                     "or split the request.\n",
                     static_cast<long long>(num_blocks), static_cast<long long>(block_size),
                     static_cast<long long>(num_blocks) * static_cast<long long>(ppb),
                     MPCOMM_CRC32_NOALLOC_MAX_WORDS);
        return -1;
    }
    // A runtime error left pending by the caller's earlier work is returned
    // untouched (and not cleared) before anything is queued.
    cudaError_t pending = cudaPeekAtLastError();
    if (pending != cudaSuccess) return pending;
    uint32_t *scratch = nullptr;
    int e = scratch_for_current_device(&scratch);
    if (e != cudaSuccess) return e;
    static const Powers pw = powers_table();
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    noalloc_crc_pieces<<<static_cast<unsigned>(num_blocks * ppb), kThreads, 0, st>>>(
        static_cast<const unsigned char *>(data), block_size, ppb, scratch, pw);
    mpcomm::kern::note_launch();
    cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) return le;
    const int fin = 128;
    noalloc_crc_finalize<<<static_cast<unsigned>((num_blocks + fin - 1) / fin), fin, 0, st>>>(
        scratch, num_blocks, block_size, ppb, out, pw);
    mpcomm::kern::note_launch();
    return cudaGetLastError();
}
