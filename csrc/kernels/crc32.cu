// CRC-32 (IEEE 802.3 / zlib: reflected polynomial 0xEDB88320, init and
// final xor 0xFFFFFFFF) of many blocks, computed in parallel.
//
// Method. CRC is linear over GF(2). Let R(M) be the register after feeding
// M into a zero-initialised register with no final xor. Then
//     R(A || B) = shift(R(A), |B|) ^ R(B),  shift(c, L) = c * x^(8L) mod P
//     CRC(M)    = shift(0xFFFFFFFF, |M|) ^ R(M) ^ 0xFFFFFFFF.
// This is the polynomial-combination identity behind zlib's crc32_combine
// (Mark Adler); the code below is written from the algebra.
//
// Kernel layout. A CTA of 256 threads owns a 256 KiB piece of a block; each
// thread computes R() of its 1 KiB segment as two independent 512 B streams
// (two dependency chains in flight) with slicing-by-4 tables, then the
// segments are folded by a shuffle tree and across warps. Shared-memory
// lookups use 8 bank-interleaved copies of every table (lane l reads copy
// l % 8), so only the 4 lanes sharing a copy can collide on a bank. A
// finalize kernel folds the pieces of each block with one CTA per block:
// each thread folds a contiguous run of pieces (one multiply per piece by
// x^(8 * 256 KiB)), then a tree combines the runs. Multiplication by
// x^(8*2^k) uses a 41-entry table of powers, so a shift costs popcount(L)
// carry-less multiplies.
#include <cuda_runtime.h>

#include <mutex>

#include "kernels/common.cuh"

namespace mpcomm {
namespace kern {

namespace {

constexpr uint32_t kPoly = 0xEDB88320u;
constexpr int kCrcThreads = 256;
constexpr uint32_t kHalfBytes = 512;            // one dependency chain
constexpr uint32_t kSegBytes = 2 * kHalfBytes;  // per thread
constexpr uint64_t kPieceBytes = static_cast<uint64_t>(kCrcThreads) * kSegBytes;  // 256 KiB
constexpr int kPieceLog2 = 18;
constexpr int kCopies = 8;
constexpr int kFinThreads = 256;

struct Powers {
    uint32_t x[41];  // x[k] = x^(8 * 2^k) mod P, reflected
};

// a * b mod P, reflected bit order (bit 31 is the x^0 coefficient).
__host__ __device__ __forceinline__ uint32_t gf2_mul(uint32_t a, uint32_t b) {
    uint32_t prod = 0;
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
        if (a & (0x80000000u >> i)) prod ^= b;
        b = (b & 1u) ? (b >> 1) ^ kPoly : (b >> 1);
    }
    return prod;
}

__host__ __device__ __forceinline__ uint32_t gf2_shift(uint32_t c, uint64_t len, const uint32_t *x) {
    for (int k = 0; len && k < 41; ++k, len >>= 1)
        if (len & 1) c = gf2_mul(c, x[k]);
    return c;
}

Powers make_powers() {
    Powers p;
    uint32_t v = 0x00800000u;  // x^8
    for (int k = 0; k < 41; ++k) {
        p.x[k] = v;
        v = gf2_mul(v, v);
    }
    return p;
}

// Table T[s][e] replicated kCopies times: word ((s * 256 + e) * kCopies + c).
__device__ __forceinline__ uint32_t lookup(const uint32_t *tab, int s, uint32_t e, int c) {
    return tab[((s * 256 + e) << 3) + c];
}

__device__ __forceinline__ uint32_t step4(const uint32_t *tab, uint32_t c, uint32_t w, int cp) {
    c ^= w;
    return lookup(tab, 3, c & 0xFFu, cp) ^ lookup(tab, 2, (c >> 8) & 0xFFu, cp) ^
           lookup(tab, 1, (c >> 16) & 0xFFu, cp) ^ lookup(tab, 0, c >> 24, cp);
}

// R() of [p, p+len) (len <= kHalfBytes). Vector loads when 16-byte aligned.
__device__ __forceinline__ uint32_t crc_span(const uint32_t *tab, const unsigned char *p, uint32_t len, int cp) {
    uint32_t c = 0, i = 0;
    if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
        for (; i + 16 <= len; i += 16) {
            const int4 v = *reinterpret_cast<const int4 *>(p + i);
            c = step4(tab, c, static_cast<uint32_t>(v.x), cp);
            c = step4(tab, c, static_cast<uint32_t>(v.y), cp);
            c = step4(tab, c, static_cast<uint32_t>(v.z), cp);
            c = step4(tab, c, static_cast<uint32_t>(v.w), cp);
        }
    }
    for (; i < len; ++i) c = (c >> 8) ^ lookup(tab, 0, (c ^ p[i]) & 0xFFu, cp);
    return c;
}

__global__ void __launch_bounds__(kCrcThreads)
    crc_pieces_kernel(const unsigned char *__restrict__ data, int64_t bs, int64_t ppb,
                      uint32_t *__restrict__ piece_crc, const __grid_constant__ Powers pw) {
    __shared__ uint32_t tab[4 * 256 * kCopies];  // 32 KiB
    __shared__ uint32_t t0[256];
    __shared__ uint32_t warp_crc[kCrcThreads / 32];
    __shared__ uint32_t warp_len[kCrcThreads / 32];
    const int tid = threadIdx.x;
    {
        uint32_t c = static_cast<uint32_t>(tid);
        for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ kPoly : (c >> 1);
        t0[tid] = c;
    }
    __syncthreads();
    {
        uint32_t c = t0[tid];
        for (int s = 0; s < 4; ++s) {
            if (s) c = (c >> 8) ^ t0[c & 0xFFu];
#pragma unroll
            for (int k = 0; k < kCopies; ++k) tab[((s * 256 + tid) << 3) + k] = c;
        }
    }
    __syncthreads();

    const int cp = tid & (kCopies - 1);
    const int64_t block = blockIdx.y;
    const int64_t piece = blockIdx.x;
    const int64_t piece_off = piece * static_cast<int64_t>(kPieceBytes);
    int64_t piece_len = bs - piece_off;
    if (piece_len > static_cast<int64_t>(kPieceBytes)) piece_len = kPieceBytes;
    const unsigned char *base = data + block * bs + piece_off + static_cast<int64_t>(tid) * kSegBytes;

    int64_t slen = piece_len - static_cast<int64_t>(tid) * kSegBytes;
    slen = slen < 0 ? 0 : (slen > kSegBytes ? kSegBytes : slen);
    const uint32_t la = static_cast<uint32_t>(slen < kHalfBytes ? slen : kHalfBytes);
    const uint32_t lb = static_cast<uint32_t>(slen) - la;
    // Two independent chains interleaved by the compiler's scheduler.
    uint32_t ca, cb;
    if (la == kHalfBytes && lb == kHalfBytes && (reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
        ca = 0;
        cb = 0;
        const unsigned char *pb = base + kHalfBytes;
#pragma unroll 2
        for (uint32_t i = 0; i < kHalfBytes; i += 16) {
            const int4 va = *reinterpret_cast<const int4 *>(base + i);
            const int4 vb = *reinterpret_cast<const int4 *>(pb + i);
            ca = step4(tab, ca, static_cast<uint32_t>(va.x), cp);
            cb = step4(tab, cb, static_cast<uint32_t>(vb.x), cp);
            ca = step4(tab, ca, static_cast<uint32_t>(va.y), cp);
            cb = step4(tab, cb, static_cast<uint32_t>(vb.y), cp);
            ca = step4(tab, ca, static_cast<uint32_t>(va.z), cp);
            cb = step4(tab, cb, static_cast<uint32_t>(vb.z), cp);
            ca = step4(tab, ca, static_cast<uint32_t>(va.w), cp);
            cb = step4(tab, cb, static_cast<uint32_t>(vb.w), cp);
        }
    } else {
        ca = crc_span(tab, base, la, cp);
        cb = crc_span(tab, base + la, lb, cp);
    }
    uint32_t c = gf2_shift(ca, lb, pw.x) ^ cb;

    // Fold segments in order: (crc, len) pairs, left absorbs right.
    uint32_t len = static_cast<uint32_t>(slen);
    const int lane = tid & 31;
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const uint32_t oc = __shfl_down_sync(0xffffffffu, c, 1 << k);
        const uint32_t ol = __shfl_down_sync(0xffffffffu, len, 1 << k);
        if ((lane & ((2 << k) - 1)) == 0) {
            c = gf2_shift(c, ol, pw.x) ^ oc;
            len += ol;
        }
    }
    if (lane == 0) {
        warp_crc[tid >> 5] = c;
        warp_len[tid >> 5] = len;
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0;
        for (int w = 0; w < kCrcThreads / 32; ++w) acc = gf2_shift(acc, warp_len[w], pw.x) ^ warp_crc[w];
        piece_crc[block * ppb + piece] = acc;
    }
}

// One CTA per block: thread t folds pieces [t*k, (t+1)*k) in order, then the
// runs are folded by a shuffle tree and across warps.
__global__ void __launch_bounds__(kFinThreads)
    crc_finalize_kernel(const uint32_t *__restrict__ piece_crc, int64_t n, int64_t bs, int64_t ppb,
                        uint32_t *__restrict__ out, const __grid_constant__ Powers pw) {
    __shared__ uint32_t wc[kFinThreads / 32];
    __shared__ uint64_t wl[kFinThreads / 32];
    const int64_t b = blockIdx.x;
    const int tid = threadIdx.x;
    const int64_t per = (ppb + kFinThreads - 1) / kFinThreads;
    const int64_t p0 = tid * per, p1 = p0 + per < ppb ? p0 + per : ppb;
    uint32_t c = 0;
    uint64_t len = 0;
    for (int64_t p = p0; p < p1; ++p) {
        int64_t l = bs - p * static_cast<int64_t>(kPieceBytes);
        if (l > static_cast<int64_t>(kPieceBytes)) l = kPieceBytes;
        // all pieces but the block's last are exactly 2^18 bytes: one multiply
        c = (l == static_cast<int64_t>(kPieceBytes) ? gf2_mul(c, pw.x[kPieceLog2])
                                                      : gf2_shift(c, static_cast<uint64_t>(l), pw.x)) ^
            piece_crc[b * ppb + p];
        len += static_cast<uint64_t>(l);
    }
    const int lane = tid & 31;
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const uint32_t oc = __shfl_down_sync(0xffffffffu, c, 1 << k);
        const uint64_t ol = __shfl_down_sync(0xffffffffu, len, 1 << k);
        if ((lane & ((2 << k) - 1)) == 0) {
            c = gf2_shift(c, ol, pw.x) ^ oc;
            len += ol;
        }
    }
    if (lane == 0) {
        wc[tid >> 5] = c;
        wl[tid >> 5] = len;
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0;
        for (int w = 0; w < kFinThreads / 32; ++w) acc = gf2_shift(acc, wl[w], pw.x) ^ wc[w];
        out[b] = gf2_shift(0xFFFFFFFFu, static_cast<uint64_t>(bs), pw.x) ^ acc ^ 0xFFFFFFFFu;
    }
}

const Powers &powers() {
    static const Powers p = make_powers();
    return p;
}

}  // namespace

size_t crc32_scratch_words(int64_t n, int64_t bs) {
    const int64_t ppb = (bs + static_cast<int64_t>(kPieceBytes) - 1) / static_cast<int64_t>(kPieceBytes);
    return static_cast<size_t>(n * ppb);
}

int crc32_blocks_scratch(const void *data, int64_t n, int64_t bs, uint32_t *out, uint32_t *scratch,
                         size_t scratch_words, void *stream) {
    if (!data || !out || !scratch || n <= 0 || bs <= 0) return cudaErrorInvalidValue;
    const int64_t ppb = (bs + static_cast<int64_t>(kPieceBytes) - 1) / static_cast<int64_t>(kPieceBytes);
    if (static_cast<size_t>(n * ppb) > scratch_words) return cudaErrorInvalidValue;
    if (n > 65535 || ppb > 0x7fffffff) return cudaErrorInvalidValue;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    dim3 grid(static_cast<unsigned>(ppb), static_cast<unsigned>(n));
    crc_pieces_kernel<<<grid, kCrcThreads, 0, st>>>(static_cast<const unsigned char *>(data), bs, ppb,
                                                   scratch, powers());
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    crc_finalize_kernel<<<static_cast<unsigned>(n), kFinThreads, 0, st>>>(scratch, n, bs, ppb, out, powers());
    note_launch();
    return cudaGetLastError();
}

int crc32_blocks(const void *data, int64_t n, int64_t bs, uint32_t *out, void *stream) {
    // Scratch from a per-device cache that only grows (released at exit).
    static std::mutex mu;
    static uint32_t *bufs[64] = {nullptr};
    static size_t caps[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const size_t need = crc32_scratch_words(n, bs);
    uint32_t *buf = nullptr;
    {
        std::lock_guard<std::mutex> g(mu);
        if (caps[dev] < need) {
            // The old buffer may still be read by queued work on another
            // stream, so it is not freed; it is small (4 bytes / 256 KiB).
            void *p = nullptr;
            cudaError_t e = cudaMalloc(&p, need * sizeof(uint32_t));
            if (e != cudaSuccess) return e;
            bufs[dev] = static_cast<uint32_t *>(p);
            caps[dev] = need;
        }
        buf = bufs[dev];
    }
    return crc32_blocks_scratch(data, n, bs, out, buf, need, stream);
}

uint32_t crc32_host(const void *data, size_t len, uint32_t crc) {
    static uint32_t tab[256];
    static std::once_flag once;
    std::call_once(once, [] {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ kPoly : (c >> 1);
            tab[i] = c;
        }
    });
    const unsigned char *p = static_cast<const unsigned char *>(data);
    crc = ~crc;
    for (size_t i = 0; i < len; ++i) crc = (crc >> 8) ^ tab[(crc ^ p[i]) & 0xFFu];
    return ~crc;
}

}  // namespace kern
}  // namespace mpcomm
