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
// Kernel layout (crc_rows_kernel). Each block is cut into spans of S bytes
// (S chosen so the whole input gives about one span per resident warp);
// a warp owns a span and reads it as 512-byte rows, lane l loading bytes
// [16l, 16l+16) of every row — fully coalesced 16-byte loads. Lane l thus
// sees a "column" of its span, 16 bytes every 512. Its register X follows
//     X <- shift(X, 512) ^ R(row piece)
// computed as one table shift by 496 bytes (four lookups in the U tables)
// followed by the ordinary slicing-by-4 steps over the 16 bytes (which
// shift by the remaining 16). At the end lane l's column contributes
// shift(X_l, 496 - 16l) to the span and the lanes are xor-reduced. The
// span's rows are split in two halves so each lane runs two independent
// chains. Lookup tables (4 slicing tables + 4 shift tables, 8 KiB) are
// replicated 16 times, bank-interleaved, and lane l reads copy l % 16, so
// only lanes l and l + 16 can collide on a bank. A finalize kernel folds
// the spans of each block with one CTA per block: each thread folds a
// contiguous run of spans (one multiply by x^(8S) per span), then a tree
// combines the runs. Multiplication by x^(8L) uses a 41-entry table of
// powers x^(8*2^k), so a shift costs popcount(L) carry-less multiplies.
#include <cuda_runtime.h>

#include <mutex>

#include "kernels/common.cuh"

namespace mpcomm {
namespace kern {

namespace {

constexpr uint32_t kPoly = 0xEDB88320u;
constexpr uint32_t kOne = 0x80000000u;  // x^0 in the reflected representation
constexpr int kRowThreads = 1024;
constexpr int kRowBytes = 512;           // one warp-wide row: 32 lanes x 16 bytes
constexpr int kTables = 8;               // T0..T3 (slicing), U0..U3 (shift by 496 bytes)
constexpr int kCopies = 16;
constexpr size_t kTabSmem = static_cast<size_t>(kTables) * 256 * kCopies * sizeof(uint32_t);  // 128 KiB
constexpr int64_t kNominalWarps = 148 * (kRowThreads / 32);  // one CTA per SM on a B200
constexpr int64_t kMinSpan = 4096;
constexpr int kFinThreads = 256;

struct Powers {
    uint32_t x[41];    // x[k] = x^(8 * 2^k) mod P, reflected
    uint32_t tab[8];   // table multipliers: T_s = x^(8(s+1)), U_k = x^(8(496-k))
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
    for (int s = 0; s < 4; ++s) p.tab[s] = gf2_shift(kOne, static_cast<uint64_t>(s + 1), p.x);
    for (int k = 0; k < 4; ++k) p.tab[4 + k] = gf2_shift(kOne, static_cast<uint64_t>(kRowBytes - 16 - k), p.x);
    return p;
}

// Table t, entry e, copy c: word ((t * 256 + e) * kCopies + c).
__device__ __forceinline__ uint32_t lookup(const uint32_t *tab, int t, uint32_t e, int c) {
    return tab[((t * 256 + static_cast<int>(e)) << 4) + c];
}

// Four slicing-by-4 lookups: shift(c ^ w, 4).
__device__ __forceinline__ uint32_t step4(const uint32_t *tab, uint32_t c, uint32_t w, int cp) {
    c ^= w;
    return lookup(tab, 3, c & 0xFFu, cp) ^ lookup(tab, 2, (c >> 8) & 0xFFu, cp) ^
           lookup(tab, 1, (c >> 16) & 0xFFu, cp) ^ lookup(tab, 0, c >> 24, cp);
}

// shift(c, 496) by the U tables.
__device__ __forceinline__ uint32_t shift496(const uint32_t *tab, uint32_t c, int cp) {
    return lookup(tab, 4, c & 0xFFu, cp) ^ lookup(tab, 5, (c >> 8) & 0xFFu, cp) ^
           lookup(tab, 6, (c >> 16) & 0xFFu, cp) ^ lookup(tab, 7, c >> 24, cp);
}

__device__ __forceinline__ uint32_t row16(const uint32_t *tab, uint32_t c, int4 v, int cp) {
    c = shift496(tab, c, cp);
    c = step4(tab, c, static_cast<uint32_t>(v.x), cp);
    c = step4(tab, c, static_cast<uint32_t>(v.y), cp);
    c = step4(tab, c, static_cast<uint32_t>(v.z), cp);
    return step4(tab, c, static_cast<uint32_t>(v.w), cp);
}

// R() of [p, p+len), one byte at a time (tails and unaligned data).
__device__ __forceinline__ uint32_t crc_bytes(const uint32_t *tab, const unsigned char *p, uint64_t len, int cp) {
    uint32_t c = 0;
    for (uint64_t i = 0; i < len; ++i) c = (c >> 8) ^ lookup(tab, 0, (c ^ p[i]) & 0xFFu, cp);
    return c;
}

__device__ __forceinline__ uint32_t warp_xor(uint32_t v) {
#pragma unroll
    for (int k = 16; k; k >>= 1) v ^= __shfl_xor_sync(0xffffffffu, v, k);
    return v;
}

// R() of one span, computed by the whole warp (result valid in every lane).
__device__ __forceinline__ uint32_t warp_span_crc(const uint32_t *tab, const unsigned char *base, uint64_t len,
                                                  int lane, uint32_t lane_k, const Powers &pw) {
    const int cp = lane & (kCopies - 1);
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) {
        // Unaligned: lane l takes a contiguous 1/32 of the span, byte by byte.
        const uint64_t q = (len + 31) / 32;
        const uint64_t a = q * static_cast<uint64_t>(lane) < len ? q * lane : len;
        const uint64_t b = a + q < len ? a + q : len;
        return warp_xor(gf2_shift(crc_bytes(tab, base + a, b - a, cp), len - b, pw.x));
    }
    const uint64_t nrows = len / kRowBytes;
    const uint64_t tail = len - nrows * kRowBytes;
    const uint64_t ha = nrows / 2, hb = nrows - ha;  // rows of chain A / chain B (hb >= ha)
    const int4 *pa = reinterpret_cast<const int4 *>(base) + lane;
    const int4 *pb = reinterpret_cast<const int4 *>(base + ha * kRowBytes) + lane;
    constexpr int kStride = kRowBytes / 16;
    uint32_t ca = 0, cb = 0;
    if (hb) {
        int4 na = ha ? ld_stream_v4(pa) : make_int4(0, 0, 0, 0);
        int4 nb = ld_stream_v4(pb);
        for (uint64_t r = 0; r < hb; ++r) {
            const int4 va = na, vb = nb;
            if (r + 1 < ha) na = ld_stream_v4(pa + (r + 1) * kStride);
            if (r + 1 < hb) nb = ld_stream_v4(pb + (r + 1) * kStride);
            if (r < ha) ca = row16(tab, ca, va, cp);
            cb = row16(tab, cb, vb, cp);
        }
    }
    // Column l ends 496 - 16l bytes before the end of its half.
    const uint32_t ya = warp_xor(gf2_mul(ca, lane_k));
    const uint32_t yb = warp_xor(gf2_mul(cb, lane_k));
    uint32_t yt = 0;
    if (tail) {
        const unsigned char *t = base + nrows * kRowBytes;
        const uint64_t a = 16u * lane < tail ? 16u * lane : tail;
        const uint64_t b = a + 16 < tail ? a + 16 : tail;
        yt = warp_xor(gf2_shift(crc_bytes(tab, t + a, b - a, cp), tail - b, pw.x));
    }
    return gf2_shift(ya, hb * kRowBytes + tail, pw.x) ^ gf2_shift(yb, tail, pw.x) ^ yt;
}

// Persistent: warp g of the grid computes spans g, g + #warps, ... of the
// n * spb spans (block b = span / spb) and writes R(span) to span_crc.
__global__ void __launch_bounds__(kRowThreads, 1)
    crc_rows_kernel(const unsigned char *__restrict__ data, int64_t n, int64_t bs, int64_t span, int64_t spb,
                    uint32_t *__restrict__ span_crc, const __grid_constant__ Powers pw) {
    extern __shared__ __align__(16) uint32_t tab[];
    for (int i = threadIdx.x; i < kTables * 256; i += blockDim.x) {
        const uint32_t v = gf2_mul(static_cast<uint32_t>(i & 255), pw.tab[i >> 8]);
#pragma unroll
        for (int c = 0; c < kCopies; ++c) tab[(i << 4) + c] = v;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const uint32_t lane_k = gf2_shift(kOne, static_cast<uint64_t>(kRowBytes - 16 - 16 * lane), pw.x);
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t total = n * spb;
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < total;
         g += nw) {
        const int64_t b = g / spb, p = g - b * spb;
        const int64_t off = p * span;
        const int64_t len = bs - off < span ? bs - off : span;
        const uint32_t r = warp_span_crc(tab, data + b * bs + off, static_cast<uint64_t>(len), lane, lane_k, pw);
        if (lane == 0) span_crc[g] = r;
    }
}

// One CTA per block: thread t folds spans [t*k, (t+1)*k) in order, then the
// runs are folded by a shuffle tree and across warps.
__global__ void __launch_bounds__(kFinThreads)
    crc_finalize_kernel(const uint32_t *__restrict__ span_crc, int64_t n, int64_t bs, int64_t span, int64_t spb,
                        uint32_t x_span, uint32_t *__restrict__ out, const __grid_constant__ Powers pw) {
    __shared__ uint32_t wc[kFinThreads / 32];
    __shared__ uint64_t wl[kFinThreads / 32];
    const int64_t b = blockIdx.x;
    const int tid = threadIdx.x;
    const int64_t per = (spb + kFinThreads - 1) / kFinThreads;
    const int64_t p0 = tid * per < spb ? tid * per : spb;
    const int64_t p1 = p0 + per < spb ? p0 + per : spb;
    uint32_t c = 0;
    uint64_t len = 0;
    for (int64_t p = p0; p < p1; ++p) {
        const int64_t l = bs - p * span < span ? bs - p * span : span;
        // every span but the block's last is exactly `span` bytes: one multiply
        c = (l == span ? gf2_mul(c, x_span) : gf2_shift(c, static_cast<uint64_t>(l), pw.x)) ^ span_crc[b * spb + p];
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

// Span length for n blocks of bs bytes: about one span per resident warp of
// a B200 (deterministic in (n, bs), so scratch sizing needs no device).
int64_t span_bytes(int64_t n, int64_t bs) {
    const int64_t total = n * bs;
    int64_t s = (total + kNominalWarps - 1) / kNominalWarps;
    s = (s + 1023) / 1024 * 1024;
    return s < kMinSpan ? kMinSpan : s;
}

const Powers &powers() {
    static const Powers p = make_powers();
    return p;
}

}  // namespace

size_t crc32_scratch_words(int64_t n, int64_t bs) {
    if (n <= 0 || bs <= 0) return 0;
    const int64_t span = span_bytes(n, bs);
    return static_cast<size_t>(n * ((bs + span - 1) / span));
}

int crc32_blocks_scratch(const void *data, int64_t n, int64_t bs, uint32_t *out, uint32_t *scratch,
                         size_t scratch_words, void *stream) {
    if (!data || !out || !scratch || n <= 0 || bs <= 0) return cudaErrorInvalidValue;
    const int64_t span = span_bytes(n, bs);
    const int64_t spb = (bs + span - 1) / span;
    if (static_cast<size_t>(n * spb) > scratch_words) return cudaErrorInvalidValue;
    if (n > 0x7fffffff) return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        static std::mutex mu;
        static uint64_t configured = 0;  // bit per device
        std::lock_guard<std::mutex> g(mu);
        if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
        if (!(configured & (1ull << dev))) {
            cudaError_t e = cudaFuncSetAttribute(crc_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(kTabSmem));
            if (e != cudaSuccess) return e;
            configured |= 1ull << dev;
        }
    }
    const int64_t warps = n * spb;
    const int64_t need = (warps + kRowThreads / 32 - 1) / (kRowThreads / 32);
    const int sms = sm_count(dev) > 0 ? sm_count(dev) : 148;
    const int ctas = static_cast<int>(need < sms ? need : sms);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const Powers &pw = powers();
    crc_rows_kernel<<<ctas, kRowThreads, kTabSmem, st>>>(static_cast<const unsigned char *>(data), n, bs, span, spb,
                                                         scratch, pw);
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const uint32_t x_span = gf2_shift(kOne, static_cast<uint64_t>(span), pw.x);
    crc_finalize_kernel<<<static_cast<unsigned>(n), kFinThreads, 0, st>>>(scratch, n, bs, span, spb, x_span, out,
                                                                         pw);
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
            // stream, so it is not freed; it is small (4 bytes per span).
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
