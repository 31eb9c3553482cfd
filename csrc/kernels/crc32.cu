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
// a warp owns a span and reads it as 1 KiB rows, lane l loading bytes
// [32l, 32l+32) of every row with one 256-bit load — fully coalesced. Lane
// l thus sees a "column" of its span, 32 bytes every 1,024. Its register X
// follows
//     X <- shift(X, 1024) ^ R(row piece)
// computed as one table shift by 992 bytes (eight nibble-table lookups)
// followed by the ordinary slicing-by-4 steps over the 32 bytes (which
// shift by the remaining 32). At the end lane l's column contributes
// shift(X_l, 992 - 32l) to the span and the lanes are xor-reduced. The
// span's rows are split in two halves so each lane runs two independent
// chains. Lookup tables (4 slicing tables of 256 entries + 8 nibble shift
// tables of 16 entries, 4.5 KiB) are replicated 32 times, bank-interleaved,
// and lane l reads copy l at 32-bit shared addresses: no bank conflicts.
//
// crc_finalize_kernel (one CTA per block, launched with programmatic
// dependent launch so its launch overlaps the row kernel) folds the block's
// full spans: thread t folds a power-of-two run of spans (one multiply by
// x^(8S) each), runs are combined by a shuffle tree and across warps with
// multipliers x^(8S*2^j) from the host, then the partial last span, the
// initial register and the final xor are applied with host constants.
// Multiplication by x^(8L) in general uses a 41-entry table of powers
// x^(8*2^k), so a shift costs popcount(L) carry-less multiplies.
#include <cuda_runtime.h>

#include <mutex>

#include "kernels/common.cuh"

namespace mpcomm {
namespace kern {

namespace {

constexpr uint32_t kPoly = 0xEDB88320u;
constexpr uint32_t kOne = 0x80000000u;  // x^0 in the reflected representation
constexpr int kRowThreads = 1024;
constexpr int kRowBytes = 1024;          // one warp-wide row: 32 lanes x 32 bytes
constexpr int kCopies = 32;             // one table copy per lane: conflict-free lookups
// Slicing tables T0..T3 (256 entries) then nibble shift tables N0..N7 (16
// entries), each entry replicated kCopies times (128 bytes per entry).
constexpr uint32_t kEntryBytes = kCopies * 4;
constexpr uint32_t kTBytes = 256 * kEntryBytes;                 // 32 KiB per slicing table
constexpr uint32_t kNBase = 4 * kTBytes;                        // nibble tables start at 128 KiB
constexpr uint32_t kNBytes = 16 * kEntryBytes;                  // 2 KiB per nibble table
constexpr size_t kTabBytes = kNBase + 8 * kNBytes;              // 144 KiB
constexpr size_t kTabSmem = kTabBytes + 32768;                  // room to align the tables to 32 KiB
constexpr int64_t kNominalWarps = 148 * (kRowThreads / 32);  // one CTA per SM on a B200
constexpr int64_t kMinSpan = 4096;
constexpr int kFinThreads = 256;

struct Powers {
    uint32_t x[41];    // x[k] = x^(8 * 2^k) mod P, reflected
    uint32_t tab[4];   // slicing-table multipliers: T_s = x^(8(s+1))
    uint32_t nib[8];   // nibble-table multipliers: x^(8 * 992) (entry v of N_j is (v << 4j) times it)
};

// Host-computed constants of one crc32_blocks call (every block has the
// same size, so one set serves all blocks; cached per (bs, span)).
struct FinalizeConsts {
    uint32_t mtab[4][256];         // c -> c * x^(8S): xor of mtab[k][byte k of c]
    uint32_t mult[kFinThreads];    // thread t's run -> block end: x^(8 S (nfull - end_t))
    uint32_t x_last;               // x^(8 * last_len)
    uint32_t init_term;            // shift(0xFFFFFFFF, bs) ^ 0xFFFFFFFF
    int64_t nfull;                 // full spans per block
    int64_t last_len;              // bytes of the partial last span (0: none)
    int64_t spb;                   // spans per block
    int64_t per;                   // full spans folded per thread
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
    // Nibble j of the register sits 4j bits into it: N_j[v] = (v << 4j) * x^(8*992).
    const uint32_t row = gf2_shift(kOne, static_cast<uint64_t>(kRowBytes - 32), p.x);
    for (int j = 0; j < 8; ++j) p.nib[j] = row;
    return p;
}

// Lookups. The tables start on a 32 KiB boundary of shared memory and
// lane l reads copy l, so the 32-bit address of an entry is
// (entry << 7) | lane_base (lane_base = table base + 4 * lane) plus the
// table's immediate offset: a shift and one LOP3 per lookup.
template <uint32_t OFF>
__device__ __forceinline__ uint32_t lut_addr(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
    return v;
}
// Byte k of c as a slicing-table entry address: PRMT extracts the byte and
// a multiply-add scales it (mad.lo runs on the FMA pipe, which the table
// walk leaves idle, instead of a shift and a LOP3 on the integer ALU).
__device__ __forceinline__ uint32_t mad128(uint32_t e, uint32_t lb) {
    uint32_t a;
    asm("mad.lo.u32 %0, %1, 128, %2;" : "=r"(a) : "r"(e), "r"(lb));
    return a;
}
__device__ __forceinline__ uint32_t at0(uint32_t lb, uint32_t c) { return mad128(__byte_perm(c, 0u, 0x4440u), lb); }
__device__ __forceinline__ uint32_t at1(uint32_t lb, uint32_t c) { return mad128(__byte_perm(c, 0u, 0x4441u), lb); }
__device__ __forceinline__ uint32_t at2(uint32_t lb, uint32_t c) { return mad128(__byte_perm(c, 0u, 0x4442u), lb); }
__device__ __forceinline__ uint32_t at3(uint32_t lb, uint32_t c) { return mad128(c >> 24, lb); }

// Four slicing-by-4 lookups: shift(c ^ w, 4).
__device__ __forceinline__ uint32_t step4(uint32_t lb, uint32_t c, uint32_t w) {
    c ^= w;
    return lut_addr<3 * kTBytes>(at0(lb, c)) ^ lut_addr<2 * kTBytes>(at1(lb, c)) ^
           lut_addr<1 * kTBytes>(at2(lb, c)) ^ lut_addr<0>(at3(lb, c));
}

// shift(c, 992) by the nibble tables: nibble j of c, address bits [7, 11).
__device__ __forceinline__ uint32_t shift_row(uint32_t lb, uint32_t c) {
    return lut_addr<kNBase + 0 * kNBytes>(((c << 7) & 0x780u) | lb) ^
           lut_addr<kNBase + 1 * kNBytes>(((c << 3) & 0x780u) | lb) ^
           lut_addr<kNBase + 2 * kNBytes>(((c >> 1) & 0x780u) | lb) ^
           lut_addr<kNBase + 3 * kNBytes>(((c >> 5) & 0x780u) | lb) ^
           lut_addr<kNBase + 4 * kNBytes>(((c >> 9) & 0x780u) | lb) ^
           lut_addr<kNBase + 5 * kNBytes>(((c >> 13) & 0x780u) | lb) ^
           lut_addr<kNBase + 6 * kNBytes>(((c >> 17) & 0x780u) | lb) ^
           lut_addr<kNBase + 7 * kNBytes>(((c >> 21) & 0x780u) | lb);
}

struct V8 {
    uint32_t w[8];
};

__device__ __forceinline__ V8 ld_v8(const void *p) {
    V8 v;
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                   "=r"(v.w[6]), "=r"(v.w[7])
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t row32(uint32_t lb, uint32_t c, const V8 &v) {
    c = shift_row(lb, c);
#pragma unroll
    for (int k = 0; k < 8; ++k) c = step4(lb, c, v.w[k]);
    return c;
}

// R() of [p, p+len), one byte at a time (tails and unaligned data).
__device__ __forceinline__ uint32_t crc_bytes(uint32_t lb, const unsigned char *p, uint64_t len) {
    uint32_t c = 0;
    for (uint64_t i = 0; i < len; ++i) c = (c >> 8) ^ lut_addr<0>(at0(lb, c ^ p[i]));  // T0
    return c;
}

__device__ __forceinline__ uint32_t warp_xor(uint32_t v) {
#pragma unroll
    for (int k = 16; k; k >>= 1) v ^= __shfl_xor_sync(0xffffffffu, v, k);
    return v;
}

// R() of one span, computed by the whole warp (result valid in every lane).
__device__ __forceinline__ uint32_t warp_span_crc(uint32_t lb, const unsigned char *base, uint64_t len, int lane,
                                                  uint32_t lane_k, const Powers &pw) {
    if ((reinterpret_cast<uintptr_t>(base) & 31u) != 0) {
        // Not 32-byte aligned: lane l takes a contiguous 1/32 of the span.
        const uint64_t q = (len + 31) / 32;
        const uint64_t a = q * static_cast<uint64_t>(lane) < len ? q * lane : len;
        const uint64_t b = a + q < len ? a + q : len;
        return warp_xor(gf2_shift(crc_bytes(lb, base + a, b - a), len - b, pw.x));
    }
    const uint64_t nrows = len / kRowBytes;
    const uint64_t tail = len - nrows * kRowBytes;
    const uint64_t ha = nrows / 2, hb = nrows - ha;  // rows of chain A / chain B (hb >= ha)
    const unsigned char *pa = base + 32 * lane;
    const unsigned char *pb = base + ha * kRowBytes + 32 * lane;
    uint32_t ca = 0, cb = 0;
    if (hb) {
        V8 na = ha ? ld_v8(pa) : V8{};
        V8 nb = ld_v8(pb);
        for (uint64_t r = 0; r < hb; ++r) {
            const V8 va = na, vb = nb;
            if (r + 1 < ha) na = ld_v8(pa + (r + 1) * kRowBytes);
            if (r + 1 < hb) nb = ld_v8(pb + (r + 1) * kRowBytes);
            if (r < ha) ca = row32(lb, ca, va);
            cb = row32(lb, cb, vb);
        }
    }
    // Column l ends 992 - 32l bytes before the end of its half.
    const uint32_t ya = warp_xor(gf2_mul(ca, lane_k));
    const uint32_t yb = warp_xor(gf2_mul(cb, lane_k));
    uint32_t yt = 0;
    if (tail) {
        const unsigned char *t = base + nrows * kRowBytes;
        const uint64_t a = 32u * lane < tail ? 32u * lane : tail;
        const uint64_t b = a + 32 < tail ? a + 32 : tail;
        yt = warp_xor(gf2_shift(crc_bytes(lb, t + a, b - a), tail - b, pw.x));
    }
    return gf2_shift(ya, hb * kRowBytes + tail, pw.x) ^ gf2_shift(yb, tail, pw.x) ^ yt;
}

// Persistent: warp g of the grid computes spans g, g + #warps, ... of the
// n * spb spans (block b = span / spb) and writes R(span) to span_crc.
__global__ void __launch_bounds__(kRowThreads, 1)
    crc_rows_kernel(const unsigned char *__restrict__ data, int64_t n, int64_t bs, int64_t span, int64_t spb,
                    uint32_t *__restrict__ span_crc, const __grid_constant__ Powers pw) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t tab_base = (raw + 32767u) & ~32767u;
    uint32_t *tab = reinterpret_cast<uint32_t *>(smem_raw + (tab_base - raw));
    for (int i = threadIdx.x; i < 4 * 256 + 8 * 16; i += blockDim.x) {
        // slicing entries first (i < 1024), then the nibble entries
        const uint32_t v = i < 1024 ? gf2_mul(static_cast<uint32_t>(i & 255), pw.tab[i >> 8])
                                    : gf2_mul(static_cast<uint32_t>((i - 1024) & 15) << (4 * ((i - 1024) >> 4)),
                                              pw.nib[(i - 1024) >> 4]);
#pragma unroll 8
        for (int c = 0; c < kCopies; ++c) tab[i * kCopies + c] = v;
    }
    __syncthreads();
    // The finalize kernel may be scheduled now; it waits for this grid's
    // completion (griddepcontrol.wait) before reading span_crc.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const uint32_t lb = tab_base + static_cast<uint32_t>(lane) * 4u;
    const uint32_t lane_k = gf2_shift(kOne, static_cast<uint64_t>(kRowBytes - 32 - 32 * lane), pw.x);
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t total = n * spb;
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < total;
         g += nw) {
        const int64_t b = g / spb, p = g - b * spb;
        const int64_t off = p * span;
        const int64_t len = bs - off < span ? bs - off : span;
        const uint32_t r = warp_span_crc(lb, data + b * bs + off, static_cast<uint64_t>(len), lane, lane_k, pw);
        if (lane == 0) span_crc[g] = r;
    }
}

// One CTA per block (see the layout note at the top of the file).
__global__ void __launch_bounds__(kFinThreads)
    crc_finalize_kernel(const uint32_t *__restrict__ span_crc, uint32_t *__restrict__ out,
                        const __grid_constant__ FinalizeConsts fc) {
    __shared__ uint32_t mt[4][256];
    __shared__ uint32_t wx[kFinThreads / 32];
    const int tid = threadIdx.x;
    for (int i = tid; i < 1024; i += kFinThreads) mt[i >> 8][i & 255] = fc.mtab[i >> 8][i & 255];
    __syncthreads();
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int64_t b = blockIdx.x;
    const int64_t p0 = tid * fc.per < fc.nfull ? tid * fc.per : fc.nfull;
    const int64_t p1 = p0 + fc.per < fc.nfull ? p0 + fc.per : fc.nfull;
    const uint32_t *sc = span_crc + b * fc.spb;
    uint32_t c = 0;
    for (int64_t p = p0; p < p1; ++p)
        c = mt[0][c & 255u] ^ mt[1][(c >> 8) & 255u] ^ mt[2][(c >> 16) & 255u] ^ mt[3][c >> 24] ^ sc[p];
    // Each run's contribution, already shifted to the end of the full spans:
    // xor-combining needs no further shifts.
    c = warp_xor(gf2_mul(c, fc.mult[tid]));
    if ((tid & 31) == 0) wx[tid >> 5] = c;
    __syncthreads();
    if (tid == 0) {
        uint32_t acc = 0;
        for (int w = 0; w < kFinThreads / 32; ++w) acc ^= wx[w];
        if (fc.last_len) acc = gf2_mul(acc, fc.x_last) ^ sc[fc.nfull];
        out[b] = fc.init_term ^ acc;
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
    // Finalize constants (all blocks have the same size), cached per (bs, span).
    static std::mutex fmu;
    static int64_t f_bs = -1, f_span = -1;
    static FinalizeConsts fc;
    FinalizeConsts fcl;
    {
        std::lock_guard<std::mutex> g(fmu);
        if (f_bs != bs || f_span != span) {
            const uint32_t q = gf2_shift(kOne, static_cast<uint64_t>(span), pw.x);
            for (int k = 0; k < 4; ++k)
                for (uint32_t v = 0; v < 256; ++v) fc.mtab[k][v] = gf2_mul(v << (8 * k), q);
            fc.nfull = bs / span;
            fc.last_len = bs - fc.nfull * span;
            fc.spb = spb;
            fc.per = (fc.nfull + kFinThreads - 1) / kFinThreads;
            if (fc.per < 1) fc.per = 1;
            for (int t = 0; t < kFinThreads; ++t) {
                int64_t end = (t + 1) * fc.per;
                if (end > fc.nfull) end = fc.nfull;
                fc.mult[t] = gf2_shift(kOne, static_cast<uint64_t>((fc.nfull - end) * span), pw.x);
            }
            fc.x_last = gf2_shift(kOne, static_cast<uint64_t>(fc.last_len), pw.x);
            fc.init_term = gf2_shift(0xFFFFFFFFu, static_cast<uint64_t>(bs), pw.x) ^ 0xFFFFFFFFu;
            f_bs = bs;
            f_span = span;
        }
        fcl = fc;
    }
    // Programmatic dependent launch: the finalize grid is set up while the
    // row kernel runs and waits on griddepcontrol.wait for its completion.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(n));
    cfg.blockDim = dim3(kFinThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, crc_finalize_kernel, static_cast<const uint32_t *>(scratch), out, fcl);
    note_launch();
    if (e != cudaSuccess) return e;
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
