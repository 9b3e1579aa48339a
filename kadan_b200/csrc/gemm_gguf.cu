// GGUF prefill GEMM on the fifth-generation tensor cores (sm_100a): Q4_K,
// Q6_K and Q8_0 weights.
//
// Replaces the reference's prefill projection for packed weights
// (services/hikari/inference_worker/src/cuda/h3_compute.cu:1781-2480:
// gguf_decode_kernel to an fp32 tile in scratch, :76-95 / :2201-2218, then an
// FP32 cublasSgemm, :2435-2468): Y[t, n] = sum_k decode(W[n, k]) * X[t, k] for
// T input rows, without the fp32 tile in HBM and on the tensor pipe.
//
//   activations : each input row t is scaled by 2^-e_t (e_t puts its absmax in
//                 [2^14, 2^15), exact) and rounded to fp16 once, by a small
//                 kernel, into [T, K] scratch; the epilogue multiplies by 2^e_t
//   weights     : per weight tile and 256 values of K, one TMA load of the
//                 packed bytes of every row of the tile (a "raw stage"):
//                   Q4_K  one 144-byte super-block (3-D map, the GEMV's)
//                   Q6_K  240 bytes from the 16-byte boundary at or below the
//                         210-byte super-block (it starts 2 (kb mod 8) bytes in)
//                   Q8_0  eight 34-byte blocks, 272 bytes (16-byte aligned)
//                 Eight dequant warps turn each raw stage into four 64-value
//                 fp16 B stages in the 128-byte-swizzled K-major layout:
//                   Q4_K  q*sc = fma(1024 + q, sc, -1024 sc)   exact in fp16
//                         w    = fma(q*sc, d, -(dmin*m))       one rounding
//                   Q6_K  q - 32 exact (1024 + q, less 1056), times
//                         fp16(d * sc)                          two roundings
//                   Q8_0  q exact (1152 + q, less 1152), times d  one rounding
//                 (1024 + q comes from the code bits by a byte permute)
//   MMA         : tcgen05.mma kind::f16, M = 128 input rows, N = 256 weight
//                 rows (Q4_K, when 256-row tiles still give every SM a tile)
//                 or 128, K = 16 per instruction, fp32 accumulators in TMEM
//                 (two N-column buffers, so the epilogue of one tile overlaps
//                 the next tile's MMAs)
//   epilogue    : TMEM -> registers (32x32b.x32), * 2^e_t, fp32 rows of Y
//
// fp16 operands hold every weight whose magnitude is below 65504; a block whose
// scales could exceed that is reported (status bit 2 and the workspace's range
// word) and the caller recomputes the job on the GEMV path.
//
// CTA = 14 warps: TMA producer, MMA issuer, 8 dequant warps (one weight row
// per thread, or half a row for 128-row tiles), 4 epilogue warps (one TMEM
// lane quarter each). Persistent
// over tiles; consecutive CTAs take the M tiles of one weight tile, so the
// weight bytes come from DRAM once and from L2 for the other input rows.
// Every wait is bounded and reports to the watchdog word.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <mutex>

#include "gguf_formats.cuh"
#include "kb200_host.hpp"
#include "tcgen05.cuh"

namespace kb200 {
namespace {

constexpr int BM = 128, BK = 64;
constexpr int kABytes = BM * BK * 2;
constexpr int kDequantWarps = 8;
constexpr int kThreads = 32 * (2 + kDequantWarps + 4);
constexpr float kHalfMax = 65504.f;

// Weight formats of the GEMM. kPitch: bytes per row of a raw stage (the TMA
// box of one 256-value step of K; a multiple of 16, and an odd number of
// 16-byte words, so the dequant warps' 16-byte reads of 8 consecutive rows hit
// distinct banks). kBlockBytes/kBlockValues: the GGUF block.
enum Fmt : int { kQ4K = 0, kQ6K = 1, kQ80 = 2 };
template <int F> struct Format;
template <> struct Format<kQ4K> {
    static constexpr int kPitch = 144, kBlockBytes = 144, kBlockValues = 256;
};
template <> struct Format<kQ6K> {
    static constexpr int kPitch = 240, kBlockBytes = 210, kBlockValues = 256;
};
template <> struct Format<kQ80> {
    static constexpr int kPitch = 272, kBlockBytes = 34, kBlockValues = 32;
};

// Tile geometry per format and weight-tile height BN (the MMA's N: 128 or 256
// weight rows). Rings hold one K step of 64 per A/B stage and 256 values of K
// per raw stage. A 256-row tile halves the activation bytes per FLOP: the
// activation tiles arrive at about 30 GB/s per SM (measured, a 16 KB tile
// every ~0.5 us with ~2 us of latency), which caps 128-row tiles; only Q4_K's
// raw stages are small enough for 256-row tiles in shared memory.
template <int F, int BN> struct Tile {
    static constexpr int kAStages = BN == 256 ? 5 : 4;
    static constexpr int kBStages = BN == 256 ? 2 : 4;
    static constexpr int kRawStages = 2;
    static constexpr int kBBytes = BN * BK * 2, kRawBytes = BN * Format<F>::kPitch;
    static constexpr int kThreadsPerRow = 32 * kDequantWarps / BN;  // 2 or 1
    static constexpr int kSmemA = 0;
    static constexpr int kSmemB = kSmemA + kAStages * kABytes;
    static constexpr int kSmemRaw = kSmemB + kBStages * kBBytes;
    static constexpr int kSmemBars = kSmemRaw + kRawStages * kRawBytes;
};

struct Bars {
    uint64_t a_full[5], a_empty[5], b_full[4], b_empty[4];
    uint64_t raw_full[2], raw_empty[2];
    uint64_t acc_full[2], acc_empty[2];
    uint32_t tmem_base;
    int abort;
};

template <int F, int BN> constexpr int smem_total() {
    return Tile<F, BN>::kSmemBars + int(sizeof(Bars)) + 1024;  // + 1024-byte alignment slack
}
static_assert(smem_total<kQ4K, 256>() <= 227 * 1024, "Q4_K 256-row tile fits shared memory");
static_assert(smem_total<kQ6K, 128>() <= 227 * 1024, "Q6_K 128-row tile fits shared memory");
static_assert(smem_total<kQ80, 128>() <= 227 * 1024, "Q8_0 128-row tile fits shared memory");

struct GemmParams {
    CUtensorMap a_map;   // fp16 [T, K], box {64, 128}, 128-byte swizzle
    CUtensorMap w_map;   // Q4_K: u64 {18, K/256, N}, box {18, 1, BN};
                         // Q6_K / Q8_0: u64 {row_bytes/8, N}, box {30 / 34, BN}
    const int* row_exp;  // [T] e_t
    float* out;          // [T][stride]
    unsigned* status;    // or null: bit 0 a weight is not finite, bit 1 out of fp16 range
    unsigned* range;     // workspace word: nonzero when a weight may exceed the fp16 range
    unsigned* watchdog;
    int T, N, nblocks, m_tiles, n_tiles;
    uint32_t stride;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_addr(dst)
        ),
        "l"(map),
        "r"(c0),
        "r"(c1),
        "r"(c2),
        "r"(smem_addr(bar))
        : "memory"
    );
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t half2_bits(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// fp16 pairs (1024 + low nibble) of code bytes b and b+1 of `w` (b = 0 or 2,
// chosen by `sel`), and (1024 + high nibble) of the same bytes.
__device__ __forceinline__ void nibble_pairs(uint32_t w, uint32_t sel, uint32_t& lo, uint32_t& hi) {
    const uint32_t p = __byte_perm(w, 0x64646464u, sel);  // [w.b, 0x64, w.b+1, 0x64]
    lo = p & 0xFF0FFF0Fu;
    hi = ((p >> 4) & 0x000F000Fu) | 0x64006400u;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// Eight words starting `shift` bits (0 or 16) into word WQ of `w`.
template <int WQ> __device__ __forceinline__ void take8(const uint32_t (&w)[12], uint32_t shift, uint32_t (&out)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
        out[i] = __funnelshift_r(w[WQ + i], w[WQ + i + 1], shift);
}

// The 32 bytes at offset `o` (even, below 16) of 16-byte aligned shared memory
// `at`, as 8 words: three 16-byte reads and a funnel shift (`o` is the same
// for every thread of the warp, so the switch does not diverge).
__device__ __forceinline__ void bytes32(const uint8_t* at, uint32_t o, uint32_t (&out)[8]) {
    uint32_t w[12];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const uint4 v = *reinterpret_cast<const uint4*>(at + 16 * k);
        w[4 * k] = v.x, w[4 * k + 1] = v.y, w[4 * k + 2] = v.z, w[4 * k + 3] = v.w;
    }
    const uint32_t shift = 8u * (o & 3u);
    switch (o >> 2) {
    case 0: take8<0>(w, shift, out); break;
    case 1: take8<1>(w, shift, out); break;
    case 2: take8<2>(w, shift, out); break;
    default: take8<3>(w, shift, out); break;
    }
}

// Per raw stage (256 values of K of one weight row), what the four 64-value
// steps of a dequant thread share.
template <int F> struct RowState;
template <> struct RowState<kQ4K> {
    uint32_t d2, sw[8], cw[8], mn[8];
};
template <> struct RowState<kQ6K> {
    uint32_t o;          // byte offset of the super-block in the raw row
    uint32_t dsc[4][2];  // fp16 d * sc of this thread's two sub-blocks of each step
};
template <> struct RowState<kQ80> {};

// Q4_K super-block (ggml block_q4_K: fp16 d, dmin, 12 bytes of 6-bit scales
// and mins, 128 bytes of nibbles; w = d*sc*q - dmin*m per sub-block of 32).
__device__ __forceinline__ void prepare(RowState<kQ4K>& st, const uint8_t* blk, int, int, bool valid, bool& finite,
                                        bool& range) {
    const uint4 head = *reinterpret_cast<const uint4*>(blk);
    const float d = half_bits_to_float(head.x & 0xffffu), dmin = half_bits_to_float(head.x >> 16);
    if (valid) {
        finite = finite && isfinite(d) && isfinite(dmin);
        // Scales that are not finite are reported as such, not as out of range.
        range = range || (isfinite(d) && isfinite(dmin) && fabsf(d) * (63.f * 15.f) + fabsf(dmin) * 63.f > kHalfMax);
    }
    // 6-bit scales and mins of sub-blocks 0-3 / 4-7, one per byte.
    const uint32_t sc_lo = head.y & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (head.w & 0x0F0F0F0Fu) | ((head.y >> 2) & 0x30303030u);
    const uint32_t m_lo = head.z & 0x3F3F3F3Fu;
    const uint32_t m_hi = ((head.w >> 4) & 0x0F0F0F0Fu) | ((head.z >> 2) & 0x30303030u);
    st.d2 = half2_bits(d, d);
    // Per sub-block g: sw = sc, cw = -1024 sc (exact: sc < 64), mn = -(dmin m).
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const uint32_t scw = g < 4 ? sc_lo : sc_hi, mw = g < 4 ? m_lo : m_hi;
        const float sc = float((scw >> (8 * (g & 3))) & 0xFFu), m = float((mw >> (8 * (g & 3))) & 0xFFu);
        st.sw[g] = half2_bits(sc, sc);
        st.cw[g] = half2_bits(-1024.f * sc, -1024.f * sc);
        st.mn[g] = half2_bits(-dmin * m, -dmin * m);
    }
}

// Step j (values 64j..64j+63: sub-blocks 2j, low nibbles, and 2j+1, high
// nibbles, of code bytes 32j..32j+31) for this thread's chunks of row r.
template <int TPR>
__device__ __forceinline__ void step(const RowState<kQ4K>& st, const uint8_t* blk, int j, int part, int r, uint8_t* brow,
                                     bool, bool&, bool&) {
    constexpr int kChunks = 4 / TPR;  // 16-byte B chunks per half-stage row
    uint32_t words[2 * kChunks];
#pragma unroll
    for (int v = 0; v < kChunks / 2; ++v) {
        const uint4 cb = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j + 8 * kChunks * part + 16 * v);
        words[4 * v] = cb.x, words[4 * v + 1] = cb.y, words[4 * v + 2] = cb.z, words[4 * v + 3] = cb.w;
    }
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
        // Code bytes 8c..8c+7 -> values 8c..8c+7 of sub-block 2j (chunk c)
        // and of sub-block 2j+1 (chunk 4 + c).
        const int c = kChunks * part + cc;
        uint32_t lo[4], hi[4];
        nibble_pairs(words[2 * cc], 0x5140u, lo[0], hi[0]);
        nibble_pairs(words[2 * cc], 0x7362u, lo[1], hi[1]);
        nibble_pairs(words[2 * cc + 1], 0x5140u, lo[2], hi[2]);
        nibble_pairs(words[2 * cc + 1], 0x7362u, lo[3], hi[3]);
        uint32_t wl[4], wh[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wl[i] = hfma2(hfma2(lo[i], st.sw[2 * j], st.cw[2 * j]), st.d2, st.mn[2 * j]);
            wh[i] = hfma2(hfma2(hi[i], st.sw[2 * j + 1], st.cw[2 * j + 1]), st.d2, st.mn[2 * j + 1]);
        }
        *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
        *reinterpret_cast<uint4*>(brow + (((4 + c) ^ (r & 7)) << 4)) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
    }
}

// Q6_K super-block (ggml block_q6_K: ql[128] low nibbles, qh[64] high bit
// pairs, int8 scales[16], fp16 d; w = d*sc*(q - 32) per sub-block of 16).
// Value 64j + 8c + e of step j, chunk c: low bits = nibble (j & 1) of ql byte
// 64(j/2) + 8c + e; high bits = bits 4(j & 1) + 2(c/4) of qh byte
// 32(j/2) + 8(c % 4) + e; scale sc[4j + c/2]. The block starts `o` bytes into
// the raw row (`row`, 16-byte aligned). Two threads per row: `part` takes
// chunks 4 part .. 4 part + 3.
__device__ __forceinline__ void prepare(RowState<kQ6K>& st, const uint8_t* row, int kb, int part, bool valid,
                                        bool& finite, bool& range) {
    st.o = (210u * uint32_t(kb)) & 15u;
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + st.o + 208));
    if (valid) {
        finite = finite && isfinite(d);
        range = range || (isfinite(d) && fabsf(d) * 4096.f > kHalfMax);  // |sc| <= 128, |q - 32| <= 32
    }
    const auto* sc = reinterpret_cast<const int8_t*>(row + st.o + 192);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float v = d * float(sc[4 * j + 2 * part + h]);  // exact in fp32
            st.dsc[j][h] = half2_bits(v, v);
        }
}

__device__ __forceinline__ void step6(const RowState<kQ6K>& st, const uint8_t* row, int j, int part, int r,
                                      uint8_t* brow) {
    uint32_t ql[8], qh[8];
    bytes32(row + 64 * (j >> 1) + 32 * part, st.o, ql);
    bytes32(row + 128 + 32 * (j >> 1), st.o, qh);
    const uint32_t ls = 4u * uint32_t(j & 1), hs = ls + 2u * uint32_t(part);
    constexpr uint32_t k1056 = 0x64206420u;  // fp16 (1056, 1056): 1024 + 32
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
        const int c = 4 * part + cc;
        const uint32_t q0 = ((ql[2 * cc] >> ls) & 0x0F0F0F0Fu) | (((qh[2 * cc] >> hs) & 0x03030303u) << 4);
        const uint32_t q1 = ((ql[2 * cc + 1] >> ls) & 0x0F0F0F0Fu) | (((qh[2 * cc + 1] >> hs) & 0x03030303u) << 4);
        const uint32_t ds = st.dsc[j][cc >> 1];
        uint4 out;
        out.x = hmul2(hsub2(__byte_perm(q0, 0x64646464u, 0x5140u), k1056), ds);
        out.y = hmul2(hsub2(__byte_perm(q0, 0x64646464u, 0x7362u), k1056), ds);
        out.z = hmul2(hsub2(__byte_perm(q1, 0x64646464u, 0x5140u), k1056), ds);
        out.w = hmul2(hsub2(__byte_perm(q1, 0x64646464u, 0x7362u), k1056), ds);
        *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = out;
    }
}

template <int TPR>
__device__ __forceinline__ void step(const RowState<kQ6K>& st, const uint8_t* row, int j, int part, int r,
                                     uint8_t* brow, bool, bool&, bool&) {
    static_assert(TPR == 2, "Q6_K tiles are 128 rows: two dequant threads per row");
    step6(st, row, j, part, r, brow);
}

// Q8_0: the raw row holds eight 34-byte blocks (fp16 d, 32 int8 q; w = d*q);
// step j is blocks 2j (chunks 0-3) and 2j+1 (chunks 4-7), one per `part`.
__device__ __forceinline__ void prepare(RowState<kQ80>&, const uint8_t*, int, int, bool, bool&, bool&) {}

template <int P>
__device__ __forceinline__ void step8(const uint8_t* row, int j, int r, uint8_t* brow, bool valid, bool& finite,
                                      bool& range) {
    const int at = 34 * (2 * j + P);
    const uint32_t dbits = *reinterpret_cast<const uint16_t*>(row + at);
    const float d = half_bits_to_float(dbits);
    if (valid) {
        finite = finite && isfinite(d);
        range = range || (isfinite(d) && fabsf(d) * 128.f > kHalfMax);
    }
    const uint32_t d2 = dbits | (dbits << 16);
    const int qs = at + 2, base = qs & ~15, o = qs & 15;
    uint32_t q[8];
    if (o == 0) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint4 v = *reinterpret_cast<const uint4*>(row + base + 16 * k);
            q[4 * k] = v.x, q[4 * k + 1] = v.y, q[4 * k + 2] = v.z, q[4 * k + 3] = v.w;
        }
    } else {
        bytes32(row + base, uint32_t(o), q);
    }
    constexpr uint32_t k1152 = 0x64806480u;  // fp16 (1152, 1152): 1024 + 128
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
        const int c = 4 * P + cc;
        const uint32_t b0 = q[2 * cc] ^ 0x80808080u, b1 = q[2 * cc + 1] ^ 0x80808080u;  // q + 128
        uint4 out;
        out.x = hmul2(hsub2(__byte_perm(b0, 0x64646464u, 0x5140u), k1152), d2);
        out.y = hmul2(hsub2(__byte_perm(b0, 0x64646464u, 0x7362u), k1152), d2);
        out.z = hmul2(hsub2(__byte_perm(b1, 0x64646464u, 0x5140u), k1152), d2);
        out.w = hmul2(hsub2(__byte_perm(b1, 0x64646464u, 0x7362u), k1152), d2);
        *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = out;
    }
}

template <int TPR>
__device__ __forceinline__ void step(const RowState<kQ80>&, const uint8_t* row, int j, int part, int r, uint8_t* brow,
                                     bool valid, bool& finite, bool& range) {
    static_assert(TPR == 2, "Q8_0 tiles are 128 rows: two dequant threads per row");
    if (part)
        step8<1>(row, j, r, brow, valid, finite, range);
    else
        step8<0>(row, j, r, brow, valid, finite, range);
}

// Tile order: the M tiles of one weight tile are consecutive.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int tile, int& mt, int& nt) {
    nt = tile / p.m_tiles;
    mt = tile % p.m_tiles;
}

// The tile's i-th super-block. Each weight tile starts its K walk at a
// different super-block: the CTAs working at the same time then read
// different activation columns instead of all queueing on the same L2 lines
// (measured: a 16 KB activation tile took 2 us to arrive when every CTA
// walked K in step). The order is fixed per tile, so results are reproducible.
__device__ __forceinline__ int k_block(const GemmParams& p, int nt, int i) {
    const int b = i + nt % p.nblocks;
    return b < p.nblocks ? b : b - p.nblocks;
}

// The raw stage of weight tile nt at 256-value step kb of K.
template <int F, int BN>
__device__ __forceinline__ void load_raw(uint8_t* dst, const GemmParams& p, int kb, int nt, uint64_t* bar) {
    if constexpr (F == kQ4K)
        tma_load_3d(dst, &p.w_map, 0, kb, nt * BN, bar);
    else if constexpr (F == kQ6K)
        tma_load_2d(dst, &p.w_map, int(((210u * uint32_t(kb)) & ~15u) / 8u), nt * BN, bar);
    else
        tma_load_2d(dst, &p.w_map, 34 * kb, nt * BN, bar);
}

template <int F, int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_gguf_kernel(const __grid_constant__ GemmParams p) {
    using C = Tile<F, BN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    auto* bars = reinterpret_cast<Bars*>(smem + C::kSmemBars);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int total = p.m_tiles * p.n_tiles;
    const int KS = p.nblocks * 4;

    if (tid == 0) {
        for (int s = 0; s < C::kAStages; ++s) {
            mbar_init(&bars->a_full[s], 1);
            mbar_init(&bars->a_empty[s], 1);
        }
        for (int s = 0; s < C::kBStages; ++s) {
            mbar_init(&bars->b_full[s], 32 * kDequantWarps);
            mbar_init(&bars->b_empty[s], 1);
        }
        for (int s = 0; s < C::kRawStages; ++s) {
            mbar_init(&bars->raw_full[s], 1);
            mbar_init(&bars->raw_empty[s], kDequantWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 4);
        }
        bars->abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    volatile int* abort_flag = &bars->abort;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer
        uint32_t it = 0, rt = 0;
        for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x) {
            int mt, nt;
            tile_coords(p, tile, mt, nt);
            for (int sb = 0; sb < p.nblocks && !*abort_flag; ++sb, ++rt) {
                const int rs = int(rt % C::kRawStages);
                if (rt >= C::kRawStages
                    && !mbar_wait(&bars->raw_empty[rs], ((rt / C::kRawStages) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog)) {
                    *abort_flag = 1;
                    break;
                }
                const int kb = k_block(p, nt, sb);
                mbar_expect_tx(&bars->raw_full[rs], uint32_t(C::kRawBytes));
                load_raw<F, BN>(smem + C::kSmemRaw + rs * C::kRawBytes, p, kb, nt, &bars->raw_full[rs]);
                for (int j = 0; j < 4; ++j, ++it) {
                    const int s = int(it % C::kAStages);
                    if (it >= C::kAStages
                        && !mbar_wait(&bars->a_empty[s], ((it / C::kAStages) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog)) {
                        *abort_flag = 1;
                        break;
                    }
                    mbar_expect_tx(&bars->a_full[s], uint32_t(kABytes));
                    tma_load_2d(smem + C::kSmemA + s * kABytes, &p.a_map, (kb * 4 + j) * BK, mt * BM, &bars->a_full[s]);
                }
            }
        }
        // Every copy this thread issued lands before the CTA can exit.
        for (uint32_t k = 0; k < uint32_t(C::kAStages) && k < it; ++k) {
            const uint32_t last = it - 1 - k;
            mbar_wait(&bars->a_full[last % C::kAStages], (last / C::kAStages) & 1u, watchdog_drain, p.watchdog);
        }
        for (uint32_t k = 0; k < uint32_t(C::kRawStages) && k < rt; ++k) {
            const uint32_t last = rt - 1 - k;
            mbar_wait(&bars->raw_full[last % C::kRawStages], (last / C::kRawStages) & 1u, watchdog_drain, p.watchdog);
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------ MMA issuer
        const uint32_t idesc = idesc_f16(BM, BN);
        uint32_t it = 0, lt = 0;
        bool issued = false;
        for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x, ++lt) {
            const int acc = int(lt & 1u);
            if (lt >= 2 && !mbar_wait(&bars->acc_empty[acc], ((lt >> 1) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int sa = int(it % C::kAStages), sb = int(it % C::kBStages);
                if (!mbar_wait(&bars->a_full[sa], (it / C::kAStages) & 1u, watchdog_full_barrier, p.watchdog)
                    || !mbar_wait(&bars->b_full[sb], (it / C::kBStages) & 1u, watchdog_full_barrier, p.watchdog)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = sw128_desc(smem_addr(smem + C::kSmemA + sa * kABytes));
                const uint64_t bd = sw128_desc(smem_addr(smem + C::kSmemB + sb * C::kBBytes));
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                    umma_f16(tmem + uint32_t(acc * BN), ad + uint64_t(2 * kk), bd + uint64_t(2 * kk), idesc,
                             (ks | kk) != 0);
                umma_commit(&bars->a_empty[sa]);
                umma_commit(&bars->b_empty[sb]);
                issued = true;
            }
            umma_commit(&bars->acc_full[acc]);
        }
        if (issued && *abort_flag) {
            // Let the MMAs in flight finish before TMEM is released.
            const uint32_t last = it - 1;
            mbar_wait(&bars->b_empty[last % C::kBStages], (last / C::kBStages) & 1u, watchdog_drain, p.watchdog);
        }
    } else if (warp >= 2 && warp < 2 + kDequantWarps) {
        // ------------------------------------------------ dequant warps
        const int r = (tid - 64) % BN;     // weight row of the tile (B-operand row)
        const int part = (tid - 64) / BN;  // which half of the row's chunks (128-row tiles)
        uint32_t it = 0, rt = 0;
        bool finite = true, range = false;
        for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x) {
            int mt, nt;
            tile_coords(p, tile, mt, nt);
            const bool row_valid = nt * BN + r < p.N;
            for (int sb = 0; sb < p.nblocks && !*abort_flag; ++sb, ++rt) {
                const int rs = int(rt % C::kRawStages);
                if (!mbar_wait(&bars->raw_full[rs], (rt / C::kRawStages) & 1u, watchdog_full_barrier, p.watchdog)) {
                    *abort_flag = 1;
                    break;
                }
                const uint8_t* row = smem + C::kSmemRaw + rs * C::kRawBytes + r * Format<F>::kPitch;
                RowState<F> st;
                prepare(st, row, k_block(p, nt, sb), part, row_valid, finite, range);
#pragma unroll
                for (int j = 0; j < 4; ++j, ++it) {
                    const int s = int(it % C::kBStages);
                    // B of the stage is free once the MMAs of its previous use completed.
                    if (it >= C::kBStages
                        && !mbar_wait(&bars->b_empty[s], ((it / C::kBStages) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog)) {
                        *abort_flag = 1;
                        break;
                    }
                    step<C::kThreadsPerRow>(st, row, j, part, r, smem + C::kSmemB + s * C::kBBytes + r * 128, row_valid,
                                            finite, range);
                    fence_proxy_async();
                    mbar_arrive(&bars->b_full[s]);
                }
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&bars->raw_empty[rs]);
            }
        }
        if (!finite && p.status)
            atomicOr(p.status, 1u);
        if (range) {
            atomicOr(p.range, 1u);
            if (p.status)
                atomicOr(p.status, 2u);
        }
    } else if (warp >= 2 + kDequantWarps) {
        // ------------------------------------------------ epilogue warps
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int row = 32 * q + lane;
        uint32_t lt = 0;
        for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x, ++lt) {
            int mt, nt;
            tile_coords(p, tile, mt, nt);
            const int acc = int(lt & 1u);
            if (!mbar_wait(&bars->acc_full[acc], (lt >> 1) & 1u, watchdog_full_barrier, p.watchdog)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int t = mt * BM + row;
            const bool valid = t < p.T;
            const float scale = valid ? ldexpf(1.f, p.row_exp[t]) : 0.f;
            const uint32_t taddr = tmem + uint32_t(acc * BN) + (uint32_t(32 * q) << 16);
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                tmem_ld32(taddr + uint32_t(32 * c), v);
                tmem_wait_ld();
                const int n0 = nt * BN + 32 * c;
                if (valid && n0 < p.N) {
                    float* dst = p.out + size_t(t) * p.stride + n0;
                    const int n = min(32, p.N - n0);
                    if (n == 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            reinterpret_cast<float4*>(dst)[k] =
                                make_float4(__uint_as_float(v[4 * k]) * scale, __uint_as_float(v[4 * k + 1]) * scale,
                                            __uint_as_float(v[4 * k + 2]) * scale, __uint_as_float(v[4 * k + 3]) * scale);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i < n)
                                dst[i] = __uint_as_float(v[i]) * scale;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&bars->acc_empty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        tmem_dealloc(tmem, 2 * BN);
}

// One CTA per input row: e_t = ilogb(absmax) - 14 (0 for an all-zero row),
// xh[t, k] = fp16(x[t, k] * 2^-e_t). Rows are read as float4 when `in` is a
// multiple of 4 (always: the GEMM takes whole super-blocks). Also clears the
// range word the GEMM of the same call reports to.
__global__ void __launch_bounds__(256)
    prefill_rows_kernel(const float* x, size_t in, __half* xh, int* row_exp, unsigned* range) {
    const size_t t = blockIdx.x;
    if (t == 0 && threadIdx.x == 0)
        *range = 0u;
    const float4* xr = reinterpret_cast<const float4*>(x + t * in);
    const size_t n4 = in / 4;
    float m = 0.f;
    for (size_t k = threadIdx.x; k < n4; k += blockDim.x) {
        const float4 v = xr[k];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    __shared__ float part[8];
    if ((threadIdx.x & 31) == 0)
        part[threadIdx.x >> 5] = m;
    __syncthreads();
    float absmax = 0.f;
    for (int w = 0; w < 8; ++w)
        absmax = fmaxf(absmax, part[w]);
    const int e = absmax > 0.f && isfinite(absmax) ? max(ilogbf(absmax) - 14, -100) : 0;
    const float inv = ldexpf(1.f, -e);
    auto* dst = reinterpret_cast<uint2*>(xh + t * in);
    for (size_t k = threadIdx.x; k < n4; k += blockDim.x) {
        const float4 v = xr[k];
        dst[k] = make_uint2(half2_bits(v.x * inv, v.y * inv), half2_bits(v.z * inv, v.w * inv));
    }
    if (threadIdx.x == 0)
        row_exp[t] = e;
}

// ------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess
            && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

template <int F, int BN> int gemm_slots() {
    static int set[64] = {};
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> guard(lock);
    if (!set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(gemm_gguf_kernel<F, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   smem_total<F, BN>());
        if (e != cudaSuccess)
            return -cuda_fail(e, "gemm_gguf_kernel attribute");
        set[dev] = 1;
    }
    return sm_count();
}

size_t align256(size_t v) {
    return (v + 255) / 256 * 256;
}

size_t xh_bytes(uint32_t rows, uint32_t in) {
    return align256(size_t(rows) * in * sizeof(__half));
}

size_t exp_bytes(uint32_t rows) {
    return align256(size_t(rows) * sizeof(int));
}

template <int F, int BN> void launch_gemm(const GemmParams& p, int grid, cudaStream_t stream) {
    TraceScope trace(KB200_KERNEL_GEMM_GGUF, stream);
    gemm_gguf_kernel<F, BN><<<grid, kThreads, smem_total<F, BN>(), stream>>>(p);
}

}  // namespace

// The weights of `j` suit the GEMM: Q4_K, Q6_K or Q8_0 in whole 256-value
// steps, 16-byte aligned rows whose pitch is a multiple of 16 bytes.
bool gemm_eligible(const kb200_gemv_job& j) {
    if (j.encoding != KB200_Q4_K && j.encoding != KB200_Q6_K && j.encoding != KB200_Q8_0)
        return false;
    if (!j.in || j.in % 256 || j.row_bytes % 16 || !aligned(j.weights, 16) || j.stride > 0xffffffffu)
        return false;
    const size_t values = j.encoding == KB200_Q8_0 ? 32 : 256;
    const size_t bytes = j.encoding == KB200_Q4_K ? 144 : j.encoding == KB200_Q6_K ? 210 : 34;
    return j.row_bytes >= size_t(j.in) / values * bytes;
}

}  // namespace kb200

using namespace kb200;

extern "C" {

size_t kb200_gguf_gemm_workspace_bytes(uint32_t rows, uint32_t in) {
    return xh_bytes(rows, in) + exp_bytes(rows) + 256;
}

int kb200_gguf_gemm_supported(const kb200_gemv_job* job) {
    return job && gemm_eligible(*job) ? 1 : 0;
}

size_t kb200_gguf_gemm_range_offset(uint32_t rows, uint32_t in) {
    return xh_bytes(rows, in) + exp_bytes(rows);
}

int kb200_gguf_gemm(const kb200_gemv_job* job, void* workspace, size_t workspace_bytes, void* stream_ptr) {
    if (!job)
        return fail(KB200_INVALID, "null job");
    const kb200_gemv_job& j = *job;
    if (j.encoding != KB200_Q4_K && j.encoding != KB200_Q6_K && j.encoding != KB200_Q8_0)
        return fail(KB200_UNSUPPORTED, "the prefill GEMM takes Q4_K, Q6_K or Q8_0 weights");
    if (!j.weights || !j.input || !j.output || !j.rows || !j.columns || !j.in)
        return fail(KB200_INVALID, "empty GEMM job");
    if (!gemm_eligible(j))
        return fail(KB200_UNSUPPORTED, "the GEMM wants whole 256-value steps in 16-byte aligned rows");
    if (j.stride < j.columns)
        return fail(KB200_INVALID, "output stride shorter than the row");
    if (overlap(j.output, (size_t(j.rows - 1) * j.stride + j.columns) * sizeof(float), j.input,
                size_t(j.rows) * j.in * sizeof(float)))
        return fail(KB200_ALIAS, "output overlaps the input");
    if (!workspace || workspace_bytes < kb200_gguf_gemm_workspace_bytes(j.rows, j.in) || !aligned(workspace, 256))
        return fail(KB200_INVALID, "GEMM workspace missing, short or not 256-byte aligned");
    auto encode = encoder();
    if (!encode)
        return fail(KB200_CUDA, "cuTensorMapEncodeTiled unavailable");
    const int F = j.encoding == KB200_Q4_K ? kQ4K : j.encoding == KB200_Q6_K ? kQ6K : kQ80;
    // Q4_K: 256-row weight tiles when they still give every SM a tile.
    const int sms = sm_count();
    const int m_tiles = int((j.rows + BM - 1) / BM);
    const int BN = F == kQ4K && m_tiles * int((j.columns + 255) / 256) >= sms ? 256 : 128;
    const int slots = F == kQ6K ? gemm_slots<kQ6K, 128>()
                    : F == kQ80 ? gemm_slots<kQ80, 128>()
                    : BN == 256 ? gemm_slots<kQ4K, 256>() : gemm_slots<kQ4K, 128>();
    if (slots <= 0)
        return -slots;
    auto stream = static_cast<cudaStream_t>(stream_ptr);

    auto* base = static_cast<uint8_t*>(workspace);
    auto* xh = reinterpret_cast<__half*>(base);
    auto* row_exp = reinterpret_cast<int*>(base + xh_bytes(j.rows, j.in));
    auto* range = reinterpret_cast<unsigned*>(base + xh_bytes(j.rows, j.in) + exp_bytes(j.rows));
    cudaError_t e;
    {
        TraceScope trace(KB200_KERNEL_GEMM_PREFILL_ROWS, stream);
        prefill_rows_kernel<<<j.rows, 256, 0, stream>>>(j.input, j.in, xh, row_exp, range);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess)
        return cuda_fail(e, "prefill_rows_kernel launch");

    GemmParams p;
    std::memset(&p, 0, sizeof(p));
    {
        const cuuint64_t dims[2] = {j.in, j.rows};
        const cuuint64_t strides[1] = {uint64_t(j.in) * sizeof(__half)};
        const cuuint32_t box[2] = {BK, BM};
        const cuuint32_t es[2] = {1, 1};
        if (encode(&p.a_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)
            != CUDA_SUCCESS)
            return fail(KB200_INVALID, "cuTensorMapEncodeTiled rejected the activations");
    }
    CUresult wr;
    if (F == kQ4K) {
        // Super-blocks of 18 words, one per box column.
        const cuuint64_t dims[3] = {18, j.in / 256, j.columns};
        const cuuint64_t strides[2] = {144, j.row_bytes};
        const cuuint32_t box[3] = {18, 1, uint32_t(BN)};
        const cuuint32_t es[3] = {1, 1, 1};
        wr = encode(&p.w_map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(j.weights), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        // Rows as u64 words; a box is the raw stage's pitch of 128 rows
        // (bytes past the row's end read as zero).
        const cuuint64_t dims[2] = {j.row_bytes / 8, j.columns};
        const cuuint64_t strides[1] = {j.row_bytes};
        const cuuint32_t box[2] = {uint32_t(F == kQ6K ? Format<kQ6K>::kPitch / 8 : Format<kQ80>::kPitch / 8), 128u};
        const cuuint32_t es[2] = {1, 1};
        wr = encode(&p.w_map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(j.weights), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (wr != CUDA_SUCCESS)
        return fail(KB200_INVALID, "cuTensorMapEncodeTiled rejected the weights");
    p.row_exp = row_exp;
    p.out = j.output;
    p.status = j.status;
    p.range = range;
    p.watchdog = watchdog_word();
    p.T = int(j.rows);
    p.N = int(j.columns);
    p.nblocks = int(j.in / 256);
    p.m_tiles = m_tiles;
    p.n_tiles = int((j.columns + BN - 1) / BN);
    p.stride = uint32_t(j.stride);
    const int grid = std::max(1, std::min(slots, p.m_tiles * p.n_tiles));
    if (F == kQ6K)
        launch_gemm<kQ6K, 128>(p, grid, stream);
    else if (F == kQ80)
        launch_gemm<kQ80, 128>(p, grid, stream);
    else if (BN == 256)
        launch_gemm<kQ4K, 256>(p, grid, stream);
    else
        launch_gemm<kQ4K, 128>(p, grid, stream);
    e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "gemm_gguf_kernel launch");
}

}  // extern "C"
