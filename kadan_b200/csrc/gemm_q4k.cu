// Q4_K prefill GEMM on the fifth-generation tensor cores (sm_100a).
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
//   weights     : per weight tile and super-block, one 3-D TMA load of the
//                 packed 144-byte blocks (the GEMV's tensor map); eight dequant
//                 warps turn each into four 64-value fp16 B stages in the
//                 128-byte-swizzled K-major layout:
//                   q*sc   = fma(1024 + q, sc, -1024 sc)      exact in fp16
//                   w      = fma(q*sc, d, -(dmin*m))           one rounding
//                 (1024 + q comes from the nibble by a byte permute + mask)
//   MMA         : tcgen05.mma kind::f16, M = 128 input rows, N = 256 weight
//                 rows (128 when 256-row tiles would leave SMs idle), K = 16
//                 per instruction, fp32 accumulators in TMEM (two N-column
//                 buffers, so the epilogue of one tile overlaps the next
//                 tile's MMAs)
//   epilogue    : TMEM -> registers (32x32b.x32), * 2^e_t, fp32 rows of Y
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
constexpr int kBlock = 144;  // Q4_K super-block bytes
constexpr int kABytes = BM * BK * 2;
constexpr int kDequantWarps = 8;
constexpr int kThreads = 32 * (2 + kDequantWarps + 4);

// Tile geometry per weight-tile height BN (the MMA's N: 128 or 256 weight
// rows). Rings hold one K step of 64 per A/B stage and one super-block (four
// K steps) per raw stage. A 256-row tile halves the activation bytes per
// FLOP: the activation tiles arrive at about 30 GB/s per SM (measured, a
// 16 KB tile every ~0.5 us with ~2 us of latency), which caps 128-row tiles.
template <int BN> struct Tile {
    static constexpr int kAStages = BN == 256 ? 5 : 4;
    static constexpr int kBStages = BN == 256 ? 2 : 4;
    static constexpr int kRawStages = 2;
    static constexpr int kBBytes = BN * BK * 2, kRawBytes = BN * kBlock;
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

template <int BN> constexpr int smem_total() {
    return Tile<BN>::kSmemBars + int(sizeof(Bars)) + 1024;  // + 1024-byte alignment slack
}

struct GemmParams {
    CUtensorMap a_map;   // fp16 [T, K], box {64, 128}, 128-byte swizzle
    CUtensorMap w_map;   // u64 {18, K/256, N}, box {18, 1, 128}
    const int* row_exp;  // [T] e_t
    float* out;          // [T][stride]
    unsigned* status;    // or null
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

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_q4k_kernel(const __grid_constant__ GemmParams p) {
    using C = Tile<BN>;
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
                tma_load_3d(smem + C::kSmemRaw + rs * C::kRawBytes, &p.w_map, 0, kb, nt * BN, &bars->raw_full[rs]);
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
        constexpr int kChunks = 4 / C::kThreadsPerRow;  // 16-byte B chunks per half-stage row
        const int r = (tid - 64) % BN;                 // weight row of the tile (B-operand row)
        const int part = (tid - 64) / BN;              // which code bytes of each 32-byte chunk
        uint32_t it = 0, rt = 0;
        bool finite = true;
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
                const uint8_t* blk = smem + C::kSmemRaw + rs * C::kRawBytes + r * kBlock;
                const uint4 head = *reinterpret_cast<const uint4*>(blk);
                const float d = half_bits_to_float(head.x & 0xffffu), dmin = half_bits_to_float(head.x >> 16);
                if (row_valid)
                    finite = finite && isfinite(d) && isfinite(dmin);
                // 6-bit scales and mins of sub-blocks 0-3 / 4-7, one per byte.
                const uint32_t sc_lo = head.y & 0x3F3F3F3Fu;
                const uint32_t sc_hi = (head.w & 0x0F0F0F0Fu) | ((head.y >> 2) & 0x30303030u);
                const uint32_t m_lo = head.z & 0x3F3F3F3Fu;
                const uint32_t m_hi = ((head.w >> 4) & 0x0F0F0F0Fu) | ((head.z >> 2) & 0x30303030u);
                const uint32_t d2 = half2_bits(d, d);
                // Per sub-block g: sw = sc, cw = -1024 sc (exact: sc < 64), mn = -(dmin m).
                uint32_t sw[8], cw[8], mn[8];
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const uint32_t scw = g < 4 ? sc_lo : sc_hi, mw = g < 4 ? m_lo : m_hi;
                    const float sc = float((scw >> (8 * (g & 3))) & 0xFFu), m = float((mw >> (8 * (g & 3))) & 0xFFu);
                    sw[g] = half2_bits(sc, sc);
                    cw[g] = half2_bits(-1024.f * sc, -1024.f * sc);
                    mn[g] = half2_bits(-dmin * m, -dmin * m);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j, ++it) {
                    const int s = int(it % C::kBStages);
                    // B of the stage is free once the MMAs of its previous use completed.
                    if (it >= C::kBStages
                        && !mbar_wait(&bars->b_empty[s], ((it / C::kBStages) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog)) {
                        *abort_flag = 1;
                        break;
                    }
                    // Low nibbles are sub-block 2j, high nibbles 2j+1.
                    uint32_t words[2 * kChunks];
#pragma unroll
                    for (int v = 0; v < kChunks / 2; ++v) {
                        const uint4 cb = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j + 8 * kChunks * part + 16 * v);
                        words[4 * v] = cb.x, words[4 * v + 1] = cb.y, words[4 * v + 2] = cb.z, words[4 * v + 3] = cb.w;
                    }
                    uint8_t* brow = smem + C::kSmemB + s * C::kBBytes + r * 128;
#pragma unroll
                    for (int cc = 0; cc < kChunks; ++cc) {
                        // Code bytes 8c..8c+7 -> values 8c..8c+7 of sub-block 2j
                        // (chunk c) and of sub-block 2j+1 (chunk 4 + c).
                        const int c = kChunks * part + cc;
                        uint32_t lo[4], hi[4];
                        nibble_pairs(words[2 * cc], 0x5140u, lo[0], hi[0]);
                        nibble_pairs(words[2 * cc], 0x7362u, lo[1], hi[1]);
                        nibble_pairs(words[2 * cc + 1], 0x5140u, lo[2], hi[2]);
                        nibble_pairs(words[2 * cc + 1], 0x7362u, lo[3], hi[3]);
                        uint32_t wl[4], wh[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            wl[i] = hfma2(hfma2(lo[i], sw[2 * j], cw[2 * j]), d2, mn[2 * j]);
                            wh[i] = hfma2(hfma2(hi[i], sw[2 * j + 1], cw[2 * j + 1]), d2, mn[2 * j + 1]);
                        }
                        *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
                        *reinterpret_cast<uint4*>(brow + (((4 + c) ^ (r & 7)) << 4)) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
                    }
                    fence_proxy_async();
                    mbar_arrive(&bars->b_full[s]);
                }
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&bars->raw_empty[rs]);
            }
        }
        if (!finite && p.status && part == 0)
            atomicOr(p.status, 1u);
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
// multiple of 4 (always: the GEMM takes whole super-blocks).
__global__ void __launch_bounds__(256) prefill_rows_kernel(const float* x, size_t in, __half* xh, int* row_exp) {
    const size_t t = blockIdx.x;
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

template <int BN> int gemm_slots() {
    static int set[64] = {};
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> guard(lock);
    if (!set[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(gemm_q4k_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_total<BN>());
        if (e != cudaSuccess)
            return -cuda_fail(e, "gemm_q4k_kernel attribute");
        set[dev] = 1;
    }
    return sm_count();
}

size_t align256(size_t v) {
    return (v + 255) / 256 * 256;
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

size_t kb200_gguf_gemm_workspace_bytes(uint32_t rows, uint32_t in) {
    return align256(size_t(rows) * in * sizeof(__half)) + align256(size_t(rows) * sizeof(int));
}

int kb200_gguf_gemm(const kb200_gemv_job* job, void* workspace, size_t workspace_bytes, void* stream_ptr) {
    if (!job)
        return fail(KB200_INVALID, "null job");
    const kb200_gemv_job& j = *job;
    if (j.encoding != KB200_Q4_K)
        return fail(KB200_UNSUPPORTED, "the prefill GEMM takes Q4_K weights");
    if (!j.weights || !j.input || !j.output || !j.rows || !j.columns || !j.in)
        return fail(KB200_INVALID, "empty GEMM job");
    if (j.in % 256 || j.row_bytes < size_t(j.in) / 256 * kBlock || j.row_bytes % 16 || !aligned(j.weights, 16))
        return fail(KB200_UNSUPPORTED, "Q4_K GEMM wants whole super-blocks in 16-byte aligned rows");
    if (j.stride < j.columns || j.stride > 0xffffffffu)
        return fail(KB200_INVALID, "output stride shorter than the row");
    if (overlap(j.output, (size_t(j.rows - 1) * j.stride + j.columns) * sizeof(float), j.input,
                size_t(j.rows) * j.in * sizeof(float)))
        return fail(KB200_ALIAS, "output overlaps the input");
    if (!workspace || workspace_bytes < kb200_gguf_gemm_workspace_bytes(j.rows, j.in) || !aligned(workspace, 256))
        return fail(KB200_INVALID, "GEMM workspace missing, short or not 256-byte aligned");
    auto encode = encoder();
    if (!encode)
        return fail(KB200_CUDA, "cuTensorMapEncodeTiled unavailable");
    // 256-row weight tiles when they still give every SM a tile.
    const int sms = sm_count();
    const int m_tiles = int((j.rows + BM - 1) / BM);
    const int BN = m_tiles * int((j.columns + 255) / 256) >= sms ? 256 : 128;
    const int slots = BN == 256 ? gemm_slots<256>() : gemm_slots<128>();
    if (slots <= 0)
        return -slots;
    auto stream = static_cast<cudaStream_t>(stream_ptr);

    auto* xh = static_cast<__half*>(workspace);
    auto* row_exp = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + align256(size_t(j.rows) * j.in * sizeof(__half)));
    prefill_rows_kernel<<<j.rows, 256, 0, stream>>>(j.input, j.in, xh, row_exp);
    cudaError_t e = cudaGetLastError();
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
    {
        const cuuint64_t dims[3] = {kBlock / 8, j.in / 256, j.columns};
        const cuuint64_t strides[2] = {kBlock, j.row_bytes};
        const cuuint32_t box[3] = {kBlock / 8, 1, uint32_t(BN)};
        const cuuint32_t es[3] = {1, 1, 1};
        if (encode(&p.w_map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(j.weights), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)
            != CUDA_SUCCESS)
            return fail(KB200_INVALID, "cuTensorMapEncodeTiled rejected the Q4_K weights");
    }
    p.row_exp = row_exp;
    p.out = j.output;
    p.status = j.status;
    p.watchdog = watchdog_word();
    p.T = int(j.rows);
    p.N = int(j.columns);
    p.nblocks = int(j.in / 256);
    p.m_tiles = m_tiles;
    p.n_tiles = int((j.columns + BN - 1) / BN);
    p.stride = uint32_t(j.stride);
    const int grid = std::max(1, std::min(slots, p.m_tiles * p.n_tiles));
    if (BN == 256)
        gemm_q4k_kernel<256><<<grid, kThreads, smem_total<256>(), stream>>>(p);
    else
        gemm_q4k_kernel<128><<<grid, kThreads, smem_total<128>(), stream>>>(p);
    e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "gemm_q4k_kernel launch");
}

}  // extern "C"
