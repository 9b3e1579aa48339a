// Packed GGUF GEMV for decode (input rows T <= KB200_BATCH_ROWS per pass).
//
// Replaces the reference's gguf_matvec_kernel / gguf_matvec_batch_kernel
// (services/hikari/inference_worker/src/cuda/h3_compute.cu:165-257), which use
// one warp per output column and byte loads. Here each CTA is a small
// pipeline built for HBM streaming on sm_100a:
//
//   * one producer lane streams the packed rows of NC output columns, one
//     4096-value K chunk at a time, into a 4-stage shared-memory ring with
//     bulk async copies (cp.async.bulk, completion on mbarriers);
//   * four consumer warps decode the staged blocks in registers. Every thread
//     owns one 32-value "unit" of the chunk, keeps that unit's activations in
//     registers and reuses them for all NC columns of the stage;
//   * codes become floats with one byte-permute each (f = 0.5 + code/256 for
//     6-bit codes, 1 + code/256 for 8-bit ones), are multiplied on the packed
//     fp32x2 FMA pipe, and the GGUF group scales are applied once per group:
//       sum_i w_i x_i = scale * 256 * sum_i f_i x_i - (constant) * sum_i x_i
//     with sum_i x_i computed once per unit and row;
//   * the per-thread partial sums are reduced by warp shuffles and a small
//     shared-memory step at the end of each tile.
//
// Decoded weights are never materialised, so the non-finite check of the
// reference (isfinite of every decoded weight, :207-217) becomes the
// equivalent check that the block's fp16 scales are finite: a block decodes
// to a non-finite value exactly when one of its fp16 scales is non-finite.
//
// Rows whose bytes are not 16-byte aligned (row_bytes % 16 != 0, or an
// unaligned base) go to gemv_generic_kernel, a warp-per-column kernel that
// decodes with the exact per-value decoder.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "gemv_mma.hpp"
#include "gguf_formats.cuh"
#include "kb200_device.cuh"
#include "kb200_host.hpp"

namespace kb200 {
namespace {

constexpr int kConsumerWarps = 4;
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kStages = 4;
constexpr int kChunkValues = 4096;  // 128 units of 32 values
constexpr int kUnits = kChunkValues / 32;
constexpr int kMaxJobs = 64;
constexpr int kColumns = 8;  // NC: output columns per tile

struct DevJob {
    const uint8_t* weights;
    const float* input;
    float* output;
    unsigned* status;
    uint64_t row_bytes, stride;
    uint32_t in, columns, rows, first_tile;
    uint32_t row_groups, group_rows;
};

struct GemvParams {
    DevJob jobs[kMaxJobs];
    uint32_t count, total_tiles;
    int32_t encoding;  // one encoding per launch
    unsigned* watchdog;
};

__device__ __forceinline__ int find_job(const GemvParams& p, uint32_t tile) {
    int low = 0, high = int(p.count);
    while (high - low > 1) {
        const int mid = (low + high) / 2;
        if (p.jobs[mid].first_tile <= tile)
            low = mid;
        else
            high = mid;
    }
    return low;
}

// Byte i (0..3) of `v` placed at bits 16..23 under exponent byte 0x3F:
// 0.5 + code * 2^-8 for codes below 128.
template <int I> __device__ __forceinline__ float byte_half_code(uint32_t v) {
    return __uint_as_float(__byte_perm(v, 0x3F000000u, 0x7054u | (I << 8)));
}

// Eight bytes starting at a 2-byte aligned shared address.
__device__ __forceinline__ uint2 load8_unaligned(const uint8_t* p) {
    const auto a = reinterpret_cast<uintptr_t>(p);
    const auto* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = uint32_t(a & 3u) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

__device__ __forceinline__ void load16f(const float* x, float* v) {
    const float4* q = reinterpret_cast<const float4*>(x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 t = __ldg(q + i);
        v[4 * i] = t.x, v[4 * i + 1] = t.y, v[4 * i + 2] = t.z, v[4 * i + 3] = t.w;
    }
}

__device__ __forceinline__ void load8f(const float* x, float* v) {
    const float4* q = reinterpret_cast<const float4*>(x);
    const float4 a = __ldg(q), b = __ldg(q + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
    v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

// sum_i f[i] * x[i] over N values (N even) on the f32x2 pipe.
template <int N> __device__ __forceinline__ float dot_pairs(const float* f, const float* x) {
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < N; i += 2)
        acc = fma2(make_float2(f[i], f[i + 1]), make_float2(x[i], x[i + 1]), acc);
    return acc.x + acc.y;
}

template <int N> __device__ __forceinline__ float sum_of(const float* x) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i)
        s += x[i];
    return s;
}

// --- Q4_K: 144-byte super-blocks of 256 values ------------------------------
// Unit u of a chunk: block u/8, 32-byte code chunk j = (u/2)%4, half h = u%2:
// 16 code bytes whose low nibbles are values 16h..16h+15 of sub-block 2j and
// whose high nibbles are the same values of sub-block 2j+1.
struct Q4K {
    static constexpr int kEncoding = KB200_Q4_K, kBlockBytes = 144, kSums = 2;
    static constexpr int kChunkBytes = kChunkValues / 256 * kBlockBytes;

    template <int T>
    __device__ static void load_x(const float* x, size_t in, int rows, int u, float (&xv)[T][32], float (&sx)[T][kSums]) {
        const int a = (u >> 3) * 256 + ((u >> 1) & 3) * 64 + (u & 1) * 16;
#pragma unroll
        for (int r = 0; r < T; ++r) {
            if (r < rows) {
                load16f(x + r * in + a, xv[r]);
                load16f(x + r * in + a + 32, xv[r] + 16);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    xv[r][i] = 0.f;
            }
            sx[r][0] = sum_of<16>(xv[r]);
            sx[r][1] = sum_of<16>(xv[r] + 16);
        }
    }

    template <int T>
    __device__ static void dot(const uint8_t* chunk, int u, const float (&xv)[T][32], const float (&sx)[T][kSums], float (&acc)[T], bool& finite) {
        const int j = (u >> 1) & 3;
        const uint8_t* blk = chunk + (u >> 3) * kBlockBytes;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 codes = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j + 16 * (u & 1));
        // Scale/min bytes of sub-blocks 2j and 2j+1 (see gguf_formats.cuh).
        const uint32_t sel = uint32_t(2 * (j & 1));
        const uint32_t a0 = (hdr.y >> (8 * sel)) & 255u, a1 = (hdr.y >> (8 * sel + 8)) & 255u;
        const uint32_t b0 = (hdr.z >> (8 * sel)) & 255u, b1 = (hdr.z >> (8 * sel + 8)) & 255u;
        const uint32_t c0 = (hdr.w >> (8 * sel)) & 255u, c1 = (hdr.w >> (8 * sel + 8)) & 255u;
        uint32_t scA, mA, scB, mB;
        if (j < 2) {
            scA = a0 & 63u, mA = b0 & 63u, scB = a1 & 63u, mB = b1 & 63u;
        } else {
            scA = (c0 & 15u) | ((a0 >> 6) << 4), mA = (c0 >> 4) | ((b0 >> 6) << 4);
            scB = (c1 & 15u) | ((a1 >> 6) << 4), mB = (c1 >> 4) | ((b1 >> 6) << 4);
        }
        const float d = half_bits_to_float(hdr.x & 0xffffu), dmin = half_bits_to_float(hdr.x >> 16);
        finite = finite && isfinite(d) && isfinite(dmin);
        const float scaledA = __fmul_rn(d, float(scA)), offA = __fmul_rn(dmin, float(mA));
        const float scaledB = __fmul_rn(d, float(scB)), offB = __fmul_rn(dmin, float(mB));
        float fa[16], fb[16];
        const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t lo = words[k] & 0x0F0F0F0Fu, hi = (words[k] >> 4) & 0x0F0F0F0Fu;
            fa[4 * k] = byte_half_code<0>(lo), fa[4 * k + 1] = byte_half_code<1>(lo);
            fa[4 * k + 2] = byte_half_code<2>(lo), fa[4 * k + 3] = byte_half_code<3>(lo);
            fb[4 * k] = byte_half_code<0>(hi), fb[4 * k + 1] = byte_half_code<1>(hi);
            fb[4 * k + 2] = byte_half_code<2>(hi), fb[4 * k + 3] = byte_half_code<3>(hi);
        }
        const float kA = 256.f * scaledA, kB = 256.f * scaledB;
        const float tA = fmaf(128.f, scaledA, offA), tB = fmaf(128.f, scaledB, offB);
#pragma unroll
        for (int r = 0; r < T; ++r) {
            const float sA = dot_pairs<16>(fa, xv[r]), sB = dot_pairs<16>(fb, xv[r] + 16);
            float v = acc[r];
            v = fmaf(kA, sA, v);
            v = fmaf(-tA, sx[r][0], v);
            v = fmaf(kB, sB, v);
            v = fmaf(-tB, sx[r][1], v);
            acc[r] = v;
        }
    }
};

// --- Q8_0: 34-byte blocks of 32 int8 codes ----------------------------------
// Unit u = block u. Codes sit at a 2-byte aligned offset; aligned words are
// funnel-shifted into place.
struct Q80 {
    static constexpr int kEncoding = KB200_Q8_0, kBlockBytes = 34, kSums = 1;
    static constexpr int kChunkBytes = kChunkValues / 32 * kBlockBytes;

    template <int T>
    __device__ static void load_x(const float* x, size_t in, int rows, int u, float (&xv)[T][32], float (&sx)[T][kSums]) {
#pragma unroll
        for (int r = 0; r < T; ++r) {
            if (r < rows) {
                load16f(x + r * in + 32 * u, xv[r]);
                load16f(x + r * in + 32 * u + 16, xv[r] + 16);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    xv[r][i] = 0.f;
            }
            sx[r][0] = sum_of<32>(xv[r]);
        }
    }

    // 1 + (q + 128) * 2^-8 from byte I of v ^ 0x80808080.
    template <int I> __device__ static float code_f(uint32_t v) {
        const uint32_t t = I == 0 ? v << 15 : I == 1 ? v << 7 : I == 2 ? v >> 1 : v >> 9;
        return __uint_as_float((t & 0x007F8000u) | 0x3F800000u);
    }

    template <int T>
    __device__ static void dot(const uint8_t* chunk, int u, const float (&xv)[T][32], const float (&sx)[T][kSums], float (&acc)[T], bool& finite) {
        const uint8_t* blk = chunk + u * kBlockBytes;
        const float d = half_bits_to_float(*reinterpret_cast<const unsigned short*>(blk));
        finite = finite && isfinite(d);
        const auto a = reinterpret_cast<uintptr_t>(blk + 2);
        const auto* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
        const uint32_t sh = uint32_t(a & 3u) * 8u;
        uint32_t raw[9];
#pragma unroll
        for (int k = 0; k < 9; ++k)
            raw[k] = w[k];
        float f[32];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t v = __funnelshift_r(raw[k], raw[k + 1], sh) ^ 0x80808080u;
            f[4 * k] = code_f<0>(v), f[4 * k + 1] = code_f<1>(v);
            f[4 * k + 2] = code_f<2>(v), f[4 * k + 3] = code_f<3>(v);
        }
        const float k1 = 256.f * d, k0 = 384.f * d;
#pragma unroll
        for (int r = 0; r < T; ++r) {
            const float s = dot_pairs<32>(f, xv[r]);
            acc[r] = fmaf(-k0, sx[r][0], fmaf(k1, s, acc[r]));
        }
    }
};

// --- Q6_K: 210-byte super-blocks of 256 values ------------------------------
// Unit u: block u/8, 128-value half h = (u/4)%2, lanes L..L+7 with
// L = 8*(u%4), all four 32-value quarters of those lanes (one int8 scale each).
struct Q6K {
    static constexpr int kEncoding = KB200_Q6_K, kBlockBytes = 210, kSums = 4;
    static constexpr int kChunkBytes = kChunkValues / 256 * kBlockBytes;

    template <int T>
    __device__ static void load_x(const float* x, size_t in, int rows, int u, float (&xv)[T][32], float (&sx)[T][kSums]) {
        const int a = (u >> 3) * 256 + ((u >> 2) & 1) * 128 + (u & 3) * 8;
#pragma unroll
        for (int r = 0; r < T; ++r) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (r < rows)
                    load8f(x + r * in + a + 32 * q, xv[r] + 8 * q);
                else
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        xv[r][8 * q + i] = 0.f;
                sx[r][q] = sum_of<8>(xv[r] + 8 * q);
            }
        }
    }

    template <int T>
    __device__ static void dot(const uint8_t* chunk, int u, const float (&xv)[T][32], const float (&sx)[T][kSums], float (&acc)[T], bool& finite) {
        const int h = (u >> 2) & 1, L = (u & 3) * 8;
        const uint8_t* blk = chunk + (u >> 3) * kBlockBytes;
        const uint2 ql0 = load8_unaligned(blk + 64 * h + L);
        const uint2 ql1 = load8_unaligned(blk + 64 * h + 32 + L);
        const uint2 qh = load8_unaligned(blk + 128 + 32 * h + L);
        const uint2 sc = load8_unaligned(blk + 192 + 8 * h);
        const float d = half_bits_to_float(*reinterpret_cast<const unsigned short*>(blk + 208));
        finite = finite && isfinite(d);
        // int8 scale of quarter q for these lanes: byte (L/16) + 2q of sc.
        const uint32_t s_lo = L >= 16 ? sc.x >> 8 : sc.x, s_hi = L >= 16 ? sc.y >> 8 : sc.y;
        float D[4];
        D[0] = __fmul_rn(d, float(int8_t(s_lo & 255u)));
        D[1] = __fmul_rn(d, float(int8_t((s_lo >> 16) & 255u)));
        D[2] = __fmul_rn(d, float(int8_t(s_hi & 255u)));
        D[3] = __fmul_rn(d, float(int8_t((s_hi >> 16) & 255u)));
        float f[4][8];
        const uint32_t l0[2] = {ql0.x, ql0.y}, l1[2] = {ql1.x, ql1.y}, hh[2] = {qh.x, qh.y};
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t c0 = (l0[k] & 0x0F0F0F0Fu) | ((hh[k] << 4) & 0x30303030u);
            const uint32_t c1 = (l1[k] & 0x0F0F0F0Fu) | ((hh[k] << 2) & 0x30303030u);
            const uint32_t c2 = ((l0[k] >> 4) & 0x0F0F0F0Fu) | (hh[k] & 0x30303030u);
            const uint32_t c3 = ((l1[k] >> 4) & 0x0F0F0F0Fu) | ((hh[k] >> 2) & 0x30303030u);
            const uint32_t c[4] = {c0, c1, c2, c3};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                f[q][4 * k] = byte_half_code<0>(c[q]), f[q][4 * k + 1] = byte_half_code<1>(c[q]);
                f[q][4 * k + 2] = byte_half_code<2>(c[q]), f[q][4 * k + 3] = byte_half_code<3>(c[q]);
            }
        }
#pragma unroll
        for (int r = 0; r < T; ++r) {
            float v = acc[r];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float s = dot_pairs<8>(f[q], xv[r] + 8 * q);
                // sum (code-32) x = 256 s - 160 sum x, code = 6-bit unsigned.
                v = fmaf(256.f * D[q], s, v);
                v = fmaf(-160.f * D[q], sx[r][q], v);
            }
            acc[r] = v;
        }
    }
};

struct Shared {
    uint64_t full[kStages], empty[kStages];
    int abort;
};

template <class F, int T> __host__ __device__ constexpr int slot_bytes() {
    return (F::kChunkBytes + 16 + 15) / 16 * 16;
}

template <class F, int T> __host__ __device__ constexpr size_t smem_bytes() {
    return size_t(kStages) * kColumns * slot_bytes<F, T>() + sizeof(Shared) + 16
           + sizeof(float) * kConsumerWarps * kColumns * T;
}

template <class F, int T>
__global__ void __launch_bounds__(kThreads) gemv_staged_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int kSlot = slot_bytes<F, T>();
    uint8_t* stages = smem;
    auto* sh = reinterpret_cast<Shared*>(smem + size_t(kStages) * kColumns * kSlot);
    auto* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sh) + sizeof(Shared) + 16);
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sh->full[s], 1);
            mbar_init(&sh->empty[s], kConsumerWarps);
        }
        sh->abort = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer: one lane issues every bulk copy ----------------
        if (lane != 0)
            return;
        uint32_t it = 0;
        for (uint32_t tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x) {
            const DevJob& job = p.jobs[find_job(p, tile)];
            const uint32_t local = tile - job.first_tile;
            const uint32_t c0 = (local / job.row_groups) * kColumns;
            const uint32_t ncols = min(uint32_t(kColumns), job.columns - c0);
            const uint32_t chunks = (job.in + kChunkValues - 1) / kChunkValues;
            for (uint32_t kc = 0; kc < chunks; ++kc, ++it) {
                const int slot = int(it % kStages);
                if (it >= kStages
                    && !mbar_wait(&sh->empty[slot], ((it / kStages) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog)) {
                    atomicExch(&sh->abort, 1);
                }
                if (*reinterpret_cast<volatile int*>(&sh->abort))
                    goto drain;
                const uint64_t offset = uint64_t(kc) * F::kChunkBytes;
                const uint32_t bytes = uint32_t(min(uint64_t(F::kChunkBytes), job.row_bytes - offset));
                mbar_expect_tx(&sh->full[slot], bytes * ncols);
                for (uint32_t c = 0; c < ncols; ++c)
                    bulk_g2s(
                        stages + (size_t(slot) * kColumns + c) * kSlot,
                        job.weights + uint64_t(c0 + c) * job.row_bytes + offset,
                        bytes,
                        &sh->full[slot]
                    );
            }
        }
    drain:
        // Wait (bounded) for the last copy issued into every slot to land.
        for (uint32_t k = 0; k < kStages && k < it; ++k) {
            const uint32_t last = it - 1 - k;
            mbar_wait(&sh->full[last % kStages], (last / kStages) & 1u, watchdog_drain, p.watchdog);
        }
        return;
    }

    // -------------------- consumers: 4 warps, one unit each --------------------
    uint32_t it = 0;
    float xv[T][32], sx[T][F::kSums];
    // Activations stay in registers while consecutive stages read the same
    // rows of the same input (every column tile of a K <= 4096 job).
    const float* x_key = nullptr;
    int x_rows = -1;
    uint32_t x_in = 0;
    for (uint32_t tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x) {
        const DevJob& job = p.jobs[find_job(p, tile)];
        const uint32_t local = tile - job.first_tile;
        const uint32_t c0 = (local / job.row_groups) * kColumns;
        const uint32_t r0 = (local % job.row_groups) * job.group_rows;
        const int rows = int(min(job.group_rows, job.rows - r0));
        const uint32_t ncols = min(uint32_t(kColumns), job.columns - c0);
        const uint32_t chunks = (job.in + kChunkValues - 1) / kChunkValues;
        const bool check = job.status != nullptr;
        float acc[kColumns][T];
#pragma unroll
        for (int c = 0; c < kColumns; ++c)
#pragma unroll
            for (int r = 0; r < T; ++r)
                acc[c][r] = 0.f;
        bool finite = true;
        for (uint32_t kc = 0; kc < chunks; ++kc, ++it) {
            const int slot = int(it % kStages);
            const int units = int(min(uint32_t(kUnits), (job.in - kc * kChunkValues) / 32));
            const bool active = tid < units;
            const float* xsrc = job.input + size_t(r0) * job.in + size_t(kc) * kChunkValues;
            if (active && (xsrc != x_key || rows != x_rows || job.in != x_in)) {
                F::template load_x<T>(xsrc, job.in, rows, tid, xv, sx);
                x_key = xsrc, x_rows = rows, x_in = job.in;
            }
            const bool aborted = *reinterpret_cast<volatile int*>(&sh->abort) != 0;
            if (!aborted && !mbar_wait(&sh->full[slot], (it / kStages) & 1u, watchdog_full_barrier, p.watchdog))
                atomicExch(&sh->abort, 1);
            if (active && !aborted) {
                const uint8_t* base = stages + size_t(slot) * kColumns * kSlot;
#pragma unroll
                for (int c = 0; c < kColumns; ++c)
                    if (c < int(ncols))
                        F::template dot<T>(base + c * kSlot, tid, xv, sx, acc[c], finite);
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&sh->empty[slot]);
        }
        if (check && !finite)
            atomicOr(job.status, 1u);
        // Reduce acc[c][r] over the 128 consumer threads.
#pragma unroll
        for (int c = 0; c < kColumns; ++c)
#pragma unroll
            for (int r = 0; r < T; ++r) {
                float v = acc[c][r];
#pragma unroll
                for (int o = 16; o; o >>= 1)
                    v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0)
                    red[(warp * kColumns + c) * T + r] = v;
            }
        named_sync(1, kConsumers);
        if (tid < kColumns * T) {
            const int c = tid / T, r = tid % T;
            if (c < int(ncols) && r < rows) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w)
                    v += red[(w * kColumns + c) * T + r];
                job.output[size_t(r0 + r) * job.stride + c0 + c] = v;
            }
        }
        named_sync(1, kConsumers);
        if (*reinterpret_cast<volatile int*>(&sh->abort))
            return;
    }
}

// --- generic path: any decodable encoding or F32 rows, any alignment --------
// One warp per output column, lanes stride K in runs of 8 values, up to
// KB200_BATCH_ROWS input rows per pass (the reference's matvec_rows shape).
constexpr int kGenericWarps = 8;

template <int Rows, bool Grids>
__global__ void __launch_bounds__(32 * kGenericWarps) gemv_generic_kernel(const __grid_constant__ GemvParams p) {
    const uint32_t tile = blockIdx.x;
    const DevJob& job = p.jobs[find_job(p, tile)];
    const uint32_t local = tile - job.first_tile;
    const uint32_t column = (local / job.row_groups) * kGenericWarps + threadIdx.x / 32;
    const uint32_t r0 = (local % job.row_groups) * job.group_rows;
    if (column >= job.columns)
        return;
    const int rows = int(min(job.group_rows, job.rows - r0));
    const int lane = threadIdx.x % 32;
    const int encoding = p.encoding;
    const uint8_t* row = job.weights + uint64_t(column) * job.row_bytes;
    float sums[Rows];
#pragma unroll
    for (int r = 0; r < Rows; ++r)
        sums[r] = 0.f;
    bool finite = true;
    for (uint32_t i = lane * 8; i < job.in; i += 256) {
        float w[8];
        if (encoding == KB200_F32) {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                w[k] = reinterpret_cast<const float*>(row)[i + k];
        } else {
            const int values = block_values(encoding), bytes = block_bytes(encoding);
#pragma unroll
            for (int k = 0; k < 8; ++k)
                w[k] = decode_value<Grids>(encoding, row + size_t((i + k) / values) * bytes, (i + k) % values);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
            finite = finite && isfinite(w[k]);
#pragma unroll
        for (int r = 0; r < Rows; ++r)
            if (r < rows) {
                const float* x = job.input + size_t(r0 + r) * job.in + i;
                float s = sums[r];
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    s = fmaf(w[k], x[k], s);
                sums[r] = s;
            }
    }
    if (!finite && job.status)
        atomicOr(job.status, 1u);
#pragma unroll
    for (int r = 0; r < Rows; ++r) {
        float v = sums[r];
#pragma unroll
        for (int o = 16; o; o >>= 1)
            v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && r < rows)
            job.output[size_t(r0 + r) * job.stride + column] = v;
    }
}

}  // namespace
}  // namespace kb200

// ------------------------------------------------------------------- host side
namespace kb200 {

int sm_count() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return 148;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

namespace {

// Per-device, per-kernel launch geometry, computed once.
struct KernelInfo {
    bool ready = false;
    int blocks_per_sm = 1;
};

template <class F, int T> int launch_staged(const GemvParams& p, cudaStream_t stream) {
    static KernelInfo info[64];
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    constexpr size_t smem = smem_bytes<F, T>();
    {
        std::lock_guard<std::mutex> guard(lock);
        if (!info[dev].ready) {
            cudaError_t e = cudaFuncSetAttribute(
                gemv_staged_kernel<F, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)
            );
            if (e != cudaSuccess)
                return cuda_fail(e, "gemv_staged_kernel attribute");
            int n = 0;
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_staged_kernel<F, T>, kThreads, smem);
            if (e != cudaSuccess)
                return cuda_fail(e, "gemv_staged_kernel occupancy");
            info[dev].blocks_per_sm = n > 0 ? n : 1;
            info[dev].ready = true;
        }
    }
    const uint32_t slots = uint32_t(sm_count() * info[dev].blocks_per_sm);
    const uint32_t grid = std::min(p.total_tiles, slots);
    TraceScope trace(KB200_KERNEL_GEMV_STAGED, stream);
    gemv_staged_kernel<F, T><<<grid, kThreads, smem, stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "gemv_staged_kernel launch");
}

template <int Rows> int launch_generic(const GemvParams& p, cudaStream_t stream) {
    TraceScope trace(KB200_KERNEL_GEMV_GENERIC, stream);
    if (grid_coded(p.encoding))
        gemv_generic_kernel<Rows, true><<<p.total_tiles, 32 * kGenericWarps, 0, stream>>>(p);
    else
        gemv_generic_kernel<Rows, false><<<p.total_tiles, 32 * kGenericWarps, 0, stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "gemv_generic_kernel launch");
}

bool staged_format(int e) {
    return e == KB200_Q4_K || e == KB200_Q8_0 || e == KB200_Q6_K;
}

int check_job(const kb200_gemv_job& j) {
    if (!kb200_encoding_supported(j.encoding))
        return fail(KB200_UNSUPPORTED, "encoding has no device decoder");
    if (const int s = ensure_iq_grids(j.encoding))
        return s;
    const size_t values = block_values(j.encoding), bytes = block_bytes(j.encoding);
    // gguf_batch_supported (IW/include/kadan/gguf_batch_partition.hpp:12-31).
    if (!j.in || !j.columns || !j.rows || j.rows > KB200_BATCH_MAX_ROWS || j.in % 8 || j.in % values)
        return fail(KB200_UNSUPPORTED, "job shape outside the batched GEMV contract");
    if (!j.weights || !j.input || !j.output)
        return fail(KB200_INVALID, "null pointer");
    if (j.row_bytes < j.in / values * bytes || j.stride < j.columns)
        return fail(KB200_INVALID, "row_bytes or stride too small");
    const size_t out_bytes = ((size_t(j.rows) - 1) * j.stride + j.columns) * sizeof(float);
    if (overlap(j.output, out_bytes, j.input, size_t(j.rows) * j.in * sizeof(float))
        || overlap(j.output, out_bytes, j.weights, size_t(j.columns) * j.row_bytes))
        return fail(KB200_ALIAS, "output overlaps an input");
    return KB200_OK;
}

// 2 = tensor-pipe kernel (Q4_K, Q6_K), 1 = bulk-copy staged CUDA-core kernel,
// 0 = generic kernel.
int path_of(const kb200_gemv_job& j) {
    if (mma_eligible(j))
        return 2;
    return staged_format(j.encoding) && aligned(j.weights, 16) && j.row_bytes % 16 == 0
                   && aligned(j.input, 16)
               ? 1
               : 0;
}

}  // namespace
}  // namespace kb200

namespace kb200 {

int gemv_batch(const kb200_gemv_job* jobs, size_t count, cudaStream_t stream, bool synchronous) {
    if (!count)
        return KB200_OK;
    if (!jobs)
        return fail(KB200_INVALID, "null job array");
    // Unsupported or invalid jobs reject the whole batch before any launch.
    for (size_t i = 0; i < count; ++i)
        if (const int s = check_job(jobs[i]))
            return s;
    for (size_t i = 0; i < count; ++i)
        for (size_t k = 0; k < count; ++k) {
            const auto& a = jobs[i];
            const auto& b = jobs[k];
            const size_t out_bytes = ((size_t(a.rows) - 1) * a.stride + a.columns) * sizeof(float);
            if (overlap(a.output, out_bytes, b.input, size_t(b.rows) * b.in * sizeof(float)))
                return fail(KB200_ALIAS, "output overlaps another job's input");
        }
    // One launch per (path, encoding, rows-per-pass), like plan_matvec's
    // per-format launches (IW/src/cuda/h3_compute.cu:325-345).
    struct Key {
        int path, encoding, group;
    };
    std::vector<std::pair<Key, std::vector<const kb200_gemv_job*>>> groups;
    for (size_t i = 0; i < count; ++i) {
        const auto& j = jobs[i];
        const int path = path_of(j);
        const int group = path == 2 ? 0 : path ? (j.rows == 1 ? 1 : 2) : (j.rows == 1 ? 1 : KB200_BATCH_ROWS);
        auto it = std::find_if(groups.begin(), groups.end(), [&](const auto& g) {
            return g.first.path == path && g.first.encoding == j.encoding && g.first.group == group;
        });
        if (it == groups.end()) {
            groups.push_back({{path, int(j.encoding), group}, {}});
            it = groups.end() - 1;
        }
        it->second.push_back(&j);
    }
    for (const auto& [key, members] : groups) {
        if (key.path == 2) {
            if (const int s = launch_mma(members, stream, nullptr, synchronous))
                return s;
            continue;
        }
        for (size_t first = 0; first < members.size(); first += kMaxJobs) {
            GemvParams p;
            std::memset(&p, 0, sizeof(p));
            p.encoding = key.encoding;
            p.watchdog = watchdog_word();
            if (!p.watchdog)
                return fail(KB200_CUDA, "watchdog word unavailable");
            uint32_t tiles = 0;
            const size_t n = std::min(members.size() - first, size_t(kMaxJobs));
            const uint32_t tile_columns = key.path ? kColumns : kGenericWarps;
            for (size_t m = 0; m < n; ++m) {
                const auto& j = *members[first + m];
                DevJob& d = p.jobs[m];
                d.weights = static_cast<const uint8_t*>(j.weights);
                d.input = j.input;
                d.output = j.output;
                d.status = j.status;
                d.row_bytes = j.row_bytes;
                d.stride = j.stride;
                d.in = j.in;
                d.columns = j.columns;
                d.rows = j.rows;
                d.group_rows = uint32_t(key.group);
                d.row_groups = (j.rows + d.group_rows - 1) / d.group_rows;
                d.first_tile = tiles;
                tiles += (j.columns + tile_columns - 1) / tile_columns * d.row_groups;
            }
            p.count = uint32_t(n);
            p.total_tiles = tiles;
            int s = KB200_OK;
            if (key.path) {
                const bool one = key.group == 1;
                switch (key.encoding) {
                case KB200_Q4_K: s = one ? launch_staged<Q4K, 1>(p, stream) : launch_staged<Q4K, 2>(p, stream); break;
                case KB200_Q8_0: s = one ? launch_staged<Q80, 1>(p, stream) : launch_staged<Q80, 2>(p, stream); break;
                case KB200_Q6_K: s = one ? launch_staged<Q6K, 1>(p, stream) : launch_staged<Q6K, 2>(p, stream); break;
                default: s = fail(KB200_UNSUPPORTED, "no staged kernel for encoding");
                }
            } else {
                s = key.group == 1 ? launch_generic<1>(p, stream) : launch_generic<KB200_BATCH_ROWS>(p, stream);
            }
            if (s)
                return s;
        }
    }
    return KB200_OK;
}

}  // namespace kb200

using namespace kb200;

extern "C" {

int kb200_gemv_path(const kb200_gemv_job* job) {
    if (!job || check_job(*job) != KB200_OK)
        return -1;
    return path_of(*job);
}

int kb200_gguf_gemv_batch(const kb200_gemv_job* jobs, size_t count, void* stream_ptr) {
    return gemv_batch(jobs, count, static_cast<cudaStream_t>(stream_ptr), false);
}

// A row-parallel projection and the sum of its partial outputs over the
// group in one call: on the tensor-pipe path the GEMV's epilogue stores each
// finished output into every peer's buffer as it is written (so the exchange
// overlaps the rest of the GEMV) and the peer all-reduce kernel only gathers
// and adds; other paths run the GEMV and then the full all-reduce.
int kb200_gguf_gemv_allreduce(const kb200_gemv_job* job, void* const* peers, int world, int rank, size_t max_count,
                              double timeout_s, void* stream_ptr) {
    if (!job)
        return fail(KB200_INVALID, "null job");
    if (const int s = check_job(*job))
        return s;
    if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world)
        return fail(KB200_UNSUPPORTED, "1..8 ranks");
    if (job->stride != job->columns)
        return fail(KB200_INVALID, "the all-reduced output must be contiguous rows");
    const size_t count = size_t(job->rows) * job->columns;
    if (world > 1 && (!peers || count % 2 || count > max_count))
        return fail(KB200_INVALID, "output must be an even number of floats within the peer buffers");
    auto stream = static_cast<cudaStream_t>(stream_ptr);
    if (world == 1)
        return kb200_gguf_gemv_batch(job, 1, stream_ptr);
    PeerOut g;
    std::memset(&g, 0, sizeof(g));
    for (int r = 0; r < world; ++r)
        g.peers[r] = static_cast<uint8_t*>(peers[r]);
    g.max_count = max_count;
    g.rank = rank;
    g.world = world;
    const bool fused = path_of(*job) == 2;
    if (fused) {
        if (const int s = launch_mma({job}, stream, &g))
            return s;
    } else if (const int s = kb200_gguf_gemv_batch(job, 1, stream_ptr)) {
        return s;
    }
    return launch_peer_allreduce(job->output, count, g, timeout_s, !fused, stream);
}

}  // extern "C"
