// MXFP4 mixture-of-experts layer on sm_100a.
//
// Semantics follow the reference MoeLayer::forward
// (services/hikari/inference_worker/src/models/text/qwen_layers.cpp:378-492):
// a max-subtracted softmax router whose sum is taken in double, top-k by
// probability (ties to the lower expert index), renormalisation by
// max(sum, 2^-14), a stable per-expert gather in slot order, gate/up, the
// activation, down, and a weighted sum of the k expert outputs in selection
// order. The MXFP4 values follow kadan::quantization::weight
// (IW/src/weights/quantization.cpp:89-96): e2m1(code) * 2^(scale - 127).
//
// Device pipeline per call (all on one stream):
//   route   one warp per token: softmax, top-k, weights, expert counts
//   sort    one CTA: stable counting sort -> expert offsets, permutation,
//           inverse positions and the per-expert 128-row m-tile prefix
//   gather  token rows (bf16) -> expert-sorted rows (fp16)
//   gemm    grouped GEMM on the tensor cores (tcgen05, TMEM accumulators),
//           twice: gate/up with the activation in the epilogue (fp16 out),
//           then down (fp32 out). Expert weights stay MXFP4 in HBM; four
//           dequant warps turn each 128x64 code tile into fp16 with
//           cvt.rn.f16x2.e2m1x2 and the block scale (exact for scale bytes
//           104..140), straight into the 128-byte-swizzled operand layout.
//           With at most 8 token rows per expert on average (decode sizes)
//           the two GEMMs are replaced by a grouped GEMV (moe_gemv_kernel)
//           that streams only the routed experts' weights.
//   combine out[t] = sum_i w[t,i] * Y[pos(t,i)] in selection order (fp32)
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <map>
#include <mutex>

#include "kb200_device.cuh"
#include "kb200_host.hpp"
#include "tcgen05.cuh"

namespace kb200 {
namespace {

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 32;

// Programmatic dependent launch between the layer's kernels: each lets the
// next kernel of the stream start launching, then waits until the previous
// one has completed and its writes are visible before touching them. Launch
// latency overlaps; the order of the work does not change. Without the launch
// attribute both instructions do nothing.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <class... Params, class... Args>
cudaError_t launch_pdl(kb200_kernel id, void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
    TraceScope trace(id, stream);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// ---------------------------------------------------------------- routing
// Routing of one token by one warp; experts strided over lanes (<= 8 per
// lane). Lane 0 writes the K choices and weights (and counts them when
// `counts` is not null).
__device__ __forceinline__ void route_token(const float* l, int E, int K, int* chosen, float* weight, int* counts) {
    const int lane = threadIdx.x & 31;
    float v[8];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < E ? l[e] : -INFINITY;
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float p[8];
    double total = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        p[i] = lane + 32 * i < E ? expf(v[i] - mx) : 0.f;
        total += double(p[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
        total += __shfl_xor_sync(0xffffffffu, total, o);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        p[i] = float(double(p[i]) / total);
    unsigned taken = 0;
    float sum = 0.f, picked[kMaxTopK];
    int idx[kMaxTopK];
    for (int s = 0; s < K; ++s) {
        float best = -1.f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((taken >> i) & 1u) && (p[i] > best || (p[i] == best && e < bi)))
                best = p[i], bi = e;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi))
                best = ob, bi = oi;
        }
        if ((bi & 31) == lane)
            taken |= 1u << (bi >> 5);
        picked[s] = best;
        idx[s] = bi;
        sum += best;
    }
    sum = fmaxf(sum, 6.103515625e-5f);
    if (lane == 0)
        for (int s = 0; s < K; ++s) {
            chosen[s] = idx[s];
            weight[s] = picked[s] / sum;
            if (counts)
                atomicAdd(&counts[idx[s]], 1);
        }
}

// One warp per token.
__global__ void moe_route_kernel(
    const float* logits, int tokens, int E, int K, int* chosen, float* weight, int* counts
) {
    pdl_enter();
    const int warp = int((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (warp >= tokens)
        return;
    route_token(logits + size_t(warp) * E, E, K, chosen + size_t(warp) * K, weight + size_t(warp) * K, counts);
}

// ------------------------------------------------------------------- sort
// One CTA of 1024 threads: stable counting sort of the tokens*K slots by
// expert (slot order within an expert), plus m-tile prefix sums.
__global__ void __launch_bounds__(1024) moe_sort_kernel(
    const int* chosen, int n, int E, const int* counts, int* offsets, int* perm, int* pos, int* mtile_prefix
) {
    __shared__ int off[kMaxExperts + 1], running[kMaxExperts], total[kMaxExperts];
    __shared__ int warp_base[32][kMaxExperts];
    pdl_enter();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        int acc = 0, tiles = 0;
        for (int e = 0; e < E; ++e) {
            off[e] = acc;
            mtile_prefix[e] = tiles;
            acc += counts[e];
            tiles += (counts[e] + 127) / 128;
        }
        off[E] = acc;
        mtile_prefix[E] = tiles;
    }
    for (int e = tid; e < E; e += blockDim.x)
        running[e] = 0;
    __syncthreads();
    for (int e = tid; e <= E; e += blockDim.x)
        offsets[e] = off[e];
    for (int base = 0; base < n; base += 1024) {
        for (int i = tid; i < 32 * E; i += 1024)
            warp_base[i / E][i % E] = 0;
        __syncthreads();
        const int slot = base + tid;
        const int e = slot < n ? chosen[slot] : -1;
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(same & ((1u << lane) - 1u));
        if (e >= 0 && rank == 0)
            warp_base[warp][e] = __popc(same);
        __syncthreads();
        for (int x = tid; x < E; x += 1024) {
            int acc = 0;
            for (int w = 0; w < 32; ++w) {
                const int c = warp_base[w][x];
                warp_base[w][x] = acc;
                acc += c;
            }
            total[x] = acc;
        }
        __syncthreads();
        if (e >= 0) {
            const int p = off[e] + running[e] + warp_base[warp][e] + rank;
            perm[p] = slot;
            pos[slot] = p;
        }
        __syncthreads();
        for (int x = tid; x < E; x += 1024)
            running[x] += total[x];
        __syncthreads();
    }
}

// ----------------------------------------------------------------- gather
// Eight values of a token row as fp32 pairs: bf16 rows (the layer's input)
// or fp32 rows (the host-span call's).
__device__ __forceinline__ void load8(const __nv_bfloat16* row, float2 (&f)[4]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k)
        f[k] = __bfloat1622float2(b[k]);
}

__device__ __forceinline__ void load8(const float* row, float2 (&f)[4]) {
    const float4 a = *reinterpret_cast<const float4*>(row), b = *reinterpret_cast<const float4*>(row + 4);
    f[0] = make_float2(a.x, a.y), f[1] = make_float2(a.z, a.w), f[2] = make_float2(b.x, b.y), f[3] = make_float2(b.z, b.w);
}

// Xs[p, :] = fp16(x[perm[p] / K, :]) for p < n, 8 values per thread.
template <class T>
__global__ void moe_gather_kernel(
    const T* x, const int* perm, int n, int K, int H, __half* xs, unsigned* status
) {
    pdl_enter();
    const int per_row = H / 8;
    const size_t total = size_t(n) * per_row;
    bool bad = false;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int p = int(i / per_row), c = int(i % per_row);
        const int token = perm[p] / K;
        float2 vals[4];
        load8(x + size_t(token) * H + c * 8, vals);
        uint4 outv;
        __half2* o = reinterpret_cast<__half2*>(&outv);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = vals[k];
            bad |= fabsf(f.x) > 65504.f || fabsf(f.y) > 65504.f;
            o[k] = __floats2half2_rn(f.x, f.y);
        }
        *reinterpret_cast<uint4*>(xs + size_t(p) * H + c * 8) = outv;
    }
    if (bad && status)
        atomicOr(status, 4u);
}

// ---------------------------------------------------------------- combine
__global__ void moe_combine_kernel(
    const float* y, const float* weight, const int* pos, int tokens, int K, int H, float* out
) {
    pdl_enter();
    const int per_row = H / 4;
    const size_t total = size_t(tokens) * per_row;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int t = int(i / per_row), c = int(i % per_row);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < K; ++s) {
            const float w = weight[size_t(t) * K + s];
            const float4 v = *reinterpret_cast<const float4*>(y + size_t(pos[size_t(t) * K + s]) * H + c * 4);
            acc.x = fmaf(w, v.x, acc.x), acc.y = fmaf(w, v.y, acc.y);
            acc.z = fmaf(w, v.z, acc.z), acc.w = fmaf(w, v.w, acc.w);
        }
        *reinterpret_cast<float4*>(out + size_t(t) * H + c * 4) = acc;
    }
}

// ----------------------------------------------------------- shared expert
__global__ void silu_mul_kernel(const float* gate, const float* up, size_t n, float* out) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        const float g = gate[i];
        out[i] = g / (1.f + expf(-g)) * up[i];
    }
}

// One CTA per token: the gate dot product, its sigmoid, then the gated add.
__global__ void __launch_bounds__(256) moe_shared_kernel(const float* x, const float* shared_gate, const float* down,
                                                         int hidden, float* out) {
    __shared__ float part[8];
    const size_t t = blockIdx.x;
    const float* xt = x + t * hidden;
    float dot = 0.f;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x)
        dot = fmaf(shared_gate[c], xt[c], dot);
    for (int o = 16; o; o >>= 1)
        dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if ((threadIdx.x & 31) == 0)
        part[threadIdx.x >> 5] = dot;
    __syncthreads();
    float g = 0.f;
    for (int w = 0; w < int(blockDim.x >> 5); ++w)
        g += part[w];
    g = 1.f / (1.f + expf(-g));
    for (int d = threadIdx.x; d < hidden; d += blockDim.x)
        out[t * hidden + d] += down[t * hidden + d] * g;
}

// ----------------------------------------------------------- grouped GEMM
// Tiles of 128 sorted rows (M) x 256 weight rows (N): each 16 KB activation
// tile feeds 256 output columns, half the L2 -> SM bytes per FLOP of 128-row
// weight tiles (measured: with 128-row tiles the activation TMA tiles took ~2
// us to arrive and the tensor pipe sat at 26 %). Activation and raw-code
// stages (kStagesG) and dequantised B stages (kStagesB) are separate rings.
// The dequant threads read their rows' block scales straight from global
// memory (L2 hits after the first m-tile of an expert), one K step ahead, so
// shared memory holds four dequantised B stages.
constexpr int BM = 128, BN = 256, BK = 64, kStagesG = 4, kStagesB = 4;
constexpr int kABytes = BM * BK * 2, kBBytes = BN * BK * 2, kRawBytes = BN * BK / 2;
constexpr int kMaxK = 4096;
constexpr int kDequantWarpsG = 8;                    // one B row per thread
constexpr int kThreadsG = 32 * (2 + kDequantWarpsG + 4);  // producer, MMA, dequant, 4 epilogue warps

struct GroupParams {
    CUtensorMap a_map;  // fp16 [rows, K], box {64, 128}, 128-byte swizzle
    CUtensorMap b_map;  // u8 codes [E * Nrows, K/2], box {32, 128} or {32, 64} (split)
    const uint8_t* scales;  // [E * Nrows, K/32]
    const float* bias;      // [E * Nrows] or null
    const int* offsets;     // [E + 1]
    const int* mtile_prefix;
    void* out;
    int K, Nrows, E, n_tiles, split, epilogue, out_cols, act_kind;
    float limit, alpha;
    unsigned* status;
    unsigned* watchdog;
};

struct GemmShared {
    uint64_t tma_full[kStagesG], stage_empty[kStagesG], b_full[kStagesB], b_empty[kStagesB];
    uint64_t acc_full[2], acc_empty[2];
    uint32_t tmem_base;
    int abort;
};

constexpr int kSmemA = 0;
constexpr int kSmemB = kSmemA + kStagesG * kABytes;
constexpr int kSmemRaw = kSmemB + kStagesB * kBBytes;
constexpr int kSmemShared = kSmemRaw + kStagesG * kRawBytes;
constexpr int kSmemTotal = kSmemShared + int(sizeof(GemmShared)) + 1024;
static_assert(kSmemTotal <= 232448, "shared memory per CTA");

struct TileInfo {
    int e, m0, mend, nt;
};

__device__ __forceinline__ TileInfo tile_info(const GroupParams& p, int tile) {
    const int mt = tile / p.n_tiles, nt = tile % p.n_tiles;
    int lo = 0, hi = p.E;  // largest e with mtile_prefix[e] <= mt
    while (hi - lo > 1) {
        const int mid = (lo + hi) / 2;
        if (p.mtile_prefix[mid] <= mt)
            lo = mid;
        else
            hi = mid;
    }
    TileInfo t;
    t.e = lo;
    t.m0 = p.offsets[lo] + (mt - p.mtile_prefix[lo]) * BM;
    t.mend = p.offsets[lo + 1];
    t.nt = nt;
    return t;
}

// The K step a tile takes at position ks of its walk: each weight tile
// starts at a different K step, so the CTAs that share an activation tile at
// the same time read different columns of it instead of queueing on the same
// L2 lines. The order is fixed per tile, so results are reproducible.
__device__ __forceinline__ int k_step(int ks, int nt, int KS) {
    const int k = ks + nt % KS;
    return k < KS ? k : k - KS;
}

// First weight row of the tile's lower and upper halves (split: gate and up).
__device__ __forceinline__ void tile_rows(const GroupParams& p, const TileInfo& t, int& r_lo, int& r_hi) {
    if (p.split) {
        r_lo = t.e * p.Nrows + t.nt * (BN / 2);
        r_hi = t.e * p.Nrows + p.Nrows / 2 + t.nt * (BN / 2);
    } else {
        r_lo = t.e * p.Nrows + t.nt * BN;
        r_hi = r_lo + BN / 2;
    }
}

// f16 2^(s-127), and whether s keeps every e2m1 * 2^(s-127) exact in fp16.
__device__ __forceinline__ uint32_t e8m0_half2(uint32_t s, bool& ok) {
    ok = s >= 104u && s <= 140u;
    uint32_t h;
    if (s >= 113u)
        h = min(s - 112u, 30u) << 10;
    else if (s >= 103u)
        h = 1u << (s - 103u);
    else
        h = 0u;
    return h | (h << 16);
}

__device__ __forceinline__ uint32_t e2m1x2_to_half2(uint32_t byte) {
    uint32_t r;
    asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(r) : "r"(byte));
    return r;
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ float act_fn(float gate, float up, int kind, float limit, float alpha) {
    if (kind == KB200_MOE_SWIGLU_OAI) {
        const float g = fminf(gate, limit);
        const float u = fminf(fmaxf(up, -limit), limit);
        return g / (1.f + expf(-alpha * g)) * (u + 1.f);
    }
    return gate / (1.f + expf(-gate)) * up;
}

__global__ void __launch_bounds__(kThreadsG, 1) moe_gemm_kernel(const __grid_constant__ GroupParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    pdl_enter();
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    auto* sh = reinterpret_cast<GemmShared*>(smem + kSmemShared);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int KS = p.K / BK, sc_row = p.K / 32;
    const int total = p.mtile_prefix[p.E] * p.n_tiles;

    if (tid == 0) {
        for (int s = 0; s < kStagesG; ++s) {
            mbar_init(&sh->tma_full[s], 1);
            mbar_init(&sh->stage_empty[s], 1);
        }
        for (int s = 0; s < kStagesB; ++s) {
            mbar_init(&sh->b_full[s], 32 * kDequantWarpsG);
            mbar_init(&sh->b_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sh->acc_full[b], 1);
            mbar_init(&sh->acc_empty[b], 4);
        }
        sh->abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&sh->tmem_base, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh->tmem_base;
    volatile int* abort_flag = &sh->abort;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ producer (TMA)
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x) {
            const TileInfo t = tile_info(p, tile);
            int r_lo, r_hi;
            tile_rows(p, t, r_lo, r_hi);
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int s = int(it % kStagesG);
                if (it >= kStagesG
                    && !mbar_wait(&sh->stage_empty[s], ((it / kStagesG) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog)) {
                    *abort_flag = 1;
                    break;
                }
                const int kx = k_step(ks, t.nt, KS);
                mbar_expect_tx(&sh->tma_full[s], uint32_t(kABytes + kRawBytes));
                tma_load_2d(smem + kSmemA + s * kABytes, &p.a_map, kx * BK, t.m0, &sh->tma_full[s]);
                // Two boxes of 128 code rows: gate and up halves (split), or
                // the tile's lower and upper 128 rows.
                uint8_t* raw = smem + kSmemRaw + s * kRawBytes;
                tma_load_2d(raw, &p.b_map, kx * (BK / 2), r_lo, &sh->tma_full[s]);
                tma_load_2d(raw + (BN / 2) * (BK / 2), &p.b_map, kx * (BK / 2), r_hi, &sh->tma_full[s]);
            }
        }
        // Drain: every copy this thread issued lands before the CTA can exit.
        for (uint32_t k = 0; k < kStagesG && k < it; ++k) {
            const uint32_t last = it - 1 - k;
            mbar_wait(&sh->tma_full[last % kStagesG], (last / kStagesG) & 1u, watchdog_drain, p.watchdog);
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------- MMA issuer
        const uint32_t idesc = idesc_f16(BM, BN);
        uint32_t it = 0, lt = 0;
        bool issued = false;
        for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x, ++lt) {
            const int acc = int(lt & 1u);
            if (lt >= 2 && !mbar_wait(&sh->acc_empty[acc], ((lt >> 1) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int s = int(it % kStagesG), sb = int(it % kStagesB);
                if (!mbar_wait(&sh->tma_full[s], (it / kStagesG) & 1u, watchdog_full_barrier, p.watchdog)
                    || !mbar_wait(&sh->b_full[sb], (it / kStagesB) & 1u, watchdog_full_barrier, p.watchdog)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = sw128_desc(smem_addr(smem + kSmemA + s * kABytes));
                const uint64_t bd = sw128_desc(smem_addr(smem + kSmemB + sb * kBBytes));
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                    umma_f16(tmem + uint32_t(acc * BN), ad + uint64_t(2 * kk), bd + uint64_t(2 * kk), idesc,
                             (ks | kk) != 0);
                umma_commit(&sh->stage_empty[s]);
                umma_commit(&sh->b_empty[sb]);
                issued = true;
            }
            umma_commit(&sh->acc_full[acc]);
        }
        if (issued && *abort_flag) {
            // Let the MMAs in flight finish before TMEM is released.
            const uint32_t last = it - 1;
            mbar_wait(&sh->stage_empty[last % kStagesG], (last / kStagesG) & 1u, watchdog_drain, p.watchdog);
        }
    } else if (warp >= 2 && warp < 2 + kDequantWarpsG) {
        // ------------------------------------------------- dequant warps
        const int r = tid - 64;  // B-operand row of this thread
        uint32_t it = 0;
        bool scale_ok = true;
        for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x) {
            // Rows past the weight tensor were zero-filled and have no scale
            // bytes: they take scale byte 0 (a zero factor).
            int r_lo, r_hi;
            const TileInfo ti = tile_info(p, tile);
            tile_rows(p, ti, r_lo, r_hi);
            const int wrow = r < BN / 2 ? r_lo + r : r_hi + (r - BN / 2);
            const bool row_in_tensor = wrow < p.E * p.Nrows;
            const uint8_t* srow = p.scales + size_t(row_in_tensor ? wrow : 0) * sc_row;
            // The two block scales of K step kx, loaded one step ahead.
            auto scales_of = [&](int kx) -> uint32_t {
                return row_in_tensor ? uint32_t(__ldg(srow + 2 * kx)) | uint32_t(__ldg(srow + 2 * kx + 1)) << 8 : 0u;
            };
            uint32_t next_sc = scales_of(k_step(0, ti.nt, KS));
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const uint32_t sc_pair = next_sc;
                if (ks + 1 < KS)
                    next_sc = scales_of(k_step(ks + 1, ti.nt, KS));
                const int s = int(it % kStagesG), sbs = int(it % kStagesB);
                if (!mbar_wait(&sh->tma_full[s], (it / kStagesG) & 1u, watchdog_full_barrier, p.watchdog)
                    || (it >= kStagesB
                        && !mbar_wait(&sh->b_empty[sbs], ((it / kStagesB) & 1u) ^ 1u, watchdog_empty_barrier,
                                      p.watchdog))) {
                    *abort_flag = 1;
                    break;
                }
                const uint8_t* raw = smem + kSmemRaw + s * kRawBytes + r * (BK / 2);
                const uint4 c0 = *reinterpret_cast<const uint4*>(raw);
                const uint4 c1 = *reinterpret_cast<const uint4*>(raw + 16);
                bool ok0, ok1;
                const uint32_t s0 = e8m0_half2(sc_pair & 0xFFu, ok0), s1 = e8m0_half2(sc_pair >> 8, ok1);
                scale_ok = scale_ok && (!row_in_tensor || (ok0 && ok1));
                const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                uint8_t* brow = smem + kSmemB + sbs * kBBytes + r * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    // 16-byte chunk c = values 8c..8c+7 = code bytes 4c..4c+3.
                    const uint32_t w = words[c], sc = c < 4 ? s0 : s1;
                    uint4 h;
                    h.x = hmul2_bits(e2m1x2_to_half2(w & 0xFFu), sc);
                    h.y = hmul2_bits(e2m1x2_to_half2((w >> 8) & 0xFFu), sc);
                    h.z = hmul2_bits(e2m1x2_to_half2((w >> 16) & 0xFFu), sc);
                    h.w = hmul2_bits(e2m1x2_to_half2(w >> 24), sc);
                    *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = h;
                }
                fence_proxy_async();
                mbar_arrive(&sh->b_full[sbs]);
            }
        }
        if (!scale_ok && p.status)
            atomicOr(p.status, 2u);
    } else if (warp >= 2 + kDequantWarpsG) {
        // ------------------------------------------------- epilogue warps
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int row = 32 * q + lane;
        uint32_t lt = 0;
        for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x, ++lt) {
            const TileInfo t = tile_info(p, tile);
            const int acc = int(lt & 1u);
            if (!mbar_wait(&sh->acc_full[acc], (lt >> 1) & 1u, watchdog_full_barrier, p.watchdog)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int prow = t.m0 + row;
            const bool valid = prow < t.mend;
            const uint32_t taddr = tmem + uint32_t(acc * BN) + (uint32_t(32 * q) << 16);
            if (p.epilogue == 0) {
                // Activation of (gate, up) pairs -> fp16 act[prow, j].
                auto* act = static_cast<__half*>(p.out);
                const int I = p.Nrows / 2;
                for (int c = 0; c < BN / 64; ++c) {
                    uint32_t g[32], u[32];
                    if (p.split) {
                        tmem_ld32(taddr + uint32_t(32 * c), g);
                        tmem_ld32(taddr + uint32_t(BN / 2 + 32 * c), u);
                    } else {
                        // Interleaved: column 2i gate, 2i+1 up.
                        uint32_t a[32], b[32];
                        tmem_ld32(taddr + uint32_t(64 * c), a);
                        tmem_ld32(taddr + uint32_t(64 * c + 32), b);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            g[i] = a[2 * i], u[i] = a[2 * i + 1];
                            g[16 + i] = b[2 * i], u[16 + i] = b[2 * i + 1];
                        }
                    }
                    tmem_wait_ld();
                    const int j0 = t.nt * (BN / 2) + 32 * c;
                    if (valid && j0 < I) {
                        // Pairs of fp16 outputs in registers (constant indices only).
                        uint32_t hv[16];
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const int j = j0 + i;
                            float gv = __uint_as_float(g[i]), uv = __uint_as_float(u[i]);
                            if (p.bias) {
                                const int gr = p.split ? j : 2 * j, ur = p.split ? I + j : 2 * j + 1;
                                gv += p.bias[size_t(t.e) * p.Nrows + gr];
                                uv += p.bias[size_t(t.e) * p.Nrows + ur];
                            }
                            const uint32_t h = __half_as_ushort(__float2half_rn(act_fn(gv, uv, p.act_kind, p.limit, p.alpha)));
                            hv[i / 2] = (i & 1) ? hv[i / 2] | (h << 16) : h;
                        }
                        __half* dst = act + size_t(prow) * p.out_cols + j0;
                        const int n = min(32, I - j0);
                        if (n == 32) {
#pragma unroll
                            for (int v = 0; v < 4; ++v)
                                reinterpret_cast<uint4*>(dst)[v] = make_uint4(hv[4 * v], hv[4 * v + 1], hv[4 * v + 2], hv[4 * v + 3]);
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (i < n)
                                    dst[i] = __ushort_as_half(uint16_t(hv[i / 2] >> (16 * (i & 1))));
                        }
                    }
                }
            } else {
                auto* y = static_cast<float*>(p.out);
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(taddr + uint32_t(32 * c), v);
                    tmem_wait_ld();
                    const int n0 = t.nt * BN + 32 * c;
                    if (valid && n0 < p.Nrows) {
                        float* dst = y + size_t(prow) * p.out_cols + n0;
                        const int n = min(32, p.Nrows - n0);
                        float f[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            f[i] = __uint_as_float(v[i])
                                   + (p.bias && i < n ? p.bias[size_t(t.e) * p.Nrows + n0 + i] : 0.f);
                        if (n == 32) {
#pragma unroll
                            for (int k = 0; k < 8; ++k)
                                reinterpret_cast<float4*>(dst)[k] = make_float4(f[4 * k], f[4 * k + 1], f[4 * k + 2], f[4 * k + 3]);
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (i < n)
                                    dst[i] = f[i];
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&sh->acc_empty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        tmem_dealloc(tmem, 2 * BN);
}

// ----------------------------------------------------------- grouped GEMV
// Decode-sized batches (a few tokens per expert): the layer is a weight
// stream. Items are (expert, 16 weight rows), dealt round-robin over the CTAs
// and skipped for experts without tokens; the four warps of a CTA split the
// item's K range and add their partial sums through shared memory. Rows are
// multiplied by the expert's tokens 8 at a time with mma.m16n8k16 (fp16
// operands, fp32 accumulation). Lane (g, t) loads, per 128 columns, MXFP4
// block t of its rows g and g+8 (16 contiguous code bytes each) and the 32
// matching activations of token g; inside each MMA the k order is the same
// permutation on both operands (slot pair 2t,2t+1 of MMA m <- block values
// 4m, 4m+1; pair 2t+8,2t+9 <- 4m+2, 4m+3), so no data crosses lanes. For
// gate/up the item's MMA rows are gate rows of 8 outputs (rows 0-7) and the
// matching up rows (8-15), so each lane finishes its outputs in registers.
// Weights decode exactly as in the GEMM (cvt.rn.f16x2.e2m1x2 times the
// power-of-two block scale).
constexpr int kGemvWarps = 4;

struct GemvParams {
    const uint8_t* blocks;  // [E, Nrows, K/2]
    const uint8_t* scales;  // [E, Nrows, K/32]
    const float* bias;      // [E, Nrows] or null
    const __half* x;        // [n, K], expert-sorted rows
    const int* offsets;     // [E + 1]
    void* out;              // epilogue 0: fp16 act [n, out_cols]; 1: fp32 y [n, out_cols]
    int K, Nrows, E, chunks, epilogue, split, out_cols, act_kind;
    float limit, alpha;
    unsigned* status;
};

__device__ __forceinline__ void hmma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1)
    );
}

// Weight row of MMA row i (0..15) of item chunk c. Gate/up: rows 0-7 are the
// gate rows of outputs 8c..8c+7, rows 8-15 the matching up rows.
__device__ __forceinline__ int gemv_row(const GemvParams& p, int c, int i) {
    if (p.epilogue == 0) {
        const int j = 8 * c + (i & 7);
        const bool up = i >= 8;
        return p.split ? (up ? p.Nrows / 2 + j : j) : 2 * j + (up ? 1 : 0);
    }
    return 16 * c + i;
}

// The MMAs of one 128-column step: the lane's 32-value blocks of rows g (w0,
// E8M0 byte s0b) and g + 8 (w1, s1b) and its 32 fp16 activations (x0..x3).
// live: the lane holds a block of K (else zeros, which every lane feeds).
__device__ __forceinline__ void gemv_step(uint4 w0, uint4 w1, uint32_t s0b, uint32_t s1b, uint4 x0, uint4 x1,
                                          uint4 x2, uint4 x3, bool live, float (&acc)[4], bool& scale_ok) {
    bool ok0, ok1;
    const uint32_t s0 = e8m0_half2(s0b, ok0), s1 = e8m0_half2(s1b, ok1);
    scale_ok = scale_ok && ((ok0 && ok1) || !live);
    const uint32_t cw0[4] = {w0.x, w0.y, w0.z, w0.w}, cw1[4] = {w1.x, w1.y, w1.z, w1.w};
    const uint32_t xw[16] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w,
                             x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        // Code bytes 2m, 2m+1 of the block: values 4m..4m+3.
        const uint32_t wa = cw0[m >> 1] >> (16 * (m & 1)), wb = cw1[m >> 1] >> (16 * (m & 1));
        const uint32_t a0 = hmul2_bits(e2m1x2_to_half2(wa & 0xFFu), s0);
        const uint32_t a2 = hmul2_bits(e2m1x2_to_half2((wa >> 8) & 0xFFu), s0);
        const uint32_t a1 = hmul2_bits(e2m1x2_to_half2(wb & 0xFFu), s1);
        const uint32_t a3 = hmul2_bits(e2m1x2_to_half2((wb >> 8) & 0xFFu), s1);
        hmma16816(acc, a0, a1, a2, a3, xw[2 * m], xw[2 * m + 1]);
    }
}

// One 16-row x 8-token MMA item over all of K: this warp's K steps (128
// columns each; steps warp, warp + 4, ...), each step's operands loaded a
// step ahead of its MMAs. code0/code1 and sc0/sc1: the lane's rows g and
// g + 8 (codes, E8M0 bytes); xr: the lane's token row (fp16, global or
// shared memory). acc: the mma C fragment (rows g, g + 8 x tokens 2t, 2t+1).
__device__ __forceinline__ void gemv_item(const uint8_t* code0, const uint8_t* code1, const uint8_t* sc0,
                                          const uint8_t* sc1, const __half* xr, int K, int warp, float (&acc)[4],
                                          bool& scale_ok) {
    const int t = threadIdx.x & 3, iters = (K + 127) / 128;
    struct Step {
        uint4 w0, w1, x0, x1, x2, x3;
        uint32_t s0, s1;  // E8M0 scale bytes (decoded at MMA time, so no load is waited on early)
        bool live;
    };
    auto load = [&](int it, Step& st) {
        const int k0 = 128 * it + 32 * t;  // first column of this lane's block
        // Past K (K % 128 == 64 leaves lanes t = 2, 3 without a block in the
        // last step): zeros, since every lane takes part in the MMAs.
        const bool live = it < iters && k0 < K;
        const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
        st.w0 = live ? __ldg(reinterpret_cast<const uint4*>(code0 + k0 / 2)) : zero;
        st.w1 = live ? __ldg(reinterpret_cast<const uint4*>(code1 + k0 / 2)) : zero;
        st.live = live;
        st.s0 = live ? uint32_t(sc0[k0 / 32]) : 127u;
        st.s1 = live ? uint32_t(sc1[k0 / 32]) : 127u;
        const uint4* xq = reinterpret_cast<const uint4*>(xr + (live ? k0 : 0));
        st.x0 = live ? xq[0] : zero, st.x1 = live ? xq[1] : zero;
        st.x2 = live ? xq[2] : zero, st.x3 = live ? xq[3] : zero;
    };
    auto mma = [&](const Step& st) {
        gemv_step(st.w0, st.w1, st.s0, st.s1, st.x0, st.x1, st.x2, st.x3, st.live, acc, scale_ok);
    };
    Step cur, nxt;
    load(warp, cur);
    for (int it = warp; it < iters; it += 2 * kGemvWarps) {
        load(it + kGemvWarps, nxt);
        mma(cur);
        load(it + 2 * kGemvWarps, cur);
        if (it + kGemvWarps < iters)
            mma(nxt);
    }
}

// gemv_item with every weight and scale load of the warp's steps issued
// before its first MMA (K <= kSteps * kGemvWarps * 128), so an item costs one
// memory round trip instead of one per two steps; the activations (shared
// memory) are read at each step. The same MMAs in the same order, hence the
// same sums.
template <int kSteps>
__device__ __forceinline__ void gemv_item_all(const uint8_t* code0, const uint8_t* code1, const uint8_t* sc0,
                                              const uint8_t* sc1, const __half* xr, int K, int warp, float (&acc)[4],
                                              bool& scale_ok) {
    const int t = threadIdx.x & 3, iters = (K + 127) / 128;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    uint4 w0[kSteps], w1[kSteps];
    uint32_t s0[kSteps], s1[kSteps];
#pragma unroll
    for (int j = 0; j < kSteps; ++j) {
        const int it = warp + kGemvWarps * j, k0 = 128 * it + 32 * t;
        const bool live = it < iters && k0 < K;
        w0[j] = live ? __ldg(reinterpret_cast<const uint4*>(code0 + k0 / 2)) : zero;
        w1[j] = live ? __ldg(reinterpret_cast<const uint4*>(code1 + k0 / 2)) : zero;
        s0[j] = live ? uint32_t(sc0[k0 / 32]) : 127u;
        s1[j] = live ? uint32_t(sc1[k0 / 32]) : 127u;
    }
#pragma unroll
    for (int j = 0; j < kSteps; ++j) {
        const int it = warp + kGemvWarps * j, k0 = 128 * it + 32 * t;
        if (it >= iters)
            break;
        const bool live = k0 < K;
        const uint4* xq = reinterpret_cast<const uint4*>(xr + (live ? k0 : 0));
        gemv_step(w0[j], w1[j], s0[j], s1[j], live ? xq[0] : zero, live ? xq[1] : zero, live ? xq[2] : zero,
                  live ? xq[3] : zero, live, acc, scale_ok);
    }
}
constexpr int kAllSteps = 6;                               // gemv_item_all in the decode kernel
constexpr int kAllK = kAllSteps * kGemvWarps * 128;        // K up to 3072 (gpt-oss: 2880)

__global__ void __launch_bounds__(32 * kGemvWarps) moe_gemv_kernel(const __grid_constant__ GemvParams p) {
    __shared__ float4 part[kGemvWarps][32];  // each lane's four accumulators, per warp
    __shared__ int off[kMaxExperts + 1];     // expert row offsets: the skip test costs no global load
    pdl_enter();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int blocks_per_row = p.K / 32;
    for (int i = threadIdx.x; i <= p.E; i += blockDim.x)
        off[i] = p.offsets[i];
    __syncthreads();
    bool scale_ok = true;
    for (int item = blockIdx.x; item < p.E * p.chunks; item += gridDim.x) {
        const int e = item / p.chunks, c = item % p.chunks;
        const int p0 = off[e], count = off[e + 1] - p0;
        if (count == 0)
            continue;
        const int r0 = gemv_row(p, c, g), r1 = gemv_row(p, c, g + 8);
        const uint8_t* code0 = p.blocks + (size_t(e) * p.Nrows + r0) * (p.K / 2);
        const uint8_t* code1 = p.blocks + (size_t(e) * p.Nrows + r1) * (p.K / 2);
        const uint8_t* sc0 = p.scales + (size_t(e) * p.Nrows + r0) * blocks_per_row;
        const uint8_t* sc1 = p.scales + (size_t(e) * p.Nrows + r1) * blocks_per_row;
        for (int q = 0; q < count; q += 8) {
            const int tok = min(q + g, count - 1);  // B column g: token q+g (clamped; unused columns ignored)
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            gemv_item(code0, code1, sc0, sc1, p.x + size_t(p0 + tok) * p.K, p.K, warp, acc, scale_ok);
            // Sum the warps' K ranges (fixed order), then warp 0 finishes.
            part[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            __syncthreads();
            if (warp == 0) {
                float4 sum = part[0][lane];
                for (int w = 1; w < kGemvWarps; ++w) {
                    const float4 o = part[w][lane];
                    sum.x += o.x, sum.y += o.y, sum.z += o.z, sum.w += o.w;
                }
                // sum: (row r0: tokens q+2t, q+2t+1), (row r1: same tokens)
                const float b0 = p.bias ? p.bias[size_t(e) * p.Nrows + r0] : 0.f;
                const float b1 = p.bias ? p.bias[size_t(e) * p.Nrows + r1] : 0.f;
                const float v0[2] = {sum.x + b0, sum.y + b0}, v1[2] = {sum.z + b1, sum.w + b1};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int tl = q + 2 * t + h;
                    if (tl >= count)
                        continue;
                    if (p.epilogue == 1) {
                        auto* y = static_cast<float*>(p.out);
                        y[size_t(p0 + tl) * p.out_cols + r0] = v0[h];
                        y[size_t(p0 + tl) * p.out_cols + r1] = v1[h];
                    } else {
                        // r0 is the gate row, r1 the up row of output 8c + g.
                        auto* act = static_cast<__half*>(p.out);
                        act[size_t(p0 + tl) * p.out_cols + 8 * c + g] =
                            __float2half_rn(act_fn(v0[h], v1[h], p.act_kind, p.limit, p.alpha));
                    }
                }
            }
            __syncthreads();
        }
    }
    if (!scale_ok && p.status)
        atomicOr(p.status, 2u);
}

// --------------------------------------------------------- fused decode
// The whole layer for a few tokens (T <= kDecodeTokens) in one cooperative
// launch. Every CTA routes all T tokens itself (the same warp code as
// moe_route_kernel, so the same choices) and converts their rows to fp16 in
// shared memory; phase 1 deals (routed expert, 8 gate/up outputs) items over
// the CTAs with the activation written as fp16 rows in slot order; a grid
// barrier; phase 2 deals (routed expert, 16 down rows) items, fp32 rows in
// slot order; a grid barrier; phase 3 adds each token's k rows in selection
// order, as moe_combine_kernel does. Items use the same per-item loop as
// moe_gemv_kernel, so the outputs are the staged path's. The barrier words
// are zero at launch and the waits bounded: a grid that cannot meet reports
// to the watchdog and leaves the outputs.
constexpr int kDecodeTokens = 8;
constexpr int kDecodeSlots = kDecodeTokens * kMaxTopK;

struct DecodeParams {
    const uint8_t *gu_blocks, *gu_scales, *dn_blocks, *dn_scales;
    const float *gu_bias, *dn_bias;
    const void* x;  // [T][H] bf16 (x_f32 0) or fp32
    const float* logits;  // [T][E]
    __half* act;          // [T * K][I] workspace
    float* y;             // [T * K][H] workspace
    float* out;           // [T][H]
    unsigned* barrier;    // two words, zero at launch
    unsigned* status;
    unsigned* watchdog;
    int T, H, I, E, K, split, act_kind, x_f32;
    int act_smem;         // 1: phase 2 reads the activation rows from a shared-memory copy
    float limit, alpha;
};

struct DecodeShared {
    int chosen[kDecodeSlots];
    float weight[kDecodeSlots];
    int pos[kDecodeSlots];               // act row of (token, selection)
    int slot_expert[kDecodeSlots];       // routed experts, ascending
    int slot_base[kDecodeSlots + 1];     // first act row of each
    int slot_token[kDecodeSlots];        // token of each act row
    int slots;
    float4 part[kGemvWarps][32];
};

// All CTAs of the (co-resident) grid arrive; false when the wait ran out.
__device__ bool decode_barrier(unsigned* word, unsigned* watchdog, int* failed) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(word, 1u);
        uint32_t polls = 0;
        while (*reinterpret_cast<volatile unsigned*>(word) < gridDim.x) {
            if (++polls == wait_polls) {
                atomicOr(watchdog, watchdog_full_barrier);
                *failed = 1;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
    }
    __syncthreads();
    return !*failed;
}

__global__ void __launch_bounds__(32 * kGemvWarps) moe_decode_kernel(const __grid_constant__ DecodeParams p) {
    __shared__ DecodeShared sh;
    extern __shared__ __align__(16) __half xh[];  // [T][H]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int T = p.T, H = p.H, I = p.I, K = p.K;
    // Routing of every token (warp per token) and the fp16 rows.
    for (int tok = warp; tok < T; tok += kGemvWarps)
        route_token(p.logits + size_t(tok) * p.E, p.E, K, sh.chosen + tok * K, sh.weight + tok * K, nullptr);
    bool bad = false;
    for (int i = threadIdx.x; i < T * H / 8; i += blockDim.x) {
        float2 v[4];
        if (p.x_f32)
            load8(static_cast<const float*>(p.x) + size_t(i) * 8, v);
        else
            load8(static_cast<const __nv_bfloat16*>(p.x) + size_t(i) * 8, v);
        uint4 o;
        __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            bad |= fabsf(v[k].x) > 65504.f || fabsf(v[k].y) > 65504.f;
            h[k] = __floats2half2_rn(v[k].x, v[k].y);
        }
        *reinterpret_cast<uint4*>(xh + size_t(i) * 8) = o;
    }
    // Any input value beyond fp16 range, from whichever thread converted it.
    bad = __syncthreads_or(bad) != 0;
    if (T * K <= 32) {
        // Routed experts in ascending order, their tokens in token order (the
        // stable counting sort's order), and each (token, selection)'s row:
        // entry l = tok * K + s goes to row rank(e_l, l), one lane per entry.
        if (warp == 0) {
            const int n = T * K;
            const int e = lane < n ? sh.chosen[lane] : 0x7fffffff;
            bool first = lane < n;
            int rank = 0;
            for (int m = 0; m < n; ++m) {
                const int em = __shfl_sync(0xffffffffu, e, m);
                rank += em < e || (em == e && m < lane);
                first = first && !(em == e && m < lane);
            }
            const unsigned firsts = __ballot_sync(0xffffffffu, first);
            int slot = 0;
            for (int m = 0; m < n; ++m) {
                const int em = __shfl_sync(0xffffffffu, e, m);
                slot += ((firsts >> m) & 1u) && em < e;
            }
            if (lane < n) {
                sh.pos[lane] = rank;
                sh.slot_token[rank] = lane / K;
                if (first)
                    sh.slot_expert[slot] = e, sh.slot_base[slot] = rank;
            }
            if (lane == 0) {
                const int slots = __popc(firsts);
                sh.slot_base[slots] = n;
                sh.slots = slots;
                if (bad && blockIdx.x == 0 && p.status)
                    atomicOr(p.status, 4u);
            }
        }
    } else if (threadIdx.x == 0) {
        // The same order, one thread.
        int n = 0, row = 0;
        for (int e = 0; e < p.E; ++e) {
            int cnt = 0;
            for (int tok = 0; tok < T; ++tok)
                for (int s = 0; s < K; ++s)
                    if (sh.chosen[tok * K + s] == e) {
                        sh.slot_token[row + cnt] = tok;
                        sh.pos[tok * K + s] = row + cnt;
                        ++cnt;
                    }
            if (cnt) {
                sh.slot_expert[n] = e;
                sh.slot_base[n] = row;
                ++n;
                row += cnt;
            }
        }
        sh.slot_base[n] = row;
        sh.slots = n;
        if (bad && blockIdx.x == 0 && p.status)
            atomicOr(p.status, 4u);
    }
    __syncthreads();
    const int slots = sh.slots;
    bool scale_ok = true;

    // Phase 1: gate/up items (slot, 8 outputs).
    const int chunks1 = I / 8;
    for (int item = blockIdx.x; item < slots * chunks1; item += gridDim.x) {
        const int s = item / chunks1, c = item % chunks1, e = sh.slot_expert[s];
        const int b0 = sh.slot_base[s], count = sh.slot_base[s + 1] - b0;
        const int j0 = 8 * c + g;
        const int r0 = p.split ? j0 : 2 * j0, r1 = p.split ? I + j0 : 2 * j0 + 1;  // gate, up rows
        const size_t N1 = size_t(2) * I;
        const uint8_t* code0 = p.gu_blocks + (size_t(e) * N1 + r0) * (H / 2);
        const uint8_t* code1 = p.gu_blocks + (size_t(e) * N1 + r1) * (H / 2);
        const uint8_t* sc0 = p.gu_scales + (size_t(e) * N1 + r0) * (H / 32);
        const uint8_t* sc1 = p.gu_scales + (size_t(e) * N1 + r1) * (H / 32);
        const int tok = sh.slot_token[b0 + min(g, count - 1)];
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (H <= kAllK)
            gemv_item_all<kAllSteps>(code0, code1, sc0, sc1, xh + size_t(tok) * H, H, warp, acc, scale_ok);
        else
            gemv_item(code0, code1, sc0, sc1, xh + size_t(tok) * H, H, warp, acc, scale_ok);
        sh.part[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncthreads();
        if (warp == 0) {
            float4 sum = sh.part[0][lane];
            for (int w = 1; w < kGemvWarps; ++w) {
                const float4 o = sh.part[w][lane];
                sum.x += o.x, sum.y += o.y, sum.z += o.z, sum.w += o.w;
            }
            const float bg = p.gu_bias ? p.gu_bias[size_t(e) * N1 + r0] : 0.f;
            const float bu = p.gu_bias ? p.gu_bias[size_t(e) * N1 + r1] : 0.f;
            const float v0[2] = {sum.x + bg, sum.y + bg}, v1[2] = {sum.z + bu, sum.w + bu};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int tl = 2 * t + h;
                if (tl < count)
                    p.act[size_t(b0 + tl) * I + j0] = __float2half_rn(act_fn(v0[h], v1[h], p.act_kind, p.limit, p.alpha));
            }
        }
        __syncthreads();
    }

    // Every activation row is written before any is read.
    __shared__ int failed;
    if (threadIdx.x == 0)
        failed = 0;
    if (!decode_barrier(p.barrier, p.watchdog, &failed))
        return;

    // The activation rows into shared memory (the phase-1 rows' buffer) when
    // they fit: phase 2 then reads them without a round trip to L2.
    __half* act_rows = p.act;
    if (p.act_smem) {
        const int rows = sh.slot_base[slots];
        const uint4* src = reinterpret_cast<const uint4*>(p.act);
        uint4* dst = reinterpret_cast<uint4*>(xh);
        for (int i = threadIdx.x; i < rows * I / 8; i += blockDim.x)
            dst[i] = src[i];
        __syncthreads();
        act_rows = xh;
    }

    // Phase 2: down items (routed expert, 16 rows), fp32 rows in slot order.
    const int chunks2 = H / 16;
    for (int item = blockIdx.x; item < slots * chunks2; item += gridDim.x) {
        const int s = item / chunks2, c = item % chunks2;
        const int e = sh.slot_expert[s], b0 = sh.slot_base[s], count = sh.slot_base[s + 1] - b0;
        const int r0 = 16 * c + g, r1 = r0 + 8;
        const uint8_t* code0 = p.dn_blocks + (size_t(e) * H + r0) * (I / 2);
        const uint8_t* code1 = p.dn_blocks + (size_t(e) * H + r1) * (I / 2);
        const uint8_t* sc0 = p.dn_scales + (size_t(e) * H + r0) * (I / 32);
        const uint8_t* sc1 = p.dn_scales + (size_t(e) * H + r1) * (I / 32);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const __half* xr = act_rows + size_t(b0 + min(g, count - 1)) * I;
        if (p.act_smem && I <= kAllK)
            gemv_item_all<kAllSteps>(code0, code1, sc0, sc1, xr, I, warp, acc, scale_ok);
        else
            gemv_item(code0, code1, sc0, sc1, xr, I, warp, acc, scale_ok);
        sh.part[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncthreads();
        if (warp == 0) {
            float4 sum = sh.part[0][lane];
            for (int w = 1; w < kGemvWarps; ++w) {
                const float4 o = sh.part[w][lane];
                sum.x += o.x, sum.y += o.y, sum.z += o.z, sum.w += o.w;
            }
            const float b_0 = p.dn_bias ? p.dn_bias[size_t(e) * H + r0] : 0.f;
            const float b_1 = p.dn_bias ? p.dn_bias[size_t(e) * H + r1] : 0.f;
            const float v0[2] = {sum.x + b_0, sum.y + b_0}, v1[2] = {sum.z + b_1, sum.w + b_1};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int tl = 2 * t + h;
                if (tl < count) {
                    p.y[size_t(b0 + tl) * H + r0] = v0[h];
                    p.y[size_t(b0 + tl) * H + r1] = v1[h];
                }
            }
        }
        __syncthreads();
    }
    if (!scale_ok && p.status)
        atomicOr(p.status, 2u);
    if (!decode_barrier(p.barrier + 1, p.watchdog, &failed))
        return;

    // Phase 3: each token's k rows in selection order.
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < size_t(T) * H;
         i += size_t(gridDim.x) * blockDim.x) {
        const int tok = int(i / H), d = int(i % H);
        float acc = 0.f;
        for (int k = 0; k < K; ++k)
            acc = fmaf(sh.weight[tok * K + k], p.y[size_t(sh.pos[tok * K + k]) * H + d], acc);
        p.out[i] = acc;
    }
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

bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, int esize, const void* base, uint64_t inner, uint64_t rows,
               uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto enc = encoder();
    if (!enc)
        return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {inner * uint64_t(esize)};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(map, type, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)
           == CUDA_SUCCESS;
}

size_t align_up(size_t v, size_t a) {
    return (v + a - 1) / a * a;
}

struct Workspace {
    int *chosen, *counts, *offsets, *perm, *pos, *mtile;
    float* weight;
    __half *xs, *act;
    float* y;
    size_t bytes;
};

// Workspace of the whole layer for `tokens` tokens. The dispatch stage uses
// the part up to xs (carve with inter = 0 and no y for it alone).
Workspace carve_shape(void* base, size_t tokens, size_t hidden, size_t inter, size_t experts, size_t top_k, bool y) {
    const size_t n = tokens * top_k, E = experts;
    auto* b = static_cast<uint8_t*>(base);
    size_t at = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = b ? b + at : nullptr;
        at = align_up(at + bytes, 256);
        return p;
    };
    Workspace ws;
    ws.chosen = reinterpret_cast<int*>(take(n * 4));
    ws.weight = reinterpret_cast<float*>(take(n * 4));
    ws.counts = reinterpret_cast<int*>(take(E * 4));
    ws.offsets = reinterpret_cast<int*>(take((E + 1) * 4));
    ws.perm = reinterpret_cast<int*>(take(n * 4));
    ws.pos = reinterpret_cast<int*>(take(n * 4));
    ws.mtile = reinterpret_cast<int*>(take((E + 1) * 4));
    ws.xs = reinterpret_cast<__half*>(take(n * hidden * 2));
    ws.act = inter ? reinterpret_cast<__half*>(take(n * inter * 2)) : nullptr;
    ws.y = y ? reinterpret_cast<float*>(take(n * hidden * 4)) : nullptr;
    ws.bytes = at;
    return ws;
}

Workspace carve(void* base, const kb200_moe_weights& w, size_t tokens) {
    return carve_shape(base, tokens, size_t(w.hidden), size_t(w.inter), size_t(w.experts), size_t(w.top_k), true);
}

// Workspace of the expert stage alone over `rows` grouped rows: the m-tile
// prefix and the fp16 activations between the two GEMMs.
struct ExpertWs {
    int* mtile;
    __half* act;
    size_t bytes;
};

ExpertWs carve_experts(void* base, const kb200_moe_weights& w, size_t rows) {
    auto* b = static_cast<uint8_t*>(base);
    ExpertWs ws;
    ws.mtile = reinterpret_cast<int*>(b);
    const size_t act_at = align_up(size_t(w.experts + 1) * 4, 256);
    ws.act = b ? reinterpret_cast<__half*>(b + act_at) : nullptr;
    ws.bytes = act_at + align_up(rows * size_t(w.inter) * 2, 256);
    return ws;
}

int check_shape(int hidden, int experts, int top_k) {
    if (hidden <= 0 || experts <= 0 || top_k <= 0)
        return fail(KB200_INVALID, "MoE shape must be positive");
    if (hidden % 64 || hidden > kMaxK)
        return fail(KB200_UNSUPPORTED, "hidden and inter must be multiples of 64, at most 4096");
    if (experts > kMaxExperts || top_k > std::min(experts, kMaxTopK))
        return fail(KB200_UNSUPPORTED, "at most 256 experts and top_k <= min(experts, 32)");
    return KB200_OK;
}

// routed: the weights route tokens themselves (top_k is checked); the
// expert stage alone ignores top_k (a rank may hold fewer experts than k).
int check_weights(const kb200_moe_weights* w, bool routed = true) {
    if (!w)
        return fail(KB200_INVALID, "null MoE weights");
    if (const int s = check_shape(w->hidden, w->experts, routed ? w->top_k : 1))
        return s;
    if (w->inter <= 0)
        return fail(KB200_INVALID, "MoE shape must be positive");
    if (w->inter % 64 || w->inter > kMaxK)
        return fail(KB200_UNSUPPORTED, "hidden and inter must be multiples of 64, at most 4096");
    if (!w->gate_up_blocks || !w->gate_up_scales || !w->down_blocks || !w->down_scales)
        return fail(KB200_INVALID, "null MoE weight pointer");
    if (!aligned(w->gate_up_blocks, 16) || !aligned(w->down_blocks, 16) || !aligned(w->gate_up_scales, 16)
        || !aligned(w->down_scales, 16))
        return fail(KB200_INVALID, "MoE weights must be 16-byte aligned");
    if (w->activation != KB200_MOE_SWIGLU_OAI && w->activation != KB200_MOE_SILU)
        return fail(KB200_UNSUPPORTED, "unknown MoE activation");
    return KB200_OK;
}

int gemm_slots() {
    static int set[64] = {};
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> guard(lock);
    if (!set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(moe_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal);
        if (e != cudaSuccess)
            return -cuda_fail(e, "moe_gemm_kernel attribute");
        set[dev] = 1;
    }
    return sm_count();
}

int launch_gemm(GroupParams& p, int max_tiles, cudaStream_t stream) {
    const int slots = gemm_slots();
    if (slots <= 0)
        return -slots;
    p.watchdog = watchdog_word();
    const int grid = std::max(1, std::min(slots, max_tiles));
    // A plain launch: GEMM CTAs launched early would hold SMs (225 KB of
    // shared memory each) that the gather kernel before them still needs.
    TraceScope trace(KB200_KERNEL_MOE_GEMM, stream);
    moe_gemm_kernel<<<grid, kThreadsG, kSmemTotal, stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "moe_gemm_kernel launch");
}

}  // namespace
}  // namespace kb200

using namespace kb200;

namespace kb200 {
namespace {

// Scratch of kb200_moe_forward_noalloc: a file-scope device array, so every
// GPU that loads this library holds KB200_MOE_STATIC_SCRATCH_BYTES of it
// until the process exits. Host code must not use the symbol itself as a
// pointer (that is a host-side stand-in); static_scratch() returns the
// device address.
__device__ __align__(256) uint8_t moe_static_scratch[KB200_MOE_STATIC_SCRATCH_BYTES];

// Device address of moe_static_scratch on the current device, looked up once
// per device (with that device current) on its first use.
int static_scratch(void** ptr) {
    static void* address[64] = {};
    static std::mutex lock;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64)
        return fail(KB200_UNSUPPORTED, "device index above 63");
    std::lock_guard<std::mutex> guard(lock);
    if (!address[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, moe_static_scratch);
        if (e != cudaSuccess)
            return cuda_fail(e, "cudaGetSymbolAddress(moe_static_scratch)");
        address[dev] = p;
    }
    *ptr = address[dev];
    return KB200_OK;
}

}  // namespace
}  // namespace kb200

namespace kb200 {
namespace {

// m-tile prefix of caller-grouped rows: mtile[e] = sum over e' < e of
// ceil(rows(e') / 128).
__global__ void moe_mtile_kernel(const int* offsets, int E, int* mtile) {
    if (threadIdx.x || blockIdx.x)
        return;
    int tiles = 0;
    for (int e = 0; e < E; ++e) {
        mtile[e] = tiles;
        tiles += (offsets[e + 1] - offsets[e] + 127) / 128;
    }
    mtile[E] = tiles;
}

// dst rows [d, d + n) = src rows [s, s + n) for each segment {s, d, n}
// (blockIdx.y); 16-byte words, grid-stride over the segment.
__global__ void rows_regroup_kernel(const uint4* src, uint4* dst, size_t row_words, const long long* seg) {
    const long long s = seg[3 * blockIdx.y], d = seg[3 * blockIdx.y + 1], n = seg[3 * blockIdx.y + 2];
    const size_t words = size_t(n) * row_words;
    const uint4* from = src + size_t(s) * row_words;
    uint4* to = dst + size_t(d) * row_words;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < words; i += size_t(gridDim.x) * blockDim.x)
        to[i] = from[i];
}

// Routing, stable sort by expert and the gather of the sorted fp16 rows
// from bf16 token rows (x_f32 false) or fp32 rows.
int dispatch_launch(const float* logits, const void* x, size_t tokens, int H, int E, int K,
                    const Workspace& ws, unsigned* status, cudaStream_t stream, bool x_f32 = false) {
    const size_t n = tokens * size_t(K);
    cudaError_t e = cudaMemsetAsync(ws.counts, 0, size_t(E) * 4, stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "counts memset");
    e = launch_pdl(KB200_KERNEL_MOE_ROUTE, moe_route_kernel, dim3(unsigned((tokens * 32 + 255) / 256)), dim3(256), 0, stream, logits,
                   int(tokens), E, K, ws.chosen, ws.weight, ws.counts);
    if (e == cudaSuccess)
        e = launch_pdl(KB200_KERNEL_MOE_SORT, moe_sort_kernel, dim3(1), dim3(1024), 0, stream, static_cast<const int*>(ws.chosen), int(n), E,
                       static_cast<const int*>(ws.counts), ws.offsets, ws.perm, ws.pos, ws.mtile);
    const size_t work = n * size_t(H / 8);
    const int blocks = int(std::min<size_t>((work + 255) / 256, size_t(sm_count()) * 16));
    if (e == cudaSuccess)
        e = x_f32 ? launch_pdl(KB200_KERNEL_MOE_GATHER, moe_gather_kernel<float>, dim3(blocks), dim3(256), 0, stream,
                               static_cast<const float*>(x), static_cast<const int*>(ws.perm), int(n), K, H, ws.xs,
                               status)
                  : launch_pdl(KB200_KERNEL_MOE_GATHER, moe_gather_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, stream,
                               static_cast<const __nv_bfloat16*>(x), static_cast<const int*>(ws.perm), int(n), K, H,
                               ws.xs, status);
    if (e != cudaSuccess || (e = cudaGetLastError()) != cudaSuccess)
        return cuda_fail(e, "MoE routing launches");
    return KB200_OK;
}

// The expert stage over n rows grouped by expert (offsets[E + 1], mtile[E + 1]
// on the device): gate/up with the activation, then down into y (fp32 [n, H]).
int experts_launch(const kb200_moe_weights* w, const __half* xs, const int* offsets, const int* mtile, size_t n,
                   __half* act, float* y, unsigned* status, cudaStream_t stream) {
    if (!encoder())
        return fail(KB200_CUDA, "cuTensorMapEncodeTiled unavailable");
    const int H = w->hidden, I = w->inter, E = w->experts;
    cudaError_t e;
    const int mtiles_max = int((n + BM - 1) / BM) + E;

    // Decode-sized batches (at most 8 token rows per expert on average) are a
    // weight stream: the grouped GEMV reads each routed expert once per 8 of
    // its rows. KB200_MOE_PATH=gemm|gemv overrides the choice.
    bool gemv = n <= size_t(8) * size_t(E);
    if (const char* path = std::getenv("KB200_MOE_PATH"))
        gemv = std::strcmp(path, "gemv") == 0 ? true : std::strcmp(path, "gemm") == 0 ? false : gemv;
    if (gemv) {
        const int grid_cap = sm_count() * 8;
        GemvParams v;
        std::memset(&v, 0, sizeof(v));
        v.blocks = w->gate_up_blocks;
        v.scales = w->gate_up_scales;
        v.bias = w->gate_up_bias;
        v.x = xs;
        v.offsets = offsets;
        v.out = act;
        v.K = H;
        v.Nrows = 2 * I;
        v.E = E;
        v.chunks = I / 8;
        v.epilogue = 0;
        v.split = w->interleaved ? 0 : 1;
        v.out_cols = I;
        v.act_kind = w->activation;
        v.limit = w->limit;
        v.alpha = w->alpha;
        v.status = status;
        e = launch_pdl(KB200_KERNEL_MOE_GEMV, moe_gemv_kernel, dim3(std::min(E * v.chunks, grid_cap)), dim3(32 * kGemvWarps), 0, stream, v);
        if (e != cudaSuccess)
            return cuda_fail(e, "moe_gemv_kernel launch");
        v.blocks = w->down_blocks;
        v.scales = w->down_scales;
        v.bias = w->down_bias;
        v.x = act;
        v.out = y;
        v.K = I;
        v.Nrows = H;
        v.chunks = H / 16;
        v.epilogue = 1;
        v.split = 0;
        v.out_cols = H;
        e = launch_pdl(KB200_KERNEL_MOE_GEMV, moe_gemv_kernel, dim3(std::min(E * v.chunks, grid_cap)), dim3(32 * kGemvWarps), 0, stream, v);
        if (e != cudaSuccess)
            return cuda_fail(e, "moe_gemv_kernel launch");
        return KB200_OK;
    }

    // gate/up: [n, H] x [2I, H]^T per expert, activation in the epilogue.
    GroupParams g1;
    std::memset(&g1, 0, sizeof(g1));
    const bool split = !w->interleaved;
    if (!encode_2d(&g1.a_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xs, uint64_t(H), n, BK, BM,
                   CU_TENSOR_MAP_SWIZZLE_128B)
        || !encode_2d(&g1.b_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->gate_up_blocks, uint64_t(H / 2),
                      uint64_t(E) * 2 * I, BK / 2, BN / 2, CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(KB200_INVALID, "tensor map encoding (gate/up)");
    g1.scales = w->gate_up_scales;
    g1.bias = w->gate_up_bias;
    g1.offsets = offsets;
    g1.mtile_prefix = mtile;
    g1.out = act;
    g1.K = H;
    g1.Nrows = 2 * I;
    g1.E = E;
    // 128 (gate, up) pairs per tile; the last tile of an expert may be partial
    // (its extra rows are read and their outputs dropped).
    g1.n_tiles = (I + BN / 2 - 1) / (BN / 2);
    g1.split = split ? 1 : 0;
    g1.epilogue = 0;
    g1.out_cols = I;
    g1.act_kind = w->activation;
    g1.limit = w->limit;
    g1.alpha = w->alpha;
    g1.status = status;
    if (const int s = launch_gemm(g1, mtiles_max * g1.n_tiles, stream))
        return s;

    // down: [n, I] x [H, I]^T per expert -> fp32 rows.
    GroupParams g2;
    std::memset(&g2, 0, sizeof(g2));
    if (!encode_2d(&g2.a_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, act, uint64_t(I), n, BK, BM,
                   CU_TENSOR_MAP_SWIZZLE_128B)
        || !encode_2d(&g2.b_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->down_blocks, uint64_t(I / 2), uint64_t(E) * H,
                      BK / 2, BN / 2, CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(KB200_INVALID, "tensor map encoding (down)");
    g2.scales = w->down_scales;
    g2.bias = w->down_bias;
    g2.offsets = offsets;
    g2.mtile_prefix = mtile;
    g2.out = y;
    g2.K = I;
    g2.Nrows = H;
    g2.E = E;
    g2.n_tiles = (H + BN - 1) / BN;
    g2.split = 0;
    g2.epilogue = 1;
    g2.out_cols = H;
    g2.status = status;
    return launch_gemm(g2, mtiles_max * g2.n_tiles, stream);
}

int combine_launch(const float* y, const float* weight, const int* pos, size_t tokens, int K, int H, float* out,
                   cudaStream_t stream) {
    const size_t work = tokens * size_t(H / 4);
    const int blocks = int(std::min<size_t>((work + 255) / 256, size_t(sm_count()) * 16));
    const cudaError_t e = launch_pdl(KB200_KERNEL_MOE_COMBINE, moe_combine_kernel, dim3(blocks), dim3(256), 0, stream, y, weight, pos,
                                     int(tokens), K, H, out);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "moe_combine_kernel launch");
}

}  // namespace
}  // namespace kb200

extern "C" {

size_t kb200_moe_workspace_bytes(const kb200_moe_weights* w, size_t tokens) {
    if (!w || check_weights(w) != KB200_OK)
        return 0;
    return carve(nullptr, *w, tokens).bytes;
}

int kb200_moe_route(const float* logits, size_t tokens, int32_t experts, int32_t top_k, int32_t* chosen, float* weight,
                    void* stream) {
    if (experts <= 0 || experts > kMaxExperts || top_k <= 0 || top_k > std::min(experts, kMaxTopK))
        return fail(KB200_UNSUPPORTED, "routing shape");
    if (!tokens)
        return KB200_OK;
    if (!logits || !chosen || !weight)
        return fail(KB200_INVALID, "null pointer");
    const int threads = 256, blocks = int((tokens * 32 + threads - 1) / threads);
    TraceScope trace(KB200_KERNEL_MOE_ROUTE, static_cast<cudaStream_t>(stream));
    moe_route_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(logits, int(tokens), experts, top_k,
                                                                              chosen, weight, nullptr);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "moe_route_kernel launch");
}

}  // extern "C"

namespace kb200 {
namespace {

// The whole layer over token rows x (bf16, or fp32 when x_f32).
// The fused decode kernel takes the layer for at most kDecodeAuto tokens
// (measured on B200 at the gpt-oss-20b shape: T=1 47 us against 54 us
// staged, T=8 219 us against 175 us), rows that fit its shared memory, unless
// KB200_MOE_DECODE=0 or a staged path named by KB200_MOE_PATH says otherwise;
// KB200_MOE_DECODE=1 takes it up to kDecodeTokens (both read at every call).
constexpr int kDecodeAuto = 2;

bool decode_eligible(const kb200_moe_weights* w, size_t tokens) {
    size_t most = size_t(kDecodeAuto);
    if (const char* v = std::getenv("KB200_MOE_DECODE")) {
        if (std::strcmp(v, "0") == 0)
            return false;
        if (std::strcmp(v, "1") == 0)
            most = size_t(kDecodeTokens);
    }
    if (std::getenv("KB200_MOE_PATH"))
        return false;
    return tokens <= most && w->top_k <= kMaxTopK && w->hidden <= kMaxK && w->hidden % 16 == 0 && w->inter % 8 == 0;
}

int decode_launch(const kb200_moe_weights* w, const void* x, bool x_f32, const float* logits, size_t tokens, float* out,
                  const Workspace& ws, unsigned* status, cudaStream_t stream) {
    // Dynamic shared memory: the tokens' fp16 rows (phase 1), reused for the
    // activation rows of phase 2 when those fit kDecodeActSmem.
    constexpr size_t kMaxDyn = size_t(kDecodeTokens) * kMaxK * sizeof(__half);
    constexpr size_t kDecodeActSmem = 48 * 1024;
    const size_t act_bytes = tokens * size_t(w->top_k) * size_t(w->inter) * sizeof(__half);
    const bool act_smem = act_bytes <= kDecodeActSmem;
    const size_t dyn = std::max(tokens * size_t(w->hidden) * sizeof(__half), act_smem ? act_bytes : size_t(0));
    // Co-resident CTAs per SM for each (device, shared memory size), queried once.
    static std::map<std::pair<int, size_t>, int> blocks_per_sm;
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    int resident = 0;
    {
        std::lock_guard<std::mutex> guard(lock);
        int& slot = blocks_per_sm[{dev, dyn}];
        if (!slot) {
            cudaError_t e = cudaFuncSetAttribute(moe_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 int(kMaxDyn));
            int n = 0;
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, moe_decode_kernel, 32 * kGemvWarps, dyn);
            if (e != cudaSuccess)
                return cuda_fail(e, "moe_decode_kernel set-up");
            slot = n > 0 ? n : 1;
        }
        resident = slot;
    }
    DecodeParams p;
    std::memset(&p, 0, sizeof(p));
    p.gu_blocks = w->gate_up_blocks, p.gu_scales = w->gate_up_scales, p.gu_bias = w->gate_up_bias;
    p.dn_blocks = w->down_blocks, p.dn_scales = w->down_scales, p.dn_bias = w->down_bias;
    p.x = x, p.logits = logits, p.act = ws.act, p.y = ws.y, p.out = out;
    p.barrier = reinterpret_cast<unsigned*>(ws.counts);
    p.status = status, p.watchdog = watchdog_word();
    p.T = int(tokens), p.H = w->hidden, p.I = w->inter, p.E = w->experts, p.K = w->top_k;
    p.split = w->interleaved ? 0 : 1, p.act_kind = w->activation, p.x_f32 = x_f32 ? 1 : 0;
    p.limit = w->limit, p.alpha = w->alpha;
    p.act_smem = act_smem ? 1 : 0;
    cudaError_t e = cudaMemsetAsync(p.barrier, 0, 2 * sizeof(unsigned), stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "decode barrier reset");
    // Co-resident CTAs only (the grid barrier waits for all of them).
    const int grid = sm_count() * std::min(resident, 8);
    void* args[] = {&p};
    TraceScope trace(KB200_KERNEL_MOE_DECODE, stream);
    e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(moe_decode_kernel), dim3(grid),
                                    dim3(32 * kGemvWarps), args, dyn, stream);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "moe_decode_kernel launch");
}

int forward_layer(const kb200_moe_weights* w, const void* x, bool x_f32, const float* logits, size_t tokens, float* out,
                  void* workspace, size_t workspace_bytes, unsigned* status, void* stream_ptr) {
    if (const int s = check_weights(w))
        return s;
    if (!tokens)
        return KB200_OK;
    if (!x || !logits || !out || !workspace)
        return fail(KB200_INVALID, "null pointer");
    if (!aligned(x, 16) || !aligned(out, 16) || !aligned(workspace, 256))
        return fail(KB200_INVALID, "MoE activations must be 16-byte aligned, workspace 256-byte aligned");
    const size_t n = tokens * size_t(w->top_k);
    if (n > size_t(INT32_MAX) / 4)
        return fail(KB200_UNSUPPORTED, "too many tokens");
    const Workspace ws = carve(workspace, *w, tokens);
    if (ws.bytes > workspace_bytes)
        return fail(KB200_NO_MEMORY, "MoE workspace too small (see kb200_moe_workspace_bytes)");
    if (!encoder())
        return fail(KB200_CUDA, "cuTensorMapEncodeTiled unavailable");
    auto stream = static_cast<cudaStream_t>(stream_ptr);
    if (decode_eligible(w, tokens))
        return decode_launch(w, x, x_f32, logits, tokens, out, ws, status, stream);
    if (const int s = dispatch_launch(logits, x, tokens, w->hidden, w->experts, w->top_k, ws, status, stream, x_f32))
        return s;
    if (const int s = experts_launch(w, ws.xs, ws.offsets, ws.mtile, n, ws.act, ws.y, status, stream))
        return s;
    return combine_launch(ws.y, ws.weight, ws.pos, tokens, w->top_k, w->hidden, out, stream);
}

}  // namespace
}  // namespace kb200

extern "C" {

int kb200_moe_forward(const kb200_moe_weights* w, const uint16_t* x_bf16, const float* logits, size_t tokens, float* out,
                      void* workspace, size_t workspace_bytes, unsigned* status, void* stream) {
    return forward_layer(w, x_bf16, false, logits, tokens, out, workspace, workspace_bytes, status, stream);
}

int kb200_moe_forward_f32(const kb200_moe_weights* w, const float* x, const float* logits, size_t tokens, float* out,
                          void* workspace, size_t workspace_bytes, unsigned* status, void* stream) {
    return forward_layer(w, x, true, logits, tokens, out, workspace, workspace_bytes, status, stream);
}

size_t kb200_moe_dispatch_workspace_bytes(size_t tokens, int32_t hidden, int32_t experts, int32_t top_k) {
    if (check_shape(hidden, experts, top_k) != KB200_OK)
        return 0;
    return carve_shape(nullptr, tokens, size_t(hidden), 0, size_t(experts), size_t(top_k), false).bytes;
}

int kb200_moe_dispatch_rows(const float* logits, const uint16_t* x_bf16, size_t tokens, int32_t hidden,
                            int32_t experts, int32_t top_k, void* workspace, size_t workspace_bytes,
                            kb200_moe_dispatch* result, unsigned* status, void* stream) {
    if (const int s = check_shape(hidden, experts, top_k))
        return s;
    if (!result)
        return fail(KB200_INVALID, "null dispatch result");
    if (!tokens) {
        *result = {nullptr, nullptr, nullptr, nullptr, 0};
        return KB200_OK;
    }
    if (!x_bf16 || !logits || !workspace)
        return fail(KB200_INVALID, "null pointer");
    if (!aligned(x_bf16, 16) || !aligned(workspace, 256))
        return fail(KB200_INVALID, "MoE activations must be 16-byte aligned, workspace 256-byte aligned");
    const size_t n = tokens * size_t(top_k);
    if (n > size_t(INT32_MAX) / 4)
        return fail(KB200_UNSUPPORTED, "too many tokens");
    const Workspace ws = carve_shape(workspace, tokens, size_t(hidden), 0, size_t(experts), size_t(top_k), false);
    if (ws.bytes > workspace_bytes)
        return fail(KB200_NO_MEMORY, "dispatch workspace too small (see kb200_moe_dispatch_workspace_bytes)");
    if (const int s = dispatch_launch(logits, x_bf16, tokens, hidden, experts, top_k, ws, status,
                                      static_cast<cudaStream_t>(stream)))
        return s;
    *result = {ws.offsets, ws.pos, ws.weight, reinterpret_cast<uint16_t*>(ws.xs), n};
    return KB200_OK;
}

size_t kb200_moe_experts_workspace_bytes(const kb200_moe_weights* w, size_t rows) {
    if (!w || check_weights(w, false) != KB200_OK)
        return 0;
    return carve_experts(nullptr, *w, rows).bytes;
}

int kb200_moe_experts(const kb200_moe_weights* w, const uint16_t* rows_f16, const int32_t* offsets, size_t rows,
                      float* y, void* workspace, size_t workspace_bytes, unsigned* status, void* stream_ptr) {
    if (const int s = check_weights(w, false))
        return s;
    if (!rows)
        return KB200_OK;
    if (!rows_f16 || !offsets || !y || !workspace)
        return fail(KB200_INVALID, "null pointer");
    if (!aligned(rows_f16, 16) || !aligned(y, 16) || !aligned(workspace, 256))
        return fail(KB200_INVALID, "MoE rows must be 16-byte aligned, workspace 256-byte aligned");
    if (rows > size_t(INT32_MAX) / 4)
        return fail(KB200_UNSUPPORTED, "too many rows");
    const ExpertWs ws = carve_experts(workspace, *w, rows);
    if (ws.bytes > workspace_bytes)
        return fail(KB200_NO_MEMORY, "expert workspace too small (see kb200_moe_experts_workspace_bytes)");
    auto stream = static_cast<cudaStream_t>(stream_ptr);
    cudaError_t e;
    {
        TraceScope trace(KB200_KERNEL_MOE_MTILE, stream);
        moe_mtile_kernel<<<1, 32, 0, stream>>>(offsets, w->experts, ws.mtile);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess)
        return cuda_fail(e, "moe_mtile_kernel launch");
    return experts_launch(w, reinterpret_cast<const __half*>(rows_f16), offsets, ws.mtile, rows, ws.act, y, status,
                          stream);
}

int kb200_silu_mul(const float* gate, const float* up, size_t n, float* out, void* stream) {
    if (!n)
        return KB200_OK;
    if (!gate || !up || !out)
        return fail(KB200_INVALID, "null pointer");
    if ((out != gate && overlap(out, n * 4, gate, n * 4)) || (out != up && overlap(out, n * 4, up, n * 4)))
        return fail(KB200_ALIAS, "output partly overlaps an input");
    const unsigned grid = unsigned(std::min<size_t>((n + 255) / 256, size_t(sm_count()) * 8));
    TraceScope trace(KB200_KERNEL_SILU_MUL, static_cast<cudaStream_t>(stream));
    silu_mul_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(gate, up, n, out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "silu_mul_kernel launch");
}

int kb200_moe_add_shared(const float* x, const float* shared_gate, const float* down, size_t tokens, size_t hidden,
                         float* out, void* stream) {
    if (!tokens)
        return KB200_OK;
    if (!x || !shared_gate || !down || !out || !hidden)
        return fail(KB200_INVALID, "null pointer or zero width");
    if (hidden > (1u << 30) || tokens > 0x7FFFFFFFu)
        return fail(KB200_UNSUPPORTED, "shape");
    const size_t bytes = tokens * hidden * 4;
    if (overlap(out, bytes, x, bytes) || overlap(out, bytes, down, bytes) || overlap(out, bytes, shared_gate, hidden * 4))
        return fail(KB200_ALIAS, "output overlaps an input");
    TraceScope trace(KB200_KERNEL_MOE_SHARED, static_cast<cudaStream_t>(stream));
    moe_shared_kernel<<<unsigned(tokens), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, shared_gate, down,
                                                                                       int(hidden), out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "moe_shared_kernel launch");
}

int kb200_moe_combine(const float* y, const float* weight, const int32_t* pos, size_t tokens, int32_t top_k,
                      int32_t hidden, float* out, void* stream) {
    if (top_k <= 0 || top_k > kMaxTopK || hidden <= 0 || hidden % 4)
        return fail(KB200_UNSUPPORTED, "combine shape");
    if (!tokens)
        return KB200_OK;
    if (!y || !weight || !pos || !out)
        return fail(KB200_INVALID, "null pointer");
    if (!aligned(y, 16) || !aligned(out, 16))
        return fail(KB200_INVALID, "combine rows must be 16-byte aligned");
    return combine_launch(y, weight, pos, tokens, top_k, hidden, out, static_cast<cudaStream_t>(stream));
}

int kb200_rows_regroup(const void* src, void* dst, size_t row_bytes, const int64_t* segments, size_t count,
                       size_t max_rows, void* stream) {
    if (!count)
        return KB200_OK;
    if (!src || !dst || !segments)
        return fail(KB200_INVALID, "null pointer");
    if (row_bytes % 16 || !aligned(src, 16) || !aligned(dst, 16) || !aligned(segments, 8))
        return fail(KB200_INVALID, "rows must be whole 16-byte words and 16-byte aligned");
    if (count > 65535)
        return fail(KB200_UNSUPPORTED, "at most 65535 segments");
    const size_t words = std::max<size_t>(1, max_rows) * (row_bytes / 16);
    const dim3 grid(unsigned(std::min<size_t>((words + 255) / 256, 64)), unsigned(count));
    TraceScope trace(KB200_KERNEL_ROWS_REGROUP, static_cast<cudaStream_t>(stream));
    rows_regroup_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), row_bytes / 16,
        reinterpret_cast<const long long*>(segments));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "rows_regroup_kernel launch");
}

// For callers that cannot allocate device memory per call (workers whose
// device memory is admitted to a ledger in advance, callers that must not let
// an allocation synchronise the device): the same layer on the library's
// fixed scratch.
// Allocates nothing; only the counts it must clear are reset (by the
// asynchronous memset inside kb200_moe_forward), everything else it reads is
// first written by the same call.
int kb200_moe_forward_noalloc(const kb200_moe_weights* w, const uint16_t* x_bf16, const float* logits, size_t tokens,
                              float* out, unsigned* status, void* stream) {
    if (const int s = check_weights(w))
        return s;
    if (!tokens)
        return KB200_OK;
    const size_t need = carve(nullptr, *w, tokens).bytes;
    if (need > KB200_MOE_STATIC_SCRATCH_BYTES)
        return fail(KB200_NO_MEMORY, "tokens need more than the 16 MiB static MoE scratch of kb200_moe_forward_noalloc");
    void* scratch = nullptr;
    if (const int s = static_scratch(&scratch))
        return s;
    return kb200_moe_forward(w, x_bf16, logits, tokens, out, scratch, KB200_MOE_STATIC_SCRATCH_BYTES, status, stream);
}

}  // extern "C"
