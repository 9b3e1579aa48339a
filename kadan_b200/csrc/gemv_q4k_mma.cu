// Q4_K decode GEMV on the tensor pipe (sm_100a), T <= 8 input rows per pass.
//
// Replaces gguf_matvec_batch_kernel<q4_k>
// (services/hikari/inference_worker/src/cuda/h3_compute.cu:165-257) for
// 16-byte aligned rows. The reference decodes every weight to fp32 on the
// CUDA cores, several instructions per weight; at HBM speed that is more work
// than an SM can issue. Here the products run on the integer tensor pipe:
//
//   Q4_K value :  w = d*sc_g*q - dmin*m_g   (q 4-bit, sc_g/m_g 6-bit per 32)
//   A operand  :  low nibbles  q      = packed & 0x0F0F0F0F  (u8, 0..15)
//                 high nibbles 16*q   = packed & 0xF0F0F0F0  (u8, 0..240)
//   B operand  :  the activations of one super-block, quantised to two int8
//                 levels, x ~= s*(h + l/254) with s = absmax/127 per 256
//                 values and token (about 15 bits); h and l sit in adjacent
//                 N columns, 4 input rows x {h, l} = 8 columns per MMA
//   MMA        :  mma.m16n8k32.u8.s8 -> exact int32 sum over one sub-block
//   scales     :  I = sum_g (16 sc_g) C_g(low) + sc_g C_g(high)   (IMAD)
//   min term   :  sum_g m_g * sum_{k in g} x_k, one fp16 m16n8k8 MMA per block
//                 (m exact, the fp32 group sums split into fp16 hi + lo)
//   epilogue   :  acc += (d*s/16) * (I_h + I_l/254) - (256 dmin) * C_min
//
// CTA = 4 consumer warps + 1 producer lane. A tile is R weight rows (R = 64,
// 32 or 16) for one group of input rows; with R < 64 the warps split K (2 or 4
// ways) and reduce in shared memory at the end. The producer streams each
// stage (R rows x 128/R super-blocks, 18 KB) with one 3-D TMA tile load per
// super-block column into a 3-stage ring, optionally running an L2 prefetch
// of the same boxes a few stages ahead; a 144-byte row pitch keeps every
// fragment load free of bank conflicts. The activations of a K segment (all
// of K at decode shapes) are quantised once per CTA and input, so consumer
// warps run without any barrier between them: wait for a stage, issue its
// MMAs, release it.
//
// Work split (balanced, "stream-K"): the launch's work is the sequence of
// units (tile, super-block), tiles of all jobs in order, K innermost. CTA c of
// G takes units [c*U/G, (c+1)*U/G), so every CTA streams the same number of
// bytes and no CTA is left with a second wave (tiles are 64 rows). A tile cut
// by CTA boundaries is computed in pieces. The CTA holding its first unit
// reaches it last (it is that CTA's final piece) and writes the outputs; every
// other piece is the first piece of a later CTA ("head piece"), done early:
// its consumers store each partial sum with a "present" tag as one 64-bit
// word (single-copy atomic, so no fence or flag is needed) in the CTA's slot
// of a fixup buffer. The first CTA's consumers, at the end of their own
// piece, read those words (re-reading any whose tag is not there yet), add
// them in CTA order, so the sum does not depend on timing, and zero them for
// the next launch. Without a fixup buffer (first use of a stream inside graph
// capture) the launch falls back to whole tiles dealt round-robin.
//
// Launched with programmatic dependent launch: the producer starts streaming
// weights while the previous kernel in the stream is still finishing; the
// consumers wait (griddepcontrol.wait) before they read activations or write
// outputs. Weights must therefore not be produced by the immediately
// preceding kernel of the stream.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <map>
#include <mutex>
#include <vector>

#include "gemv_mma.hpp"
#include "gguf_formats.cuh"
#include "kb200_device.cuh"
#include "kb200_host.hpp"

namespace kb200 {
namespace {

constexpr int kWarps = 4;
constexpr int kConsumerThreads = 32 * kWarps;
constexpr int kThreadsQ = kConsumerThreads + 32;
constexpr int kBlockBytes = 144;
constexpr int kStageUnits = 128;  // rows x super-blocks per stage
constexpr int kStages = 3;
constexpr int kStageBytes = kStageUnits * kBlockBytes;  // 18432
constexpr int kMaxJobsQ = 32;

struct alignas(64) MmaJob {
    CUtensorMap map;  // dims {18 x u64, blocks, rows}, box {18, 1, R}
    const float* input;
    float* output;
    unsigned* status;
    const uint8_t* staged;  // Q6_K pair kernel: quantised activations, chunk after chunk (or null)
    uint32_t stride, in, columns, rows;
    uint32_t first_tile, first_unit;  // prefix of tiles / of tiles x nblocks
    uint32_t row_groups, group_rows, nblocks;
};

// Partial sums of one piece: acc[NT <= 2][2] of each consumer thread, for
// up to 256 consumer threads (the 8-row Q6_K pair kernel's eight warps).
constexpr int kSlotFloats = 2 * 2 * 256;
// Fewest 64-row x 1 super-block units per CTA for which the balanced split
// pays for its fixup (a round trip to L2 at the end of each cut tile).
constexpr int kMinUnitsPerCta = 6;

struct MmaParams {
    MmaJob jobs[kMaxJobsQ];
    uint32_t count, total_tiles;
    uint32_t tile_rows;    // R: 64, 32 or 16
    uint32_t total_units;  // balanced split over units; 0 = whole tiles round-robin
    uint32_t prefetch;     // L2 prefetch distance in stages (0 = off)
    // [gridDim.x][kSlotFloats] head-piece partial sums as {fp32 bits, 1}
    // words; zero between launches.
    unsigned long long* partials;
    unsigned* watchdog;
    // Tensor-parallel exchange (world > 1): the outputs of the launch's one
    // job also go to slot [rank] of every peer's buffer, as words tagged
    // with the group's next call number.
    PeerOut peer;
};

// One output value into slot [rank] of every peer: 64-bit {call, value}
// words, which the gather kernel of the same call reads and adds.
__device__ __forceinline__ void push_peers(const PeerOut& g, uint32_t call, size_t index, float v) {
    const unsigned long long w = (unsigned long long)call << 32 | __float_as_uint(v);
    const size_t slot = (size_t(call & 1u) * kPeerMaxRanks + g.rank) * g.max_count + index;
    for (int q = 0; q < g.world; ++q)
        if (q != g.rank) {
            unsigned long long* at = reinterpret_cast<unsigned long long*>(g.peers[q] + kPeerWordsOff) + slot;
            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(at), "l"(w) : "memory");
        }
}

// Relaxed 64-bit global accesses: single-copy atomic, so a partial sum and
// its "present" tag, stored as one word, are seen together or not at all.
__device__ __forceinline__ void store_relaxed(unsigned long long* at, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(at), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long load_relaxed(const unsigned long long* at) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(at) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long tagged(float v) {
    return (1ull << 32) | __float_as_uint(v);
}

// A contiguous run of one tile's super-blocks [k0, k1) taken by this CTA.
struct Piece {
    int job;
    uint32_t tile;            // tile within the job: column tile * row_groups + row group
    uint32_t k0, k1;
    bool whole;               // k0 == 0 && k1 == nblocks
    uint32_t c_first, c_last; // CTAs holding the tile's first / last unit (cut tiles)
};

__device__ __forceinline__ uint32_t range_begin(uint32_t total_units, uint32_t cta) {
    return uint32_t(uint64_t(cta) * total_units / gridDim.x);
}

// CTA whose unit range holds unit x (every range is non-empty: G <= U).
__device__ __forceinline__ uint32_t cta_of(uint32_t total_units, uint32_t x) {
    return uint32_t((uint64_t(x + 1) * gridDim.x - 1) / total_units);
}

// Activation segment: per super-block and token, the quantised h/l operands
// in B-fragment order ([j][t][part][4 words], 512 bytes), the minimum-term B
// operands ([part][t] fp16x2, 32 bytes) and the scale s (4 bytes).
constexpr int kTokenBlockBytes = 512;
constexpr int kMinBytes = 32;
constexpr int kTokenBlockTotal = kTokenBlockBytes + kMinBytes + 4;
constexpr int kSegBudget = 16 * 1024;

// One (block, token set) record of the staged Q4_K activations: the rows'
// operands, minimum-term operands and scales, padded to 16 bytes.
__host__ __device__ constexpr int q4k_record_bytes(int rows) {
    return (rows * kTokenBlockTotal + 15) / 16 * 16;
}

// kStaged: a stage (64 rows x 2 super-blocks) also holds the activation
// records of its super-blocks for up to 4 NT tokens, copied from the launch's
// staging buffer, and there is no activation segment. Staged 8-row passes
// keep two stages, so that three CTAs still fit an SM.
template <bool kStaged = false, int NT = 1> struct LayoutQ4 {
    static constexpr int kStages = kStaged && NT == 2 ? 2 : ::kb200::kStages;
    // A stage starts on a 128-byte boundary (the TMA tile destinations).
    static constexpr int kStride =
        kStaged ? (kStageBytes + 2 * q4k_record_bytes(4 * NT) + 127) / 128 * 128 : kStageBytes;
    static constexpr int kStagesOff = 0;
    static constexpr int kSegOff = kStages * kStride;
    static constexpr int kRedOff = kSegOff + (kStaged ? 0 : kSegBudget);  // split-K partials
    static constexpr int kRedBytes = kConsumerThreads * 4 * 4;  // [nt<=2][2][thread]
    static constexpr int kBarOff = kRedOff + kRedBytes;  // full[], empty[], abort flag
    static constexpr int kTotal = kBarOff + 2 * kStages * 8 + 16;
};
using Layout = LayoutQ4<false>;
static_assert(kStageBytes % 128 == 0 && LayoutQ4<true>::kStride % 128 == 0 && LayoutQ4<true, 2>::kStride % 128 == 0,
              "tensor copies land on 128-byte boundaries");
static_assert(3 * (LayoutQ4<true>::kTotal + 128 + 1024) <= 228 * 1024, "three staged Q4_K CTAs per SM");
static_assert(3 * (LayoutQ4<true, 2>::kTotal + 128 + 1024) <= 228 * 1024, "three staged 8-row Q4_K CTAs per SM");

// Segment of `rows` tokens: the most whole stages (multiples of `bps`
// super-blocks) that fit kSegBudget; operands first, then minimum-term
// operands, then scales. blocks == 0 means not even one stage fits (the host
// never launches such a geometry).
__host__ __device__ constexpr int segment_blocks(int rows, int bps, int budget = kSegBudget) {
    return budget / (rows * kTokenBlockTotal) / bps * bps;
}

// off: byte offset of the segment buffer in the kernel's shared memory.
struct Segment {
    int blocks, rows, off;
    __device__ Segment(int r, int bps, int budget = kSegBudget, int offset = Layout::kSegOff)
        : blocks(segment_blocks(r, bps, budget)), rows(r), off(offset) {}
    __device__ uint8_t* frag(uint8_t* smem) const { return smem + off; }
    __device__ uint32_t* minb(uint8_t* smem) const {
        return reinterpret_cast<uint32_t*>(smem + off + blocks * rows * kTokenBlockBytes);
    }
    __device__ float* scales(uint8_t* smem) const {
        return reinterpret_cast<float*>(minb(smem) + blocks * rows * (kMinBytes / 4));
    }
};

// Last job whose first tile (units = false) or first unit (units = true) is <= at.
__device__ __forceinline__ int find_job(const MmaParams& p, uint32_t at, bool units) {
    int low = 0, high = int(p.count);
    while (high - low > 1) {
        const int mid = (low + high) / 2;
        if ((units ? p.jobs[mid].first_unit : p.jobs[mid].first_tile) <= at)
            low = mid;
        else
            high = mid;
    }
    return low;
}

// The pieces of this CTA in order. Producer, prefetcher and consumers each
// walk their own copy and see the same sequence.
struct PieceIter {
    uint32_t cur, end;

    __device__ explicit PieceIter(const MmaParams& p) {
        if (p.total_units) {
            cur = range_begin(p.total_units, blockIdx.x);
            end = range_begin(p.total_units, blockIdx.x + 1);
        } else {
            cur = blockIdx.x;
            end = p.total_tiles;
        }
    }

    __device__ bool next(const MmaParams& p, Piece& pc) {
        if (cur >= end)
            return false;
        if (!p.total_units) {
            pc.job = find_job(p, cur, false);
            pc.tile = cur - p.jobs[pc.job].first_tile;
            pc.k0 = 0;
            pc.k1 = p.jobs[pc.job].nblocks;
            pc.whole = true;
            cur += gridDim.x;
            return true;
        }
        pc.job = find_job(p, cur, true);
        const MmaJob& job = p.jobs[pc.job];
        const uint32_t local = cur - job.first_unit, nb = job.nblocks;
        pc.tile = local / nb;
        pc.k0 = local % nb;
        pc.k1 = min(nb, pc.k0 + (end - cur));
        pc.whole = pc.k0 == 0 && pc.k1 == nb;
        if (!pc.whole) {
            const uint32_t x0 = cur - pc.k0;
            pc.c_first = cta_of(p.total_units, x0);
            pc.c_last = cta_of(p.total_units, x0 + nb - 1);
        }
        cur += pc.k1 - pc.k0;
        return true;
    }
};

__device__ __forceinline__ void prefetch_l2_3d(const CUtensorMap* map, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(map), "r"(c0), "r"(c1), "r"(c2)
        : "memory"
    );
}

// L2 prefetch cursor: walks the producer's stage sequence ahead of it.
struct Prefetcher {
    PieceIter pieces;
    Piece pc;
    uint32_t b0 = 0;
    bool live = false;

    __device__ explicit Prefetcher(const MmaParams& p) : pieces(p) {}

    // Prefetch the next stage (BPS super-blocks of R rows) into L2.
    __device__ void step(const MmaParams& p, int R, int BPS) {
        if (!live || b0 >= pc.k1) {
            if (!pieces.next(p, pc))
                return;
            live = true;
            b0 = pc.k0;
        }
        const MmaJob& job = p.jobs[pc.job];
        const int row0 = int((pc.tile / job.row_groups) * uint32_t(R));
        const uint32_t stop = min(pc.k1, b0 + uint32_t(BPS));
        for (uint32_t b = b0; b < stop; ++b)
            prefetch_l2_3d(&job.map, 0, int(b), row0);
        b0 = stop;
    }
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

__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// C = A(16x32 u8) * B(32x8 s8), exact int32.
__device__ __forceinline__ void imma(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0)
    );
}

__device__ __forceinline__ void mma1688(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(b0)
    );
}

__device__ __forceinline__ uint32_t pack_half2(__half2 h) {
    return *reinterpret_cast<uint32_t*>(&h);
}

// 1.5 * 2^23: for |y| < 2^22, the low mantissa bits of y + kMagic hold
// round-to-nearest-even(y) as a two's-complement integer.
constexpr float kMagic = 12582912.f;

__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)));
    return *reinterpret_cast<float2*>(&d);
}

__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    return add2(a, make_float2(-b.x, -b.y));
}

__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)));
    return *reinterpret_cast<float2*>(&d);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return __byte_perm(__byte_perm(uint32_t(a), uint32_t(b), 0x0040u), __byte_perm(uint32_t(c), uint32_t(d), 0x0040u), 0x5410u);
}

__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void grid_dependents_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Values 8 lane .. 8 lane + 7 of 256 at xr (16-byte vectors when `vec`).
__device__ __forceinline__ void load_lane8(float (&v)[8], const float* xr, bool vec) {
    if (vec) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(xr)), b = __ldg(reinterpret_cast<const float4*>(xr) + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
        v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            v[i] = __ldg(xr + i);
    }
}

// The two int8 levels of 8 values with absmax m: pairs of values at a time,
// y = v/s, r1 = y + M (M = 1.5 * 2^23, so r1's low bits are round(y) as an
// integer), d = y - round(y) in [-1/2, 1/2] (exact), r2 = d * 254 + M (low
// bits round(254 d), within [-127, 127]). The int8 codes are the low bytes
// of h (r1) and l (r2).
__device__ __forceinline__ void quantise_levels(const float (&v)[8], float m, uint32_t (&h)[8], uint32_t (&l)[8]) {
    const float inv = m > 0.f ? 127.f / m : 0.f;
    const float2 inv2 = make_float2(inv, inv), magic = make_float2(kMagic, kMagic);
    const float2 neg_magic = make_float2(-kMagic, -kMagic), k254 = make_float2(254.f, 254.f);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const float2 y = mul2(make_float2(v[i], v[i + 1]), inv2);
        const float2 r1 = add2(y, magic);
        const float2 d = sub2(y, add2(r1, neg_magic));
        const float2 r2 = fma2(d, k254, magic);
        h[i] = __float_as_uint(r1.x), h[i + 1] = __float_as_uint(r1.y);
        l[i] = __float_as_uint(r2.x), l[i + 1] = __float_as_uint(r2.y);
    }
}

// One (block, token) item of the Q4_K activation operands: lane L holds
// values 8L..8L+7 (v), m is the block's absmax, sum the sum of the lane's
// sub-block G = L/4 and next that of G ^ 1. Writes the lane's B words of the
// 512-byte record frag, (lanes 8t') the minimum-term operands of the 32-byte
// record minb and (lane 0) the scale.
__device__ __forceinline__ void q4k_store_item(const float (&v)[8], float m, float sum, float next, uint32_t* frag,
                                               uint32_t* minb, float* scale, int lane) {
    const int G = lane >> 2, t = lane & 3;
    uint32_t h[8], l[8];
    quantise_levels(v, m, h, l);
    const int idx = (((G >> 1) * 4 + t) * 2) * 4 + (G & 1) * 2;  // part h; part l is +4
    frag[idx] = pack4(int(h[0]), int(h[1]), int(h[2]), int(h[3]));
    frag[idx + 1] = pack4(int(h[4]), int(h[5]), int(h[6]), int(h[7]));
    frag[idx + 4] = pack4(int(l[0]), int(l[1]), int(l[2]), int(l[3]));
    frag[idx + 5] = pack4(int(l[4]), int(l[5]), int(l[6]), int(l[7]));
    // Minimum term B' for lane (g, t') = sums of sub-blocks 2t', 2t'+1
    // (scaled by 1/256) split into fp16 hi and lo: written by lanes 8t'.
    if ((lane & 7) == 0) {
        const float s0 = sum * (1.f / 256.f), s1 = next * (1.f / 256.f);
        const __half2 hi = __floats2half2_rn(s0, s1);
        const float2 hf = __half22float2(hi);
        const __half2 lo = __floats2half2_rn(s0 - hf.x, s1 - hf.y);
        minb[lane >> 3] = pack_half2(hi);
        minb[4 + (lane >> 3)] = pack_half2(lo);
    }
    if (lane == 0)
        *scale = m > 0.f ? m / 127.f : 0.f;
}

// Absmax, own sub-block sum and the neighbouring sub-block's sum of a
// warp's 256 values (lane L: values 8L..8L+7).
__device__ __forceinline__ void q4k_block_stats(const float (&v)[8], float& m, float& sum, float& next) {
    m = 0.f, sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        m = fmaxf(m, fabsf(v[i]));
        sum += v[i];
    }
    // Non-negative floats order as their bit patterns.
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    next = __shfl_xor_sync(0xffffffffu, sum, 4);  // sum of sub-block G ^ 1
}

// Quantise the activations of super-blocks [blk0, blk0 + nblk) for the
// segment's tokens. One warp per (block, token): lane L owns values
// 8L..8L+7, which are the B registers b0 (k = 4t..4t+3 <-> values 8t..8t+3)
// and b1 (k = 16+4t.. <-> values 8t+4..8t+7) of sub-block G = L/4, t = L%4.
//
// kQ6: the Q6_K kernel's operand order instead (m16n8k16, sub-blocks of 16):
// words [block][sub-block s][token][h, l][t'] with t' = values 4t'..4t'+3 of
// the sub-block, and no minimum-term operands.
template <bool kQ6 = false>
__device__ void prep_segment(uint8_t* smem, const Segment& seg, const float* x, size_t in, int blk0, int nblk) {
    const int rows = seg.rows;
    auto* frag = reinterpret_cast<uint32_t*>(seg.frag(smem));
    uint32_t* minb = seg.minb(smem);
    float* scales = seg.scales(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (in & 3) == 0;
    const int items = nblk * rows;
    // kBatch items per warp at a time, without branches between them: all
    // their loads are in flight before the first is used (the activations
    // come from L2, a microsecond away under full HBM load) and the four
    // reduction chains interleave.
    constexpr int kBatch = 4;
    for (int base = warp; base < items; base += kWarps * kBatch) {
        float v[kBatch][8];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int item = min(base + q * kWarps, items - 1);  // past the end: reload the last, store nothing
            const int blk = item / rows, tok = item % rows;
            load_lane8(v[q], x + size_t(tok) * in + size_t(blk0 + blk) * 256 + lane * 8, vec);
        }
        float m[kBatch], sum[kBatch], next[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
            q4k_block_stats(v[q], m[q], sum[q], next[q]);
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int item = base + q * kWarps;
            if (item >= items)
                break;
            const int blk = item / rows, tok = item % rows;
            const int slot = blk * rows + tok;
            if constexpr (kQ6) {
                uint32_t h[8], l[8];
                quantise_levels(v[q], m[q], h, l);
                // Lane L: values 8L..8L+7 = words 2(L&1), 2(L&1)+1 of sub-block L/2.
                uint32_t* dst = frag + blk * rows * (kTokenBlockBytes / 4);
                const int idx = (((lane >> 1) * rows + tok) * 2) * 4 + 2 * (lane & 1);
                dst[idx] = pack4(int(h[0]), int(h[1]), int(h[2]), int(h[3]));
                dst[idx + 1] = pack4(int(h[4]), int(h[5]), int(h[6]), int(h[7]));
                dst[idx + 4] = pack4(int(l[0]), int(l[1]), int(l[2]), int(l[3]));
                dst[idx + 5] = pack4(int(l[4]), int(l[5]), int(l[6]), int(l[7]));
                if (lane == 0)
                    scales[slot] = m[q] > 0.f ? m[q] / 127.f : 0.f;
            } else {
                q4k_store_item(v[q], m[q], sum[q], next[q], frag + slot * (kTokenBlockBytes / 4),
                               minb + slot * (kMinBytes / 4), scales + slot, lane);
            }
        }
    }
}

// End of a piece, common to the K-quant kernels: sum the K-split warps of
// each row group, then either publish the partial sums (head piece of a cut
// tile), add the later pieces' sums in CTA order (tail piece), or write the
// outputs (whole tile or tail piece). acc[nt][0/1]: rows my_row, my_row + 8
// for token nt*4 + t.
template <int NT, class Await, int CT = kConsumerThreads>
__device__ __forceinline__ void finish_piece(const MmaParams& p, const Piece& pc, const MmaJob& job, float (&acc)[NT][2],
                                             int KS, int ks, int tid, uint32_t my_row, bool valid_lo, bool valid_hi,
                                             uint32_t r0, int rows, float* red, int* abort_flag, Await& await_dependency) {
    static_assert(2 * NT * CT <= kSlotFloats, "a fixup slot holds every consumer thread's partial sums");
    const int warp = tid >> 5, lane = tid & 31, t = lane & 3;
    if (KS > 1) {
        // Sum the K splits of each row group: warp (rg, 0) collects.
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            red[(nt * 2 + 0) * CT + tid] = acc[nt][0];
            red[(nt * 2 + 1) * CT + tid] = acc[nt][1];
        }
        named_sync(1, CT);
        if (ks == 0) {
            for (int k = 1; k < KS; ++k) {
                const int other = (warp + k) * 32 + lane;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    acc[nt][0] += red[(nt * 2 + 0) * CT + other];
                    acc[nt][1] += red[(nt * 2 + 1) * CT + other];
                }
            }
        }
        named_sync(1, CT);
    }
    await_dependency();
    bool write = ks == 0;
    if (!pc.whole && pc.k0 > 0) {
        // Head piece of a cut tile (R = 64, every warp holds final sums):
        // store the partial sums; the fixup lanes publish them.
        // store the tagged partial sums (the slot was zeroed by the previous
        // launch, which finished before the grid-dependency wait).
        unsigned long long* mine = p.partials + size_t(blockIdx.x) * kSlotFloats;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            store_relaxed(mine + (nt * 2 + 0) * CT + tid, tagged(acc[nt][0]));
            store_relaxed(mine + (nt * 2 + 1) * CT + tid, tagged(acc[nt][1]));
        }
        write = false;
    } else if (!pc.whole) {
        // Tail piece holding the tile's first unit: add the later pieces'
        // sums in CTA order as their tags appear, and zero the words for
        // the next launch on this stream.
        constexpr int kAhead = 4;  // CTAs whose words are in flight together
        const uint32_t others = pc.c_last - pc.c_first;
        for (uint32_t c0 = 0; c0 < others; c0 += kAhead) {
            unsigned long long w[kAhead][NT][2];
#pragma unroll
            for (int q = 0; q < kAhead; ++q) {
                const uint32_t c = pc.c_first + 1 + min(c0 + q, others - 1);
                const unsigned long long* part = p.partials + size_t(c) * kSlotFloats;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    w[q][nt][0] = load_relaxed(part + (nt * 2 + 0) * CT + tid);
                    w[q][nt][1] = load_relaxed(part + (nt * 2 + 1) * CT + tid);
                }
            }
#pragma unroll
            for (int q = 0; q < kAhead; ++q) {
                if (c0 + q >= others)
                    break;
                unsigned long long* part = p.partials + size_t(pc.c_first + 1 + c0 + q) * kSlotFloats;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                    for (int hl = 0; hl < 2; ++hl) {
                        unsigned long long* at = part + (nt * 2 + hl) * CT + tid;
                        unsigned long long v = w[q][nt][hl];
                        for (uint32_t poll = 0; (v >> 32) != 1ull; ++poll) {
                            if (poll == wait_polls) {
                                atomicOr(p.watchdog, watchdog_fixup);
                                atomicExch(abort_flag, 1);
                                break;
                            }
                            __nanosleep(32);
                            v = load_relaxed(at);
                        }
                        acc[nt][hl] += __uint_as_float(uint32_t(v));
                        store_relaxed(at, 0ull);
                    }
                }
            }
        }
    }
    if (write) {
        // The group's call number: the gather kernels of earlier calls have
        // finished (grid-dependency wait above), and each advanced the counters.
        const bool push = p.peer.world > 1;
        const uint32_t call = push ? reinterpret_cast<const uint32_t*>(p.peer.peers[p.peer.rank])[0] + 1u : 0u;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int tok = nt * 4 + t;
            if (tok < rows) {
                const size_t row = size_t(r0 + tok) * job.stride;
                float* out = job.output + row;
                if (valid_lo) {
                    out[my_row] = acc[nt][0];
                    if (push)
                        push_peers(p.peer, call, row + my_row, acc[nt][0]);
                }
                if (valid_hi) {
                    out[my_row + 8] = acc[nt][1];
                    if (push)
                        push_peers(p.peer, call, row + my_row + 8, acc[nt][1]);
                }
            }
        }
    }
}

// kStaged (64-row tiles, one row group of at most 8 input rows): the activations come
// quantised from the launch's staging buffer (q4k_quant_kernel, launched just
// before), one record per super-block copied with the stage's weights; the
// producer issues the first stages' weight loads before it waits for the
// quantisation kernel. Otherwise the consumers quantise activation segments.
template <int NT, bool kStaged = false>
__global__ void __launch_bounds__(kThreadsQ, 3) gemv_q4k_mma_kernel(const __grid_constant__ MmaParams p) {
    using L = LayoutQ4<kStaged, NT>;
    constexpr int kStages = L::kStages;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // TMA destinations (no swizzle) want 128-byte alignment.
    uint8_t* smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
    auto* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
    auto* empty = full + kStages;
    auto* abort_flag = reinterpret_cast<int*>(empty + kStages);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int R = int(p.tile_rows), KS = 64 / R, BPS = kStageUnits / R;
    auto* red = reinterpret_cast<float*>(smem + L::kRedOff);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        *abort_flag = 0;
        fence_barrier_init();
        // The next kernel of the stream may start its own weight streaming.
        grid_dependents_launch();
    }
    __syncthreads();

    if (warp == kWarps) {
        // ------------------------------ producer ------------------------------
        if (lane != 0)
            return;
        uint32_t it = 0;
        // Staged: activation copies of the first stages, held back until the
        // quantisation kernel has finished.
        bool staged_ready = false;
        const uint8_t* held_src[kStages];
        uint32_t held_bytes[kStages];
        uint32_t held = 0;
        auto release_held = [&] {
            grid_dependency_wait();
            asm volatile("fence.proxy.async.global;" ::: "memory");
            staged_ready = true;
            for (uint32_t k = 0; k < held; ++k)
                bulk_g2s(smem + L::kStagesOff + k * L::kStride + kStageBytes, held_src[k], held_bytes[k], &full[k]);
            held = 0;
        };
        PieceIter pieces(p);
        Prefetcher ahead(p);
        for (uint32_t i = 0; i < p.prefetch; ++i)
            ahead.step(p, R, BPS);
        Piece pc;
        while (pieces.next(p, pc)) {
            const MmaJob& job = p.jobs[pc.job];
            const int row0 = int((pc.tile / job.row_groups) * uint32_t(R));
            const uint32_t record = kStaged ? uint32_t(q4k_record_bytes(int(job.rows))) : 0u;
            asm volatile("prefetch.tensormap [%0];" ::"l"(&job.map) : "memory");
            for (uint32_t b0 = pc.k0; b0 < pc.k1; b0 += BPS, ++it) {
                const int slot = int(it % kStages);
                if (it >= kStages && !mbar_wait(&empty[slot], ((it / kStages) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog))
                    atomicExch(abort_flag, 1);
                if (*reinterpret_cast<volatile int*>(abort_flag))
                    goto drain;
                const int nb = int(min(uint32_t(BPS), pc.k1 - b0));
                uint8_t* stage = smem + L::kStagesOff + slot * L::kStride;
                mbar_expect_tx(&full[slot], uint32_t(nb * R * kBlockBytes) + uint32_t(nb) * record);
                for (int b = 0; b < nb; ++b)
                    tma_load_3d(stage + b * R * kBlockBytes, &job.map, 0, int(b0 + b), row0, &full[slot]);
                if constexpr (kStaged) {
                    const uint8_t* src = job.staged + size_t(b0) * record;
                    if (staged_ready) {
                        bulk_g2s(stage + kStageBytes, src, uint32_t(nb) * record, &full[slot]);
                    } else {
                        held_src[held] = src, held_bytes[held] = uint32_t(nb) * record;
                        if (++held == uint32_t(kStages))
                            release_held();
                    }
                }
                if (p.prefetch)
                    ahead.step(p, R, BPS);
            }
        }
        if constexpr (kStaged)
            if (!staged_ready)
                release_held();
    drain:
        for (uint32_t k = 0; k < kStages && k < it; ++k) {
            const uint32_t last = it - 1 - k;
            mbar_wait(&full[last % kStages], (last / kStages) & 1u, watchdog_drain, p.watchdog);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    // Activations, outputs and the fixup words may belong to the previous
    // kernel of the stream: the grid-dependency wait comes right before the
    // first of those accesses, so walking the job table (constant-cache misses
    // at kernel start) overlaps the previous kernel's tail.
    bool dependency_met = false;
    auto await_dependency = [&] {
        if (!dependency_met) {
            grid_dependency_wait();
            dependency_met = true;
        }
    };
    const int g = lane >> 2, t = lane & 3;
    const int rg = warp / KS, ks = warp % KS;  // row group and K split of this warp
    uint32_t it = 0;
    // (input, rows, first block, blocks) of the activation segment held in shared memory.
    const float* seg_x = nullptr;
    int seg_rows = -1, seg_blk0 = -1, seg_nblk = 0;
    PieceIter pieces(p);
    Piece pc;
    while (pieces.next(p, pc)) {
        const MmaJob& job = p.jobs[pc.job];
        const uint32_t row0 = (pc.tile / job.row_groups) * uint32_t(R);
        const uint32_t r0 = (pc.tile % job.row_groups) * job.group_rows;
        const int rows = int(min(job.group_rows, job.rows - r0));
        const float* x = job.input + size_t(r0) * job.in;
        const Segment seg(rows, BPS);
        if (!kStaged && seg.blocks < BPS)  // a stage's activations would overflow the segment buffer
            atomicExch(abort_flag, 1);
        const int record = q4k_record_bytes(rows);
        const uint32_t my_row = row0 + 16 * rg + g;  // and my_row + 8
        const bool valid_lo = my_row < job.columns, valid_hi = my_row + 8 < job.columns;
        const bool check = job.status != nullptr;
        bool finite = true;
        float acc[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            acc[nt][0] = acc[nt][1] = 0.f;

        for (uint32_t b0 = pc.k0; b0 < pc.k1; b0 += BPS, ++it) {
            const int slot = int(it % kStages);
            const int nb = int(min(uint32_t(BPS), pc.k1 - b0));
            const int blk_first = int(b0);
            if (!kStaged
                && (x != seg_x || rows != seg_rows || blk_first < seg_blk0 || blk_first + nb > seg_blk0 + seg_nblk)
                && seg.blocks >= BPS) {
                // The window covers all of K when the segment buffer holds
                // it (one quantisation per input however the work is cut),
                // else this stage and what follows, as far as it reaches.
                // The CTA's last piece needs only its own blocks (small
                // launches: a piece of a few units would otherwise quantise
                // all of K).
                const int nbk = int(job.nblocks);
                const bool last = pieces.cur >= pieces.end;
                const int start = last || nbk > seg.blocks ? blk_first : 0;
                const int count = min(seg.blocks, (last ? int(pc.k1) : nbk) - start);
                await_dependency();
                // Every warp is done with the previous segment before it is replaced.
                named_sync(1, kConsumerThreads);
                prep_segment(smem, seg, x, job.in, start, count);
                named_sync(1, kConsumerThreads);
                seg_x = x, seg_rows = rows, seg_blk0 = start, seg_nblk = count;
            }
            const bool aborted = *reinterpret_cast<volatile int*>(abort_flag) != 0;
            if (!aborted && !mbar_wait(&full[slot], (it / kStages) & 1u, watchdog_full_barrier, p.watchdog))
                atomicExch(abort_flag, 1);
            if (!aborted) {
                const uint8_t* stage = smem + L::kStagesOff + slot * L::kStride;
#pragma unroll
                for (int bb = 0; bb < 2; ++bb) {
                    const int b = 2 * ks + bb;  // this warp's super-blocks of the stage
                    if (b >= nb)
                        break;
                    // Activation operands of (block, token): the stage's record of
                    // block b (staged) or the segment's arrays.
                    const int sblk = kStaged ? 0 : blk_first + b - seg_blk0;  // block index within the segment
                    const uint8_t* rec = stage + kStageBytes + b * record;
                    const uint8_t* frag = kStaged ? rec : seg.frag(smem);
                    const uint32_t* minb = kStaged ? reinterpret_cast<const uint32_t*>(rec + rows * kTokenBlockBytes)
                                                   : seg.minb(smem);
                    const float* scales = kStaged ? reinterpret_cast<const float*>(rec + rows * (kTokenBlockBytes + kMinBytes))
                                                  : seg.scales(smem);
                    const uint8_t* rgp = stage + b * R * kBlockBytes + (16 * rg + g) * kBlockBytes;
                    const uint8_t* r8p = rgp + 8 * kBlockBytes;
                    const uint4 hg = *reinterpret_cast<const uint4*>(rgp);
                    const uint4 h8 = *reinterpret_cast<const uint4*>(r8p);
                    const float dg = half_bits_to_float(hg.x & 0xffffu), mg = half_bits_to_float(hg.x >> 16);
                    const float d8 = half_bits_to_float(h8.x & 0xffffu), m8 = half_bits_to_float(h8.x >> 16);
                    if (check)
                        finite = finite && (!valid_lo || (isfinite(dg) && isfinite(mg)))
                                 && (!valid_hi || (isfinite(d8) && isfinite(m8)));
                    // 6-bit scales of sub-blocks 0-3 / 4-7, one per byte.
                    const uint32_t scLo_g = hg.y & 0x3F3F3F3Fu;
                    const uint32_t scHi_g = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
                    const uint32_t scLo_8 = h8.y & 0x3F3F3F3Fu;
                    const uint32_t scHi_8 = (h8.w & 0x0F0F0F0Fu) | ((h8.y >> 2) & 0x30303030u);
                    // B operand rows of this lane: token (nt*4 + g/2) clamped to the
                    // last present one (absent tokens only feed ignored columns).
                    const uint8_t* bsrc[NT];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const int tok = min(nt * 4 + (g >> 1), rows - 1);
                        bsrc[nt] = frag + (sblk * rows + tok) * kTokenBlockBytes + t * 32 + (g & 1) * 16;
                    }
                    // int32 sums 16 * sum_g sc_g * C_g: [nt][row g / g+8][h, l].
                    int I[NT][2][2];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        I[nt][0][0] = I[nt][0][1] = I[nt][1][0] = I[nt][1][1] = 0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        // Code bytes 8t..8t+7 of 32-byte chunk j, rows g and g+8.
                        const uint2 cg = *reinterpret_cast<const uint2*>(rgp + 16 + 32 * j + 8 * t);
                        const uint2 c8 = *reinterpret_cast<const uint2*>(r8p + 16 + 32 * j + 8 * t);
                        const uint32_t wg = j < 2 ? scLo_g : scHi_g, w8 = j < 2 ? scLo_8 : scHi_8;
                        // bytes 2(j%2) (sub-block 2j) and 2(j%2)+1 (2j+1) of the scale word.
                        const uint32_t selA = 0x4440u | (2u * uint32_t(j & 1)), selB = selA + 1u;
                        const int scAg = int(__byte_perm(wg, 0u, selA)) << 4, scA8 = int(__byte_perm(w8, 0u, selA)) << 4;
                        const int scBg = int(__byte_perm(wg, 0u, selB)), scB8 = int(__byte_perm(w8, 0u, selB));
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            const uint4 bf = *reinterpret_cast<const uint4*>(bsrc[nt] + j * 128);
                            int Ca[4], Cb[4];
                            // Sub-block 2j: low nibbles (q); 2j+1: high nibbles in place (16 q).
                            imma(Ca, cg.x & 0x0F0F0F0Fu, c8.x & 0x0F0F0F0Fu, cg.y & 0x0F0F0F0Fu, c8.y & 0x0F0F0F0Fu, bf.x, bf.y);
                            imma(Cb, cg.x & 0xF0F0F0F0u, c8.x & 0xF0F0F0F0u, cg.y & 0xF0F0F0F0u, c8.y & 0xF0F0F0F0u, bf.z, bf.w);
                            I[nt][0][0] += scAg * Ca[0] + scBg * Cb[0];
                            I[nt][0][1] += scAg * Ca[1] + scBg * Cb[1];
                            I[nt][1][0] += scA8 * Ca[2] + scB8 * Cb[2];
                            I[nt][1][1] += scA8 * Ca[3] + scB8 * Cb[3];
                        }
                    }
                    // Minimum term: A' = m of sub-blocks 2t, 2t+1 for rows g, g+8.
                    const uint32_t mLo_g = hg.z & 0x3F3F3F3Fu;
                    const uint32_t mHi_g = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
                    const uint32_t mLo_8 = h8.z & 0x3F3F3F3Fu;
                    const uint32_t mHi_8 = ((h8.w >> 4) & 0x0F0F0F0Fu) | ((h8.z >> 2) & 0x30303030u);
                    const uint32_t mwg = t < 2 ? mLo_g : mHi_g, mw8 = t < 2 ? mLo_8 : mHi_8;
                    const uint32_t mb = 2u * uint32_t(t & 1);
                    // bytes [m(2t), 0x64, m(2t+1), 0x64] -> (m(2t), m(2t+1)).
                    const uint32_t sel = (4u << 12) | ((mb + 1u) << 8) | (4u << 4) | mb;
                    const uint32_t am_g = hadd2_u(__byte_perm(mwg, 0x64646464u, sel), 0xE400E400u);
                    const uint32_t am_8 = hadd2_u(__byte_perm(mw8, 0x64646464u, sel), 0xE400E400u);
                    const float mg256 = mg * 256.f, m8256 = m8 * 256.f;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const int tokb = min(nt * 4 + (g >> 1), rows - 1);
                        const uint32_t bm = minb[(sblk * rows + tokb) * (kMinBytes / 4) + (g & 1) * 4 + t];
                        float Cm[4] = {0.f, 0.f, 0.f, 0.f};
                        mma1688(Cm, am_g, am_8, bm);
                        // Columns 2t, 2t+1 = token nt*4 + t (h, l).
                        const int tokc = min(nt * 4 + t, rows - 1);
                        const float sc = scales[sblk * rows + tokc] * (1.f / 16.f);
                        const float kg = dg * sc, k8 = d8 * sc;
                        acc[nt][0] = fmaf(kg, fmaf(float(I[nt][0][1]), 1.f / 254.f, float(I[nt][0][0])), acc[nt][0]);
                        acc[nt][0] = fmaf(-mg256, Cm[0] + Cm[1], acc[nt][0]);
                        acc[nt][1] = fmaf(k8, fmaf(float(I[nt][1][1]), 1.f / 254.f, float(I[nt][1][0])), acc[nt][1]);
                        acc[nt][1] = fmaf(-m8256, Cm[2] + Cm[3], acc[nt][1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[slot]);
        }
        if (check && !finite)
            atomicOr(job.status, 1u);
        finish_piece<NT>(p, pc, job, acc, KS, ks, tid, my_row, valid_lo, valid_hi, r0, rows, red, abort_flag,
                         await_dependency);
        // After an abort the remaining pieces still run (without waits or
        // MMAs) so that every cut tile's counter is re-armed.
    }
}

// ------------------------------------------------------------------- Q6_K
// Q6_K value: w = d * sc_s * (q - 32), q 6-bit (low 4 bits in ql, high 2 in
// qh), sc_s int8 per sub-block of 16 (IW/include/kadan/gguf_quantization.hpp
// decode of q6_k; ggml-common.h block_q6_K: ql[128], qh[64], scales[16], d).
// Sub-block s = 8 ip + 2 qt + h holds values 128 ip + 32 qt + 16 h + i
// (i < 16): low bits = nibble (qt >> 1) of ql[64 ip + 32 (qt & 1) + 16 h + i],
// high bits = bits 2 qt..2 qt+1 of qh[32 ip + 16 h + i].
//
//   A operand : q - 32 as s8, built per 4 values with two masks, one add and
//               one xor ((q + 96) ^ 128 = q - 32 mod 256, no carries since
//               q + 96 < 256)
//   MMA       : mma.m16n8k16.s8.s8 -> exact int32 sum over one sub-block
//   scales    : I = sum_s sc_s C_s (IMAD, exact)
//   epilogue  : acc += d * s_x * (I_h + I_l / 254)
// A 210-byte block is not a whole number of 16-byte words, so the TMA unit
// is a chunk of 8 blocks (1680 bytes) of 16 rows, one 2-D box per stage;
// blocks at odd positions of a chunk start 2 bytes off a word boundary and
// are read as half-word pairs.
constexpr int kQ6Block = 210;
constexpr int kQ6Chunk = 8;                       // blocks per TMA unit
constexpr int kQ6Rows = 16;                       // rows per tile
constexpr int kQ6StageBytes = kQ6Rows * kQ6Chunk * kQ6Block;  // 26880
// Activation segment: one chunk of 4 * NT tokens.
template <int NT> constexpr int q6_seg_budget() {
    return 4 * NT * kQ6Chunk * kTokenBlockTotal;
}
constexpr uint32_t kQ6MinUnitsPerCta = 2;

// S stages of one chunk each. NT = 1 (4 rows per pass): 3 stages (two CTAs per
// SM) or 2 stages (three CTAs per SM: more warps to hide the integer chains
// of the 6-bit unpack, the same bytes in flight); NT = 2 (8 rows): 2 stages,
// so that the twice larger activation segment still leaves room for two CTAs.
template <int NT, int S> struct Q6Layout {
    static constexpr int kStages = S;
    static constexpr int kSegBudget = q6_seg_budget<NT>();
    static constexpr int kStagesOff = 0;
    static constexpr int kSegOff = kStages * kQ6StageBytes;
    static constexpr int kRedOff = kSegOff + kSegBudget;
    static constexpr int kRedBytes = kConsumerThreads * 4 * 4;
    static constexpr int kBarOff = kRedOff + kRedBytes;
    static constexpr int kTotal = kBarOff + 2 * kStages * 8 + 16;
};
static_assert(2 * (Q6Layout<1, 3>::kTotal + 128 + 1024) <= 228 * 1024, "two Q6_K CTAs per SM (NT = 1)");
static_assert(3 * (Q6Layout<1, 2>::kTotal + 128 + 1024) <= 228 * 1024, "three Q6_K CTAs per SM (NT = 1, 2 stages)");
static_assert(2 * (Q6Layout<2, 2>::kTotal + 128 + 1024) <= 228 * 1024, "two Q6_K CTAs per SM (NT = 2)");

// CTAs per SM the kernel is compiled for (register budget).
template <int NT, int S> constexpr int q6_min_ctas() {
    return NT == 1 && S == 2 ? 3 : 2;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)
        ),
        "l"(map),
        "r"(c0),
        "r"(c1),
        "r"(smem_addr(bar))
        : "memory"
    );
}

// C = A(16x16 s8) * B(16x8 s8), exact int32.
__device__ __forceinline__ void imma16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0)
    );
}

// 4 bytes at p: one word load when p is word aligned, else two half-words
// (p is always 2-byte aligned here).
template <bool kOdd> __device__ __forceinline__ uint32_t ld_word(const uint8_t* p) {
    if constexpr (kOdd) {
        const uint32_t lo = *reinterpret_cast<const uint16_t*>(p), hi = *reinterpret_cast<const uint16_t*>(p + 2);
        return lo | (hi << 16);
    } else {
        return *reinterpret_cast<const uint32_t*>(p);
    }
}

// One block of rows g (bg) and g + 8 (b8) for one n-tile of tokens: adds the
// block's contribution to acc. bq: this lane's B words of the block, indexed
// [(s * rows + tok) * 2 + part] * 4 + t.
template <bool kOdd, int NT>
__device__ __forceinline__ void q6k_block(const uint8_t* bg, const uint8_t* b8, const uint32_t* bq, int rows,
                                          const int (&tokb)[NT], int part, int t, const float (&sc_tok)[NT],
                                          float (&acc)[NT][2], bool& finite_g, bool& finite_8) {
    const float dg = half_bits_to_float(*reinterpret_cast<const uint16_t*>(bg + 208));
    const float d8 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(b8 + 208));
    finite_g = finite_g && isfinite(dg);
    finite_8 = finite_8 && isfinite(d8);
    uint32_t scg[4], sc8[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        scg[w] = ld_word<kOdd>(bg + 192 + 4 * w);
        sc8[w] = ld_word<kOdd>(b8 + 192 + 4 * w);
    }
    // int32 sums sum_s sc_s C_s: [nt][h, l] for rows g and g + 8.
    int Ig[NT][2], I8[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
        Ig[nt][0] = Ig[nt][1] = I8[nt][0] = I8[nt][1] = 0;
#pragma unroll
    for (int ip = 0; ip < 2; ++ip)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int o = 64 * ip + 16 * h + 4 * t, oh = 128 + 32 * ip + 16 * h + 4 * t;
            const uint32_t qa_g = ld_word<kOdd>(bg + o), qb_g = ld_word<kOdd>(bg + o + 32), qh_g = ld_word<kOdd>(bg + oh);
            const uint32_t qa_8 = ld_word<kOdd>(b8 + o), qb_8 = ld_word<kOdd>(b8 + o + 32), qh_8 = ld_word<kOdd>(b8 + oh);
#pragma unroll
            for (int qt = 0; qt < 4; ++qt) {
                const int sb = 8 * ip + 2 * qt + h;
                const uint32_t ng = ((qt & 1) ? qb_g : qa_g) >> (4 * (qt >> 1));
                const uint32_t n8 = ((qt & 1) ? qb_8 : qa_8) >> (4 * (qt >> 1));
                // Bits 2qt, 2qt+1 of each qh byte moved to bits 4, 5.
                const uint32_t hg = qt == 3 ? qh_g >> 2 : qh_g << (4 - 2 * qt);
                const uint32_t h8 = qt == 3 ? qh_8 >> 2 : qh_8 << (4 - 2 * qt);
                const uint32_t vg = (((ng & 0x0F0F0F0Fu) | (hg & 0x30303030u)) + 0x60606060u) ^ 0x80808080u;
                const uint32_t v8 = (((n8 & 0x0F0F0F0Fu) | (h8 & 0x30303030u)) + 0x60606060u) ^ 0x80808080u;
                const int sg = int(int8_t(scg[sb >> 2] >> (8 * (sb & 3))));
                const int s8 = int(int8_t(sc8[sb >> 2] >> (8 * (sb & 3))));
                // One A operand (the weights) for every n-tile of tokens.
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const uint32_t b = bq[((sb * rows + tokb[nt]) * 2 + part) * 4 + t];
                    int C[4];
                    imma16(C, vg, v8, b);
                    Ig[nt][0] += sg * C[0], Ig[nt][1] += sg * C[1];
                    I8[nt][0] += s8 * C[2], I8[nt][1] += s8 * C[3];
                }
            }
        }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        acc[nt][0] = fmaf(dg * sc_tok[nt], fmaf(float(Ig[nt][1]), 1.f / 254.f, float(Ig[nt][0])), acc[nt][0]);
        acc[nt][1] = fmaf(d8 * sc_tok[nt], fmaf(float(I8[nt][1]), 1.f / 254.f, float(I8[nt][0])), acc[nt][1]);
    }
}

// Q6_K decode GEMV, T <= 4 NT input rows per pass. Tiles of 16 rows; a unit of
// the balanced split is (tile, chunk of 8 blocks); each stage is one chunk,
// its 8 blocks split over the 4 consumer warps (2 each), which add up in
// shared memory at the end of a piece. Everything else (pieces, fixup,
// programmatic dependent launch) is the Q4_K kernel's.
template <int NT, int S>
__global__ void __launch_bounds__(kThreadsQ, q6_min_ctas<NT, S>()) gemv_q6k_mma_kernel(const __grid_constant__ MmaParams p) {
    using L = Q6Layout<NT, S>;
    constexpr int kStages = L::kStages;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
    auto* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
    auto* empty = full + kStages;
    auto* abort_flag = reinterpret_cast<int*>(empty + kStages);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int KS = kWarps;
    auto* red = reinterpret_cast<float*>(smem + L::kRedOff);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        *abort_flag = 0;
        fence_barrier_init();
        grid_dependents_launch();
    }
    __syncthreads();

    if (warp == kWarps) {
        // ------------------------------ producer ------------------------------
        if (lane != 0)
            return;
        uint32_t it = 0;
        PieceIter pieces(p);
        Piece pc;
        while (pieces.next(p, pc)) {
            const MmaJob& job = p.jobs[pc.job];
            const int row0 = int((pc.tile / job.row_groups) * uint32_t(kQ6Rows));
            asm volatile("prefetch.tensormap [%0];" ::"l"(&job.map) : "memory");
            for (uint32_t ch = pc.k0; ch < pc.k1; ++ch, ++it) {
                const int slot = int(it % kStages);
                if (it >= kStages && !mbar_wait(&empty[slot], ((it / kStages) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog))
                    atomicExch(abort_flag, 1);
                if (*reinterpret_cast<volatile int*>(abort_flag))
                    goto drain;
                // The whole box lands (rows and blocks past the matrix are zero-filled).
                mbar_expect_tx(&full[slot], uint32_t(kQ6StageBytes));
                tma_load_2d(smem + L::kStagesOff + slot * kQ6StageBytes, &job.map, int(ch) * (kQ6Chunk * kQ6Block / 8),
                            row0, &full[slot]);
            }
        }
    drain:
        for (uint32_t k = 0; k < kStages && k < it; ++k) {
            const uint32_t last = it - 1 - k;
            mbar_wait(&full[last % kStages], (last / kStages) & 1u, watchdog_drain, p.watchdog);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    bool dependency_met = false;
    auto await_dependency = [&] {
        if (!dependency_met) {
            grid_dependency_wait();
            dependency_met = true;
        }
    };
    const int g = lane >> 2, t = lane & 3, ks = warp;
    uint32_t it = 0;
    const float* seg_x = nullptr;
    int seg_rows = -1, seg_blk0 = -1, seg_nblk = 0;
    PieceIter pieces(p);
    Piece pc;
    while (pieces.next(p, pc)) {
        const MmaJob& job = p.jobs[pc.job];
        const uint32_t row0 = (pc.tile / job.row_groups) * uint32_t(kQ6Rows);
        const uint32_t r0 = (pc.tile % job.row_groups) * job.group_rows;
        const int rows = int(min(job.group_rows, job.rows - r0));
        const int nblocks = int(job.in / 256);
        const float* x = job.input + size_t(r0) * job.in;
        const Segment seg(rows, kQ6Chunk, L::kSegBudget, L::kSegOff);
        if (seg.blocks < kQ6Chunk)
            atomicExch(abort_flag, 1);
        const uint32_t* frag = reinterpret_cast<const uint32_t*>(seg.frag(smem));
        const float* scales = seg.scales(smem);
        const uint32_t my_row = row0 + g;
        const bool valid_lo = my_row < job.columns, valid_hi = my_row + 8 < job.columns;
        const bool check = job.status != nullptr;
        bool finite_g = true, finite_8 = true;
        float acc[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            acc[nt][0] = acc[nt][1] = 0.f;

        for (uint32_t ch = pc.k0; ch < pc.k1; ++ch, ++it) {
            const int slot = int(it % kStages);
            const int blk_first = int(ch) * kQ6Chunk;
            const int nb = min(kQ6Chunk, nblocks - blk_first);
            if ((x != seg_x || rows != seg_rows || blk_first < seg_blk0 || blk_first + nb > seg_blk0 + seg_nblk)
                && seg.blocks >= kQ6Chunk) {
                // The CTA's last piece needs only its own chunks.
                const bool last = pieces.cur >= pieces.end;
                const int start = last || nblocks > seg.blocks ? blk_first : 0;
                const int count = min(seg.blocks, (last ? min(nblocks, int(pc.k1) * kQ6Chunk) : nblocks) - start);
                await_dependency();
                named_sync(1, kConsumerThreads);
                prep_segment<true>(smem, seg, x, job.in, start, count);
                named_sync(1, kConsumerThreads);
                seg_x = x, seg_rows = rows, seg_blk0 = start, seg_nblk = count;
            }
            const bool aborted = *reinterpret_cast<volatile int*>(abort_flag) != 0;
            if (!aborted && !mbar_wait(&full[slot], (it / kStages) & 1u, watchdog_full_barrier, p.watchdog))
                atomicExch(abort_flag, 1);
            if (!aborted) {
                const uint8_t* stage = smem + L::kStagesOff + slot * kQ6StageBytes;
#pragma unroll
                for (int bb = 0; bb < 2; ++bb) {
                    const int b = 2 * ks + bb;  // block of the chunk; odd b sits 2 bytes off a word
                    if (b >= nb)
                        break;
                    const int sblk = blk_first + b - seg_blk0;
                    const uint8_t* bg = stage + g * (kQ6Chunk * kQ6Block) + b * kQ6Block;
                    const uint8_t* b8 = bg + 8 * (kQ6Chunk * kQ6Block);
                    const uint32_t* bq = frag + sblk * rows * (kTokenBlockBytes / 4);
                    int tokb[NT];
                    float sc_tok[NT];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        tokb[nt] = min(nt * 4 + (g >> 1), rows - 1);
                        sc_tok[nt] = scales[sblk * rows + min(nt * 4 + t, rows - 1)];
                    }
                    if (bb)
                        q6k_block<true, NT>(bg, b8, bq, rows, tokb, g & 1, t, sc_tok, acc, finite_g, finite_8);
                    else
                        q6k_block<false, NT>(bg, b8, bq, rows, tokb, g & 1, t, sc_tok, acc, finite_g, finite_8);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[slot]);
        }
        if (check && !((finite_g || !valid_lo) && (finite_8 || !valid_hi)))
            atomicOr(job.status, 1u);
        finish_piece<NT>(p, pc, job, acc, KS, ks, tid, my_row, valid_lo, valid_hi, r0, rows, red, abort_flag,
                         await_dependency);
    }
}

// ------------------------------------------------------- Q6_K, 1-2 input rows
// Decode-size Q6_K (T <= 2) with half the tensor-pipe work and a third of the
// integer work of the kernel above. One mma.m16n8k32.u8.s8 covers two
// sub-blocks of 16 values (an even one in k 0..15, the odd one after it) and
// keeps them apart in the N dimension: column n = 4 tok + 2 par + hl holds
// token tok's activations at level hl (h or l) in the k half of sub-block
// parity par and zeros in the other half, so each lane's C values belong to
// one sub-block (par = lane % 2) and take that sub-block's scale alone.
//   A   : the unsigned 6-bit codes q (no -32 bias: two masks and a select per
//         4 values)
//   -32 : sum_s sc_s * 32 * X_s per row and token, X_s = sum of sub-block s's
//         quantised activations, from one mma.m16n8k16.s8 per block with A =
//         the row's 16 int8 scales as stored and B = X_s split as 64 X1 + X0
//         (both int8; column 4 tok + 2 digit + hl)
//   sums: lane pairs (par 0, 1) hold disjoint sub-blocks of one token and are
//         added once at the end of a piece
// Activation segment per (block, token): B words [pair p = 4 ip + qt][par]
// [hl][t] (512 bytes; lane (g, t) of pair p reads word (g % 4) * 4 + t of its
// token), X words [digit][hl][t] (64 bytes), the scale s (4 bytes).
constexpr int kPairWordBytes = 512, kPairXBytes = 64, kPairTokenBlock = kPairWordBytes + kPairXBytes + 4;
// Segment of S stages: 48 blocks of one token with 3 stages (two CTAs per SM
// still fit: a long-K launch such as K = 28672 re-quantises its window a
// third less often), all of K = 8192 with 2 stages (three CTAs per SM).
template <int S> constexpr int pair_seg_budget() {
    return (S == 3 ? 48 : 32) * kPairTokenBlock;
}

__host__ __device__ constexpr int pair_segment_blocks(int rows, int budget) {
    return budget / (rows * kPairTokenBlock) / kQ6Chunk * kQ6Chunk;
}

// Chunk of kQ6Chunk blocks in the pair layout (the staged path's unit): B
// words, X words and scales of `rows` tokens, 580 bytes per (block, token).
__host__ __device__ constexpr int pair_chunk_bytes(int rows) {
    return kQ6Chunk * rows * kPairTokenBlock;
}

// S stages, W consumer warps (each takes kQ6Chunk / W blocks of a stage).
// kStaged: a stage also holds its chunk's quantised activations (up to two
// tokens, copied from the launch's staging buffer), and there is no
// per-CTA activation window.
template <int S, int W = kWarps, bool kStaged = false, int TP = 1> struct PairLayout {
    static constexpr int kStages = S;
    // A stage starts on a 128-byte boundary (the TMA tile destination).
    static constexpr int kStageBytes = (kQ6StageBytes + (kStaged ? pair_chunk_bytes(2 * TP) : 0) + 127) / 128 * 128;
    static constexpr int kStagesOff = 0;
    static constexpr int kSegOff = kStages * kStageBytes;
    static constexpr int kSegBudget = kStaged ? 0 : pair_seg_budget<S>();
    static constexpr int kRedOff = kSegOff + kSegBudget;
    static constexpr int kRedBytes = 32 * W * 4 * 4;
    static constexpr int kBarOff = kRedOff + kRedBytes;
    static constexpr int kTotal = kBarOff + 2 * kStages * 8 + 16;
};
static_assert(2 * (PairLayout<3>::kTotal + 128 + 1024) <= 228 * 1024, "two Q6_K pair CTAs per SM");
static_assert(3 * (PairLayout<2>::kTotal + 128 + 1024) <= 228 * 1024, "three Q6_K pair CTAs per SM (2 stages)");
static_assert(2 * (PairLayout<3, kWarps, true>::kTotal + 128 + 1024) <= 228 * 1024, "two staged pair CTAs per SM");
static_assert(3 * (PairLayout<2, kWarps, true>::kTotal + 128 + 1024) <= 228 * 1024, "three staged pair CTAs per SM");
static_assert(2 * (PairLayout<2, kWarps, true, 2>::kTotal + 128 + 1024) <= 228 * 1024, "two staged 4-row pair CTAs per SM");
static_assert(PairLayout<2, kWarps, true, 2>::kStageBytes % 128 == 0 && PairLayout<2, 8, true, 4>::kStageBytes % 128 == 0,
              "tensor copies land on 128-byte boundaries");
static_assert(PairLayout<2, 8, true, 4>::kTotal + 128 + 1024 <= 228 * 1024, "one staged 8-row pair CTA per SM");
static_assert(kQ6StageBytes % 128 == 0 && PairLayout<3, kWarps, true>::kStageBytes % 128 == 0,
              "tensor copies land on 128-byte boundaries");
static_assert(pair_chunk_bytes(1) % 16 == 0, "bulk copy sizes and source offsets are multiples of 16 bytes");

struct PairSegment {
    int blocks, rows, off;
    __device__ PairSegment(int r, int offset, int budget)
        : blocks(pair_segment_blocks(r, budget)), rows(r), off(offset) {}
    __device__ uint32_t* words(uint8_t* smem) const { return reinterpret_cast<uint32_t*>(smem + off); }
    __device__ uint32_t* xwords(uint8_t* smem) const { return words(smem) + blocks * rows * (kPairWordBytes / 4); }
    __device__ float* scales(uint8_t* smem) const {
        return reinterpret_cast<float*>(xwords(smem) + blocks * rows * (kPairXBytes / 4));
    }
};

// Quantises one (block, token) item: lane L holds values 8L..8L+7 of the
// block in v and writes its B words, X bytes and (lane 0) the scale into a
// pair-layout area of `blocks` blocks x `rows` tokens at words / xbytes /
// scales (shared or global memory).
__device__ __forceinline__ void pair_quant_store(const float (&v)[8], uint32_t* words, uint8_t* xbytes, float* scales,
                                                 int rows, int blk, int tok, int lane) {
    const int s = lane >> 1, half = lane & 1;
    const int ip = s >> 3, qt = (s >> 1) & 3, par = s & 1;
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        m = fmaxf(m, fabsf(v[i]));
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    // 1/s to within an ulp: the levels below absorb it (x ~ s (h + l / 254)
    // with s = m / 127 exactly as stored).
    const float inv = m > 0.f ? 127.f * __frcp_rn(m) : 0.f;
    // x ~ s (h + l / 254): h = round(x / s), l = round(254 (x / s - h)).
    const float2 inv2 = make_float2(inv, inv), magic = make_float2(kMagic, kMagic);
    const float2 neg_magic = make_float2(-kMagic, -kMagic), k254 = make_float2(254.f, 254.f);
    int h[8], l[8];
    int xh = 0, xl = 0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const float2 y = mul2(make_float2(v[i], v[i + 1]), inv2);
        const float2 r1 = add2(y, magic);
        const float2 d = sub2(y, add2(r1, neg_magic));
        const float2 r2 = fma2(d, k254, magic);
        h[i] = int(__float_as_uint(r1.x) << 10) >> 10, h[i + 1] = int(__float_as_uint(r1.y) << 10) >> 10;
        l[i] = int(__float_as_uint(r2.x) << 10) >> 10, l[i + 1] = int(__float_as_uint(r2.y) << 10) >> 10;
        xh += h[i] + h[i + 1];
        xl += l[i] + l[i + 1];
    }
    // B words of this lane: pair p, parity par, t = 2 half + {0, 1}.
    uint32_t* w = words + ((blk * 8 + 4 * ip + qt) * rows + tok) * 16 + par * 8 + 2 * half;
    w[0] = pack4(h[0], h[1], h[2], h[3]);
    w[1] = pack4(h[4], h[5], h[6], h[7]);
    w[4] = pack4(l[0], l[1], l[2], l[3]);
    w[5] = pack4(l[4], l[5], l[6], l[7]);
    // Sub-block sums (both halves), split X = 64 X1 + X0, X0 in [-32, 31].
    xh += __shfl_xor_sync(0xffffffffu, xh, 1);
    xl += __shfl_xor_sync(0xffffffffu, xl, 1);
    if (!half) {
        uint8_t* xb = xbytes + (blk * rows + tok) * kPairXBytes + (s & 3);
        const int h1 = (xh + 32) >> 6, l1 = (xl + 32) >> 6;
        // [digit][hl][t = s / 4][byte s % 4]
        xb[(0 * 2 + 0) * 16 + (s >> 2) * 4] = uint8_t(h1);
        xb[(0 * 2 + 1) * 16 + (s >> 2) * 4] = uint8_t(l1);
        xb[(1 * 2 + 0) * 16 + (s >> 2) * 4] = uint8_t(xh - 64 * h1);
        xb[(1 * 2 + 1) * 16 + (s >> 2) * 4] = uint8_t(xl - 64 * l1);
    }
    if (lane == 0)
        scales[blk * rows + tok] = m > 0.f ? m / 127.f : 0.f;
}

// Quantise super-blocks [blk0, blk0 + nblk) of the segment's tokens into the
// pair layout: one warp per (block, token); lane L owns values 8L..8L+7 (half
// L % 2 of sub-block L / 2). Every load of a warp's items is in flight before
// the first is used.
template <int W>
__device__ void prep_pairs(uint8_t* smem, const PairSegment& seg, const float* x, size_t in, int blk0, int nblk) {
    const int rows = seg.rows;
    uint32_t* words = seg.words(smem);
    uint8_t* xbytes = reinterpret_cast<uint8_t*>(seg.xwords(smem));
    float* scales = seg.scales(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (in & 3) == 0;
    const int items = nblk * rows;
    constexpr int kBatch = 4;
    for (int base = warp; base < items; base += W * kBatch) {
        float v[kBatch][8];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int item = min(base + q * W, items - 1);
            const int blk = item / rows, tok = item % rows;
            load_lane8(v[q], x + size_t(tok) * in + size_t(blk0 + blk) * 256 + lane * 8, vec);
        }
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int item = base + q * W;
            if (item >= items)
                break;
            pair_quant_store(v[q], words, xbytes, scales, rows, item / rows, item % rows, lane);
        }
    }
}

// Inputs of one activation quantisation launch: each region is one distinct
// input (x, in, rows) of a GEMV launch, written at dst in the layout its
// GEMV kernel copies into its stages.
struct StageQuantRegion {
    const float* x;
    uint8_t* dst;
    uint32_t in, rows, first_item;  // items: blocks x rows, prefix over regions
    uint32_t group_rows;            // pair layout: rows per row group (groups follow one another)
};
struct StageQuantParams {
    StageQuantRegion regions[kMaxJobsQ];
    uint32_t count, items;
};

// The region holding `item` (regions in first_item order).
__device__ __forceinline__ const StageQuantRegion& quant_region(const StageQuantParams& p, uint32_t item) {
    uint32_t r = 0;
    while (r + 1 < p.count && item >= p.regions[r + 1].first_item)
        ++r;
    return p.regions[r];
}

// Q4_K: every (block, token) of the launch's inputs quantised once into one
// record per block and input (q4k_record_bytes), one warp per item. Waits for
// the previous kernel of the stream (which may write the inputs); lets the
// GEMV that follows launch only once its items are done: launched earlier,
// that GEMV's CTAs take the SMs piecemeal while the previous kernel drains
// (measured: a step of the config-4 stack 10 % slower).
__global__ void __launch_bounds__(128) q4k_quant_kernel(const __grid_constant__ StageQuantParams p) {
    grid_dependency_wait();
    const int lane = threadIdx.x & 31;
    const uint32_t warps = gridDim.x * (blockDim.x >> 5);
    for (uint32_t item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); item < p.items; item += warps) {
        const StageQuantRegion& g = quant_region(p, item);
        const int rows = int(g.rows);
        const uint32_t local = item - g.first_item;
        const int blk = int(local / g.rows), tok = int(local % g.rows);
        uint8_t* rec = g.dst + size_t(blk) * q4k_record_bytes(rows);
        const bool vec = (reinterpret_cast<uintptr_t>(g.x) & 15u) == 0 && (g.in & 3) == 0;
        float v[8], m, sum, next;
        load_lane8(v, g.x + size_t(tok) * g.in + size_t(blk) * 256 + lane * 8, vec);
        q4k_block_stats(v, m, sum, next);
        q4k_store_item(v, m, sum, next, reinterpret_cast<uint32_t*>(rec + tok * kTokenBlockBytes),
                       reinterpret_cast<uint32_t*>(rec + rows * kTokenBlockBytes + tok * kMinBytes),
                       reinterpret_cast<float*>(rec + rows * (kTokenBlockBytes + kMinBytes)) + tok, lane);
    }
    // The GEMV reads the buffer with bulk async copies.
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0)
        grid_dependents_launch();
}

// Quantises every (block, token) of the launch's inputs once into the
// staging buffer the GEMV's producer copies from, one warp per item. Waits
// for the previous kernel of the stream (which may write the inputs) and
// lets the GEMV that follows start streaming weights at once.
__global__ void __launch_bounds__(128) pair_quant_kernel(const __grid_constant__ StageQuantParams p) {
    if (threadIdx.x == 0)
        grid_dependents_launch();
    grid_dependency_wait();
    const int lane = threadIdx.x & 31;
    const uint32_t warps = gridDim.x * (blockDim.x >> 5);
    for (uint32_t item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); item < p.items; item += warps) {
        const StageQuantRegion& g = quant_region(p, item);
        const uint32_t local = item - g.first_item;
        const int blk = int(local / g.rows), row = int(local % g.rows);
        const int chunk = blk / kQ6Chunk, b = blk % kQ6Chunk;
        // Row group of this row, its rows and the row's token within it.
        const int gr = int(g.group_rows), rg = row / gr, tok = row % gr;
        const int rows = min(gr, int(g.rows) - rg * gr);
        const int chunks = int((g.in / 256 + kQ6Chunk - 1) / kQ6Chunk);
        uint8_t* base = g.dst + size_t(rg) * chunks * pair_chunk_bytes(gr) + size_t(chunk) * pair_chunk_bytes(rows);
        uint32_t* words = reinterpret_cast<uint32_t*>(base);
        uint8_t* xbytes = base + kQ6Chunk * rows * kPairWordBytes;
        float* scales = reinterpret_cast<float*>(xbytes + kQ6Chunk * rows * kPairXBytes);
        const bool vec = (reinterpret_cast<uintptr_t>(g.x) & 15u) == 0 && (g.in & 3) == 0;
        float v[8];
        load_lane8(v, g.x + size_t(row) * g.in + size_t(blk) * 256 + lane * 8, vec);
        pair_quant_store(v, words, xbytes, scales, rows, b, tok, lane);
    }
    // The GEMV reads the buffer with bulk async copies.
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Code word of 4 values: low nibbles (shift `ls`) and the high bit pairs
// placed at bits 4-5 (qh moved by `hs`: left when positive).
__device__ __forceinline__ uint32_t q6_code(uint32_t ql, uint32_t qh, int ls, int hs) {
    const uint32_t hi = (hs >= 0 ? qh << hs : qh >> -hs) & 0x30303030u;
    return ((ql >> ls) & 0x0F0F0F0Fu) | hi;
}

// prmt selector that sign-extends byte b of a word (prmt's default mode
// replicates a byte's sign where the selector nibble's top bit is set; the
// __byte_perm intrinsic ignores that bit).
__host__ __device__ constexpr uint32_t sext_sel(uint32_t b) {
    return ((b | 8u) << 12) | ((b | 8u) << 8) | ((b | 8u) << 4) | b;
}

__device__ __forceinline__ int sext_byte(uint32_t w, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
    return int(r);
}

// One block of rows g (bg) and g + 8 (b8): adds this lane's sub-blocks of
// its tokens to acc, for TP pairs of tokens (2 TP input rows per pass). A lane
// supplies B column g of every token pair (token 2 tp + g / 4, parity g / 2 %
// 2, level g % 2): bw points at its word of pair 0 for token pair 0 (pairs
// `pair_stride` words apart, token pairs 32 words apart), xw[tp] are its X
// words. It receives C columns 2t, 2t + 1: token 2 tp + t / 2, parity t % 2
// (the scales it applies), h and l; sc_tok[tp] is that token's activation
// scale. boff[tp]: word offset of token pair tp's B word from bw (tokens
// past the last present one are clamped to it). The weight operands are
// unpacked once for all token pairs.
template <bool kOdd, int TP>
__device__ __forceinline__ void q6k_pair_block(const uint8_t* bg, const uint8_t* b8, const uint32_t* bw, int pair_stride,
                                               const int (&boff)[TP], const uint32_t (&xw)[TP], int g, int t,
                                               const float (&sc_tok)[TP],
                                               float (&acc_g)[TP], float (&acc_8)[TP], bool& finite_g, bool& finite_8) {
    const float dg = half_bits_to_float(*reinterpret_cast<const uint16_t*>(bg + 208));
    const float d8 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(b8 + 208));
    finite_g = finite_g && isfinite(dg);
    finite_8 = finite_8 && isfinite(d8);
    const bool b_odd = (g >> 1) & 1;  // parity of the B column this lane supplies
    const bool odd_col = t & 1;       // parity of the C columns this lane receives
    // -32 correction: sum_s sc_s (64 X1_s + X0_s) for digit (t % 2) = X1 / X0.
    int I[TP][4];
    {
        const uint32_t sa = ld_word<kOdd>(bg + 192 + 4 * t), sb = ld_word<kOdd>(b8 + 192 + 4 * t);
        const int mult = odd_col ? -32 : -32 * 64;
#pragma unroll
        for (int tp = 0; tp < TP; ++tp) {
            int cx[4];
            imma16(cx, sa, sb, xw[tp]);
            I[tp][0] = mult * cx[0], I[tp][1] = mult * cx[1], I[tp][2] = mult * cx[2], I[tp][3] = mult * cx[3];
        }
    }
    uint32_t scg[4], sc8[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        scg[w] = ld_word<kOdd>(bg + 192 + 4 * w);
        sc8[w] = ld_word<kOdd>(b8 + 192 + 4 * w);
    }
    const uint32_t sel0 = sext_sel(odd_col ? 1u : 0u), sel1 = sext_sel(odd_col ? 3u : 2u);
#pragma unroll
    for (int ip = 0; ip < 2; ++ip) {
        // ql words [a][h] (a = qt & 1) and qh words [h] of both rows.
        uint32_t qlg[2][2], ql8[2][2], qhg[2], qh8[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int a = 0; a < 2; ++a) {
                qlg[a][h] = ld_word<kOdd>(bg + 64 * ip + 32 * a + 16 * h + 4 * t);
                ql8[a][h] = ld_word<kOdd>(b8 + 64 * ip + 32 * a + 16 * h + 4 * t);
            }
            qhg[h] = ld_word<kOdd>(bg + 128 + 32 * ip + 16 * h + 4 * t);
            qh8[h] = ld_word<kOdd>(b8 + 128 + 32 * ip + 16 * h + 4 * t);
        }
#pragma unroll
        for (int qt = 0; qt < 4; ++qt) {
            const int ls = 4 * (qt >> 1), hs = 4 - 2 * qt;
            const int a = qt & 1;
            const uint32_t a0 = q6_code(qlg[a][0], qhg[0], ls, hs), a1 = q6_code(ql8[a][0], qh8[0], ls, hs);
            const uint32_t a2 = q6_code(qlg[a][1], qhg[1], ls, hs), a3 = q6_code(ql8[a][1], qh8[1], ls, hs);
            // Scale of sub-block 8 ip + 2 qt + par: word 2 ip + qt / 2, byte 2 (qt % 2) + par.
            const uint32_t sel = (qt & 1) ? sel1 : sel0;
            const int sg = sext_byte(scg[2 * ip + (qt >> 1)], sel);
            const int s8 = sext_byte(sc8[2 * ip + (qt >> 1)], sel);
#pragma unroll
            for (int tp = 0; tp < TP; ++tp) {
                const uint32_t w = bw[(4 * ip + qt) * pair_stride + boff[tp]];
                int c[4];
                imma(c, a0, a1, a2, a3, b_odd ? 0u : w, b_odd ? w : 0u);
                I[tp][0] += sg * c[0], I[tp][1] += sg * c[1];
                I[tp][2] += s8 * c[2], I[tp][3] += s8 * c[3];
            }
        }
    }
#pragma unroll
    for (int tp = 0; tp < TP; ++tp) {
        acc_g[tp] = fmaf(dg * sc_tok[tp], fmaf(float(I[tp][1]), 1.f / 254.f, float(I[tp][0])), acc_g[tp]);
        acc_8[tp] = fmaf(d8 * sc_tok[tp], fmaf(float(I[tp][3]), 1.f / 254.f, float(I[tp][2])), acc_8[tp]);
    }
}

// Q6_K decode GEMV for one or two input rows per pass: the Q6_K kernel's
// tiles, stages, pieces, fixup and programmatic dependent launch, with the
// paired-sub-block inner loop above.
//
// kStaged: the activations come quantised from the launch's staging buffer
// (pair_quant_kernel, launched just before): the producer copies chunk ch's
// slice with the chunk's weights into the same stage, so consumers never
// quantise and never wait at a window refill. The producer issues the first
// S weight loads before it waits for the quantisation kernel, then the
// activation copies of those stages, then both parts of every later stage.
// Otherwise each CTA quantises a window of activations into shared memory
// whenever its chunks leave the current one.
//
// TP token pairs per pass (staged only for TP = 2): 2 TP input rows share
// each unpacked weight fragment; more rows are row groups, whose staged
// activations follow one another (group stride: the job's chunks x a full
// group's chunk bytes).
template <int S, int W, bool kStaged, int TP = 1>
__global__ void __launch_bounds__(32 * W + 32, TP == 1 ? (S == 2 ? 3 : 2) : TP == 2 ? 2 : 1)
    gemv_q6k_pair_kernel(const __grid_constant__ MmaParams p) {
    static_assert(TP == 1 || kStaged, "4- and 8-row passes take staged activations");
    constexpr int NF = TP >= 4 ? 2 : 1;  // groups of 4 tokens in the piece ending
    using L = PairLayout<S, W, kStaged, TP>;
    constexpr int kStages = L::kStages;
    constexpr int CT = 32 * W;               // consumer threads
    constexpr int kPerWarp = kQ6Chunk / W;   // blocks of a stage per consumer warp
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
    auto* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
    auto* empty = full + kStages;
    auto* abort_flag = reinterpret_cast<int*>(empty + kStages);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int KS = W;
    auto* red = reinterpret_cast<float*>(smem + L::kRedOff);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        *abort_flag = 0;
        fence_barrier_init();
        grid_dependents_launch();
    }
    __syncthreads();

    if (warp == W) {
        // ------------------------------ producer ------------------------------
        if (lane != 0)
            return;
        uint32_t it = 0;
        // Staged: activation copies of the first stages, held back until the
        // quantisation kernel has finished.
        bool staged_ready = false;
        const uint8_t* held_src[kStages];
        uint32_t held_bytes[kStages];
        uint32_t held = 0;
        auto release_held = [&] {
            grid_dependency_wait();
            asm volatile("fence.proxy.async.global;" ::: "memory");
            staged_ready = true;
            for (uint32_t k = 0; k < held; ++k)
                bulk_g2s(smem + L::kStagesOff + k * L::kStageBytes + kQ6StageBytes, held_src[k], held_bytes[k], &full[k]);
            held = 0;
        };
        PieceIter pieces(p);
        Piece pc;
        while (pieces.next(p, pc)) {
            const MmaJob& job = p.jobs[pc.job];
            const int row0 = int((pc.tile / job.row_groups) * uint32_t(kQ6Rows));
            // Staged activations of this tile's row group.
            const uint32_t rg = pc.tile % job.row_groups;
            const uint32_t act_bytes = kStaged ? uint32_t(pair_chunk_bytes(int(min(job.group_rows, job.rows - rg * job.group_rows)))) : 0u;
            const uint8_t* act_src = kStaged ? job.staged + size_t(rg) * job.nblocks * pair_chunk_bytes(int(job.group_rows)) : nullptr;
            asm volatile("prefetch.tensormap [%0];" ::"l"(&job.map) : "memory");
            for (uint32_t ch = pc.k0; ch < pc.k1; ++ch, ++it) {
                const int slot = int(it % kStages);
                if (it >= kStages && !mbar_wait(&empty[slot], ((it / kStages) & 1u) ^ 1u, watchdog_empty_barrier, p.watchdog))
                    atomicExch(abort_flag, 1);
                if (*reinterpret_cast<volatile int*>(abort_flag))
                    goto drain;
                uint8_t* stage = smem + L::kStagesOff + slot * L::kStageBytes;
                mbar_expect_tx(&full[slot], uint32_t(kQ6StageBytes) + act_bytes);
                tma_load_2d(stage, &job.map, int(ch) * (kQ6Chunk * kQ6Block / 8), row0, &full[slot]);
                if constexpr (kStaged) {
                    const uint8_t* src = act_src + size_t(ch) * act_bytes;
                    if (staged_ready) {
                        bulk_g2s(stage + kQ6StageBytes, src, act_bytes, &full[slot]);
                    } else {
                        held_src[held] = src, held_bytes[held] = act_bytes;
                        if (++held == uint32_t(kStages))
                            release_held();
                    }
                }
            }
        }
        if constexpr (kStaged)
            if (!staged_ready)
                release_held();
    drain:
        for (uint32_t k = 0; k < kStages && k < it; ++k) {
            const uint32_t last = it - 1 - k;
            mbar_wait(&full[last % kStages], (last / kStages) & 1u, watchdog_drain, p.watchdog);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    bool dependency_met = false;
    auto await_dependency = [&] {
        if (!dependency_met) {
            grid_dependency_wait();
            dependency_met = true;
        }
    };
    const int g = lane >> 2, t = lane & 3, ks = warp;
    uint32_t it = 0;
    const float* seg_x = nullptr;
    int seg_rows = -1, seg_blk0 = -1, seg_nblk = 0;
    PieceIter pieces(p);
    Piece pc;
    while (pieces.next(p, pc)) {
        const MmaJob& job = p.jobs[pc.job];
        const uint32_t row0 = (pc.tile / job.row_groups) * uint32_t(kQ6Rows);
        const uint32_t r0 = (pc.tile % job.row_groups) * job.group_rows;
        const int rows = int(min(job.group_rows, job.rows - r0));
        const int nblocks = int(job.in / 256);
        const float* x = job.input + size_t(r0) * job.in;
        const PairSegment seg(rows, kStaged ? 0 : L::kSegOff, kStaged ? pair_chunk_bytes(rows) : L::kSegBudget);
        if (!kStaged && seg.blocks < kQ6Chunk)
            atomicExch(abort_flag, 1);
        // B side: the token of the column this lane supplies (2 tp + g / 4)
        // and its word in every group of 16; C side: the token of the
        // columns it receives (2 tp + t / 2). Both clamped to the rows present.
        int btok[TP], ctok[TP], boff[TP];
#pragma unroll
        for (int tp = 0; tp < TP; ++tp) {
            btok[tp] = min(2 * tp + (g >> 2), rows - 1), ctok[tp] = min(2 * tp + (t >> 1), rows - 1);
            boff[tp] = (btok[tp] - btok[0]) * 16;
        }
        const int lane_word = (g & 3) * 4 + t;
        const uint32_t my_row = row0 + g;
        const bool valid_lo = my_row < job.columns, valid_hi = my_row + 8 < job.columns;
        const bool check = job.status != nullptr;
        bool finite_g = true, finite_8 = true;
        float acc_g[TP], acc_8[TP];
#pragma unroll
        for (int tp = 0; tp < TP; ++tp)
            acc_g[tp] = acc_8[tp] = 0.f;

        for (uint32_t ch = pc.k0; ch < pc.k1; ++ch, ++it) {
            const int slot = int(it % kStages);
            const int blk_first = int(ch) * kQ6Chunk;
            const int nb = min(kQ6Chunk, nblocks - blk_first);
            uint8_t* stage = smem + L::kStagesOff + slot * L::kStageBytes;
            // Activations of this chunk: the stage's own slice (staged) or the
            // CTA's window, refilled when the chunk leaves it.
            uint8_t* act_base = stage + kQ6StageBytes;
            int act_blk0 = blk_first;
            if constexpr (!kStaged) {
                act_base = smem;
                if ((x != seg_x || rows != seg_rows || blk_first < seg_blk0 || blk_first + nb > seg_blk0 + seg_nblk)
                    && seg.blocks >= kQ6Chunk) {
                    // The CTA's last piece needs only its own chunks.
                    const bool last = pieces.cur >= pieces.end;
                    const int start = last || nblocks > seg.blocks ? blk_first : 0;
                    const int count = min(seg.blocks, (last ? min(nblocks, int(pc.k1) * kQ6Chunk) : nblocks) - start);
                    await_dependency();
                    named_sync(1, CT);
                    prep_pairs<W>(smem, seg, x, job.in, start, count);
                    named_sync(1, CT);
                    seg_x = x, seg_rows = rows, seg_blk0 = start, seg_nblk = count;
                }
                act_blk0 = seg_blk0;
            }
            const uint32_t* words = seg.words(act_base);
            const uint32_t* xwords = seg.xwords(act_base);
            const float* scales = seg.scales(act_base);
            const bool aborted = *reinterpret_cast<volatile int*>(abort_flag) != 0;
            if (!aborted && !mbar_wait(&full[slot], (it / kStages) & 1u, watchdog_full_barrier, p.watchdog))
                atomicExch(abort_flag, 1);
            if (!aborted) {
#pragma unroll
                for (int bb = 0; bb < kPerWarp; ++bb) {
                    const int b = kPerWarp * ks + bb;  // block of the chunk; odd b sits 2 bytes off a word
                    if (b >= nb)
                        break;
                    const int sblk = blk_first + b - act_blk0;
                    const uint8_t* bg = stage + g * (kQ6Chunk * kQ6Block) + b * kQ6Block;
                    const uint8_t* b8 = bg + 8 * (kQ6Chunk * kQ6Block);
                    const uint32_t* bw = words + (sblk * 8 * rows + btok[0]) * 16 + lane_word;
                    uint32_t xw[TP];
                    float sc_tok[TP];
#pragma unroll
                    for (int tp = 0; tp < TP; ++tp) {
                        xw[tp] = xwords[(sblk * rows + btok[tp]) * 16 + lane_word];
                        sc_tok[tp] = scales[sblk * rows + ctok[tp]];
                    }
                    if (b & 1)
                        q6k_pair_block<true, TP>(bg, b8, bw, rows * 16, boff, xw, g, t, sc_tok, acc_g, acc_8, finite_g,
                                                 finite_8);
                    else
                        q6k_pair_block<false, TP>(bg, b8, bw, rows * 16, boff, xw, g, t, sc_tok, acc_g, acc_8, finite_g,
                                                  finite_8);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[slot]);
        }
        if (check && !((finite_g || !valid_lo) && (finite_8 || !valid_hi)))
            atomicOr(job.status, 1u);
        // Lanes t = 2k, 2k + 1 hold token 2 tp + k's even and odd
        // sub-blocks: add them, then give lane t the sums of tokens t and
        // 4 + t (token pairs t / 2 and 2 + t / 2, lane 2 (t % 2) of each group
        // of four) as the common piece ending expects.
        const int from = (lane & ~3) | ((2 * t) & 3);
        float acc[NF][2];
#pragma unroll
        for (int tp = 0; tp < TP; ++tp) {
            acc_g[tp] += __shfl_xor_sync(0xffffffffu, acc_g[tp], 1);
            acc_8[tp] += __shfl_xor_sync(0xffffffffu, acc_8[tp], 1);
            const float vg = __shfl_sync(0xffffffffu, acc_g[tp], from), v8 = __shfl_sync(0xffffffffu, acc_8[tp], from);
#pragma unroll
            for (int nf = 0; nf < NF; ++nf)
                if (tp == (TP == 1 ? 0 : 2 * nf + (t >> 1)))
                    acc[nf][0] = vg, acc[nf][1] = v8;
        }
        finish_piece<NF, decltype(await_dependency), CT>(p, pc, job, acc, KS, ks, tid, my_row, valid_lo, valid_hi, r0,
                                                         rows, red, abort_flag, await_dependency);
    }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// CTA slots of the kernel on the current device (SMs x resident CTAs), or a
// negative kb200_status.
template <int NT, bool kStaged = false> int kernel_slots() {
    static int blocks_per_sm[64] = {};
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    constexpr int smem = LayoutQ4<kStaged, NT>::kTotal + 128;  // + alignment slack
    std::lock_guard<std::mutex> guard(lock);
    if (!blocks_per_sm[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_q4k_mma_kernel<NT, kStaged>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess)
            return -cuda_fail(e, "gemv_q4k_mma_kernel attribute");
        int n = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_q4k_mma_kernel<NT, kStaged>, kThreadsQ, smem);
        if (e != cudaSuccess)
            return -cuda_fail(e, "gemv_q4k_mma_kernel occupancy");
        blocks_per_sm[dev] = n > 0 ? n : 1;
    }
    return sm_count() * blocks_per_sm[dev];
}

// Key of a stream's per-stream buffers: the handle itself, except for
// cudaStreamPerThread, one handle that names a different stream in every
// host thread (keyed by a thread-local address, which no stream handle
// equals).
cudaStream_t stream_key(cudaStream_t stream) {
    static thread_local char per_thread;
    return stream == cudaStreamPerThread ? reinterpret_cast<cudaStream_t>(&per_thread) : stream;
}

// Fixup buffer of the balanced split for one (device, stream). Launches on one
// stream run in order, and a launch touches the buffer only after its
// grid-dependency wait, so every launch of the stream can share it.
struct Fixup {
    unsigned long long* partials = nullptr;
    uint32_t ctas = 0;
};

// The stream's fixup buffer, allocated (and zeroed on the stream) by the
// first call outside graph capture; null when none can be had.
struct FixupTable {
    std::mutex lock;
    std::map<std::pair<int, cudaStream_t>, Fixup> table;
};

FixupTable& fixups() {
    static FixupTable t;
    return t;
}

const Fixup* fixup_for(cudaStream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return nullptr;
    FixupTable& t = fixups();
    std::lock_guard<std::mutex> guard(t.lock);
    Fixup& f = t.table[{dev, stream_key(stream)}];
    if (f.ctas)
        return &f;
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess || capture != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;
    }
    // At most 4 CTAs of this kernel fit on an SM (shared memory).
    const uint32_t ctas = uint32_t(sm_count()) * 4u;
    Fixup made;
    const size_t bytes = size_t(ctas) * kSlotFloats * sizeof(unsigned long long);
    if (cudaMalloc(&made.partials, bytes) != cudaSuccess
        || cudaMemsetAsync(made.partials, 0, bytes, stream) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(made.partials);
        return nullptr;
    }
    made.ctas = ctas;
    f = made;
    return &f;
}

// Staging buffer of the pair kernel's quantised activations for one (device,
// stream). The quantisation kernel writes it after its grid-dependency wait
// (the previous kernel of the stream is done) and the GEMV after it reads it
// after its own, so the launches of one stream share it. Allocated by the
// first call outside graph capture and never moved or freed: captured graphs
// hold its address. A launch whose inputs do not fit falls back to per-CTA
// quantisation.
constexpr size_t kStagingBytes = size_t(8) << 20;

struct StagingTable {
    std::mutex lock;
    std::map<std::pair<int, cudaStream_t>, uint8_t*> table;
};

uint8_t* staging_for(cudaStream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return nullptr;
    static StagingTable t;
    std::lock_guard<std::mutex> guard(t.lock);
    uint8_t*& buf = t.table[{dev, stream_key(stream)}];
    if (buf)
        return buf;
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess || capture != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;
    }
    void* p = nullptr;
    if (cudaMalloc(&p, kStagingBytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    buf = static_cast<uint8_t*>(p);
    return buf;
}

struct Tuning {
    bool balanced = true;  // KB200_GEMV_BALANCED=0: whole tiles round-robin
    uint32_t prefetch = 0; // KB200_GEMV_L2_PREFETCH=<stages>
    uint32_t min_units = kMinUnitsPerCta;       // KB200_GEMV_MIN_UNITS=<units per CTA>
    uint32_t q6_min_units = kQ6MinUnitsPerCta;  // KB200_GEMV_Q6K_MIN_UNITS=<units per CTA>
    int ctas_per_sm = 0;                        // KB200_GEMV_CTAS_PER_SM=<n>: grid slots per SM (0: all that fit)
    int q6_stages = 0;                          // KB200_GEMV_Q6K_STAGES=2|3: ring depth at 1-4 rows per pass (0: auto)
    bool q6_pair = true;                        // KB200_GEMV_Q6K_PAIR=0: 1-2 rows on the 4-row kernel
    bool q6_staged = true;                      // KB200_GEMV_Q6K_STAGED=0: pair kernel quantises per CTA
    bool q4_staged = true;                      // KB200_GEMV_Q4K_STAGED=0: Q4_K kernel quantises per CTA
};

const Tuning& tuning() {
    static const Tuning t = [] {
        Tuning v;
        if (const char* s = std::getenv("KB200_GEMV_BALANCED"))
            v.balanced = std::atoi(s) != 0;
        if (const char* s = std::getenv("KB200_GEMV_CTAS_PER_SM"))
            v.ctas_per_sm = std::max(0, std::atoi(s));
        if (const char* s = std::getenv("KB200_GEMV_MIN_UNITS"))
            v.min_units = uint32_t(std::max(1, std::atoi(s)));
        if (const char* s = std::getenv("KB200_GEMV_Q6K_MIN_UNITS"))
            v.q6_min_units = uint32_t(std::max(1, std::atoi(s)));
        if (const char* s = std::getenv("KB200_GEMV_Q6K_PAIR"))
            v.q6_pair = std::atoi(s) != 0;
        if (const char* s = std::getenv("KB200_GEMV_Q6K_STAGED"))
            v.q6_staged = std::atoi(s) != 0;
        if (const char* s = std::getenv("KB200_GEMV_Q4K_STAGED"))
            v.q4_staged = std::atoi(s) != 0;
        if (const char* s = std::getenv("KB200_GEMV_Q6K_STAGES"))
            v.q6_stages = std::atoi(s) == 2 ? 2 : 3;
        if (const char* s = std::getenv("KB200_GEMV_L2_PREFETCH"))
            v.prefetch = uint32_t(std::max(0, std::min(64, std::atoi(s))));
        return v;
    }();
    return t;
}

template <int NT, int S> int q6k_slots() {
    static int blocks_per_sm[64] = {};
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    constexpr int smem = Q6Layout<NT, S>::kTotal + 128;
    std::lock_guard<std::mutex> guard(lock);
    if (!blocks_per_sm[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_q6k_mma_kernel<NT, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess)
            return -cuda_fail(e, "gemv_q6k_mma_kernel attribute");
        int n = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_q6k_mma_kernel<NT, S>, kThreadsQ, smem);
        if (e != cudaSuccess)
            return -cuda_fail(e, "gemv_q6k_mma_kernel occupancy");
        blocks_per_sm[dev] = n > 0 ? n : 1;
    }
    return sm_count() * blocks_per_sm[dev];
}

template <int S, int W, bool kStaged, int TP = 1> int q6k_pair_slots() {
    static int blocks_per_sm[64] = {};
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    constexpr int smem = PairLayout<S, W, kStaged, TP>::kTotal + 128;
    std::lock_guard<std::mutex> guard(lock);
    if (!blocks_per_sm[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_q6k_pair_kernel<S, W, kStaged, TP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess)
            return -cuda_fail(e, "gemv_q6k_pair_kernel attribute");
        int n = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_q6k_pair_kernel<S, W, kStaged, TP>, 32 * W + 32,
                                                          smem);
        if (e != cudaSuccess)
            return -cuda_fail(e, "gemv_q6k_pair_kernel occupancy");
        blocks_per_sm[dev] = n > 0 ? n : 1;
    }
    return sm_count() * blocks_per_sm[dev];
}

template <int NT, bool kStaged = false> int launch_q4k(const MmaParams& p, uint32_t grid, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreadsQ);
    cfg.dynamicSmemBytes = LayoutQ4<kStaged, NT>::kTotal + 128;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    TraceScope trace(KB200_KERNEL_GEMV_Q4K_MMA, stream);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_q4k_mma_kernel<NT, kStaged>, p);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "gemv_q4k_mma_kernel launch");
}

}  // namespace

void clear_gemv_fixups() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return;
    FixupTable& t = fixups();
    std::lock_guard<std::mutex> guard(t.lock);
    cudaDeviceSynchronize();
    for (auto& [key, f] : t.table)
        if (key.first == dev && f.ctas)
            cudaMemset(f.partials, 0, size_t(f.ctas) * kSlotFloats * sizeof(unsigned long long));
    cudaDeviceSynchronize();
}

bool q6k_mma_enabled() {
    static const bool on = [] {
        const char* s = std::getenv("KB200_GEMV_Q6K_MMA");
        return !s || std::atoi(s) != 0;
    }();
    return on;
}

bool mma_eligible(const kb200_gemv_job& j) {
    if (!aligned(j.weights, 16) || j.row_bytes % 16 || j.in % 256 || j.stride > 0xffffffffu || !encode_fn())
        return false;
    if (j.encoding == KB200_Q4_K)
        return j.row_bytes >= size_t(j.in) / 256 * 144;
    if (j.encoding == KB200_Q6_K)
        return q6k_mma_enabled() && j.row_bytes >= size_t(j.in) / 256 * kQ6Block;
    return false;
}

// Fills q with one region per distinct input of the launch's jobs (pointer,
// length and rows), points each job at its region of the staging buffer and
// returns true, or returns false (and stages nothing) when the regions do not
// fit the buffer. Layout: Q4_K records per block (q4k) or Q6_K pair-layout
// chunks of 8 blocks.
bool stage_inputs(MmaParams& p, uint8_t* staging, StageQuantParams& q, bool q4k) {
    std::memset(&q, 0, sizeof(q));
    size_t used = 0;
    for (uint32_t m = 0; m < p.count; ++m) {
        MmaJob& d = p.jobs[m];
        uint32_t r = 0;
        while (r < q.count && !(q.regions[r].x == d.input && q.regions[r].in == d.in && q.regions[r].rows == d.rows
                                && q.regions[r].group_rows == d.group_rows))
            ++r;
        if (r == q.count) {
            const size_t blocks = d.in / 256;
            const size_t bytes = q4k ? blocks * size_t(q4k_record_bytes(int(d.rows)))
                                     : size_t(d.row_groups) * ((blocks + kQ6Chunk - 1) / kQ6Chunk)
                                           * size_t(pair_chunk_bytes(int(d.group_rows)));
            if (used + bytes > kStagingBytes) {
                for (uint32_t k = 0; k < p.count; ++k)
                    p.jobs[k].staged = nullptr;
                return false;
            }
            StageQuantRegion& g = q.regions[q.count++];
            g.x = d.input;
            g.dst = staging + used;
            g.in = d.in;
            g.rows = d.rows;
            g.group_rows = d.group_rows;
            g.first_item = q.items;
            q.items += d.in / 256 * d.rows;
            used += bytes;
        }
        d.staged = q.regions[r].dst;
    }
    if (q.items == 0)
        for (uint32_t k = 0; k < p.count; ++k)
            p.jobs[k].staged = nullptr;
    return q.items > 0;
}

int launch_stage_quant(const StageQuantParams& q, cudaStream_t stream, bool q4k) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min((q.items + 3) / 4, uint32_t(sm_count()) * 8u));  // warp per item, grid-stride
    cfg.blockDim = dim3(128);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    TraceScope trace(q4k ? KB200_KERNEL_Q4K_QUANT : KB200_KERNEL_PAIR_QUANT, stream);
    const cudaError_t e = q4k ? cudaLaunchKernelEx(&cfg, q4k_quant_kernel, q) : cudaLaunchKernelEx(&cfg, pair_quant_kernel, q);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, q4k ? "q4k_quant_kernel launch" : "pair_quant_kernel launch");
}

// Q6_K: 16-row tiles, units of (tile, chunk of 8 blocks), up to 8 input rows
// per pass (more rows become row groups), balanced split when whole tiles
// would leave a tenth of the CTA slots idle. 1-2 rows run on the pair
// kernel, with the activations quantised once per launch into the stream's
// staging buffer when it has one and they fit.
int launch_q6k_mma(const std::vector<const kb200_gemv_job*>& jobs, cudaStream_t stream, const PeerOut* peer,
                   bool synchronous) {
    auto encode = encode_fn();
    if (!encode)
        return fail(KB200_CUDA, "cuTensorMapEncodeTiled unavailable");
    // Rows per pass: up to 4 in one n-tile, up to 8 in two.
    int max_rows = 1;
    for (const auto* j : jobs)
        max_rows = std::max(max_rows, int(std::min(j->rows, uint32_t(KB200_BATCH_ROWS))));
    const int nt = max_rows <= 4 ? 1 : 2;
    // 1-2 rows: the paired-sub-block kernel (2 rows per pass). 3-4 rows: the
    // same kernel with two token pairs per pass, 5-8 rows with four (one CTA
    // of eight consumer warps per SM), when the activations can be staged;
    // else the 4/8-row kernel.
    const bool pair = max_rows <= 2 && tuning().q6_pair;
    // Ring depth: 2 stages (three CTAs per SM) for the pair kernel when no job
    // is longer than 64 super-blocks (more warps for short, launch-bound K),
    // else 3 (two CTAs per SM, deeper ring for long K); forced by the tuning.
    uint32_t max_in = 0;
    for (const auto* j : jobs)
        max_in = std::max(max_in, j->in);
    const bool two_stage = nt == 1
                           && (tuning().q6_stages == 2 || (tuning().q6_stages == 0 && pair && max_in <= 16384));
    uint8_t* staging = max_rows <= 8 && tuning().q6_pair && tuning().q6_staged ? staging_for(stream) : nullptr;
    const Fixup* fixup = tuning().balanced ? fixup_for(stream) : nullptr;
    // Both pair kernels are set up on the first call (which may be the only
    // one outside graph capture), whichever this launch takes.
    const int pair_slots = !pair ? 0 : two_stage ? q6k_pair_slots<2, 4, false>() : q6k_pair_slots<3, 4, false>();
    const int pair_slots_staged = !pair ? 0 : two_stage ? q6k_pair_slots<2, 4, true>() : q6k_pair_slots<3, 4, true>();
    const bool eight = max_rows > 4;  // 5-8 rows: four token pairs per pass
    const int quad_slots = !pair && staging ? (eight ? q6k_pair_slots<2, 8, true, 4>() : q6k_pair_slots<2, 4, true, 2>()) : 0;
    if (pair_slots < 0 || pair_slots_staged < 0 || quad_slots < 0)
        return -std::min(pair_slots, std::min(pair_slots_staged, quad_slots));
    const int quad_rows = eight ? 8 : 4;
    for (size_t first = 0; first < jobs.size(); first += kMaxJobsQ) {
        const size_t n = std::min(jobs.size() - first, size_t(kMaxJobsQ));
        // 4- or 8-row passes when this batch's distinct inputs fit the staging buffer.
        bool quad = false;
        if (!pair && staging) {
            size_t bytes = 0;
            for (size_t m = 0; m < n; ++m) {
                const auto& j = *jobs[first + m];
                bool seen = false;
                for (size_t k = 0; k < m && !seen; ++k)
                    seen = jobs[first + k]->input == j.input && jobs[first + k]->in == j.in && jobs[first + k]->rows == j.rows;
                if (!seen)
                    bytes += size_t((j.rows + quad_rows - 1) / quad_rows) * ((j.in / 256 + kQ6Chunk - 1) / kQ6Chunk)
                             * size_t(pair_chunk_bytes(quad_rows));
            }
            quad = bytes <= kStagingBytes;
        }
        const uint32_t group_rows = pair ? 2u : quad ? uint32_t(quad_rows) : uint32_t(4 * nt);
        MmaParams p;
        std::memset(&p, 0, sizeof(p));
        p.watchdog = watchdog_word();
        p.tile_rows = kQ6Rows;
        if (peer)
            p.peer = *peer;
        uint32_t tiles = 0, units = 0;
        for (size_t m = 0; m < n; ++m) {
            const auto& j = *jobs[first + m];
            MmaJob& d = p.jobs[m];
            // Rows as u64 words (the pitch is a multiple of 16 bytes); one box
            // is 8 blocks (210 words) of 16 rows.
            const cuuint64_t dims[2] = {j.row_bytes / 8, j.columns};
            const cuuint64_t strides[1] = {j.row_bytes};
            const cuuint32_t box[2] = {kQ6Chunk * kQ6Block / 8, kQ6Rows};
            const cuuint32_t estr[2] = {1, 1};
            const CUresult r = encode(&d.map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(j.weights), dims,
                                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS)
                return fail(KB200_INVALID, "cuTensorMapEncodeTiled rejected a Q6_K job");
            d.input = j.input;
            d.output = j.output;
            d.status = j.status;
            d.stride = uint32_t(j.stride);
            d.in = j.in;
            d.columns = j.columns;
            d.rows = j.rows;
            d.nblocks = (j.in / 256 + kQ6Chunk - 1) / kQ6Chunk;  // units (chunks) per tile
            d.group_rows = group_rows;
            d.row_groups = (j.rows + group_rows - 1) / group_rows;
            d.first_tile = tiles;
            d.first_unit = units;
            const uint32_t job_tiles = (j.columns + kQ6Rows - 1) / kQ6Rows * d.row_groups;
            tiles += job_tiles;
            units += job_tiles * d.nblocks;
        }
        p.count = uint32_t(n);
        p.total_tiles = tiles;
        // In a synchronous call nothing ahead on the stream hides the
        // quantisation kernel: 1-2 rows are staged there only where each CTA
        // would otherwise quantise more than two activation windows (the
        // host-span q,k,v and o launches of a 70B layer quantise per CTA;
        // [down] is staged). 3-8 rows are always staged (their other kernel
        // is far slower).
        bool worth = true;
        if (pair && synchronous) {
            const int win_rows = std::min(max_rows, 2);
            const int window = pair_segment_blocks(win_rows, two_stage ? pair_seg_budget<2>() : pair_seg_budget<3>());
            const uint64_t cta_units = (uint64_t(units) + uint64_t(pair_slots_staged) - 1) / uint64_t(pair_slots_staged);
            worth = cta_units * kQ6Chunk > 2u * uint64_t(window);
        }
        StageQuantParams q;
        const bool staged = staging && (pair || quad) && worth && stage_inputs(p, staging, q, false);
        if (quad && !staged)  // only a batch without any super-block gets here
            return fail(KB200_INVALID, "Q6_K jobs without input values");
        int slots = quad     ? quad_slots
                    : !pair  ? (nt == 2 ? q6k_slots<2, 2>() : two_stage ? q6k_slots<1, 2>() : q6k_slots<1, 3>())
                    : staged ? pair_slots_staged : pair_slots;
        if (slots <= 0)
            return -slots;
        if (tuning().ctas_per_sm > 0)
            slots = std::min(slots, sm_count() * tuning().ctas_per_sm);
        const uint64_t waves = (tiles + uint64_t(slots) - 1) / uint64_t(slots);
        const bool ragged = uint64_t(tiles) * 10 < waves * uint64_t(slots) * 9;
        const bool balanced = fixup && fixup->ctas >= uint32_t(slots) && ragged
                              && uint64_t(units) >= uint64_t(tuning().q6_min_units) * uint64_t(slots);
        uint32_t grid = std::min(tiles, uint32_t(slots));
        if (balanced) {
            grid = std::min(units, uint32_t(slots));
            p.total_units = units;
            p.partials = fixup->partials;
        }
        if (staged)
            if (const int st = launch_stage_quant(q, stream, false))
                return st;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(quad && eight ? 32 * 8 + 32 : kThreadsQ);
        cfg.dynamicSmemBytes = (quad && eight ? PairLayout<2, 8, true, 4>::kTotal
                                : quad      ? PairLayout<2, 4, true, 2>::kTotal
                                : !pair     ? (nt == 2      ? Q6Layout<2, 2>::kTotal
                                               : two_stage ? Q6Layout<1, 2>::kTotal
                                                           : Q6Layout<1, 3>::kTotal)
                                : staged    ? (two_stage ? PairLayout<2, 4, true>::kTotal : PairLayout<3, 4, true>::kTotal)
                                            : (two_stage ? PairLayout<2, 4>::kTotal : PairLayout<3, 4>::kTotal))
                               + 128;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        TraceScope trace(pair || quad ? KB200_KERNEL_GEMV_Q6K_PAIR : KB200_KERNEL_GEMV_Q6K_MMA, stream);
        cudaError_t e;
        if (quad)
            e = eight ? cudaLaunchKernelEx(&cfg, gemv_q6k_pair_kernel<2, 8, true, 4>, p)
                      : cudaLaunchKernelEx(&cfg, gemv_q6k_pair_kernel<2, 4, true, 2>, p);
        else if (pair && staged)
            e = two_stage ? cudaLaunchKernelEx(&cfg, gemv_q6k_pair_kernel<2, 4, true>, p)
                          : cudaLaunchKernelEx(&cfg, gemv_q6k_pair_kernel<3, 4, true>, p);
        else if (pair)
            e = two_stage ? cudaLaunchKernelEx(&cfg, gemv_q6k_pair_kernel<2, 4, false>, p)
                          : cudaLaunchKernelEx(&cfg, gemv_q6k_pair_kernel<3, 4, false>, p);
        else
            e = nt == 2     ? cudaLaunchKernelEx(&cfg, gemv_q6k_mma_kernel<2, 2>, p)
                : two_stage ? cudaLaunchKernelEx(&cfg, gemv_q6k_mma_kernel<1, 2>, p)
                            : cudaLaunchKernelEx(&cfg, gemv_q6k_mma_kernel<1, 3>, p);
        if (e != cudaSuccess)
            return cuda_fail(e, "gemv_q6k_mma_kernel launch");
    }
    return KB200_OK;
}

int launch_q4k_mma(const std::vector<const kb200_gemv_job*>& jobs, cudaStream_t stream, const PeerOut* peer,
                   bool synchronous) {
    auto encode = encode_fn();
    if (!encode)
        return fail(KB200_CUDA, "cuTensorMapEncodeTiled unavailable");
    // Rows per pass: up to 4 in one n-tile, up to 8 in two.
    int max_rows = 1;
    for (const auto* j : jobs)
        max_rows = std::max(max_rows, int(std::min(j->rows, uint32_t(KB200_BATCH_ROWS))));
    const int nt = max_rows <= 4 ? 1 : 2;
    const uint32_t group_rows = uint32_t(4 * nt);
    int slots = nt == 1 ? kernel_slots<1>() : kernel_slots<2>();
    if (slots <= 0)
        return -slots;
    // Activations quantised once per launch (64-row tiles, one row group)
    // when the staged kernel fits as many CTAs per SM (both are set up on
    // the first call, which may be the only one outside graph capture).
    uint8_t* staging = nullptr;
    if (tuning().q4_staged) {
        const int staged_slots = nt == 1 ? kernel_slots<1, true>() : kernel_slots<2, true>();
        if (staged_slots <= 0)
            return -staged_slots;
        if (staged_slots == slots)
            staging = staging_for(stream);
    }
    if (tuning().ctas_per_sm > 0)
        slots = std::min(slots, sm_count() * tuning().ctas_per_sm);
    const Fixup* fixup = tuning().balanced ? fixup_for(stream) : nullptr;
    for (size_t first = 0; first < jobs.size(); first += kMaxJobsQ) {
        const size_t n = std::min(jobs.size() - first, size_t(kMaxJobsQ));
        int tokens = 1;
        uint64_t units64 = 0;
        for (size_t m = 0; m < n; ++m) {
            const auto& j = *jobs[first + m];
            tokens = std::max(tokens, int(std::min(j.rows, group_rows)));
            units64 += uint64_t((j.columns + 63) / 64) * ((j.rows + group_rows - 1) / group_rows) * (j.in / 256);
        }
        if (segment_blocks(tokens, kStageUnits / 64) == 0)
            return fail(KB200_UNSUPPORTED, "activation segment too small for this many rows");
        // Whole tiles: the tallest of 64/32/16 rows that still gives every
        // CTA slot a tile; shorter tiles split K among the warps instead. A
        // tile height is only allowed if one stage of activations (128/R
        // super-blocks for every token) fits the segment buffer.
        uint32_t R = 64;
        uint64_t rr_tiles = 0;
        for (uint32_t cand : {64u, 32u, 16u}) {
            if (segment_blocks(tokens, kStageUnits / int(cand)) == 0)
                break;
            R = cand;
            rr_tiles = 0;
            for (size_t m = 0; m < n; ++m) {
                const auto& j = *jobs[first + m];
                rr_tiles += (j.columns + cand - 1) / cand * ((j.rows + group_rows - 1) / group_rows);
            }
            if (rr_tiles >= uint64_t(slots))
                break;
        }
        // Balanced split (64-row tiles, the same number of units per CTA)
        // when whole tiles would leave more than a tenth of the CTA slots of
        // their waves idle and every CTA gets enough units to pay for the
        // fixup of its cut tiles.
        const uint64_t waves = (rr_tiles + slots - 1) / uint64_t(slots);
        const bool ragged = rr_tiles * 10 < waves * uint64_t(slots) * 9;
        const bool balanced = fixup && fixup->ctas >= uint32_t(slots) && ragged
                              && units64 >= uint64_t(tuning().min_units) * uint64_t(slots) && units64 < (1ull << 31);
        if (balanced)
            R = 64;
        MmaParams p;
        std::memset(&p, 0, sizeof(p));
        p.watchdog = watchdog_word();
        p.tile_rows = R;
        if (peer)
            p.peer = *peer;
        p.prefetch = tuning().prefetch;
        uint32_t tiles = 0, units = 0;
        for (size_t m = 0; m < n; ++m) {
            const auto& j = *jobs[first + m];
            MmaJob& d = p.jobs[m];
            const cuuint64_t dims[3] = {18, j.in / 256, j.columns};
            const cuuint64_t strides[2] = {144, j.row_bytes};
            const cuuint32_t box[3] = {18, 1, R};
            const cuuint32_t estr[3] = {1, 1, 1};
            const CUresult r = encode(
                &d.map,
                CU_TENSOR_MAP_DATA_TYPE_UINT64,
                3,
                const_cast<void*>(j.weights),
                dims,
                strides,
                box,
                estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE
            );
            if (r != CUDA_SUCCESS)
                return fail(KB200_INVALID, "cuTensorMapEncodeTiled rejected a Q4_K job");
            d.input = j.input;
            d.output = j.output;
            d.status = j.status;
            d.stride = uint32_t(j.stride);
            d.in = j.in;
            d.columns = j.columns;
            d.rows = j.rows;
            d.nblocks = j.in / 256;
            d.group_rows = group_rows;
            d.row_groups = (j.rows + group_rows - 1) / group_rows;
            d.first_tile = tiles;
            d.first_unit = units;
            const uint32_t job_tiles = (j.columns + R - 1) / R * d.row_groups;
            tiles += job_tiles;
            units += job_tiles * d.nblocks;
        }
        p.count = uint32_t(n);
        p.total_tiles = tiles;
        uint32_t grid = std::min(tiles, uint32_t(slots));
        if (balanced) {
            grid = std::min(units, uint32_t(slots));
            p.total_units = units;
            p.partials = fixup->partials;
        }
        // Staged only when a CTA would quantise more than once: its share of
        // units is longer than the activation segment holds (then every CTA
        // re-quantises the same activations). Otherwise each CTA quantises
        // once, and the quantisation kernel (which lets the GEMV launch only
        // when done) would add its latency to the launch: measured on the
        // config-2 stack, [gate, up] 15.8 -> 18.2 us and [down] 12.4 -> 14.8 us.
        StageQuantParams q;
        bool one_group = true;
        for (uint32_t m = 0; m < p.count; ++m)
            one_group = one_group && p.jobs[m].row_groups == 1;
        const uint64_t units_per_cta = (uint64_t(units) + grid - 1) / grid;
        // Synchronous calls: only where a CTA would quantise more than twice.
        const bool requantises = units_per_cta > uint64_t(segment_blocks(tokens, kStageUnits / int(R))) * (synchronous ? 2u : 1u);
        const bool staged = staging && R == 64 && one_group && requantises && stage_inputs(p, staging, q, true);
        if (staged)
            if (const int st = launch_stage_quant(q, stream, true))
                return st;
        const int s = nt == 2 ? (staged ? launch_q4k<2, true>(p, grid, stream) : launch_q4k<2>(p, grid, stream))
                      : staged ? launch_q4k<1, true>(p, grid, stream) : launch_q4k<1>(p, grid, stream);
        if (s)
            return s;
    }
    return KB200_OK;
}

int launch_mma(const std::vector<const kb200_gemv_job*>& jobs, cudaStream_t stream, const PeerOut* peer,
               bool synchronous) {
    if (jobs.empty())
        return KB200_OK;
    if (peer && peer->world > 1 && (jobs.size() != 1 || jobs.front()->stride != jobs.front()->columns))
        return fail(KB200_INVALID, "a peer exchange takes one job with contiguous output rows");
    return jobs.front()->encoding == KB200_Q6_K ? launch_q6k_mma(jobs, stream, peer, synchronous)
                                                : launch_q4k_mma(jobs, stream, peer, synchronous);
}

}  // namespace kb200
