// Layer math around the quantized path, on the device: RMSNorm, L2 norm,
// RoPE, cached (decode) attention and the gated delta-net step.
//
// The reference runs these on the host (rms_norm / l2_norm / rope / attend /
// delta_rule, services/hikari/inference_worker/src/models/text/
// gguf_weights.cpp:639-818, driven by AttentionLayer and DeltaNetLayer,
// qwen_layers.cpp:74-330) unless its DenseCompute takes attend_cached /
// delta_step (dense_compute.hpp:275-330; the reference's CUDA versions are
// cached_attention_kernel, delta_conv_kernel, delta_l2_kernel and
// delta_heads_kernel, h3_compute.cu:392-630). Semantics follow the host code:
// sums of squares in double, the norm scale in float, RoPE angles formed by
// repeated float multiplication, softmax over max-subtracted scores.
//
// B200 layout of the two heavy kernels:
//   attention  one CTA per (query row, KV head, segment of 128 keys) serves
//              all query heads of the KV head's group, so every key and value
//              row is read from HBM once per group instead of once per head.
//              Each warp stages 32 key rows in shared memory (one coalesced
//              row per load, all 32 in flight), scores them one key per lane
//              (exponentials one per lane, not one per key), then adds the
//              32 value rows, several in flight, with lanes owning dim / 32
//              contiguous dims (coalesced rows). Segments are combined by a
//              second kernel.
//   delta net  one CTA per value head with the head's dim x dim state in
//              shared memory for the whole step (read and written once per
//              step, not once per row); thread j owns state column j.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "kb200_host.hpp"

namespace kb200 {
namespace {

// ------------------------------------------------------------------ norms
// Block-wide double sum; every thread receives it. `shared` holds 32 doubles.
__device__ double block_sum_f64(double v, double* shared) {
    for (int o = 16; o; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warps = (blockDim.x + 31) / 32;
    __syncthreads();
    if ((threadIdx.x & 31) == 0)
        shared[threadIdx.x / 32] = v;
    __syncthreads();
    double total = 0;
    for (int w = 0; w < warps; ++w)
        total += shared[w];
    return total;
}

// One CTA per row: rms_norm (weight non-null) or its unweighted form, then
// times `post` (the L2 norm's 1/sqrt(width); 1 otherwise).
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* x, const float* weight, size_t width, float eps,
                                                       float post, float* out, unsigned* status) {
    __shared__ double shared[32];
    const float* row = x + size_t(blockIdx.x) * width;
    float* dst = out + size_t(blockIdx.x) * width;
    double sum = 0;
    for (size_t i = threadIdx.x; i < width; i += blockDim.x)
        sum += double(row[i]) * row[i];
    sum = block_sum_f64(sum, shared);
    const float scale = 1.f / sqrtf(float(sum / double(width)) + eps);
    bool finite = true;
    for (size_t i = threadIdx.x; i < width; i += blockDim.x) {
        float v = weight ? row[i] * scale * weight[i] : row[i] * scale;
        if (post != 1.f)
            v *= post;
        dst[i] = v;
        finite = finite && isfinite(v);
    }
    if (status && !finite)
        atomicOr(status, 1u);
}

// ------------------------------------------------------------------- rope
// One thread per (row, head, pair i < rotary / 2): theta_i = (position + row)
// * scale^i with the product formed left to right in float, as the host loop
// does (theta *= theta_scale per pair).
__global__ void rope_kernel(float* x, size_t rows, size_t row_width, size_t width, size_t rotary, size_t position,
                            float theta_scale) {
    const size_t half = rotary / 2, heads = row_width / width;
    const size_t n = rows * heads * half;
    for (size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < n; idx += size_t(gridDim.x) * blockDim.x) {
        const size_t i = idx % half, head = (idx / half) % heads, r = idx / (half * heads);
        float theta = float(position + r);
        for (size_t k = 0; k < i; ++k)
            theta *= theta_scale;
        float s, c;
        sincosf(theta, &s, &c);
        float* at = x + r * row_width + head * width;
        const float a = at[i], b = at[i + half];
        at[i] = a * c - b * s;
        at[i + half] = a * s + b * c;
    }
}

// -------------------------------------------------------------- attention
constexpr int kAttnWarps = 4;
constexpr int kAttnSegment = 32 * kAttnWarps;  // keys per CTA: one 32-key chunk per warp
constexpr int kAttnMaxGE = 64;     // group heads x dims per lane held in registers
constexpr int kAttnMaxG = 16;      // query heads per KV head

struct AttnParams {
    const float* q;       // [rows][heads][dim]
    const float* keys;    // [positions][kv_heads][dim]
    const float* values;  // same
    const uint32_t* selected;
    const uint32_t* offsets;
    float* partial;       // sums [rows][heads][segments][dim], then (max, total) [rows][heads][segments][2]
    uint32_t position, heads, kv_heads, dim, segments;
    uint32_t seg_len;     // keys per segment, a multiple of 32 * kAttnWarps
    float scale;
};

__device__ __forceinline__ void load_dims(const float* p, float (&v)[8], int E) {
    if (E == 8) {
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else if (E == 4) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
    } else {
        const float2 a = *reinterpret_cast<const float2*>(p);
        v[0] = a.x, v[1] = a.y;
    }
}

// E = dim / 32 (2, 4 or 8): dims [E lane, E lane + E) of a row belong to
// lane `lane` when value rows are added. G = query heads per KV head, at most
// GM (a power of two fixed at compile time, so the per-head state stays in
// registers). Shared
// memory: the group's queries [G][dim], then per warp half of its 32 key rows
// at a time, [32][dim/2 + 4] (the pad keeps lane t's reads of row t
// conflict-free), reused at the end as merge space.
template <int E, int GM>
__global__ void __launch_bounds__(32 * kAttnWarps) attend_kernel(const __grid_constant__ AttnParams p) {
    constexpr int D = 32 * E, H = D / 2, KP = H + 4;  // head dim, staged half, key row pitch
    constexpr int VU = E >= 8 ? 4 : 8;                // value rows in flight
    extern __shared__ __align__(16) float smem_f[];
    const int row = blockIdx.x, kv = blockIdx.y, seg = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = int(p.heads / p.kv_heads);
    float* qs = smem_f;
    float* ks = smem_f + G * D + warp * 32 * KP;
    const uint32_t* chosen = p.selected ? p.selected + p.offsets[row] : nullptr;
    const int visible = int(p.selected ? p.offsets[row + 1] - p.offsets[row] : p.position + uint32_t(row) + 1u);
    const int begin = seg * int(p.seg_len), end = min(visible, begin + int(p.seg_len));
    const size_t stride = size_t(p.kv_heads) * D;  // floats between cache positions
    for (int i = threadIdx.x; i < G * D; i += blockDim.x)
        qs[i] = p.q[(size_t(row) * p.heads + size_t(kv) * G) * D + i];
    __syncthreads();

    float m[GM], l[GM], acc[GM][E];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        m[g] = -INFINITY, l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e)
            acc[g][e] = 0.f;
    }
    for (int c0 = begin + 32 * warp; c0 < end; c0 += 32 * kAttnWarps) {
        const int n = min(32, end - c0);
        // Scores: lane t takes key c0 + t, over the two halves of the dims.
        const bool live = lane < n;
        float s[GM];
#pragma unroll
        for (int g = 0; g < GM; ++g)
            s[g] = 0.f;
        const float* mine = ks + lane * KP;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            // Half of each key row into shared memory: lanes cover the half
            // row in 16-byte pieces, 32 / (H / 4) rows per warp load, every
            // load in flight before the first store.
            constexpr int PIECES = H / 4, RPL = 32 / PIECES;
            const int piece = lane % PIECES, sub = lane / PIECES;
#pragma unroll 8
            for (int r0 = 0; r0 < 32; r0 += RPL) {
                const int r = r0 + sub;
                if (r < n) {
                    const float* key = p.keys + size_t(chosen ? chosen[c0 + r] : uint32_t(c0 + r)) * stride
                                       + size_t(kv) * D + half * H;
                    *reinterpret_cast<float4*>(ks + r * KP + 4 * piece) = *reinterpret_cast<const float4*>(key + 4 * piece);
                }
            }
            __syncwarp();
#pragma unroll 4
            for (int d = 0; d < H; d += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(mine + d);
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (g >= G)
                        break;
                    const float4 q4 = *reinterpret_cast<const float4*>(qs + g * D + half * H + d);
                    s[g] = fmaf(q4.x, k4.x, s[g]);
                    s[g] = fmaf(q4.y, k4.y, s[g]);
                    s[g] = fmaf(q4.z, k4.z, s[g]);
                    s[g] = fmaf(q4.w, k4.w, s[g]);
                }
            }
            __syncwarp();
        }
        // Online softmax per head over the chunk.
        float pr[GM];
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            if (g >= G)
                break;
            const float score = live ? s[g] * p.scale : -INFINITY;
            float cm = score;
            for (int o = 16; o; o >>= 1)
                cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
            const float mn = fmaxf(m[g], cm);
            const float corr = expf(m[g] - mn);  // 0 on the first chunk (m = -inf)
            pr[g] = live ? expf(score - mn) : 0.f;
            float ps = pr[g];
            for (int o = 16; o; o >>= 1)
                ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l[g] = l[g] * corr + ps;
            m[g] = mn;
#pragma unroll
            for (int e = 0; e < E; ++e)
                acc[g][e] *= corr;
        }
        // The chunk's value rows, VU rows in flight at a time; lane owns dims
        // [E lane, E lane + E) of each (coalesced rows).
        for (int j0 = 0; j0 < n; j0 += VU) {
            float v[VU][8];
#pragma unroll
            for (int u = 0; u < VU; ++u) {
                const int tj = c0 + min(j0 + u, n - 1);
                const float* vr = p.values + size_t(chosen ? chosen[tj] : uint32_t(tj)) * stride + size_t(kv) * D;
                load_dims(vr + size_t(E) * lane, v[u], E);
            }
#pragma unroll
            for (int u = 0; u < VU; ++u) {
                if (j0 + u >= n)
                    break;
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (g >= G)
                        break;
                    const float w = __shfl_sync(0xffffffffu, pr[g], j0 + u);
#pragma unroll
                    for (int e = 0; e < E; ++e)
                        acc[g][e] = fmaf(w, v[u][e], acc[g][e]);
                }
            }
        }
    }
    // Merge the warps: each writes (m, l) and its dims, then the CTA combines.
    __syncthreads();
    float* ms = smem_f;                     // [warps][G]
    float* ls = ms + kAttnWarps * G;        // [warps][G]
    float* as = ls + kAttnWarps * G;        // [warps][G][dim]
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        if (g >= G)
            break;
        if (lane == 0)
            ms[warp * G + g] = m[g], ls[warp * G + g] = l[g];
#pragma unroll
        for (int e = 0; e < E; ++e)
            as[(warp * G + g) * D + E * lane + e] = acc[g][e];
    }
    __syncthreads();
    const size_t entries = size_t(gridDim.x) * p.heads * p.segments;
    for (int i = threadIdx.x; i < G * (D + 2); i += blockDim.x) {
        const int g = i / (D + 2), d = i % (D + 2);
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w)
            if (ls[w * G + g] > 0.f)
                M = fmaxf(M, ms[w * G + g]);
        float sum = 0.f;
        for (int w = 0; w < kAttnWarps; ++w)
            if (ls[w * G + g] > 0.f) {
                const float f = expf(ms[w * G + g] - M);
                sum += (d == 0 ? 0.f : d == 1 ? ls[w * G + g] : as[(w * G + g) * D + d - 2]) * f;
            }
        const size_t entry = (size_t(row) * p.heads + size_t(kv) * G + g) * p.segments + seg;
        if (d >= 2)
            p.partial[entry * D + d - 2] = sum;
        else
            p.partial[entries * D + entry * 2 + d] = d == 0 ? M : sum;
    }
}

// out[row][head][d] = sum_seg acc * e^(m - M) / sum_seg l * e^(m - M), over
// segments that saw a key. One CTA of 256 threads per (row, head): the
// segment weights e^(m - M) / total in parallel into shared memory, then
// threads = (dim / 4 float4 columns) x (groups of segments), a group's sums
// added through shared memory.
__global__ void __launch_bounds__(256) attend_combine_kernel(const float* partial, float* out, uint32_t heads,
                                                             uint32_t dim, uint32_t segments) {
    extern __shared__ __align__(16) float cw[];  // [segments] weights, then [groups][dim] sums
    __shared__ float red[8];
    const size_t rh = size_t(blockIdx.x) * heads + blockIdx.y;
    const size_t entries = size_t(gridDim.x) * heads * segments;
    const float* ml = partial + entries * dim + rh * segments * 2;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float M = -INFINITY;
    for (uint32_t z = tid; z < segments; z += blockDim.x)
        if (ml[2 * z + 1] > 0.f)
            M = fmaxf(M, ml[2 * z]);
    for (int o = 16; o; o >>= 1)
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (lane == 0)
        red[warp] = M;
    __syncthreads();
    M = red[0];
    for (int w = 1; w < int(blockDim.x >> 5); ++w)
        M = fmaxf(M, red[w]);
    __syncthreads();
    float total = 0.f;
    for (uint32_t z = tid; z < segments; z += blockDim.x) {
        const float l = ml[2 * z + 1];
        const float f = l > 0.f ? expf(ml[2 * z] - M) : 0.f;
        cw[z] = f;
        total += l * f;
    }
    for (int o = 16; o; o >>= 1)
        total += __shfl_xor_sync(0xffffffffu, total, o);
    if (lane == 0)
        red[warp] = total;
    __syncthreads();
    total = 0.f;
    for (int w = 0; w < int(blockDim.x >> 5); ++w)
        total += red[w];
    const int cols = int(dim / 4), groups = int(blockDim.x) / cols;
    const int col = tid % cols, grp = tid / cols;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    if (grp < groups) {
        const float* acc = partial + rh * segments * dim + 4 * col;
#pragma unroll 4
        for (uint32_t z = grp; z < segments; z += groups) {
            const float w = cw[z];
            const float4 a = *reinterpret_cast<const float4*>(acc + size_t(z) * dim);
            sum.x = fmaf(w, a.x, sum.x), sum.y = fmaf(w, a.y, sum.y);
            sum.z = fmaf(w, a.z, sum.z), sum.w = fmaf(w, a.w, sum.w);
        }
    }
    float* gs = cw + ((segments + 3) & ~3u);
    __syncthreads();
    if (grp < groups)
        *reinterpret_cast<float4*>(gs + grp * dim + 4 * col) = sum;
    __syncthreads();
    for (uint32_t d = tid; d < dim; d += blockDim.x) {
        float v = 0.f;
        for (int g = 0; g < groups; ++g)
            v += gs[g * dim + d];
        out[rh * dim + d] = v / total;
    }
}

// -------------------------------------------------------------- delta net
__device__ __forceinline__ float sigmoid_f(float x) {
    return 1.f / (1.f + expf(-x));
}

__device__ __forceinline__ float silu_f(float x) {
    return x / (1.f + expf(-x));
}

__device__ __forceinline__ float softplus_f(float x) {
    return x > 20.f ? x : log1pf(expf(x));
}

struct DeltaParams {
    const float *qkv, *z, *alpha, *beta, *conv, *dt, *a, *norm;
    const float* history;  // [past][channels], oldest first
    float* next_history;   // [past][channels]
    float* mixed;          // [rows][channels] workspace
    float* state;          // [value_heads][dim][dim]
    float* output;         // [rows][value_heads * dim]
    uint32_t rows, channels, key_heads, value_heads, dim, kernel;
    float eps;
    int sigmoid_gate;
};

// Causal depthwise convolution with SiLU over all rows at once (sequence =
// history ++ rows), and the next history (the newest kernel - 1 inputs).
__global__ void delta_conv_kernel(const __grid_constant__ DeltaParams p) {
    const uint32_t past = p.kernel - 1, C = p.channels;
    const size_t total = size_t(p.rows) * C, hist = size_t(past) * C;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < (total > hist ? total : hist);
         i += size_t(gridDim.x) * blockDim.x) {
        if (i < hist) {
            const uint32_t k = uint32_t(i / C), c = uint32_t(i % C), src = p.rows + k;
            p.next_history[i] = src < past ? p.history[size_t(src) * C + c] : p.qkv[size_t(src - past) * C + c];
        }
        if (i < total) {
            const uint32_t r = uint32_t(i / C), c = uint32_t(i % C);
            const float* w = p.conv + size_t(c) * p.kernel;
            float sum = 0.f;
            for (uint32_t k = 0; k < past; ++k) {
                const int t = int(r) - int(past) + int(k);
                const float v = t < 0 ? p.history[size_t(int(past) + t) * C + c] : p.qkv[size_t(t) * C + c];
                sum += v * w[k];
            }
            sum += p.qkv[i] * w[past];
            p.mixed[i] = silu_f(sum);
        }
    }
}

// L2 norm of every q and k head of every row, in place: one CTA per (row,
// head of the 2 key_heads q and k heads).
__global__ void delta_l2_kernel(const __grid_constant__ DeltaParams p) {
    __shared__ double shared[32];
    float* x = p.mixed + size_t(blockIdx.x) * p.channels + size_t(blockIdx.y) * p.dim;
    double sum = 0;
    for (uint32_t d = threadIdx.x; d < p.dim; d += blockDim.x)
        sum += double(x[d]) * x[d];
    sum = block_sum_f64(sum, shared);
    // rms_norm(x, dim, eps / dim), then times 1/sqrt(dim) (l2_norm).
    const float scale = 1.f / sqrtf(float(sum / double(p.dim)) + p.eps / float(p.dim));
    const float post = 1.f / sqrtf(float(p.dim));
    for (uint32_t d = threadIdx.x; d < p.dim; d += blockDim.x)
        x[d] = x[d] * scale * post;
}

// One CTA per value head, thread j = state column j; the rows in order.
// kShared: the head's state lives in shared memory for the step.
template <bool kShared>
__global__ void __launch_bounds__(256) delta_heads_kernel(const __grid_constant__ DeltaParams p) {
    extern __shared__ float dyn[];
    __shared__ float q[256], k[256];
    __shared__ double shared[32];
    const uint32_t h = blockIdx.x, j = threadIdx.x, dim = p.dim, kh = h % p.key_heads;
    const size_t inner = size_t(p.value_heads) * dim;
    float* global_s = p.state + size_t(h) * dim * dim;
    float* s = kShared ? dyn : global_s;
    if (kShared)
        for (uint32_t i = 0; i < dim; ++i)
            s[i * dim + j] = global_s[i * dim + j];
    const float scale = 1.f / sqrtf(float(dim));
    for (uint32_t r = 0; r < p.rows; ++r) {
        const float* m = p.mixed + size_t(r) * p.channels;
        __syncthreads();
        q[j] = m[kh * dim + j] * scale;
        k[j] = m[p.key_heads * dim + kh * dim + j];
        const float v = m[2 * p.key_heads * dim + h * dim + j];
        __syncthreads();
        const float g = expf(softplus_f(p.alpha[size_t(r) * p.value_heads + h] + p.dt[h]) * p.a[h]);
        const float b = sigmoid_f(p.beta[size_t(r) * p.value_heads + h]);
        float delta = v;
        for (uint32_t i = 0; i < dim; ++i)
            delta -= s[i * dim + j] * g * k[i];
        delta *= b;
        float out = 0.f;
        for (uint32_t i = 0; i < dim; ++i) {
            const float value = s[i * dim + j] * g + k[i] * delta;
            s[i * dim + j] = value;
            out += value * q[i];
        }
        const double sum = block_sum_f64(double(out) * out, shared);
        const float normalized = out * (1.f / sqrtf(float(sum / double(dim)) + p.eps)) * p.norm[j];
        const float gate = p.z[size_t(r) * inner + size_t(h) * dim + j];
        p.output[size_t(r) * inner + size_t(h) * dim + j] = normalized * (p.sigmoid_gate ? sigmoid_f(gate) : silu_f(gate));
    }
    if (kShared)
        for (uint32_t i = 0; i < dim; ++i)
            global_s[i * dim + j] = s[i * dim + j];
}

}  // namespace
}  // namespace kb200

namespace kb200 {
namespace {

int launch_status(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, what);
}

// Shared memory of attend_kernel<E, GM> for G heads per KV head: queries and
// the warps' half key rows, or the merge space, whichever is larger.
constexpr size_t attend_smem(int E, int G) {
    return sizeof(float) * std::max(size_t(G) * 32 * E + size_t(kAttnWarps) * 32 * (16 * E + 4),
                                     size_t(kAttnWarps) * G * (32 * E + 2));
}

void attend_split(size_t rows, size_t position, size_t kv_heads, size_t target, uint32_t& segments,
                  uint32_t& seg_len);

// Launch with about two waves of CTAs over the SMs (the variant's occupancy,
// queried once per device), each segment a whole number of 128-key chunks.
template <int E, int GM> int launch_attend(AttnParams& p, size_t rows, size_t position, cudaStream_t stream) {
    static int blocks_per_sm[64] = {};
    static std::mutex lock;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64)
        return fail(KB200_UNSUPPORTED, "device index above 63");
    const size_t smem_max = attend_smem(E, GM);
    {
        std::lock_guard<std::mutex> guard(lock);
        if (!blocks_per_sm[dev]) {
            cudaError_t e = cudaFuncSetAttribute(attend_kernel<E, GM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 int(smem_max));
            int n = 0;
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attend_kernel<E, GM>, 32 * kAttnWarps, smem_max);
            if (e != cudaSuccess)
                return cuda_fail(e, "attend_kernel set-up");
            blocks_per_sm[dev] = n > 0 ? n : 1;
        }
    }
    const int G = int(p.heads / p.kv_heads);
    attend_split(rows, position, p.kv_heads, size_t(sm_count()) * blocks_per_sm[dev] * 2, p.segments, p.seg_len);
    attend_kernel<E, GM><<<dim3(unsigned(rows), p.kv_heads, p.segments), 32 * kAttnWarps, attend_smem(E, G), stream>>>(p);
    return launch_status("attend_kernel launch");
}

template <int E> int launch_attend_e(AttnParams& p, size_t rows, size_t position, cudaStream_t stream) {
    const uint32_t G = p.heads / p.kv_heads;
    if (G <= 1)
        return launch_attend<E, 1>(p, rows, position, stream);
    if (G <= 2)
        return launch_attend<E, 2>(p, rows, position, stream);
    if (G <= 4)
        return launch_attend<E, 4>(p, rows, position, stream);
    if (G <= 8 || E >= 8)
        return launch_attend<E, 8>(p, rows, position, stream);
    return launch_attend<E, (E >= 8 ? 8 : 16)>(p, rows, position, stream);
}

size_t attend_segments(size_t rows, size_t position) {
    return (position + rows + kAttnSegment - 1) / kAttnSegment;
}

// Segments of a launch: about `target` CTAs in all, each segment a whole
// number of 128-key chunks; at most attend_segments (the workspace bound).
void attend_split(size_t rows, size_t position, size_t kv_heads, size_t target, uint32_t& segments,
                  uint32_t& seg_len) {
    const size_t keys = position + rows, most = attend_segments(rows, position);
    const size_t want = std::max<size_t>(1, target / std::max<size_t>(1, rows * kv_heads));
    const size_t n = std::min(most, want);
    const size_t chunks = (keys + kAttnSegment - 1) / kAttnSegment;
    seg_len = uint32_t((chunks + n - 1) / n * kAttnSegment);
    segments = uint32_t((keys + seg_len - 1) / seg_len);
}

bool delta_shape_ok(uint32_t key_heads, uint32_t value_heads, uint32_t dim, uint32_t kernel) {
    return key_heads && value_heads && value_heads % key_heads == 0 && dim && dim <= 256 && dim % 32 == 0
           && kernel >= 1 && kernel <= 64;
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

int kb200_rms_norm(const float* x, const float* weight, size_t rows, size_t width, float eps, float* out,
                   unsigned* status, void* stream) {
    if (!rows)
        return KB200_OK;
    if (!x || !out || !width)
        return fail(KB200_INVALID, "null rows or zero width");
    if (rows > 0x7FFFFFFFu)
        return fail(KB200_UNSUPPORTED, "too many rows");
    if (out != x && overlap(out, rows * width * 4, x, rows * width * 4))
        return fail(KB200_ALIAS, "output partly overlaps the input");
    if (weight && overlap(out, rows * width * 4, weight, width * 4))
        return fail(KB200_ALIAS, "output overlaps the weight");
    TraceScope trace(KB200_KERNEL_RMS_NORM, static_cast<cudaStream_t>(stream));
    rms_norm_kernel<<<unsigned(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, weight, width, eps, 1.f, out,
                                                                                  status);
    return launch_status("rms_norm_kernel launch");
}

int kb200_l2_norm(const float* x, size_t rows, size_t width, float eps, float* out, void* stream) {
    if (!rows)
        return KB200_OK;
    if (!x || !out || !width)
        return fail(KB200_INVALID, "null rows or zero width");
    if (rows > 0x7FFFFFFFu)
        return fail(KB200_UNSUPPORTED, "too many rows");
    if (out != x && overlap(out, rows * width * 4, x, rows * width * 4))
        return fail(KB200_ALIAS, "output partly overlaps the input");
    TraceScope trace(KB200_KERNEL_RMS_NORM, static_cast<cudaStream_t>(stream));
    rms_norm_kernel<<<unsigned(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, nullptr, width, eps / float(width), 1.f / sqrtf(float(width)), out, nullptr);
    return launch_status("rms_norm_kernel launch");
}

int kb200_rope(float* x, size_t rows, size_t row_width, size_t width, size_t rotary, size_t position, float base,
               void* stream) {
    if (!rows)
        return KB200_OK;
    if (!x)
        return fail(KB200_INVALID, "null rows");
    // gguf_text_rope_shape (gguf_weights.cpp:683-686).
    if (!width || !rotary || rotary % 2 || rotary > width || !row_width || row_width % width)
        return fail(KB200_INVALID, "gguf_text_rope_shape");
    const float theta_scale = std::pow(base, -2.0f / float(rotary));
    const size_t n = rows * (row_width / width) * (rotary / 2);
    const unsigned grid = unsigned(std::min<size_t>((n + 255) / 256, size_t(sm_count()) * 8));
    TraceScope trace(KB200_KERNEL_ROPE, static_cast<cudaStream_t>(stream));
    rope_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, rows, row_width, width, rotary, position,
                                                                    theta_scale);
    return launch_status("rope_kernel launch");
}

int kb200_attend_supported(size_t heads, size_t kv_heads, size_t dim) {
    if (!heads || !kv_heads || heads % kv_heads || heads > 65535 || kv_heads > 65535)
        return 0;
    const size_t G = heads / kv_heads;
    if (dim != 64 && dim != 128 && dim != 256)
        return 0;
    return G <= size_t(kAttnMaxG) && G * (dim / 32) <= size_t(kAttnMaxGE) ? 1 : 0;
}

size_t kb200_attend_workspace_bytes(size_t rows, size_t position, size_t heads, size_t dim) {
    return rows * heads * attend_segments(rows, position) * (dim + 2) * sizeof(float);
}

int kb200_attend_cached(const float* q, const float* keys, const float* values, size_t rows, size_t position,
                        size_t heads, size_t kv_heads, size_t dim, float scale, const uint32_t* selected,
                        const uint32_t* offsets, float* out, void* workspace, size_t workspace_bytes, void* stream) {
    if (!kb200_attend_supported(heads, kv_heads, dim))
        return fail(KB200_UNSUPPORTED, "attention shape (heads per KV head, head dim 64/128/256)");
    if (!rows)
        return KB200_OK;
    if (!q || !keys || !values || !out || !workspace || (selected && !offsets))
        return fail(KB200_INVALID, "null pointer");
    if (rows > 65535 || position + rows > 0x7FFFFFFFu)
        return fail(KB200_UNSUPPORTED, "too many rows or positions");
    if (!aligned(keys, 16) || !aligned(values, 16))
        return fail(KB200_INVALID, "keys and values must be 16-byte aligned");
    const size_t need = kb200_attend_workspace_bytes(rows, position, heads, dim);
    if (workspace_bytes < need)
        return fail(KB200_NO_MEMORY, "attention workspace too small (kb200_attend_workspace_bytes)");
    if (overlap(out, rows * heads * dim * 4, q, rows * heads * dim * 4))
        return fail(KB200_ALIAS, "output overlaps the queries");
    auto s = static_cast<cudaStream_t>(stream);
    AttnParams p;
    p.q = q, p.keys = keys, p.values = values, p.selected = selected, p.offsets = offsets;
    p.partial = static_cast<float*>(workspace);
    p.position = uint32_t(position), p.heads = uint32_t(heads), p.kv_heads = uint32_t(kv_heads);
    p.dim = uint32_t(dim), p.scale = scale;
    {
        TraceScope trace(KB200_KERNEL_ATTEND, s);
        const int st = dim == 64    ? launch_attend_e<2>(p, rows, position, s)
                       : dim == 128 ? launch_attend_e<4>(p, rows, position, s)
                                    : launch_attend_e<8>(p, rows, position, s);
        if (st)
            return st;
    }
    TraceScope trace(KB200_KERNEL_ATTEND_COMBINE, s);
    const size_t combine_smem = (size_t((p.segments + 3) & ~3u) + 1024) * sizeof(float);
    attend_combine_kernel<<<dim3(unsigned(rows), unsigned(heads)), 256, combine_smem, s>>>(p.partial, out, p.heads,
                                                                                          p.dim, p.segments);
    return launch_status("attend_combine_kernel launch");
}

int kb200_delta_supported(uint32_t key_heads, uint32_t value_heads, uint32_t dim, uint32_t kernel) {
    return delta_shape_ok(key_heads, value_heads, dim, kernel) ? 1 : 0;
}

size_t kb200_delta_workspace_bytes(const kb200_delta_args* a) {
    if (!a || !delta_shape_ok(a->key_heads, a->value_heads, a->dim, a->kernel))
        return 0;
    const size_t channels = (2 * size_t(a->key_heads) + a->value_heads) * a->dim;
    return ((size_t(a->rows) + a->kernel - 1) * channels * sizeof(float) + 255) / 256 * 256;
}

int kb200_delta_step(const kb200_delta_args* a, void* workspace, size_t workspace_bytes, void* stream) {
    if (!a)
        return fail(KB200_INVALID, "null arguments");
    if (!delta_shape_ok(a->key_heads, a->value_heads, a->dim, a->kernel))
        return fail(KB200_UNSUPPORTED, "delta-net shape (dim a multiple of 32 up to 256, value heads a multiple "
                                       "of key heads)");
    if (!a->rows)
        return KB200_OK;
    if (!a->qkv || !a->z || !a->alpha || !a->beta || !a->conv || !a->dt || !a->a || !a->norm || !a->state
        || !a->output || (a->kernel > 1 && !a->history) || !workspace)
        return fail(KB200_INVALID, "null pointer");
    if (workspace_bytes < kb200_delta_workspace_bytes(a))
        return fail(KB200_NO_MEMORY, "delta-net workspace too small (kb200_delta_workspace_bytes)");
    const size_t channels = (2 * size_t(a->key_heads) + a->value_heads) * a->dim;
    if (channels > 0xFFFFFFFFu || size_t(a->rows) * channels > (size_t(1) << 40))
        return fail(KB200_UNSUPPORTED, "too many channels");
    auto s = static_cast<cudaStream_t>(stream);
    DeltaParams p;
    p.qkv = a->qkv, p.z = a->z, p.alpha = a->alpha, p.beta = a->beta, p.conv = a->conv, p.dt = a->dt, p.a = a->a;
    p.norm = a->norm, p.history = a->history, p.state = a->state, p.output = a->output;
    p.mixed = static_cast<float*>(workspace);
    p.next_history = p.mixed + size_t(a->rows) * channels;
    p.rows = a->rows, p.channels = uint32_t(channels), p.key_heads = a->key_heads, p.value_heads = a->value_heads;
    p.dim = a->dim, p.kernel = a->kernel, p.eps = a->eps, p.sigmoid_gate = a->sigmoid_gate;
    const size_t past_bytes = size_t(a->kernel - 1) * channels * sizeof(float);
    {
        TraceScope trace(KB200_KERNEL_DELTA_CONV, s);
        const size_t n = std::max(size_t(a->rows) * channels, size_t(a->kernel - 1) * channels);
        delta_conv_kernel<<<unsigned(std::min<size_t>((n + 255) / 256, size_t(sm_count()) * 8)), 256, 0, s>>>(p);
        if (const int st = launch_status("delta_conv_kernel launch"))
            return st;
    }
    if (past_bytes) {
        const cudaError_t e = cudaMemcpyAsync(a->history, p.next_history, past_bytes, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess)
            return cuda_fail(e, "delta-net history copy");
    }
    {
        TraceScope trace(KB200_KERNEL_DELTA_L2, s);
        delta_l2_kernel<<<dim3(a->rows, 2 * a->key_heads), a->dim, 0, s>>>(p);
        if (const int st = launch_status("delta_l2_kernel launch"))
            return st;
    }
    TraceScope trace(KB200_KERNEL_DELTA_HEADS, s);
    if (a->dim <= 128) {
        const size_t smem = size_t(a->dim) * a->dim * sizeof(float);
        static bool attr_set[64] = {};
        static std::mutex lock;
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> guard(lock);
        if (dev >= 0 && dev < 64 && !attr_set[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(delta_heads_kernel<true>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 128 * 4);
            if (e != cudaSuccess)
                return cuda_fail(e, "delta_heads_kernel attribute");
            attr_set[dev] = true;
        }
        delta_heads_kernel<true><<<a->value_heads, a->dim, smem, s>>>(p);
    } else {
        delta_heads_kernel<false><<<a->value_heads, a->dim, 0, s>>>(p);
    }
    return launch_status("delta_heads_kernel launch");
}

}  // extern "C"
