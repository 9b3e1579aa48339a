// One-shot all-reduce of fp32 partial sums over NVLink peer memory.
//
// Tensor-parallel decode adds the row-parallel projections' partial outputs
// across ranks twice per layer (after o and after down): T x hidden fp32,
// 32 KB at T = 1. At that size a library all-reduce is bound by its
// protocol's latency, not by NVLink bandwidth. Here every rank's buffer is
// mapped into every other rank's address space (CUDA IPC, one process per
// GPU), and one kernel does the exchange:
//
//   CTA c of every rank owns chunk c of the vector. It stores its chunk into
//   slot [rank] of every peer's receive area (plain peer stores over NVLink),
//   then publishes flag [rank][c] = epoch at each peer with a system-scope
//   release. It waits (acquire, bounded by a time limit) until every peer's
//   flag [src][c] in its own buffer shows the epoch, and sums the chunk over
//   ranks in rank order 0..N-1, so every rank gets the same bits.
//
// The epoch is the number of the call, counted on the device (a graph replay
// needs no new parameters; every rank makes the same calls). Receive areas
// and flags alternate between two banks by epoch parity: a rank's call k
// starts after its call k-1 finished, for which CTA 0 saw every peer's call
// k-1 flag, so every peer has finished call k-2 and reads bank (k-1)&1 at
// most; call k writes bank k&1.
//
// Buffer of one rank (same layout on every rank, zeroed at allocation):
//   flags  [2][kMaxRanks][kMaxCtas] u32   written by peers
//   epochs [kMaxCtas] u32                 this rank's call counters
//   data   [2][kMaxRanks][max_count] f32  written by peers
// No TMA and no multicast: peer memory is only touched by plain loads and
// stores.
#include <algorithm>
#include <cstring>

#include "kb200_device.cuh"
#include "kb200_host.hpp"

namespace kb200 {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 256;
constexpr int kArThreads = 256;
constexpr size_t kChunkFloats = 1024;
constexpr size_t kFlagsBytes = size_t(2) * kMaxRanks * kMaxCtas * 4;
constexpr size_t kEpochOff = kFlagsBytes;
constexpr size_t kDataOff = (kEpochOff + kMaxCtas * 4 + 255) / 256 * 256;
constexpr unsigned watchdog_peer = 16u;  // a peer's chunk never arrived

struct ArParams {
    uint8_t* peers[kMaxRanks];  // every rank's buffer, this rank's included
    float* data;                // in/out, count floats
    size_t count, max_count, per_cta;
    int rank, world;
    unsigned long long timeout_ns;
    unsigned* watchdog;
};

__device__ __forceinline__ uint32_t* flag_at(uint8_t* base, uint32_t bank, int src, int cta) {
    return reinterpret_cast<uint32_t*>(base) + (size_t(bank) * kMaxRanks + src) * kMaxCtas + cta;
}

__device__ __forceinline__ float* data_at(uint8_t* base, uint32_t bank, int src, size_t max_count) {
    return reinterpret_cast<float*>(base + kDataOff) + (size_t(bank) * kMaxRanks + src) * max_count;
}

__device__ __forceinline__ void store_release_sys(uint32_t* at, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(at), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* at) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(at) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(kArThreads) peer_allreduce_kernel(const __grid_constant__ ArParams p) {
    __shared__ uint32_t epoch_s;
    __shared__ int ok_s;
    const int c = blockIdx.x, tid = threadIdx.x;
    // The partial sums come from the previous kernel of the stream.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    uint8_t* mine = p.peers[p.rank];
    uint32_t* epochs = reinterpret_cast<uint32_t*>(mine + kEpochOff);
    if (tid == 0) {
        epoch_s = epochs[c] + 1u;
        ok_s = 1;
    }
    __syncthreads();
    // Every counter holds the number of calls so far, whatever the grid size
    // of each call: this CTA advances counters c, c + grid, c + 2 grid, ...
    for (int i = c + int(gridDim.x) * tid; i < kMaxCtas && tid < kMaxCtas; i += int(gridDim.x) * kArThreads)
        epochs[i] = epoch_s;
    const uint32_t e = epoch_s, bank = e & 1u;
    const size_t begin = size_t(c) * p.per_cta, end = min(p.count, begin + p.per_cta);
    const size_t v0 = begin / 4, v1 = end / 4;  // float4 index range (count and per_cta are multiples of 4)
    const float4* src = reinterpret_cast<const float4*>(p.data);

    // 1. Push this rank's chunk into slot [rank] of every peer.
    for (int q = 0; q < p.world; ++q) {
        if (q == p.rank)
            continue;
        float4* dst = reinterpret_cast<float4*>(data_at(p.peers[q], bank, p.rank, p.max_count));
        for (size_t i = v0 + tid; i < v1; i += kArThreads)
            dst[i] = src[i];
    }
    __threadfence_system();
    __syncthreads();
    if (tid < p.world && tid != p.rank)
        store_release_sys(flag_at(p.peers[tid], bank, p.rank, c), e);

    // 2. Wait for every peer's chunk (one thread per source, bounded).
    if (tid < p.world && tid != p.rank) {
        const uint32_t* flag = flag_at(mine, bank, tid, c);
        const unsigned long long start = global_ns();
        while (load_acquire_sys(flag) != e) {
            if (global_ns() - start > p.timeout_ns) {
                atomicOr(p.watchdog, watchdog_peer);
                ok_s = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (!ok_s)
        return;

    // 3. Sum over ranks in rank order; this rank's term is its own data.
    float4* out = reinterpret_cast<float4*>(p.data);
    for (size_t i = v0 + tid; i < v1; i += kArThreads) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < p.world; ++s) {
            const float4 v = s == p.rank ? src[i] : reinterpret_cast<const float4*>(data_at(mine, bank, s, p.max_count))[i];
            if (s == 0)
                acc = v;
            else
                acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
        }
        out[i] = acc;
    }
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

size_t kb200_peer_buffer_bytes(int world, size_t max_count) {
    if (world < 1 || world > kMaxRanks)
        return 0;
    return kDataOff + size_t(2) * kMaxRanks * max_count * sizeof(float);
}

int kb200_device_alloc(size_t bytes, void** ptr) {
    if (!ptr || !bytes)
        return fail(KB200_INVALID, "null pointer or zero size");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess)
        return cuda_fail(e, "cudaMalloc");
    if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "cudaMemset");
    }
    *ptr = p;
    return KB200_OK;
}

int kb200_device_free(void* ptr) {
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "cudaFree");
}

int kb200_ipc_handle(const void* ptr, void* handle) {
    if (!ptr || !handle)
        return fail(KB200_INVALID, "null pointer");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess)
        return cuda_fail(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == KB200_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    return KB200_OK;
}

int kb200_ipc_open(const void* handle, void** ptr) {
    if (!ptr || !handle)
        return fail(KB200_INVALID, "null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int kb200_ipc_close(void* ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int kb200_peer_allreduce_f32(float* data, size_t count, void* const* peers, int world, int rank, size_t max_count,
                             double timeout_s, void* stream) {
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return fail(KB200_UNSUPPORTED, "1..8 ranks");
    if (!count || world == 1)
        return KB200_OK;
    if (!data || !peers)
        return fail(KB200_INVALID, "null pointer");
    if (count % 4 || !aligned(data, 16) || count > max_count)
        return fail(KB200_INVALID, "count must be a multiple of 4 floats within the buffer, data 16-byte aligned");
    ArParams p;
    std::memset(&p, 0, sizeof(p));
    for (int r = 0; r < world; ++r) {
        if (!peers[r] || !aligned(peers[r], 256))
            return fail(KB200_INVALID, "peer buffers must be 256-byte aligned");
        p.peers[r] = static_cast<uint8_t*>(peers[r]);
    }
    const size_t ctas = std::min<size_t>(kMaxCtas, (count + kChunkFloats - 1) / kChunkFloats);
    p.per_cta = ((count + ctas - 1) / ctas + 3) / 4 * 4;
    p.data = data;
    p.count = count;
    p.max_count = max_count;
    p.rank = rank;
    p.world = world;
    p.timeout_ns = static_cast<unsigned long long>(std::max(0.001, timeout_s) * 1e9);
    p.watchdog = watchdog_word();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned((count + p.per_cta - 1) / p.per_cta));
    cfg.blockDim = dim3(kArThreads);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, peer_allreduce_kernel, p);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "peer_allreduce_kernel launch");
}

}  // extern "C"
