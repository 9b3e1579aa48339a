// One-shot all-reduce of fp32 partial sums over NVLink peer memory.
//
// Tensor-parallel decode adds the row-parallel projections' partial outputs
// across ranks twice per layer (after o and after down): T x hidden fp32,
// 32 KB at T = 1. At that size an all-reduce is bound by latency, not by
// NVLink bandwidth. Every rank's exchange buffer is mapped into every other
// rank's address space (CUDA IPC, one process per GPU) and one kernel does
// the exchange with self-validating words:
//
//   each float travels as one 64-bit word {epoch, value bits}; a thread
//   stores its elements into slot [rank] of every peer's buffer (plain
//   64-bit stores over NVLink, two per 16-byte vector), then reads the same
//   elements from every peer's slot in its own buffer until their epoch
//   halves show this call, and sums over ranks in rank order 0..N-1, so all
//   ranks hold the same bits. A 64-bit access is single-copy atomic, so a
//   word with the right epoch carries the right value: no fence and no
//   separate flag are needed, and no thread waits for another.
//
// The epoch is the number of the call, counted on the device (a graph replay
// needs no new parameters; every rank makes the same calls). Receive slots
// alternate between two banks by epoch parity: a rank's call k starts after
// its call k-1 finished, for which it read every peer's call k-1 words, so
// every peer has finished call k-2 and reads bank (k-1)&1 at most while call
// k writes bank k&1.
//
// Buffer of one rank (same layout on every rank, zeroed at allocation):
//   epochs [kMaxCtas] u32                     this rank's call counters
//   words  [2][kMaxRanks][max_count] u64      written by peers
// No TMA and no multicast: peer memory is only touched by plain loads and
// stores.
#include <algorithm>
#include <cstring>

#include "gemv_mma.hpp"
#include "kb200_device.cuh"
#include "kb200_host.hpp"

namespace kb200 {
namespace {

constexpr int kMaxRanks = kPeerMaxRanks;
constexpr int kMaxCtas = 256;
constexpr int kArThreads = 256;
constexpr size_t kWordsOff = kPeerWordsOff;  // after the epoch counters
constexpr unsigned watchdog_peer = 16u;  // a peer's words never arrived

struct ArParams {
    uint8_t* peers[kMaxRanks];  // every rank's buffer, this rank's included
    float* data;                // in/out, count floats
    size_t count, max_count;
    int rank, world;
    int push;  // 0: the values are already in the peers' slots (fused GEMV)
    unsigned long long timeout_ns;
    unsigned* watchdog;
};

__device__ __forceinline__ unsigned long long* words_at(uint8_t* base, uint32_t bank, int src, size_t max_count) {
    return reinterpret_cast<unsigned long long*>(base + kWordsOff) + (size_t(bank) * kMaxRanks + src) * max_count;
}

__device__ __forceinline__ void store_pair(unsigned long long* at, unsigned long long a, unsigned long long b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(at), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void load_pair(const unsigned long long* at, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(at) : "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(kArThreads) peer_allreduce_kernel(const __grid_constant__ ArParams p) {
    __shared__ uint32_t epoch_s;
    const int c = blockIdx.x, tid = threadIdx.x;
    // The partial sums come from the previous kernel of the stream.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    uint8_t* mine = p.peers[p.rank];
    uint32_t* epochs = reinterpret_cast<uint32_t*>(mine);
    if (tid == 0)
        epoch_s = epochs[c] + 1u;
    __syncthreads();
    // Every counter holds the number of calls so far, whatever the grid size
    // of each call: this CTA advances counters c, c + grid, c + 2 grid, ...
    for (int i = c + int(gridDim.x) * tid; i < kMaxCtas; i += int(gridDim.x) * kArThreads)
        epochs[i] = epoch_s;
    const uint32_t e = epoch_s, bank = e & 1u;
    const unsigned long long tag = (unsigned long long)e << 32;
    auto* pairs = reinterpret_cast<float2*>(p.data);
    const size_t npairs = p.count / 2;
    const size_t stride = size_t(gridDim.x) * kArThreads;

    // 1. Push: this rank's elements into slot [rank] of every peer.
    for (size_t i = size_t(c) * kArThreads + tid; p.push && i < npairs; i += stride) {
        const float2 v = pairs[i];
        const unsigned long long w0 = tag | __float_as_uint(v.x), w1 = tag | __float_as_uint(v.y);
        for (int q = 0; q < p.world; ++q)
            if (q != p.rank)
                store_pair(words_at(p.peers[q], bank, p.rank, p.max_count) + 2 * i, w0, w1);
    }
    // 2. Gather the same elements from every peer's slot and sum in rank order.
    // All sources' words are loaded at once (one round trip, not one per
    // rank); only words that have not arrived yet are polled again.
    bool ok = true;
    for (size_t i = size_t(c) * kArThreads + tid; i < npairs; i += stride) {
        unsigned long long a[kMaxRanks], b[kMaxRanks];
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s)
            if (s < p.world && s != p.rank)
                load_pair(words_at(mine, bank, s, p.max_count) + 2 * i, a[s], b[s]);
        const float2 own = pairs[i];
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int s = 0; s < kMaxRanks; ++s) {
            if (s >= p.world)
                break;
            float2 v = own;
            if (s != p.rank) {
                if ((a[s] >> 32) != e || (b[s] >> 32) != e) {
                    const unsigned long long* at = words_at(mine, bank, s, p.max_count) + 2 * i;
                    const unsigned long long start = global_ns();
                    do {
                        if (!ok || global_ns() - start > p.timeout_ns) {
                            ok = false;
                            break;
                        }
                        __nanosleep(32);
                        load_pair(at, a[s], b[s]);
                    } while ((a[s] >> 32) != e || (b[s] >> 32) != e);
                }
                v = make_float2(__uint_as_float(uint32_t(a[s])), __uint_as_float(uint32_t(b[s])));
            }
            if (s == 0)
                acc = v;
            else
                acc.x += v.x, acc.y += v.y;
        }
        if (ok)
            pairs[i] = acc;
    }
    if (!ok)
        atomicOr(p.watchdog, watchdog_peer);
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

size_t kb200_peer_buffer_bytes(int world, size_t max_count) {
    if (world < 1 || world > kMaxRanks)
        return 0;
    return kWordsOff + size_t(2) * kMaxRanks * max_count * sizeof(unsigned long long);
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
    if (!peers)
        return fail(KB200_INVALID, "null pointer");
    PeerOut g;
    std::memset(&g, 0, sizeof(g));
    for (int r = 0; r < world; ++r)
        g.peers[r] = static_cast<uint8_t*>(peers[r]);
    g.max_count = max_count;
    g.rank = rank;
    g.world = world;
    return launch_peer_allreduce(data, count, g, timeout_s, true, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace kb200 {

int launch_peer_allreduce(float* data, size_t count, const PeerOut& g, double timeout_s, bool push,
                          cudaStream_t stream) {
    if (!data)
        return fail(KB200_INVALID, "null pointer");
    if (count % 2 || !aligned(data, 8) || count > g.max_count || g.max_count % 2)
        return fail(KB200_INVALID, "count must be an even number of floats within the buffer, data 8-byte aligned");
    ArParams p;
    std::memset(&p, 0, sizeof(p));
    for (int r = 0; r < g.world; ++r) {
        if (!g.peers[r] || !aligned(g.peers[r], 256))
            return fail(KB200_INVALID, "peer buffers must be 256-byte aligned");
        p.peers[r] = g.peers[r];
    }
    const size_t ctas = std::min<size_t>(kMaxCtas, (count / 2 + kArThreads - 1) / kArThreads);
    p.data = data;
    p.count = count;
    p.max_count = g.max_count;
    p.rank = g.rank;
    p.world = g.world;
    p.push = push ? 1 : 0;
    p.timeout_ns = static_cast<unsigned long long>(std::max(0.001, timeout_s) * 1e9);
    p.watchdog = watchdog_word();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(ctas));
    cfg.blockDim = dim3(kArThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    TraceScope trace(KB200_KERNEL_PEER_ALLREDUCE, stream);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, peer_allreduce_kernel, p);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "peer_allreduce_kernel launch");
}

}  // namespace kb200
