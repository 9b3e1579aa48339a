// Expert-parallel token exchange over NVLink peer memory (one process per GPU).
//
// The MoE layer with experts split over the ranks moves each routed row to
// the rank that holds its expert and the expert's result back. With a library
// all-to-all the host must first read the per-rank row counts back to size
// the transfer, which stops the host once per layer. Here the counts travel
// on the device and every row goes straight to its final place:
//
//   dispatch (ep_dispatch_kernel): every rank stores its per-expert row
//   offsets (the dispatch stage's expert-sorted order) into every rank's
//   buffer as epoch-tagged 64-bit words; each CTA waits (bounded) for all
//   ranks' offsets, derives where each of its rows lands in the owner's
//   expert-major receive area (for each local expert, the rows of source
//   0..N-1 in order), stores the rows there with plain peer stores, and
//   flags each owner after a system-scope fence. The owner's CTA 0 waits for
//   every source's flags and writes the local expert offsets, so the expert
//   GEMMs that follow in the stream see all rows.
//
//   return (ep_return_kernel): the owner stores each result row straight
//   into its source's return area at the row's position in the source's
//   expert-sorted order, flags, and waits for the rows of its own tokens,
//   which the combine then adds in selection order.
//
// Receive and return areas are single buffers: a rank writes a peer's
// receive area for layer k+1 only after its own return area for layer k is
// complete, which the peer fills after its expert GEMMs consumed layer k's
// rows. Count words and flags carry the call's epoch (counted on the device)
// and alternate between two banks. No TMA and no multicast: peer memory is
// only touched by plain loads and stores.
#include <algorithm>
#include <cstring>

#include "kb200_device.cuh"
#include "kb200_host.hpp"

namespace kb200 {
namespace {

constexpr int kEpRanks = 8;
constexpr int kEpCtas = 128;  // grid of both kernels (flags are per sending CTA)
constexpr int kEpThreads = 256;
constexpr int kEpMaxExperts = 256;
constexpr unsigned watchdog_ep = 32u;  // a peer's counts or rows never arrived

// Control area of one rank's buffer.
constexpr size_t kEpochOff = 0;                                        // [kEpCtas] u32
constexpr size_t kCountOff = 1024;                                     // [2][kEpRanks][kEpMaxExperts + 1] u64
constexpr size_t kRowFlagOff = kCountOff + 2 * kEpRanks * (kEpMaxExperts + 1) * 8;  // [2][kEpRanks][kEpCtas] u32
constexpr size_t kBackFlagOff = kRowFlagOff + 2 * kEpRanks * kEpCtas * 4;          // [2][kEpRanks][kEpCtas] u32
constexpr size_t kCtrlBytes = (kBackFlagOff + 2 * kEpRanks * kEpCtas * 4 + 4095) / 4096 * 4096;

struct EpParams {
    uint8_t* peers[kEpRanks];  // every rank's buffer, this rank's included
    const int* offsets;        // this rank's expert offsets [E + 1] (dispatch stage)
    const uint4* rows;         // dispatch: this rank's fp16 rows [n, H] in expert order
    const uint4* results;      // return: fp32 results [capacity, H] in receive order
    int* local_offsets;        // dispatch output: [E_l + 1] receive-area offsets per local expert
    size_t capacity, local_capacity;  // receive rows / return rows per rank
    int hidden, experts, world, rank;
    unsigned long long timeout_ns;
    unsigned* watchdog;
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* at, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(at), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* at) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(at) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long load_volatile_u64(const unsigned long long* at) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(at) : "memory");
    return v;
}

__device__ __forceinline__ void store_volatile_u64(unsigned long long* at, unsigned long long v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(at), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long* count_words(uint8_t* base, uint32_t bank, int src) {
    return reinterpret_cast<unsigned long long*>(base + kCountOff) + (size_t(bank) * kEpRanks + src) * (kEpMaxExperts + 1);
}

__device__ __forceinline__ uint32_t* row_flag(uint8_t* base, size_t off, uint32_t bank, int src, int cta) {
    return reinterpret_cast<uint32_t*>(base + off) + (size_t(bank) * kEpRanks + src) * kEpCtas + cta;
}

__device__ __forceinline__ uint8_t* rows_area(uint8_t* base) {
    return base + kCtrlBytes;
}

__device__ __forceinline__ uint8_t* back_area(uint8_t* base, size_t capacity, int hidden) {
    return base + kCtrlBytes + (capacity * size_t(hidden) * 2 + 4095) / 4096 * 4096;
}

// Shared per CTA: every rank's offsets [world][E + 1] and this call's epoch.
struct EpShared {
    int off[kEpRanks][kEpMaxExperts + 1];
    int base[kEpMaxExperts];  // dispatch: receive row of (expert e, this rank) at its owner
    uint32_t epoch;
    int ok;
};

// The call's epoch; every counter holds the number of calls so far.
__device__ uint32_t advance_epoch(const EpParams& p, EpShared& sh, bool advance) {
    auto* epochs = reinterpret_cast<uint32_t*>(p.peers[p.rank] + kEpochOff);
    if (threadIdx.x == 0) {
        sh.epoch = epochs[blockIdx.x] + (advance ? 1u : 0u);
        sh.ok = 1;
    }
    __syncthreads();
    if (advance)
        for (int i = int(blockIdx.x) + int(gridDim.x) * int(threadIdx.x); i < kEpCtas; i += int(gridDim.x) * kEpThreads)
            epochs[i] = sh.epoch;
    return sh.epoch;
}

// Wait (bounded) until `flag` shows `e`; false after the time limit.
__device__ bool wait_flag(const uint32_t* flag, uint32_t e, unsigned long long timeout_ns) {
    if (load_acquire_sys(flag) == e)
        return true;
    const unsigned long long start = global_ns();
    while (load_acquire_sys(flag) != e) {
        if (global_ns() - start > timeout_ns)
            return false;
        __nanosleep(64);
    }
    return true;
}

// Every rank's offsets, read from the tagged count words of this rank's buffer.
__device__ void gather_offsets(const EpParams& p, EpShared& sh, uint32_t e) {
    const int n = p.experts + 1;
    uint8_t* mine = p.peers[p.rank];
    for (int i = int(threadIdx.x); i < p.world * n; i += kEpThreads) {
        const int s = i / n, x = i % n;
        const unsigned long long* at = count_words(mine, e & 1u, s) + x;
        unsigned long long w = load_volatile_u64(at);
        if (uint32_t(w >> 32) != e) {
            const unsigned long long start = global_ns();
            while (uint32_t(w >> 32) != e) {
                if (!sh.ok || global_ns() - start > p.timeout_ns) {
                    sh.ok = 0;
                    break;
                }
                __nanosleep(64);
                w = load_volatile_u64(at);
            }
        }
        sh.off[s][x] = int(uint32_t(w));
    }
    __syncthreads();
}

// Receive-area row of the first row of (expert e, source src) at e's owner:
// the owner's earlier local experts' rows from every source, then the rows of
// expert e from sources before src.
__device__ __forceinline__ int receive_base(const EpShared& sh, int world, int local, int e, int src) {
    const int q0 = e / local * local;
    int b = 0;
    for (int s = 0; s < world; ++s) {
        b += sh.off[s][e] - sh.off[s][q0];
        if (s < src)
            b += sh.off[s][e + 1] - sh.off[s][e];
    }
    return b;
}

// Largest e with off[e] <= i (expert of row i in a rank's sorted order).
__device__ __forceinline__ int expert_of(const int* off, int experts, int i) {
    int lo = 0, hi = experts;
    while (hi - lo > 1) {
        const int mid = (lo + hi) / 2;
        if (off[mid] <= i)
            lo = mid;
        else
            hi = mid;
    }
    return lo;
}

__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(const __grid_constant__ EpParams p) {
    __shared__ EpShared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t e = advance_epoch(p, sh, true), bank = e & 1u;
    const int n1 = p.experts + 1, local = p.experts / p.world;
    // 1. CTA 0 publishes this rank's offsets to every rank (itself included).
    if (blockIdx.x == 0)
        for (int i = tid; i < p.world * n1; i += kEpThreads) {
            const int q = i / n1, x = i % n1;
            store_volatile_u64(count_words(p.peers[q], bank, p.rank) + x,
                               (unsigned long long)e << 32 | uint32_t(p.offsets[x]));
        }
    // 2. Every CTA reads all ranks' offsets.
    gather_offsets(p, sh, e);
    for (int x = tid; x < p.experts; x += kEpThreads)
        sh.base[x] = receive_base(sh, p.world, local, x, p.rank);
    __syncthreads();
    // 3. Rows of this rank, one warp per row, to their owners' receive areas.
    const int n = sh.off[p.rank][p.experts];
    const int words = p.hidden / 8;  // 16-byte words per fp16 row
    if (sh.ok)
        for (int i = int(blockIdx.x) * (kEpThreads / 32) + warp; i < n; i += int(gridDim.x) * (kEpThreads / 32)) {
            const int x = expert_of(sh.off[p.rank], p.experts, i);
            const int q = x / local;
            const size_t dst = size_t(sh.base[x] + (i - sh.off[p.rank][x]));
            if (dst >= p.capacity)
                continue;  // the host sized the areas for every row; never reached
            uint4* to = reinterpret_cast<uint4*>(rows_area(p.peers[q])) + dst * words;
            const uint4* from = p.rows + size_t(i) * words;
            for (int w = lane; w < words; w += 32)
                to[w] = from[w];
        }
    // 4. Flag every owner once this CTA's stores are visible system-wide.
    __threadfence_system();
    __syncthreads();
    if (tid < p.world)
        store_release_sys(row_flag(p.peers[tid], kRowFlagOff, bank, p.rank, blockIdx.x), e);
    // 5. CTA 0 waits for every source's rows and writes the local expert offsets.
    if (blockIdx.x == 0) {
        uint8_t* mine = p.peers[p.rank];
        for (int i = tid; i < p.world * kEpCtas; i += kEpThreads)
            if (!wait_flag(row_flag(mine, kRowFlagOff, bank, i / kEpCtas, i % kEpCtas), e, p.timeout_ns))
                sh.ok = 0;
        __syncthreads();
        if (tid <= local) {
            // After a give-up the offsets are zero: the expert stage reads no
            // rows. The receive area holds `capacity` rows at most.
            const int x = p.rank * local + tid;  // local expert tid (tid == local: the end)
            int b = 0;
            for (int s = 0; s < p.world && sh.ok; ++s)
                b += sh.off[s][x] - sh.off[s][p.rank * local];
            p.local_offsets[tid] = sh.ok ? int(min(size_t(max(b, 0)), p.capacity)) : 0;
        }
    }
    if (!sh.ok && tid == 0)
        atomicOr(p.watchdog, watchdog_ep);
}

__global__ void __launch_bounds__(kEpThreads) ep_return_kernel(const __grid_constant__ EpParams p) {
    __shared__ EpShared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // The epoch of this layer's dispatch (already advanced by it).
    const uint32_t e = advance_epoch(p, sh, false), bank = e & 1u;
    const int local = p.experts / p.world;
    gather_offsets(p, sh, e);
    // Rows received: for each local expert, the rows of source 0..N-1.
    const int x0 = p.rank * local;
    int total = 0;
    for (int s = 0; s < p.world; ++s)
        total += sh.off[s][x0 + local] - sh.off[s][x0];
    total = int(min(size_t(max(total, 0)), p.capacity));  // the results hold `capacity` rows
    const int words = p.hidden / 4;  // 16-byte words per fp32 row
    if (sh.ok)
        for (int j = int(blockIdx.x) * (kEpThreads / 32) + warp; j < total; j += int(gridDim.x) * (kEpThreads / 32)) {
            // (expert, source, index) of received row j.
            int b = 0, xe = x0, src = 0, u = 0;
            bool found = false;
            for (int x = x0; x < x0 + local && !found; ++x)
                for (int s = 0; s < p.world; ++s) {
                    const int c = sh.off[s][x + 1] - sh.off[s][x];
                    if (j < b + c) {
                        xe = x, src = s, u = j - b;
                        found = true;
                        break;
                    }
                    b += c;
                }
            const size_t dst = size_t(sh.off[src][xe] + u);
            if (dst >= p.local_capacity)
                continue;  // never reached
            uint4* to = reinterpret_cast<uint4*>(back_area(p.peers[src], p.capacity, p.hidden)) + dst * words;
            const uint4* from = p.results + size_t(j) * words;
            for (int w = lane; w < words; w += 32)
                to[w] = from[w];
        }
    __threadfence_system();
    __syncthreads();
    if (tid < p.world)
        store_release_sys(row_flag(p.peers[tid], kBackFlagOff, bank, p.rank, blockIdx.x), e);
    // CTA 0 waits for the results of this rank's rows, so the combine that
    // follows in the stream sees them all.
    if (blockIdx.x == 0) {
        uint8_t* mine = p.peers[p.rank];
        for (int i = tid; i < p.world * kEpCtas; i += kEpThreads)
            if (!wait_flag(row_flag(mine, kBackFlagOff, bank, i / kEpCtas, i % kEpCtas), e, p.timeout_ns))
                sh.ok = 0;
        __syncthreads();
    }
    if (!sh.ok && tid == 0)
        atomicOr(p.watchdog, watchdog_ep);
}

int ep_check(int hidden, int experts, int world, int rank, void* const* peers, size_t capacity, size_t local_capacity) {
    if (world < 1 || world > kEpRanks || rank < 0 || rank >= world)
        return fail(KB200_UNSUPPORTED, "1..8 ranks");
    if (experts <= 0 || experts > kEpMaxExperts || experts % world)
        return fail(KB200_UNSUPPORTED, "experts must split evenly over the ranks, at most 256");
    if (hidden <= 0 || hidden % 64)
        return fail(KB200_UNSUPPORTED, "hidden must be a multiple of 64");
    if (!peers || !capacity || !local_capacity)
        return fail(KB200_INVALID, "null peers or empty areas");
    for (int r = 0; r < world; ++r)
        if (!peers[r] || !aligned(peers[r], 256))
            return fail(KB200_INVALID, "exchange buffers must be 256-byte aligned");
    return KB200_OK;
}

int ep_launch(bool dispatch, EpParams& p, void* const* peers, double timeout_s, void* stream) {
    for (int r = 0; r < p.world; ++r)
        p.peers[r] = static_cast<uint8_t*>(peers[r]);
    p.timeout_ns = static_cast<unsigned long long>(std::max(0.001, timeout_s) * 1e9);
    p.watchdog = watchdog_word();
    // CTAs of one grid wait on each other (the counts CTA 0 publishes, the
    // flags CTA 0 collects): a cooperative launch guarantees they are all
    // resident, or fails.
    void* args[] = {&p};
    TraceScope trace(KB200_KERNEL_EP_EXCHANGE, static_cast<cudaStream_t>(stream));
    const cudaError_t e = cudaLaunchCooperativeKernel(
        dispatch ? reinterpret_cast<const void*>(ep_dispatch_kernel) : reinterpret_cast<const void*>(ep_return_kernel),
        dim3(kEpCtas), dim3(kEpThreads), args, 0, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, dispatch ? "ep_dispatch_kernel launch" : "ep_return_kernel launch");
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

size_t kb200_ep_buffer_bytes(int world, int experts, int hidden, size_t capacity, size_t local_capacity) {
    if (world < 1 || world > kEpRanks || experts <= 0 || experts > kEpMaxExperts || hidden <= 0 || hidden % 64)
        return 0;
    return kCtrlBytes + (capacity * size_t(hidden) * 2 + 4095) / 4096 * 4096 + local_capacity * size_t(hidden) * 4;
}

void* kb200_ep_rows_area(void* buffer) {
    return buffer ? static_cast<uint8_t*>(buffer) + kCtrlBytes : nullptr;
}

void* kb200_ep_return_area(void* buffer, size_t capacity, int hidden) {
    return buffer ? static_cast<uint8_t*>(buffer) + kCtrlBytes + (capacity * size_t(hidden) * 2 + 4095) / 4096 * 4096
                  : nullptr;
}

int kb200_ep_dispatch(const int32_t* offsets, const uint16_t* rows, int hidden, int experts, int world, int rank,
                      void* const* peers, size_t capacity, size_t local_capacity, int32_t* local_offsets,
                      double timeout_s, void* stream) {
    if (const int s = ep_check(hidden, experts, world, rank, peers, capacity, local_capacity))
        return s;
    if (!offsets || !rows || !local_offsets)
        return fail(KB200_INVALID, "null pointer");
    if (!aligned(rows, 16))
        return fail(KB200_INVALID, "rows must be 16-byte aligned");
    EpParams p;
    std::memset(&p, 0, sizeof(p));
    p.offsets = offsets;
    p.rows = reinterpret_cast<const uint4*>(rows);
    p.local_offsets = local_offsets;
    p.capacity = capacity;
    p.local_capacity = local_capacity;
    p.hidden = hidden;
    p.experts = experts;
    p.world = world;
    p.rank = rank;
    return ep_launch(true, p, peers, timeout_s, stream);
}

int kb200_ep_return(const float* results, int hidden, int experts, int world, int rank, void* const* peers,
                    size_t capacity, size_t local_capacity, double timeout_s, void* stream) {
    if (const int s = ep_check(hidden, experts, world, rank, peers, capacity, local_capacity))
        return s;
    if (!results)
        return fail(KB200_INVALID, "null pointer");
    if (!aligned(results, 16))
        return fail(KB200_INVALID, "results must be 16-byte aligned");
    EpParams p;
    std::memset(&p, 0, sizeof(p));
    p.results = reinterpret_cast<const uint4*>(results);
    p.capacity = capacity;
    p.local_capacity = local_capacity;
    p.hidden = hidden;
    p.experts = experts;
    p.world = world;
    p.rank = rank;
    return ep_launch(false, p, peers, timeout_s, stream);
}

}  // extern "C"
