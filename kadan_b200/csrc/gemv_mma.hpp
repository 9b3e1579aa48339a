// Tensor-pipe GEMV kernels (host entry points used by the batch dispatcher)
// and the peer-memory exchange they can feed.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include "kadan_b200.h"

namespace kb200 {

// Exchange buffers of a tensor-parallel group, as kb200_peer_allreduce_f32
// lays them out: every rank's buffer holds call counters, then epoch-tagged
// 64-bit words [2 banks][8 sources][max_count].
constexpr int kPeerMaxRanks = 8;
constexpr size_t kPeerWordsOff = 4096;

struct PeerOut {
    uint8_t* peers[kPeerMaxRanks];  // every rank's buffer, this rank's included
    size_t max_count;
    int rank, world;  // world == 0: no exchange
};

// Q4_K or Q6_K job that the mma.sync kernels can take: 16-byte aligned rows
// of whole super-blocks, and the driver's tensor-map encoder is available.
bool mma_eligible(const kb200_gemv_job& job);
// Jobs of one encoding: one launch per 32 jobs; rows above the kernel's rows
// per pass (8) become row groups. With `peer`, the
// single job's outputs (rows x columns, contiguous) also go, as words tagged
// with the group's next call number, to slot [rank] of every peer's buffer.
// synchronous: the caller waits for this launch alone (a host-span call), so
// nothing ahead on the stream hides a quantisation kernel in front of a GEMV;
// activations are then staged only where CTAs would quantise many times.
int launch_mma(const std::vector<const kb200_gemv_job*>& jobs, cudaStream_t stream, const PeerOut* peer = nullptr,
               bool synchronous = false);

// kb200_gguf_gemv_batch with the synchronous hint of launch_mma.
int gemv_batch(const kb200_gemv_job* jobs, size_t count, cudaStream_t stream, bool synchronous);

// The peer all-reduce kernel; push = false when the values were already
// pushed (by a GEMV launched with a PeerOut) and only the gather-sum is left.
int launch_peer_allreduce(float* data, size_t count, const PeerOut& peer, double timeout_s, bool push,
                          cudaStream_t stream);

}  // namespace kb200
