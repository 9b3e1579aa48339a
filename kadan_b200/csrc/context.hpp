// The host-span context (kb200_context) shared by the translation units that
// implement its calls: context.cu (projections, MoE) and layer_host.cpp
// (attention and delta-net over per-layer device state).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "kadan_b200.h"

namespace kb200 {
class ReadTeam;
struct LayerStore;  // per-layer KV mirrors and recurrent state (layer_host.cpp)

// Frees every layer's device state held in `store` and the store itself.
void release_layers(LayerStore* store);
}  // namespace kb200

struct kb200_context {
    int device = 0;
    cudaStream_t stream = nullptr;
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
    void* pinned = nullptr;
    size_t pinned_bytes = 0;
    cudaEvent_t staged[2] = {nullptr, nullptr};  // source batch: staging half done
    int read_lanes = 4;                           // source reads: 3 workers + the caller
    kb200::ReadTeam* team = nullptr;              // created by the first source batch
    kb200_context_counters counters = {};         // launches of every call, cumulative
    kb200::LayerStore* layers = nullptr;          // created by the first attention / delta-net call
};

namespace kb200 {
// Grows the context's device workspace and pinned staging to at least the
// given sizes (contents not kept).
int context_ensure(kb200_context* c, size_t device_bytes, size_t host_bytes);

inline bool cancelled(const volatile uint8_t* cancel) {
    return cancel && *cancel;
}
}  // namespace kb200
