// Multi-device column partition of a packed projection batch.
//
// The reference splits each projection's output columns across devices in
// proportion to their weight capacity and chunks each device's slice the way
// an individual projection on that device would (gguf_batch_partition,
// IW/include/kadan/gguf_batch_partition.hpp:44-83; weight_boundary and the
// projection plans, IW/include/kadan/device_placement.hpp:76-142, :341-357).
// The geometry is part of the worker's contract (retained weight chunks are
// keyed by it), so the arithmetic here follows the same steps: the
// proportional boundary in long double, and the reference's scratch
// accounting of 256..1-row tiles for the chunk width.
#include <algorithm>
#include <cstdint>

#include "gguf_geometry.hpp"
#include "kb200_host.hpp"

namespace kb200 {
namespace {

constexpr uint64_t kStatusBytes = 256;                 // projection_status_bytes
constexpr uint64_t kStagingBytes = 16ull * 1024 * 1024;  // gguf_projection_staging_bytes
constexpr uint64_t kMaxExtent = 2147483647ull;

struct Plan {
    uint64_t rows, columns, bytes;
};

// Widest chunk of `out` columns whose decode tile, scratch and slices fit
// `limit` bytes, trying row tiles 256, 128, ..., 1.
int projection_plan(uint64_t in, uint64_t out, uint64_t width, bool precise, uint64_t alignment, uint64_t limit,
                    Plan* plan) {
    if (!in || in > kMaxExtent || !out || out > kMaxExtent || (width != 1 && width != 2 && width != 4)
        || (alignment != 1 && alignment != 4) || out % alignment)
        return fail(KB200_INVALID, "projection_layout");
    const uint64_t wide = precise ? 8 : 0;
    for (uint64_t tile = 256; tile; tile /= 2) {
        const uint64_t fixed = 8ull * 1024 * 1024 + 4096 + kStatusBytes + tile * in * (9 + wide) + tile * 4;
        const uint64_t per_column = in * (width + wide) + 8 + tile * (8 + wide);
        if (fixed >= limit)
            continue;
        const uint64_t columns = std::min(out, (limit - fixed) / per_column) / alignment * alignment;
        if (columns) {
            *plan = {tile, columns, fixed + columns * per_column};
            return KB200_OK;
        }
    }
    return fail(KB200_INVALID, "projection_scratch_limit");
}

int gguf_projection_plan(uint64_t in, uint64_t out, int encoding, uint64_t limit, Plan* plan) {
    if (!gguf_geometry(encoding))
        return fail(KB200_INVALID, "gguf_projection_encoding");
    const uint64_t values = block_values(encoding), bytes = block_bytes(encoding);
    if (!in || in > kMaxExtent || in % values || in / values > kStagingBytes / bytes)
        return fail(KB200_INVALID, "gguf_projection_layout");
    const uint64_t row_bytes = in / values * bytes;
    if (!out || out > kMaxExtent || limit <= kStagingBytes + kStatusBytes)
        return fail(KB200_INVALID, "gguf_projection_layout");
    if (const int s = projection_plan(in, std::min(out, kStagingBytes / row_bytes), sizeof(float), false, 1,
                                      limit - (kStagingBytes + kStatusBytes), plan))
        return s;
    plan->bytes += kStagingBytes + kStatusBytes;
    return KB200_OK;
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

size_t kb200_weight_boundary(size_t units, const uint64_t* capacities, size_t devices, size_t index) {
    if (index >= devices || !capacities)
        return units;
    long double total = 0, prefix = 0;
    for (size_t i = 0; i < devices; ++i) {
        total += static_cast<long double>(capacities[i]);
        if (i < index)
            prefix += static_cast<long double>(capacities[i]);
    }
    if (total == 0)
        return units * index / devices;
    return std::min(units, static_cast<size_t>(static_cast<long double>(units) * prefix / total));
}

int kb200_gguf_batch_partition(size_t in, size_t out, int encoding, const uint64_t* capacities, size_t devices,
                               size_t device, uint64_t scratch_limit, kb200_partition* result) {
    if (!result)
        return fail(KB200_INVALID, "null partition result");
    const size_t first = kb200_weight_boundary(out, capacities, devices, device);
    const size_t count = kb200_weight_boundary(out, capacities, devices, device + 1) - first;
    *result = {first, count, 0};
    if (!count)
        return KB200_OK;
    Plan plan{};
    const int s = encoding == KB200_F32
                      ? projection_plan(in, std::min<uint64_t>(count, (16ull * 1024 * 1024) / (uint64_t(in) * sizeof(float))),
                                        sizeof(float), false, 1, scratch_limit, &plan)
                      : gguf_projection_plan(in, count, encoding, scratch_limit, &plan);
    if (s)
        return s;
    result->chunk_columns = size_t(plan.columns);
    return KB200_OK;
}

void kb200_partition_scatter(const kb200_partition* p, const float* local, size_t rows, float* output, size_t out) {
    if (!p || !p->count)
        return;
    for (size_t row = 0; row < rows; ++row)
        std::copy(local + row * p->count, local + (row + 1) * p->count, output + row * out + p->first);
}

}  // extern "C"
