// Host-span boundary: kb200_context, kb200_dense_gguf_batch and
// kb200_dense_gguf_source_batch, the reference's DenseCompute::dense_gguf_batch
// contract (services/hikari/inference_worker/src/cuda/h3_compute.cu:3963-4375).
// Over device-resident weights: one input upload, one launch per encoding, one
// download, one stream synchronisation per call. Over packed-row sources:
// bank hits as one launch, misses streamed through two pinned staging halves
// and admitted into the bank once they decoded finite.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "context.hpp"
#include "gemv_mma.hpp"
#include "gguf_formats.cuh"
#include "kb200_host.hpp"
#include "read_team.hpp"

namespace kb200 {

int context_ensure(kb200_context* c, size_t device_bytes, size_t host_bytes) {
    if (device_bytes > c->workspace_bytes) {
        if (c->workspace)
            cudaFree(c->workspace);
        c->workspace = nullptr;
        c->workspace_bytes = 0;
        const size_t grow = device_bytes + device_bytes / 2;
        if (cudaMalloc(&c->workspace, grow) != cudaSuccess)
            return fail(KB200_NO_MEMORY, "device workspace");
        c->workspace_bytes = grow;
    }
    if (host_bytes > c->pinned_bytes) {
        if (c->pinned)
            cudaFreeHost(c->pinned);
        c->pinned = nullptr;
        c->pinned_bytes = 0;
        const size_t grow = host_bytes + host_bytes / 2;
        if (cudaMallocHost(&c->pinned, grow) != cudaSuccess)
            return fail(KB200_NO_MEMORY, "pinned staging");
        c->pinned_bytes = grow;
    }
    return KB200_OK;
}

namespace {

int ensure(kb200_context* c, size_t device_bytes, size_t host_bytes) {
    return context_ensure(c, device_bytes, host_bytes);
}

size_t up16(size_t v) {
    return (v + 15) / 16 * 16;
}

size_t up256(size_t v) {
    return (v + 255) / 256 * 256;
}

// Input spans of a batch on the device. Jobs sharing a span (same pointer and
// length) upload and check it once (h3_compute.cu:3972-3991); every span
// starts 64-byte aligned. `owner[j]` marks the job that uploads its span.
struct InputLayout {
    std::vector<size_t> at;
    std::vector<char> owner;
    size_t floats = 0;
};

template <class Job>
int layout_inputs(const Job* jobs, size_t count, InputLayout& l) {
    l.at.assign(count, 0);
    l.owner.assign(count, 0);
    l.floats = 0;
    for (size_t j = 0; j < count; ++j) {
        const size_t n = size_t(jobs[j].rows) * jobs[j].in;
        size_t shared = 0;
        while (shared < j
               && (jobs[shared].input != jobs[j].input || size_t(jobs[shared].rows) * jobs[shared].in != n))
            ++shared;
        if (shared < j) {
            l.at[j] = l.at[shared];
            continue;
        }
        for (size_t i = 0; i < n; ++i)
            if (!std::isfinite(jobs[j].input[i]))
                return fail(KB200_NONFINITE_INPUT, "non-finite input value");
        l.at[j] = l.floats;
        l.owner[j] = 1;
        l.floats += up16(n);
    }
    return KB200_OK;
}

// No output may overlap any input (the reference's alias rule).
template <class Job>
int check_aliases(const Job* jobs, size_t count) {
    for (size_t j = 0; j < count; ++j)
        for (size_t k = 0; k < count; ++k)
            if (overlap(jobs[j].output, size_t(jobs[j].rows) * jobs[j].out * sizeof(float), jobs[k].input,
                        size_t(jobs[k].rows) * jobs[k].in * sizeof(float)))
                return fail(KB200_ALIAS, "output overlaps an input");
    return KB200_OK;
}

template <class Job>
void stage_inputs(const Job* jobs, size_t count, const InputLayout& l, uint8_t* host) {
    for (size_t j = 0; j < count; ++j)
        if (l.owner[j])
            std::memcpy(host + l.at[j] * sizeof(float), jobs[j].input, size_t(jobs[j].rows) * jobs[j].in * sizeof(float));
}

// The reference's switch between its two projection paths: packed jobs of
// more than gguf_batch_rows input rows leave the batched GEMV for decode +
// GEMM (`matvec = packed && rows <= 8`, h3_compute.cu:1863-1865). Here those
// jobs run on the tensor-core GEMM when it takes their weights
// (KB200_PREFILL_GEMM=0 keeps every job on the GEMV path).
bool prefill_gemm_enabled() {
    static const bool on = [] {
        const char* s = std::getenv("KB200_PREFILL_GEMM");
        return !s || std::atoi(s) != 0;
    }();
    return on;
}

bool to_gemm(const kb200_gemv_job& j) {
    return j.rows > KB200_BATCH_ROWS && prefill_gemm_enabled() && gemm_eligible(j);
}

// Device scratch the GEMM jobs among `jobs` need (one at a time, in stream order).
size_t gemm_scratch(const kb200_gemv_job* jobs, size_t count) {
    size_t need = 0;
    for (size_t j = 0; j < count; ++j)
        if (to_gemm(jobs[j]))
            need = std::max(need, kb200_gguf_gemm_workspace_bytes(jobs[j].rows, jobs[j].in));
    return need;
}

// Enqueue device jobs on the context's stream: one GEMM per job to_gemm
// selects (reporting to `gemm_status`: bit 0 a non-finite weight, bit 1 a
// weight beyond the fp16 operand range), every other job in one GEMV batch.
int launch_projections(kb200_context* c, const kb200_gemv_job* jobs, size_t count, void* scratch, size_t scratch_bytes,
                       unsigned* gemm_status) {
    std::vector<kb200_gemv_job> gemv;
    gemv.reserve(count);
    for (size_t j = 0; j < count; ++j) {
        if (!to_gemm(jobs[j])) {
            gemv.push_back(jobs[j]);
            continue;
        }
        kb200_gemv_job g = jobs[j];
        g.status = gemm_status;
        if (const int s = kb200_gguf_gemm(&g, scratch, scratch_bytes, c->stream))
            return s;
        ++c->counters.gemm_launches;
    }
    if (!gemv.empty()) {
        if (const int s = gemv_batch(gemv.data(), gemv.size(), c->stream, true))
            return s;
        ++c->counters.gemv_batches;
    }
    return KB200_OK;
}

// The GEMM jobs among `jobs` again, on the GEMV path (a block's scales put a
// weight beyond the fp16 operands the GEMM uses).
int rerun_gemm_jobs(kb200_context* c, const kb200_gemv_job* jobs, size_t count) {
    std::vector<kb200_gemv_job> again;
    for (size_t j = 0; j < count; ++j)
        if (to_gemm(jobs[j]))
            again.push_back(jobs[j]);
    if (again.empty())
        return KB200_OK;
    c->counters.gemm_fallbacks += again.size();
    ++c->counters.gemv_batches;
    return gemv_batch(again.data(), again.size(), c->stream, true);
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

int kb200_context_create(int device, kb200_context** out) {
    if (!out)
        return fail(KB200_INVALID, "null output");
    *out = nullptr;
    auto* c = new (std::nothrow) kb200_context;
    if (!c)
        return fail(KB200_NO_MEMORY, "context");
    c->device = device;
    DeviceScope scope(device);
    const cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "cudaStreamCreate");
    }
    *out = c;
    return KB200_OK;
}

void kb200_context_destroy(kb200_context* c) {
    if (!c)
        return;
    DeviceScope scope(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->workspace)
        cudaFree(c->workspace);
    if (c->pinned)
        cudaFreeHost(c->pinned);
    for (cudaEvent_t e : c->staged)
        if (e)
            cudaEventDestroy(e);
    delete c->team;
    release_layers(c->layers);
    cudaStreamDestroy(c->stream);
    delete c;
}

void* kb200_context_stream(kb200_context* c) {
    return c ? static_cast<void*>(c->stream) : nullptr;
}

int kb200_context_counters_get(kb200_context* c, kb200_context_counters* out) {
    if (!c || !out)
        return fail(KB200_INVALID, "null context or output");
    *out = c->counters;
    return KB200_OK;
}

int kb200_context_set_read_lanes(kb200_context* c, int lanes) {
    if (!c || lanes < 1 || lanes > 64)
        return fail(KB200_INVALID, "read lanes must be 1..64");
    if (c->team && c->team->lanes() != lanes) {
        delete c->team;
        c->team = nullptr;
    }
    c->read_lanes = lanes;
    return KB200_OK;
}

int kb200_weights_upload(kb200_context* c, const void* host, size_t bytes, void** device) {
    if (!c || !host || !device || !bytes)
        return fail(KB200_INVALID, "weights_upload arguments");
    DeviceScope scope(c->device);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess)
        return fail(KB200_NO_MEMORY, "weight bank allocation");
    e = cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "weights_upload copy");
    }
    *device = p;
    return KB200_OK;
}

int kb200_weights_free(kb200_context* c, void* device) {
    if (!c)
        return fail(KB200_INVALID, "null context");
    DeviceScope scope(c->device);
    const cudaError_t e = cudaFree(device);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "weights_free");
}

int kb200_dense_gguf_batch(
    kb200_context* c, const kb200_host_job* jobs, size_t count, const volatile uint8_t* cancel, int* result
) {
    if (result)
        *result = KB200_RESULT_UNSUPPORTED;
    // Cancellation first, then an empty batch is unsupported (h3_compute.cu:3966-3968).
    if (c && cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled before start");
    if (!c || !jobs || !count)
        return fail(KB200_UNSUPPORTED, "empty batch");
    // Unsupported precedes every read and write (gguf_batch_supported).
    for (size_t j = 0; j < count; ++j) {
        const auto& job = jobs[j];
        if (!kb200_encoding_supported(job.encoding) || !job.weights || !job.input || !job.output || !job.in
            || !job.out || !job.rows || job.rows > KB200_BATCH_MAX_ROWS || job.in % 8
            || job.in % block_values(job.encoding)
            || job.row_bytes < size_t(job.in) / block_values(job.encoding) * block_bytes(job.encoding))
            return fail(KB200_UNSUPPORTED, "job outside the batched GEMV contract");
    }
    InputLayout inputs;
    if (const int s = layout_inputs(jobs, count, inputs))
        return s;
    std::vector<size_t> output_at(count);
    size_t outputs = 0;
    for (size_t j = 0; j < count; ++j) {
        output_at[j] = outputs;
        outputs += size_t(jobs[j].rows) * jobs[j].out;
    }
    if (const int s = check_aliases(jobs, count))
        return s;

    DeviceScope scope(c->device);
    ++c->counters.calls;
    // Device jobs over the workspace's spans (addresses filled in once it exists).
    std::vector<kb200_gemv_job> device_jobs(count);
    for (size_t j = 0; j < count; ++j) {
        const auto& job = jobs[j];
        device_jobs[j] = kb200_gemv_job{job.weights, nullptr, nullptr, nullptr, job.row_bytes, job.out,
                                        job.in,      job.out, job.rows, job.encoding};
    }
    // Device layout: [inputs][status: GEMV, GEMM][outputs][GEMM scratch], so
    // one upload carries the inputs and the cleared status words and one
    // download the status words and the outputs; host staging mirrors all
    // but the scratch.
    const size_t in_bytes = inputs.floats * sizeof(float), out_bytes = outputs * sizeof(float);
    const size_t status_at = up16(in_bytes), out_at = status_at + 16;
    const size_t scratch_at = up256(out_at + out_bytes), scratch = gemm_scratch(device_jobs.data(), count);
    if (const int s = ensure(c, scratch_at + scratch, out_at + out_bytes))
        return s;
    auto* dev = static_cast<uint8_t*>(c->workspace);
    auto* host = static_cast<uint8_t*>(c->pinned);
    stage_inputs(jobs, count, inputs, host);
    std::memset(host + status_at, 0, 2 * sizeof(unsigned));
    cudaError_t e = cudaMemcpyAsync(dev, host, status_at + 2 * sizeof(unsigned), cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "input upload");
    if (cancelled(cancel)) {
        cudaStreamSynchronize(c->stream);
        return fail(KB200_CANCELLED, "cancelled after upload");
    }
    auto* status = reinterpret_cast<unsigned*>(dev + status_at);
    for (size_t j = 0; j < count; ++j) {
        device_jobs[j].input = reinterpret_cast<const float*>(dev) + inputs.at[j];
        device_jobs[j].output = reinterpret_cast<float*>(dev + out_at) + output_at[j];
        device_jobs[j].status = jobs[j].validated ? nullptr : status;
    }
    if (const int s = launch_projections(c, device_jobs.data(), count, dev + scratch_at, scratch, status + 1)) {
        cudaStreamSynchronize(c->stream);
        return s;
    }
    e = cudaMemcpyAsync(host + status_at, dev + status_at, out_at + out_bytes - status_at, cudaMemcpyDeviceToHost,
                        c->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "output download");
    if (cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled after download");
    unsigned invalid = 0, gemm = 0;
    std::memcpy(&invalid, host + status_at, sizeof(invalid));
    std::memcpy(&gemm, host + status_at + sizeof(unsigned), sizeof(gemm));
    if (invalid || (gemm & 1u))
        return fail(KB200_NONFINITE_WEIGHT, "a decoded weight is not finite");
    if (gemm & 2u) {
        // A weight beyond the GEMM's fp16 operands: those jobs again on the GEMV path.
        if (const int s = rerun_gemm_jobs(c, device_jobs.data(), count)) {
            cudaStreamSynchronize(c->stream);
            return s;
        }
        e = cudaMemcpyAsync(host + out_at, dev + out_at, out_bytes, cudaMemcpyDeviceToHost, c->stream);
        if (e == cudaSuccess)
            e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess)
            return cuda_fail(e, "output download");
    }
    for (size_t j = 0; j < count; ++j)
        std::memcpy(jobs[j].output, host + out_at + output_at[j] * sizeof(float),
                    size_t(jobs[j].rows) * jobs[j].out * sizeof(float));
    if (result)
        *result = KB200_RESULT_UNVALIDATED;
    return KB200_OK;
}

}  // extern "C"

namespace kb200 {
namespace {

constexpr size_t kHalf = KB200_SOURCE_STAGING_HALF;

// One column chunk of a source job: its bank key, its place in the output
// and, when it streams, its byte offset inside a staging half.
struct Chunk {
    size_t job;
    uint64_t first_col, cols, bytes, row_bytes;
    kb200_weight_key key;
    const void* resident;
    size_t offset;
};

// Misses [begin, end) share one staging half; `used` bytes of it.
struct Group {
    size_t begin, end, used;
};

// gguf_batch_supported (IW/include/kadan/gguf_batch_partition.hpp:14-37): a
// row must fit one 16 MiB staging buffer, sizes fit an int, and the encoding
// has a decoder here.
bool source_job_supported(const kb200_source_job& job) {
    if (!kb200_encoding_supported(job.encoding) || !job.identity || !job.source || !job.input || !job.output
        || !job.in || !job.out || job.in > uint32_t(INT_MAX) || job.out > uint32_t(INT_MAX) || !job.rows
        || job.rows > KB200_BATCH_MAX_ROWS || job.in % 8)
        return false;
    const uint64_t values = kb200_block_values(job.encoding), width = kb200_block_bytes(job.encoding);
    return job.in % values == 0 && job.in / values <= kHalf / width;
}

}  // namespace
}  // namespace kb200

extern "C" {

int kb200_dense_gguf_source_batch(kb200_context* c, kb200_bank* bank, const kb200_source_job* jobs, size_t count,
                                  uint64_t scratch_limit, const volatile uint8_t* cancel, int* result) {
    if (result)
        *result = KB200_RESULT_UNSUPPORTED;
    // Cancellation first, then an empty batch is unsupported (h3_compute.cu:3966-3968).
    if (c && cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled before start");
    if (!c || !jobs || !count)
        return fail(KB200_UNSUPPORTED, "empty batch");
    // Unsupported precedes every source read and output write (gguf_batch_supported).
    for (size_t j = 0; j < count; ++j)
        if (!source_job_supported(jobs[j]))
            return fail(KB200_UNSUPPORTED, "job outside the batched GEMV contract");
    // The reference's chunk geometry on one device (gguf_batch_partition.hpp:44-83).
    const uint64_t one_device = 1, limit = scratch_limit ? scratch_limit : (uint64_t(1) << 30);
    std::vector<kb200_partition> parts(count);
    for (size_t j = 0; j < count; ++j)
        if (const int s = kb200_gguf_batch_partition(jobs[j].in, jobs[j].out, jobs[j].encoding, &one_device, 1, 0,
                                                     limit, &parts[j]))
            return s;
    InputLayout inputs;
    if (const int s = layout_inputs(jobs, count, inputs))
        return s;
    std::vector<size_t> output_at(count);
    size_t outputs = 0;
    for (size_t j = 0; j < count; ++j) {
        output_at[j] = outputs;
        outputs += size_t(jobs[j].rows) * jobs[j].out;
    }
    if (const int s = check_aliases(jobs, count))
        return s;
    if (bank && bank_device(bank) >= 0 && bank_device(bank) != c->device)
        return fail(KB200_INVALID, "the weight bank holds another device's memory");

    DeviceScope scope(c->device);
    ++c->counters.calls;
    // Bank lookups (h3_compute.cu:4063-4115): hits run from the bank, misses stream.
    std::vector<Chunk> hits, misses;
    for (size_t j = 0; j < count; ++j) {
        const auto& job = jobs[j];
        const uint64_t values = kb200_block_values(job.encoding), width = kb200_block_bytes(job.encoding);
        const uint64_t blocks_per_row = job.in / values, row_bytes = blocks_per_row * width;
        const auto& part = parts[j];
        for (uint64_t off = 0; off < part.count; off += part.chunk_columns) {
            const uint64_t cols = std::min<uint64_t>(part.chunk_columns, part.count - off), first = part.first + off;
            Chunk ch{j, first, cols, cols * row_bytes, row_bytes,
                     kb200_weight_key{*job.identity, first * blocks_per_row, cols * blocks_per_row, width},
                     nullptr, 0};
            void* hit = nullptr;
            if (bank)
                if (const int s = kb200_bank_find(bank, &ch.key, &hit))
                    return s;
            ch.resident = hit;
            (hit ? hits : misses).push_back(ch);
        }
    }
    std::vector<Group> groups;
    for (size_t k = 0; k < misses.size();) {
        Group g{k, k, 0};
        while (g.end < misses.size() && (g.end == g.begin || g.used + up256(misses[g.end].bytes) <= kHalf)) {
            if (misses[g.end].bytes > kHalf)
                return fail(KB200_INVALID, "gguf_projection_layout");
            misses[g.end].offset = g.used;
            g.used += up256(misses[g.end].bytes);
            ++g.end;
        }
        groups.push_back(g);
        k = g.end;
    }

    // GEMM scratch: every chunk of a job has the job's rows, in and row pitch,
    // and both bank entries and staging offsets are 256-byte aligned.
    size_t scratch = 0;
    for (size_t j = 0; j < count; ++j) {
        const auto& job = jobs[j];
        const uint64_t row_bytes = job.in / kb200_block_values(job.encoding) * kb200_block_bytes(job.encoding);
        const kb200_gemv_job probe{reinterpret_cast<const void*>(uintptr_t(256)), nullptr, nullptr, nullptr,
                                   size_t(row_bytes), job.out, job.in, job.out, job.rows, job.encoding};
        scratch = std::max(scratch, gemm_scratch(&probe, 1));
    }
    // Device layout: [inputs][outputs][status: half 0, half 1, bank hits]
    // [staging half 0][half 1][GEMM scratch]; the pinned host buffer mirrors
    // all but the scratch.
    const size_t in_bytes = up256(inputs.floats * sizeof(float)), out_bytes = up256(outputs * sizeof(float));
    const size_t status_at = in_bytes + out_bytes, staging_at = status_at + 256;
    const size_t total = staging_at + (groups.empty() ? 0 : 2 * kHalf);
    if (const int s = ensure(c, total + scratch, total))
        return s;
    uint8_t* dev_scratch = static_cast<uint8_t*>(c->workspace) + total;
    for (cudaEvent_t& e : c->staged)
        if (!e)
            if (const cudaError_t err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming))
                return cuda_fail(err, "cudaEventCreate");
    auto* dev = static_cast<uint8_t*>(c->workspace);
    auto* host = static_cast<uint8_t*>(c->pinned);
    auto* dev_in = reinterpret_cast<const float*>(dev);
    auto* dev_out = reinterpret_cast<float*>(dev + in_bytes);
    auto* dev_status = reinterpret_cast<unsigned*>(dev + status_at);
    auto* host_status = reinterpret_cast<volatile unsigned*>(host + status_at);
    uint8_t* dev_stage = dev + staging_at;
    uint8_t* host_stage = host + staging_at;
    auto abandon = [&](int status) {
        cudaStreamSynchronize(c->stream);
        return status;
    };
    auto device_job = [&](const Chunk& ch, const void* weights, unsigned* status) {
        const auto& job = jobs[ch.job];
        return kb200_gemv_job{weights, dev_in + inputs.at[ch.job], dev_out + output_at[ch.job] + ch.first_col,
                              status, size_t(ch.row_bytes), job.out, job.in, uint32_t(ch.cols), job.rows,
                              job.encoding};
    };

    stage_inputs(jobs, count, inputs, host);
    if (const cudaError_t e = cudaMemcpyAsync(dev, host, inputs.floats * sizeof(float), cudaMemcpyHostToDevice,
                                              c->stream))
        return abandon(cuda_fail(e, "input upload"));
    std::vector<kb200_gemv_job> hit_jobs;
    if (!hits.empty()) {
        // Bank entries were checked finite when they were admitted.
        for (const Chunk& ch : hits)
            hit_jobs.push_back(device_job(ch, ch.resident, nullptr));
        if (const cudaError_t e = cudaMemsetAsync(dev_status + 2, 0, sizeof(unsigned), c->stream))
            return abandon(cuda_fail(e, "status clear"));
        if (const int s = launch_projections(c, hit_jobs.data(), hit_jobs.size(), dev_scratch, scratch, dev_status + 2))
            return abandon(s);
    }
    std::vector<std::vector<kb200_gemv_job>> group_jobs(groups.size());
    // Group g uses half g % 2; before it is refilled, group g - 2 is finished:
    // its status read, and its chunks admitted while their bytes are still staged.
    auto finish = [&](size_t g) -> int {
        const size_t half = g % 2;
        if (const cudaError_t e = cudaEventSynchronize(c->staged[half]))
            return cuda_fail(e, "streamed group");
        if (host_status[half] & 1u)
            return fail(KB200_NONFINITE_WEIGHT, "a decoded weight is not finite");
        // A weight beyond the GEMM's fp16 operands: the group's GEMM chunks
        // again on the GEMV path while their bytes are staged (the half is
        // refilled later on the same stream).
        if (host_status[half] & 2u)
            if (const int s = rerun_gemm_jobs(c, group_jobs[g].data(), group_jobs[g].size()))
                return s;
        if (cancelled(cancel))
            return fail(KB200_CANCELLED, "cancelled after a streamed group");
        if (!bank)
            return KB200_OK;
        for (size_t k = groups[g].begin; k < groups[g].end; ++k) {
            const Chunk& m = misses[k];
            if (!jobs[m.job].retain_misses)
                continue;
            void* kept = nullptr;
            int refusal = 0;
            if (const int s = kb200_bank_retain_device(bank, &m.key, dev_stage + half * kHalf + m.offset, m.bytes,
                                                       cancel, &kept, &refusal))
                return s;
        }
        return KB200_OK;
    };
    if (!groups.empty() && !c->team) {
        try {
            c->team = new ReadTeam(c->read_lanes);
        } catch (...) {
            return abandon(fail(KB200_NO_MEMORY, "read team threads"));
        }
    }
    std::vector<ReadItem> reads;
    for (size_t g = 0; g < groups.size(); ++g) {
        const size_t half = g % 2;
        if (g >= 2)
            if (const int s = finish(g - 2))
                return abandon(s);
        if (cancelled(cancel))
            return abandon(fail(KB200_CANCELLED, "cancelled before a streamed group"));
        uint8_t* staged = host_stage + half * kHalf;
        std::vector<kb200_gemv_job>& launch = group_jobs[g];
        reads.clear();
        for (size_t k = groups[g].begin; k < groups[g].end; ++k) {
            const Chunk& m = misses[k];
            const auto& job = jobs[m.job];
            split_read(reads, job.source, job.source_user, m.first_col, m.cols, m.row_bytes, staged + m.offset,
                       c->read_lanes);
            launch.push_back(device_job(m, dev_stage + half * kHalf + m.offset, dev_status + half));
        }
        if (const int s = c->team->run(reads))
            return abandon(fail(s, "packed-row source failed"));
        cudaError_t e = cudaMemcpyAsync(dev_stage + half * kHalf, staged, groups[g].used, cudaMemcpyHostToDevice,
                                        c->stream);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(dev_status + half, 0, sizeof(unsigned), c->stream);
        if (e != cudaSuccess)
            return abandon(cuda_fail(e, "staging upload"));
        if (const int s = launch_projections(c, launch.data(), launch.size(), dev_scratch, scratch, dev_status + half))
            return abandon(s);
        e = cudaMemcpyAsync(const_cast<unsigned*>(host_status + half), dev_status + half, sizeof(unsigned),
                            cudaMemcpyDeviceToHost, c->stream);
        if (e == cudaSuccess)
            e = cudaEventRecord(c->staged[half], c->stream);
        if (e != cudaSuccess)
            return abandon(cuda_fail(e, "staging status"));
    }
    for (size_t g = groups.size() >= 2 ? groups.size() - 2 : 0; g < groups.size(); ++g)
        if (const int s = finish(g))
            return abandon(s);
    // Outputs and, right after them, the status words (the bank hits' last).
    cudaError_t e = cudaMemcpyAsync(host + in_bytes, dev_out, out_bytes + 3 * sizeof(unsigned), cudaMemcpyDeviceToHost,
                                    c->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess)
        return abandon(cuda_fail(e, "output download"));
    if (cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled after download");
    const unsigned hit_status = hits.empty() ? 0u : host_status[2];
    if (hit_status & 1u)
        return fail(KB200_NONFINITE_WEIGHT, "a decoded weight is not finite");
    if (hit_status & 2u) {
        if (const int s = rerun_gemm_jobs(c, hit_jobs.data(), hit_jobs.size()))
            return abandon(s);
        e = cudaMemcpyAsync(host + in_bytes, dev_out, outputs * sizeof(float), cudaMemcpyDeviceToHost, c->stream);
        if (e == cudaSuccess)
            e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess)
            return abandon(cuda_fail(e, "output download"));
    }
    for (size_t j = 0; j < count; ++j)
        std::memcpy(jobs[j].output, host + in_bytes + output_at[j] * sizeof(float),
                    size_t(jobs[j].rows) * jobs[j].out * sizeof(float));
    if (result)
        *result = KB200_RESULT_UNVALIDATED;
    return KB200_OK;
}

int kb200_source_job_supported(const kb200_source_job* job) {
    return job && source_job_supported(*job) ? 1 : 0;
}

int kb200_dense_gguf_source(kb200_context* c, kb200_bank* bank, const kb200_source_job* job, const float* bias,
                            uint64_t scratch_limit, int precise, const volatile uint8_t* cancel, int* result) {
    if (result)
        *result = KB200_RESULT_UNSUPPORTED;
    if (!c || !job || !source_job_supported(*job))
        return fail(KB200_UNSUPPORTED, "job outside the projection contract");
    if (precise)
        return fail(KB200_UNSUPPORTED, "fp64 (precise) projections are not offered");
    if (bias)
        for (uint32_t o = 0; o < job->out; ++o)
            if (!std::isfinite(bias[o]))
                return fail(KB200_NONFINITE_BIAS, "non-finite bias value");
    if (bias && overlap(job->output, size_t(job->rows) * job->out * sizeof(float), bias, size_t(job->out) * sizeof(float)))
        return fail(KB200_ALIAS, "output overlaps the bias");
    int batch_result = KB200_RESULT_UNSUPPORTED;
    if (const int s = kb200_dense_gguf_source_batch(c, bank, job, 1, scratch_limit, cancel, &batch_result))
        return s;
    const size_t n = size_t(job->rows) * job->out;
    for (size_t i = 0; i < n; ++i) {
        float& y = job->output[i];
        if (bias)
            y += bias[i % job->out];
        if (!std::isfinite(y))
            return fail(KB200_NONFINITE_OUTPUT, "a projection output is not finite");
    }
    if (result)
        *result = KB200_RESULT_FINITE;
    return KB200_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- MoE layer
extern "C" {

int kb200_moe_forward_host(kb200_context* c, const kb200_moe_weights* w, const float* x, const float* logits,
                           size_t tokens, float* out, const volatile uint8_t* cancel, int* result) {
    using namespace kb200;
    if (result)
        *result = KB200_RESULT_UNSUPPORTED;
    if (c && cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled before start");
    // Unsupported first: nothing read from the caller and nothing written.
    const size_t need = w ? kb200_moe_workspace_bytes(w, tokens) : 0;
    if (!c || !w || !tokens || !x || !logits || !out || !need)
        return fail(KB200_UNSUPPORTED, "MoE call outside the layer's contract");
    const size_t H = size_t(w->hidden), E = size_t(w->experts);
    const size_t x_bytes = tokens * H * sizeof(float), l_bytes = tokens * E * sizeof(float);
    if (overlap(out, x_bytes, x, x_bytes) || overlap(out, x_bytes, logits, l_bytes))
        return fail(KB200_ALIAS, "output overlaps an input");
    for (size_t i = 0; i < tokens * H; ++i)
        if (!std::isfinite(x[i]))
            return fail(KB200_NONFINITE_INPUT, "non-finite input value");
    for (size_t i = 0; i < tokens * E; ++i)
        if (!std::isfinite(logits[i]))
            return fail(KB200_NONFINITE_INPUT, "non-finite router logit");
    DeviceScope scope(c->device);
    ++c->counters.calls;
    // Device: [x][logits][out][status][layer workspace]; host mirrors all but the workspace.
    const size_t l_at = up256(x_bytes), o_at = l_at + up256(l_bytes), s_at = o_at + up256(x_bytes);
    const size_t ws_at = s_at + 256;
    if (const int s = ensure(c, ws_at + need, ws_at))
        return s;
    auto* dev = static_cast<uint8_t*>(c->workspace);
    auto* host = static_cast<uint8_t*>(c->pinned);
    std::memcpy(host, x, x_bytes);
    std::memcpy(host + l_at, logits, l_bytes);
    std::memset(host + s_at, 0, sizeof(unsigned));
    cudaError_t e = cudaMemcpyAsync(dev, host, o_at, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(dev + s_at, host + s_at, sizeof(unsigned), cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "MoE input upload");
    auto* status = reinterpret_cast<unsigned*>(dev + s_at);
    if (const int s = kb200_moe_forward_f32(w, reinterpret_cast<const float*>(dev),
                                            reinterpret_cast<const float*>(dev + l_at), tokens,
                                            reinterpret_cast<float*>(dev + o_at), dev + ws_at, need, status,
                                            c->stream)) {
        cudaStreamSynchronize(c->stream);
        return s;
    }
    e = cudaMemcpyAsync(host + o_at, dev + o_at, s_at + sizeof(unsigned) - o_at, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "MoE output download");
    if (cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled after download");
    unsigned flags = 0;
    std::memcpy(&flags, host + s_at, sizeof(flags));
    // Scales or activations the fp16 operands cannot hold exactly: the
    // caller's own path must take the layer (nothing of its output written).
    if (flags & 6u)
        return fail(KB200_UNSUPPORTED, flags & 2u ? "MXFP4 scale outside the exact fp16 range"
                                                  : "activation outside the fp16 range");
    const auto* y = reinterpret_cast<const float*>(host + o_at);
    for (size_t i = 0; i < tokens * H; ++i)
        if (!std::isfinite(y[i]))
            return fail(KB200_NONFINITE_OUTPUT, "a layer output is not finite");
    std::memcpy(out, y, x_bytes);
    if (result)
        *result = KB200_RESULT_FINITE;
    return KB200_OK;
}

}  // extern "C"
