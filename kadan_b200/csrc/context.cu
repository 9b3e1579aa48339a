// Host-span boundary: kb200_context and kb200_dense_gguf_batch, the
// reference's DenseCompute::dense_gguf_batch contract
// (services/hikari/inference_worker/src/cuda/h3_compute.cu:3963-4375) over
// device-resident weights. One input upload, one launch per encoding, one
// download, one stream synchronisation per call.
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "gguf_formats.cuh"
#include "kb200_host.hpp"

struct kb200_context {
    int device = 0;
    cudaStream_t stream = nullptr;
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
    void* pinned = nullptr;
    size_t pinned_bytes = 0;
};

namespace kb200 {
namespace {

struct DeviceScope {
    int previous = -1;
    explicit DeviceScope(int device) {
        cudaGetDevice(&previous);
        if (previous != device)
            cudaSetDevice(device);
    }
    ~DeviceScope() {
        int now = -1;
        cudaGetDevice(&now);
        if (previous >= 0 && now != previous)
            cudaSetDevice(previous);
    }
};

int ensure(kb200_context* c, size_t device_bytes, size_t host_bytes) {
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

bool cancelled(const volatile int* cancel) {
    return cancel && *cancel;
}

size_t up16(size_t v) {
    return (v + 15) / 16 * 16;
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
    cudaStreamDestroy(c->stream);
    delete c;
}

void* kb200_context_stream(kb200_context* c) {
    return c ? static_cast<void*>(c->stream) : nullptr;
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
    kb200_context* c, const kb200_host_job* jobs, size_t count, const volatile int* cancel, int* result
) {
    if (result)
        *result = KB200_RESULT_UNSUPPORTED;
    if (!c || !jobs || !count)
        return fail(KB200_UNSUPPORTED, "empty batch");
    if (cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled before start");
    // Unsupported precedes every read and write (gguf_batch_supported).
    for (size_t j = 0; j < count; ++j) {
        const auto& job = jobs[j];
        if (!kb200_encoding_supported(job.encoding) || !job.weights || !job.input || !job.output || !job.in
            || !job.out || !job.rows || job.rows > KB200_BATCH_MAX_ROWS || job.in % 8
            || job.in % block_values(job.encoding)
            || job.row_bytes < size_t(job.in) / block_values(job.encoding) * block_bytes(job.encoding))
            return fail(KB200_UNSUPPORTED, "job outside the batched GEMV contract");
    }
    // Jobs sharing an input span upload and check it once (h3_compute.cu:3972-3991).
    std::vector<size_t> input_at(count);
    size_t inputs = 0, outputs = 0;
    for (size_t j = 0; j < count; ++j) {
        size_t shared = 0;
        while (shared < j
               && (jobs[shared].input != jobs[j].input
                   || size_t(jobs[shared].rows) * jobs[shared].in != size_t(jobs[j].rows) * jobs[j].in))
            ++shared;
        if (shared < j) {
            input_at[j] = input_at[shared];
            continue;
        }
        const size_t n = size_t(jobs[j].rows) * jobs[j].in;
        for (size_t i = 0; i < n; ++i)
            if (!std::isfinite(jobs[j].input[i]))
                return fail(KB200_NONFINITE_INPUT, "non-finite input value");
        input_at[j] = inputs;
        inputs += up16(n);  // keep every input 64-byte aligned on the device
    }
    std::vector<size_t> output_at(count);
    for (size_t j = 0; j < count; ++j) {
        output_at[j] = outputs;
        outputs += size_t(jobs[j].rows) * jobs[j].out;
    }
    for (size_t j = 0; j < count; ++j)
        for (size_t k = 0; k < count; ++k)
            if (overlap(jobs[j].output, size_t(jobs[j].rows) * jobs[j].out * sizeof(float), jobs[k].input,
                        size_t(jobs[k].rows) * jobs[k].in * sizeof(float)))
                return fail(KB200_ALIAS, "output overlaps an input");

    DeviceScope scope(c->device);
    // Device layout: [inputs][outputs][status]; host staging mirrors it.
    const size_t in_bytes = inputs * sizeof(float), out_bytes = outputs * sizeof(float);
    const size_t status_at = up16(in_bytes + out_bytes);
    const size_t total = status_at + 16;
    if (const int s = ensure(c, total, total))
        return s;
    auto* dev = static_cast<uint8_t*>(c->workspace);
    auto* host = static_cast<uint8_t*>(c->pinned);
    for (size_t j = 0; j < count; ++j) {
        bool first = true;
        for (size_t k = 0; k < j; ++k)
            if (input_at[k] == input_at[j])
                first = false;
        if (first)
            std::memcpy(host + input_at[j] * sizeof(float), jobs[j].input,
                        size_t(jobs[j].rows) * jobs[j].in * sizeof(float));
    }
    std::memset(host + status_at, 0, sizeof(unsigned));
    cudaError_t e = cudaMemcpyAsync(dev, host, in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(dev + status_at, host + status_at, sizeof(unsigned), cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "input upload");
    if (cancelled(cancel)) {
        cudaStreamSynchronize(c->stream);
        return fail(KB200_CANCELLED, "cancelled after upload");
    }
    std::vector<kb200_gemv_job> device_jobs(count);
    auto* status = reinterpret_cast<unsigned*>(dev + status_at);
    for (size_t j = 0; j < count; ++j) {
        const auto& job = jobs[j];
        device_jobs[j] = kb200_gemv_job{
            job.weights,
            reinterpret_cast<const float*>(dev) + input_at[j],
            reinterpret_cast<float*>(dev + in_bytes) + output_at[j],
            job.validated ? nullptr : status,
            job.row_bytes,
            job.out,
            job.in,
            job.out,
            job.rows,
            job.encoding};
    }
    if (const int s = kb200_gguf_gemv_batch(device_jobs.data(), count, c->stream)) {
        cudaStreamSynchronize(c->stream);
        return s;
    }
    e = cudaMemcpyAsync(host + in_bytes, dev + in_bytes, status_at + sizeof(unsigned) - in_bytes,
                        cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "output download");
    if (cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled after download");
    unsigned invalid = 0;
    std::memcpy(&invalid, host + status_at, sizeof(invalid));
    if (invalid)
        return fail(KB200_NONFINITE_WEIGHT, "a decoded weight is not finite");
    for (size_t j = 0; j < count; ++j)
        std::memcpy(jobs[j].output, host + in_bytes + output_at[j] * sizeof(float),
                    size_t(jobs[j].rows) * jobs[j].out * sizeof(float));
    if (result)
        *result = KB200_RESULT_UNVALIDATED;
    return KB200_OK;
}

}  // extern "C"
