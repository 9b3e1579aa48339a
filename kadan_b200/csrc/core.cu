// C-ABI housekeeping (status text, last error, watchdog word) and the exact
// dequantisation kernel.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "gguf_formats.cuh"
#include "kb200_device.cuh"
#include "kb200_host.hpp"

namespace kb200 {

namespace {

// Host copies of the caller's IQ code grids; published once, never changed.
uint32_t iq3xxs_grid_host[256], iq3s_grid_host[512];
unsigned long long iq2s_grid_host[1024];
const IqGrids iq_grids_host{iq3xxs_grid_host, iq2s_grid_host, iq3s_grid_host};
std::atomic<bool> iq_grids_set{false};
std::mutex iq_grids_lock;

}  // namespace

const IqGrids* registered_iq_grids() {
    return iq_grids_set.load(std::memory_order_acquire) ? &iq_grids_host : nullptr;
}

// Set (one bit per cause) by a kernel whose bounded wait ran out; read and
// cleared by kb200_take_device_error(). A file-scope device variable.
__device__ unsigned device_error = 0;

namespace {
thread_local char error_text[512];
}

unsigned* watchdog_word() {
    // One slot per device, filled on first use; threads that drive different
    // devices may race to fill a slot, so slots are atomic (every racer
    // stores the same address).
    static std::atomic<unsigned*> cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return nullptr;
    unsigned* word = cached[dev].load(std::memory_order_acquire);
    if (!word) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, device_error) == cudaSuccess) {
            word = static_cast<unsigned*>(p);
            cached[dev].store(word, std::memory_order_release);
        }
    }
    return word;
}

int fail(int status, const char* what) {
    std::snprintf(error_text, sizeof(error_text), "%s: %s", kb200_status_name(status), what);
    return status;
}

int cuda_fail(cudaError_t code, const char* where) {
    std::snprintf(error_text, sizeof(error_text), "h3_cuda: %s (%s)", cudaGetErrorString(code), where);
    return KB200_CUDA;
}

// Decode `count` values; each thread writes one value so stores stay coalesced.
template <bool Grids>
__global__ void dequant_kernel(
    int encoding, const uint8_t* packed, size_t count, float* out, unsigned* status
) {
    const int values = block_values(encoding), bytes = block_bytes(encoding);
    bool bad = false;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += size_t(gridDim.x) * blockDim.x) {
        const float v = decode_value<Grids>(encoding, packed + i / values * bytes, unsigned(i % values));
        out[i] = v;
        bad |= !isfinite(v);
    }
    if (bad && status)
        atomicOr(status, 1u);
}

}  // namespace kb200

using namespace kb200;

extern "C" {

const char* kb200_status_name(int status) {
    switch (status) {
    case KB200_OK: return "ok";
    case KB200_UNSUPPORTED: return "unsupported";
    case KB200_INVALID: return "h3_cuda_invalid_argument";
    case KB200_CUDA: return "h3_cuda";
    case KB200_NONFINITE_WEIGHT: return "h3_cuda_nonfinite_weight";
    case KB200_NONFINITE_INPUT: return "h3_cuda_nonfinite_input";
    case KB200_ALIAS: return "h3_cuda_alias";
    case KB200_CANCELLED: return "h3_cuda_cancelled";
    case KB200_TIMEOUT: return "kb200_device_wait_timeout";
    case KB200_NO_MEMORY: return "h3_cuda_projection_scratch";
    case KB200_QUARANTINED: return "weight_cleanup_unconfirmed";
    case KB200_IO: return "gguf_io";
    case KB200_NONFINITE_BIAS: return "h3_cuda_nonfinite_bias";
    case KB200_NONFINITE_OUTPUT: return "h3_cuda_nonfinite_output";
    default: return "kb200_unknown_status";
    }
}

const char* kb200_last_error(void) {
    return error_text;
}

int kb200_version(void) {
    return 1;
}

int kb200_encoding_supported(int encoding) {
    return encoding == KB200_F32 || decodable(encoding) || (grid_coded(encoding) && registered_iq_grids()) ? 1 : 0;
}

int kb200_set_iq_grids(const uint32_t* iq3xxs, const uint64_t* iq2s, const uint32_t* iq3s) {
    if (!iq3xxs || !iq2s || !iq3s)
        return fail(KB200_INVALID, "null IQ code grid");
    std::lock_guard<std::mutex> guard(iq_grids_lock);
    if (iq_grids_set.load(std::memory_order_relaxed)) {
        const bool same = !std::memcmp(iq3xxs_grid_host, iq3xxs, sizeof(iq3xxs_grid_host))
                          && !std::memcmp(iq2s_grid_host, iq2s, sizeof(iq2s_grid_host))
                          && !std::memcmp(iq3s_grid_host, iq3s, sizeof(iq3s_grid_host));
        return same ? KB200_OK : fail(KB200_INVALID, "IQ code grids are already registered with other values");
    }
    std::memcpy(iq3xxs_grid_host, iq3xxs, sizeof(iq3xxs_grid_host));
    std::memcpy(iq2s_grid_host, iq2s, sizeof(iq2s_grid_host));
    std::memcpy(iq3s_grid_host, iq3s, sizeof(iq3s_grid_host));
    iq_grids_set.store(true, std::memory_order_release);
    return KB200_OK;
}

size_t kb200_block_values(int encoding) {
    return kb200_encoding_supported(encoding) ? size_t(block_values(encoding)) : 0;
}

size_t kb200_block_bytes(int encoding) {
    return kb200_encoding_supported(encoding) ? size_t(block_bytes(encoding)) : 0;
}

int kb200_take_device_error(unsigned* value) {
    unsigned v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, device_error, sizeof(v));
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbol(device_error, &zero, sizeof(zero));
    if (e != cudaSuccess)
        return cuda_fail(e, "kb200_take_device_error");
    if (value)
        *value = v;
    // A launch that gave up may have left partial sums of cut tiles behind.
    if (v)
        clear_gemv_fixups();
    return v ? fail(KB200_TIMEOUT, "a bounded device wait gave up") : KB200_OK;
}

int kb200_gguf_dequant(
    int encoding, const void* packed, size_t count, float* out, unsigned* status, void* stream
) {
    if (encoding == KB200_F32 || !kb200_encoding_supported(encoding))
        return fail(KB200_UNSUPPORTED, "encoding has no device decoder");
    if (count % size_t(block_values(encoding)))
        return fail(KB200_INVALID, "count is not whole blocks");
    if (!count)
        return KB200_OK;
    if (!packed || !out)
        return fail(KB200_INVALID, "null pointer");
    const size_t packed_bytes = count / block_values(encoding) * block_bytes(encoding);
    if (overlap(out, count * sizeof(float), packed, packed_bytes))
        return fail(KB200_ALIAS, "output overlaps packed input");
    if (const int s = ensure_iq_grids(encoding))
        return s;
    const unsigned threads = 256;
    const size_t want = (count + threads - 1) / threads;
    const unsigned blocks = unsigned(want < 148u * 16u ? want : 148u * 16u);
    TraceScope trace(KB200_KERNEL_GGUF_DEQUANT, static_cast<cudaStream_t>(stream));
    if (grid_coded(encoding))
        dequant_kernel<true><<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
            encoding, static_cast<const uint8_t*>(packed), count, out, status
        );
    else
        dequant_kernel<false><<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
            encoding, static_cast<const uint8_t*>(packed), count, out, status
        );
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "dequant_kernel launch");
}

}  // extern "C"
