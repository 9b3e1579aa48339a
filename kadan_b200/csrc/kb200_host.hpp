// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "kadan_b200.h"

namespace kb200 {

// Record `what` as the calling thread's last error and return `status`.
int fail(int status, const char* what);
int cuda_fail(cudaError_t code, const char* where);

// Byte ranges [a, a+an) and [b, b+bn) share an address (the reference's
// alias rule, IW/src/cuda/h3_compute.cu:60-66).
inline bool overlap(const void* a, size_t an, const void* b, size_t bn) {
    if (!an || !bn)
        return false;
    const auto x = reinterpret_cast<std::uintptr_t>(a), y = reinterpret_cast<std::uintptr_t>(b);
    return x <= y ? y - x < an : x - y < bn;
}

inline bool aligned(const void* p, size_t to) {
    return reinterpret_cast<std::uintptr_t>(p) % to == 0;
}

// Makes `device` current for the scope and restores the previous device.
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
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;
};

// Device address of the watchdog word (a file-scope __device__ variable of
// core.cu) on the current device; kernels with bounded waits report there.
unsigned* watchdog_word();

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

// Zero every fixup buffer of the Q4_K GEMV on the current device (after a
// launch gave up, its cut tiles' partial words may be left behind). Synchronous.
void clear_gemv_fixups();

// The prefill GEMM (kb200_gguf_gemm) takes the job's weights.
bool gemm_eligible(const kb200_gemv_job& j);

// Counts and times one kernel launch for the calling thread's current phase
// (kb200_phase_enter): construct it right before the launch and let it go out
// of scope right after. Without a current phase it does nothing.
class TraceScope {
public:
    TraceScope(kb200_kernel id, cudaStream_t stream);
    ~TraceScope();
    TraceScope(const TraceScope&) = delete;
    TraceScope& operator=(const TraceScope&) = delete;

private:
    bool active_ = false, timed_ = false;
    int kernel_ = 0;
    cudaStream_t stream_ = nullptr;
    void* start_ = nullptr;  // CUevent
    void* end_ = nullptr;    // CUevent
    double t0_ = 0.0;
};

// The CUDA device whose memory a weight bank holds, or -1 for a bank over
// caller-supplied operations.
int bank_device(const kb200_bank* bank);

}  // namespace kb200
