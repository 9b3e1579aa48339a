// Per-kernel telemetry: phases, launch counts, host and device seconds.
//
// The reference keeps one phase per model thread (CudaPhaseScope,
// IW/include/kadan/cuda_phase_metrics.hpp:89-140) and times each launch with a
// pair of driver-API events read back without waiting (cuda_trace::kernel and
// collect, IW/src/cuda/cuda_telemetry.cuh:45-160). The same contract here: a
// thread-local ring of at most 128 pending event pairs per thread, owned by
// the phase that was current when they were recorded; pairs are read at later
// launches, at snapshots and when the thread changes phase. The driver API is
// used so that telemetry neither sets nor clears the runtime's last error,
// which the launch sites read right after their launches; its entry points
// are looked up through the runtime, so the library does not link libcuda.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cuda.h>
#include <mutex>
#include <new>
#include <type_traits>

#include "kb200_host.hpp"

struct kb200_phase {
    std::atomic<int> refs{1};
    std::mutex lock;
    kb200_phase_metrics metrics{};
};

namespace kb200 {
namespace {

using Clock = std::chrono::steady_clock;

struct Driver {
    CUresult (*event_create)(CUevent*, unsigned) = nullptr;
    CUresult (*event_record)(CUevent, CUstream) = nullptr;
    CUresult (*event_query)(CUevent) = nullptr;
    CUresult (*event_elapsed)(float*, CUevent, CUevent) = nullptr;
    CUresult (*event_destroy)(CUevent) = nullptr;
    CUresult (*stream_capturing)(CUstream, CUstreamCaptureStatus*) = nullptr;
    CUresult (*ctx_current)(CUcontext*) = nullptr;
    bool ok = false;
};

// The driver functions, looked up once; ok is false when any is missing.
const Driver& driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        auto get = [](const char* name, auto& fn) {
            void* p = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q) == cudaSuccess
                && q == cudaDriverEntryPointSuccess && p) {
                fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(p);
                return true;
            }
            cudaGetLastError();  // a failed lookup leaves no error behind for the launch sites
            return false;
        };
        d.ok = get("cuEventCreate", d.event_create) && get("cuEventRecord", d.event_record)
               && get("cuEventQuery", d.event_query) && get("cuEventElapsedTime", d.event_elapsed)
               && get("cuEventDestroy", d.event_destroy) && get("cuStreamIsCapturing", d.stream_capturing)
               && get("cuCtxGetCurrent", d.ctx_current);
    });
    return d;
}

void acquire(kb200_phase* p) {
    if (p)
        p->refs.fetch_add(1, std::memory_order_relaxed);
}

void release(kb200_phase* p) {
    if (p && p->refs.fetch_sub(1, std::memory_order_acq_rel) == 1)
        delete p;
}

template <class F> void update(kb200_phase* p, F f) {
    if (!p)
        return;
    std::lock_guard<std::mutex> guard(p->lock);
    p->metrics.observed = 1;
    f(p->metrics);
}

struct Pending {
    CUevent start = nullptr, end = nullptr;
    int kernel = 0;
};

struct Events {
    static constexpr int kCapacity = 128;
    Pending pending[kCapacity];
    int size = 0;
    kb200_phase* owner = nullptr;  // referenced
    bool disabled = false;         // an event could not be destroyed: stop making more

    void destroy(const Pending& pair) {
        for (CUevent e : {pair.start, pair.end})
            if (e && driver().event_destroy(e) != CUDA_SUCCESS) {
                disabled = true;
                update(owner, [](kb200_phase_metrics& m) { ++m.unavailable; });
            }
    }

    // Reads every finished pair; with `terminal`, unfinished ones are dropped.
    void collect(bool terminal) {
        int kept = 0;
        for (int i = 0; i < size; ++i) {
            const Pending pair = pending[i];
            const CUresult status = driver().event_query(pair.end);
            if (status == CUDA_ERROR_NOT_READY && !terminal) {
                pending[kept++] = pair;
                continue;
            }
            if (status == CUDA_SUCCESS) {
                float ms = 0.f;
                if (driver().event_elapsed(&ms, pair.start, pair.end) == CUDA_SUCCESS && std::isfinite(ms) && ms >= 0.f)
                    update(owner, [&](kb200_phase_metrics& m) {
                        ++m.kernels[pair.kernel].measured;
                        m.kernels[pair.kernel].gpu_seconds += double(ms) / 1000.0;
                    });
                else
                    update(owner, [](kb200_phase_metrics& m) { ++m.unavailable; });
            } else if (status == CUDA_ERROR_NOT_READY) {
                update(owner, [](kb200_phase_metrics& m) { ++m.dropped; });
            } else {
                update(owner, [](kb200_phase_metrics& m) { ++m.unavailable; });
            }
            destroy(pair);
        }
        size = kept;
    }

    void finalize() {
        collect(true);
        release(owner);
        owner = nullptr;
    }

    ~Events() { finalize(); }
};

struct Current {
    kb200_phase* phase = nullptr;  // referenced
    ~Current() { release(phase); }
};

thread_local Events events;
thread_local Current current;

// Binds the event ring to the thread's current phase; false when none.
bool prepare() {
    if (events.owner != current.phase) {
        events.finalize();
        acquire(current.phase);
        events.owner = current.phase;
    }
    return events.owner != nullptr;
}

const char* const kNames[KB200_KERNEL_COUNT] = {
    "dequant_kernel",         "gemv_staged_kernel",     "gemv_generic_kernel",       "gemv_q4k_mma_kernel",
    "gemv_q6k_mma_kernel",    "gemv_q6k_pair_kernel",   "prefill_rows_kernel",       "gemm_gguf_kernel",
    "moe_route_kernel",       "moe_sort_kernel",        "moe_gather_kernel",         "moe_mtile_kernel",
    "moe_gemm_kernel",        "moe_gemv_kernel",        "moe_combine_kernel",        "rows_regroup_kernel",
    "mxfp4_ggml_dequant_kernel", "mxfp4_from_ggml_kernel", "peer_allreduce_kernel",  "ep_exchange_kernel",
    "rms_norm_kernel",        "rope_kernel",            "attend_kernel",             "attend_combine_kernel",
    "delta_conv_kernel",      "delta_l2_kernel",        "delta_heads_kernel",        "silu_mul_kernel",
    "moe_shared_kernel",      "moe_decode_kernel",      "pair_quant_kernel",         "q4k_quant_kernel",
};

}  // namespace

TraceScope::TraceScope(kb200_kernel id, cudaStream_t stream) {
    if (!prepare())
        return;
    active_ = true;
    kernel_ = int(id);
    stream_ = stream;
    if (events.size == Events::kCapacity)
        events.collect(false);
    if (events.size == Events::kCapacity) {
        update(events.owner, [](kb200_phase_metrics& m) { ++m.dropped; });
    } else if (events.disabled || !driver().ok) {
        update(events.owner, [](kb200_phase_metrics& m) { ++m.unavailable; });
    } else {
        // A launch into a capturing stream runs later, as part of a graph:
        // it is counted, not timed.
        const Driver& d = driver();
        CUstreamCaptureStatus capture = CU_STREAM_CAPTURE_STATUS_NONE;
        CUcontext context = nullptr;
        if (d.stream_capturing(reinterpret_cast<CUstream>(stream), &capture) == CUDA_SUCCESS
            && capture == CU_STREAM_CAPTURE_STATUS_NONE) {
            CUevent a = nullptr, b = nullptr;
            timed_ = d.ctx_current(&context) == CUDA_SUCCESS && context
                     && d.event_create(&a, CU_EVENT_DEFAULT) == CUDA_SUCCESS
                     && d.event_create(&b, CU_EVENT_DEFAULT) == CUDA_SUCCESS
                     && d.event_record(a, reinterpret_cast<CUstream>(stream)) == CUDA_SUCCESS;
            start_ = a, end_ = b;
            if (!timed_) {
                update(events.owner, [](kb200_phase_metrics& m) { ++m.unavailable; });
                events.destroy(Pending{a, b, kernel_});
                start_ = end_ = nullptr;
            }
        }
    }
    t0_ = std::chrono::duration<double>(Clock::now().time_since_epoch()).count();
}

TraceScope::~TraceScope() {
    if (!active_)
        return;
    const double host = std::chrono::duration<double>(Clock::now().time_since_epoch()).count() - t0_;
    // Close the device interval before the phase lock, so contention on the
    // lock is not charged to the kernel.
    const bool recorded = timed_ && driver().event_record(static_cast<CUevent>(end_), reinterpret_cast<CUstream>(stream_))
                                        == CUDA_SUCCESS;
    const int k = kernel_;
    update(events.owner, [&](kb200_phase_metrics& m) {
        ++m.kernels[k].calls;
        m.kernels[k].host_seconds += host;
    });
    if (!timed_)
        return;
    const Pending pair{static_cast<CUevent>(start_), static_cast<CUevent>(end_), k};
    if (recorded && events.size < Events::kCapacity) {
        events.pending[events.size++] = pair;
    } else {
        update(events.owner, [](kb200_phase_metrics& m) { ++m.unavailable; });
        events.destroy(pair);
    }
}

}  // namespace kb200

using namespace kb200;

extern "C" {

int kb200_phase_create(uint64_t shared_batch_size, kb200_phase** out) {
    if (!out)
        return fail(KB200_INVALID, "null output");
    auto* p = new (std::nothrow) kb200_phase;
    if (!p)
        return fail(KB200_NO_MEMORY, "phase allocation");
    p->metrics.shared_batch_size = shared_batch_size ? shared_batch_size : 1;
    *out = p;
    return KB200_OK;
}

int kb200_phase_enter(kb200_phase* phase, kb200_phase** previous) {
    // Pairs recorded under the old phase are read (or dropped) first, as the
    // reference's scope change does.
    events.finalize();
    acquire(phase);
    kb200_phase* old = current.phase;
    current.phase = phase;
    if (previous)
        *previous = old;
    else
        release(old);
    return KB200_OK;
}

int kb200_phase_snapshot(kb200_phase* phase, kb200_phase_metrics* out) {
    if (!phase || !out)
        return fail(KB200_INVALID, "null phase or output");
    if (events.owner == phase)
        events.collect(false);
    std::lock_guard<std::mutex> guard(phase->lock);
    *out = phase->metrics;
    return KB200_OK;
}

void kb200_phase_release(kb200_phase* phase) {
    release(phase);
}

const char* kb200_kernel_name(int kernel) {
    return kernel >= 0 && kernel < KB200_KERNEL_COUNT ? kNames[kernel] : nullptr;
}

}  // extern "C"
