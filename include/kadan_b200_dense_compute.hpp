// Worker-side adapter: kadan::DenseCompute over the kadan_b200 C ABI.
//
// This header compiles inside the Hikari worker's tree (it needs
// kadan/dense_compute.hpp, services/hikari/inference_worker/include/kadan/
// dense_compute.hpp:60-342) and is not part of libkadan_b200.so. It overrides
// the quantized-weight hot path — dense_gguf_batch and dense_gguf_source —
// and forwards dense (the pure virtual) to the compute it wraps; a worker
// forwards its other virtuals the same way. Status codes map onto the
// reference's conventions: KB200_UNSUPPORTED -> ProjectionResult::unsupported
// (nothing read or written), KB200_OK -> the call's result, any other status
// -> std::runtime_error with the library's message. An exception thrown by a
// GgufWeightSource is rethrown after the call, as the reference propagates it.
#pragma once

#include <atomic>
#include <cstdint>
#include <exception>
#include <memory>
#include <mutex>
#include <span>
#include <stdexcept>
#include <vector>

#include "kadan/dense_compute.hpp"
#include "kadan_b200.h"

namespace kadan::b200 {

class Compute final : public DenseCompute {
public:
    // `fallback` serves every virtual this adapter does not override.
    // `bank_bytes`: envelope of the resident weight bank on `device`;
    // `scratch_bytes`: device memory kept free for projection workspaces.
    Compute(std::shared_ptr<DenseCompute> fallback, int device, std::uint64_t bank_bytes,
            std::uint64_t scratch_bytes)
        : fallback_(std::move(fallback)), scratch_(scratch_bytes) {
        check(kb200_context_create(device, &ctx_));
        if (const int s = kb200_bank_create_cuda(device, bank_bytes, scratch_bytes, &bank_)) {
            kb200_context_destroy(ctx_);
            check(s);
        }
    }

    ~Compute() override {
        kb200_bank_destroy(bank_);
        kb200_context_destroy(ctx_);
    }

    Compute(const Compute&) = delete;
    Compute& operator=(const Compute&) = delete;

    ProjectionResult dense_gguf_batch(std::span<const GgufBatchJob> jobs, const std::atomic_bool& cancel) override {
        std::lock_guard lock(mutex_);
        Sources sources;
        std::vector<kb200_weight_identity> ids(jobs.size());
        std::vector<Source> users(jobs.size());
        std::vector<kb200_source_job> out(jobs.size());
        for (std::size_t i = 0; i < jobs.size(); ++i) {
            const auto& j = jobs[i];
            if (!j.identity || !j.source || !j.in || j.input.size() % j.in)
                return ProjectionResult::unsupported;
            ids[i] = identity(*j.identity);
            users[i] = {j.source, &sources};
            out[i] = {&ids[i], &read_rows, &users[i], j.input.data(), j.output.data(),
                      std::uint32_t(j.in), std::uint32_t(j.out), std::uint32_t(j.input.size() / j.in),
                      j.encoding ? std::int32_t(*j.encoding) : KB200_F32, j.retain_misses ? 1 : 0};
        }
        int result = KB200_RESULT_UNSUPPORTED;
        const int s = kb200_dense_gguf_source_batch(ctx_, bank_, out.data(), out.size(), scratch_, cancel_byte(cancel),
                                                    &result);
        return finish(s, result, sources);
    }

    ProjectionResult dense_gguf_source(const WeightIdentity& id, gguf::Encoding encoding,
                                       const GgufWeightSource& source, std::span<const float> bias,
                                       std::span<const float> input, std::size_t in, std::size_t out,
                                       std::span<float> output, const std::atomic_bool& cancel, bool precise,
                                       bool retain_misses) override {
        std::lock_guard lock(mutex_);
        if (!in || input.size() % in || (!bias.empty() && bias.size() != out))
            return ProjectionResult::unsupported;
        Sources sources;
        Source user{&source, &sources};
        const kb200_weight_identity ident = identity(id);
        const kb200_source_job job{&ident, &read_rows, &user, input.data(), output.data(), std::uint32_t(in),
                                   std::uint32_t(out), std::uint32_t(input.size() / in), std::int32_t(encoding),
                                   retain_misses ? 1 : 0};
        int result = KB200_RESULT_UNSUPPORTED;
        const int s = kb200_dense_gguf_source(ctx_, bank_, &job, bias.empty() ? nullptr : bias.data(), scratch_,
                                              precise ? 1 : 0, cancel_byte(cancel), &result);
        return finish(s, result, sources);
    }

    void dense(std::span<const float> weights, std::span<const float> bias, std::span<const float> input,
               std::size_t in, std::size_t out, std::span<float> output, const std::atomic_bool& cancel,
               bool precise) override {
        fallback_->dense(weights, bias, input, in, out, output, cancel, precise);
    }

private:
    // The first exception a source threw during one call.
    struct Sources {
        std::mutex mutex;
        std::exception_ptr error;
    };
    struct Source {
        const GgufWeightSource* fn = nullptr;
        Sources* sources = nullptr;
    };

    static_assert(sizeof(std::atomic_bool) == 1 && std::atomic_bool::is_always_lock_free,
                  "the ABI reads the cancel flag as one byte");

    static const volatile std::uint8_t* cancel_byte(const std::atomic_bool& cancel) {
        return reinterpret_cast<const volatile std::uint8_t*>(&cancel);
    }

    static kb200_weight_identity identity(const WeightIdentity& w) {
        return {w.device, w.inode, w.file_size, w.modified_seconds, w.modified_nanoseconds,
                w.changed_seconds, w.changed_nanoseconds, w.payload_begin, w.payload_end};
    }

    // kb200_row_source over a GgufWeightSource; sources may run concurrently
    // on the library's read threads, on disjoint rows.
    static int read_rows(void* user, std::uint64_t first_row, void* dst, std::uint64_t bytes) {
        auto* u = static_cast<Source*>(user);
        try {
            (*u->fn)(std::size_t(first_row), {static_cast<std::byte*>(dst), std::size_t(bytes)});
            return KB200_OK;
        } catch (...) {
            std::lock_guard lock(u->sources->mutex);
            if (!u->sources->error)
                u->sources->error = std::current_exception();
            return KB200_INVALID;
        }
    }

    static ProjectionResult finish(int status, int result, Sources& sources) {
        if (sources.error)
            std::rethrow_exception(sources.error);
        if (status == KB200_UNSUPPORTED)
            return ProjectionResult::unsupported;
        check(status);
        return result == KB200_RESULT_FINITE ? ProjectionResult::finite : ProjectionResult::unvalidated;
    }

    static void check(int status) {
        if (status != KB200_OK)
            throw std::runtime_error(kb200_last_error());
    }

    std::shared_ptr<DenseCompute> fallback_;
    std::uint64_t scratch_;
    kb200_context* ctx_ = nullptr;
    kb200_bank* bank_ = nullptr;
    std::mutex mutex_;  // the reference serialises DenseCompute calls (h3_compute.cu:1639)
};

}  // namespace kadan::b200
