// Worker-side adapter: kadan::DenseCompute over the kadan_b200 C ABI.
//
// This header compiles inside the Hikari worker's tree (it needs
// kadan/dense_compute.hpp, services/hikari/inference_worker/include/kadan/
// dense_compute.hpp:60-342) and is not part of libkadan_b200.so. It overrides
// the quantized-weight hot path — dense_gguf_batch and dense_gguf_source —
// and forwards every other virtual to the compute it wraps (the worker's own
// CUDA compute), so it can take that object's place; release_weights and
// weight_placement also cover the B200 weight bank. Status codes map onto the
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
        : fallback_(std::move(fallback)), device_(device), scratch_(scratch_bytes) {
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

    // -- weight residency: the bank's entries of these tensors retire too.
    Bytes release_weights(std::span<const WeightIdentity> sources) override {
        Bytes released = fallback_->release_weights(sources);
        std::lock_guard lock(mutex_);
        std::vector<kb200_weight_identity> ids;
        for (const auto& w : sources)
            ids.push_back(identity(w));
        std::uint64_t ours = 0;
        check(kb200_bank_release_sources(bank_, ids.data(), ids.size(), &ours));
        return released + ours;
    }

    std::vector<DeviceWeightPlacement> weight_placement() const override {
        auto placement = fallback_->weight_placement();
        kb200_bank_state st{};
        if (kb200_bank_state_get(bank_, &st) == KB200_OK)
            placement.push_back({device_, Bytes(st.capacity), Bytes(st.allocated)});
        return placement;
    }

    void release_devices() override {
        {
            std::lock_guard lock(mutex_);
            check(kb200_bank_release(bank_));
        }
        fallback_->release_devices();
    }

    // -- everything else is the wrapped compute's.
    Footprint release_scratch(bool keep) override {
        return fallback_->release_scratch(keep);
    }
    Footprint retained_weights() const override {
        return fallback_->retained_weights();
    }
    void reserve_device_state(Bytes bytes) override {
        fallback_->reserve_device_state(bytes);
    }
    bool prepare_weights(Bytes bytes) override {
        return fallback_->prepare_weights(bytes);
    }
    void dense_weight(const WeightIdentity& id, std::span<const float> weights, std::span<const float> bias,
                      std::span<const float> input, std::size_t in, std::size_t out, std::span<float> output,
                      const std::atomic_bool& cancel, bool precise) override {
        fallback_->dense_weight(id, weights, bias, input, in, out, output, cancel, precise);
    }
    bool supports_weight_sources() const override {
        return fallback_->supports_weight_sources();
    }
    bool supports_bf16_weights() const override {
        return fallback_->supports_bf16_weights();
    }
    bool image_vae_normalize(std::span<const float> a, std::span<const float> b, std::size_t n, std::span<float> y,
                             bool silu, const std::atomic_bool& cancel) override {
        return fallback_->image_vae_normalize(a, b, n, y, silu, cancel);
    }
    bool image_silu_pair_bf16_source(const WeightIdentity& gate_id, const Bf16WeightSource& gate,
                                     const WeightIdentity& up_id, const Bf16WeightSource& up,
                                     std::span<const float> input, std::size_t in, std::size_t out,
                                     std::span<float> output, const std::atomic_bool& cancel) override {
        return fallback_->image_silu_pair_bf16_source(gate_id, gate, up_id, up, input, in, out, output, cancel);
    }
    ProjectionResult dense_bf16_source(const WeightIdentity& id, const Bf16WeightSource& source,
                                       std::span<const float> bias, std::span<const float> input, std::size_t in,
                                       std::size_t out, std::span<float> output,
                                       const std::atomic_bool& cancel) override {
        return fallback_->dense_bf16_source(id, source, bias, input, in, out, output, cancel);
    }
    bool image_vae_convolution_source(const WeightIdentity& id, const FloatWeightSource& source,
                                      std::span<const float> bias, std::span<const float> input,
                                      image::VaeConvolution shape, std::span<float> output,
                                      const std::atomic_bool& cancel) override {
        return fallback_->image_vae_convolution_source(id, source, bias, input, shape, output, cancel);
    }
    ProjectionResult dense_source(const WeightIdentity& id, const FloatWeightSource& source,
                                  std::span<const float> bias, std::span<const float> input, std::size_t in,
                                  std::size_t out, std::span<float> output, const std::atomic_bool& cancel,
                                  bool precise, ProjectionPolicy policy) override {
        return fallback_->dense_source(id, source, bias, input, in, out, output, cancel, precise, policy);
    }
    bool attend(std::span<const float> q, std::span<const float> k, std::span<const float> v, std::size_t queries,
                std::size_t keys, std::size_t heads, std::size_t kv_heads, std::size_t dim,
                std::size_t causal_queries, std::size_t window, std::size_t offset, std::span<float> y,
                const std::atomic_bool& cancel) override {
        return fallback_->attend(q, k, v, queries, keys, heads, kv_heads, dim, causal_queries, window, offset, y,
                                 cancel);
    }
    bool attend_cached(std::uint64_t layer, std::span<const float> q, std::span<const float> keys,
                       std::span<const float> values, std::size_t rows, std::size_t position, std::size_t heads,
                       std::size_t kv_heads, std::size_t dim, float scale, std::span<float> output,
                       const std::atomic_bool& cancel, std::span<const std::uint32_t> selected,
                       std::span<const std::uint32_t> offsets) override {
        return fallback_->attend_cached(layer, q, keys, values, rows, position, heads, kv_heads, dim, scale, output,
                                        cancel, selected, offsets);
    }
    void copy_recurrent_state(std::uint64_t layer, std::span<float> state, std::span<float> history) override {
        fallback_->copy_recurrent_state(layer, state, history);
    }
    bool delta_step(const DeltaStep& step, const std::atomic_bool& cancel) override {
        return fallback_->delta_step(step, cancel);
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
    int device_;
    std::uint64_t scratch_;
    kb200_context* ctx_ = nullptr;
    kb200_bank* bank_ = nullptr;
    mutable std::mutex mutex_;  // the reference serialises DenseCompute calls (h3_compute.cu:1639)
};

}  // namespace kadan::b200
