// Worker-side adapter: kadan::DenseCompute over the kadan_b200 C ABI.
//
// This header compiles inside the Hikari worker's tree (it needs
// kadan/dense_compute.hpp, services/hikari/inference_worker/include/kadan/
// dense_compute.hpp:60-342) and is not part of libkadan_b200.so. It overrides
// the quantized-weight hot path — dense_gguf_batch and dense_gguf_source —
// and the layer math around it — attend_cached, delta_step and
// copy_recurrent_state, over per-layer state that release_scratch(false)
// frees — and forwards every other virtual to the compute it wraps (the
// worker's own CUDA compute), so it can take that object's place;
// release_weights and weight_placement also cover the B200 weight bank. Status codes map onto the
// reference's conventions: KB200_UNSUPPORTED -> ProjectionResult::unsupported
// (nothing read or written), KB200_OK -> the call's result, any other status
// -> std::runtime_error: the reference's own message where the status stands
// for one ("h3_cuda_cancelled", "h3_cuda_nonfinite_weight", ...), else the
// library's text. An exception thrown by a GgufWeightSource is rethrown after
// the call, as the reference propagates it.
#pragma once

#include <atomic>
#include <cstdint>
#include <exception>
#include <memory>
#include <mutex>
#include <set>
#include <span>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "kadan/dense_compute.hpp"
#include "kadan_b200.h"

namespace kadan::b200 {

class Compute final : public DenseCompute {
public:
    // `fallback` serves every virtual this adapter does not override. One
    // context and one resident weight bank per device in `devices`;
    // `bank_bytes`: each bank's envelope; `scratch_bytes`: device memory kept
    // free for projection workspaces. With several devices every job's output
    // columns are split across them in proportion to the banks' envelopes, as
    // the reference splits them (kb200_gguf_batch_partition).
    Compute(std::shared_ptr<DenseCompute> fallback, std::vector<int> devices, std::uint64_t bank_bytes,
            std::uint64_t scratch_bytes)
        : fallback_(std::move(fallback)), scratch_(scratch_bytes) {
        if (devices.empty())
            throw std::invalid_argument("b200_devices");
        // IQ3_XXS, IQ2_S and IQ3_S decode with the worker's own code grids.
        check(kb200_set_iq_grids(gguf::detail::iq3xxs_grid_host, gguf::detail::iq2s_grid_host,
                                 gguf::detail::iq3s_grid_host));
        for (const int d : devices) {
            Device dev{d};
            int s = kb200_context_create(d, &dev.ctx);
            if (s == KB200_OK && (s = kb200_bank_create_cuda(d, bank_bytes, scratch_bytes, &dev.bank)) != KB200_OK)
                kb200_context_destroy(dev.ctx);
            if (s != KB200_OK) {
                const std::string error = kb200_last_error();
                close();
                throw std::runtime_error(error);
            }
            devices_.push_back(dev);
        }
    }

    ~Compute() override {
        close();
    }

    Compute(const Compute&) = delete;
    Compute& operator=(const Compute&) = delete;

    ProjectionResult dense_gguf_batch(std::span<const GgufBatchJob> jobs, const std::atomic_bool& cancel) override {
        // A cancelled call throws before anything else, an empty batch is
        // unsupported (h3_compute.cu:3966-3968).
        if (cancel.load())
            throw std::runtime_error(kb200_status_name(KB200_CANCELLED));
        if (jobs.empty())
            return ProjectionResult::unsupported;
        std::lock_guard lock(mutex_);
        Sources sources;
        std::vector<kb200_weight_identity> ids(jobs.size());
        std::vector<Source> users(jobs.size());
        std::vector<kb200_source_job> full(jobs.size());
        for (std::size_t i = 0; i < jobs.size(); ++i) {
            const auto& j = jobs[i];
            if (!j.identity || !j.source || !j.in || j.input.size() % j.in
                || j.output.size() != j.input.size() / j.in * j.out)
                return ProjectionResult::unsupported;
            ids[i] = identity(*j.identity);
            users[i] = {j.source, &sources};
            full[i] = {&ids[i], &read_rows, &users[i], j.input.data(), j.output.data(), std::uint32_t(j.in),
                       std::uint32_t(j.out), std::uint32_t(j.input.size() / j.in),
                       j.encoding ? std::int32_t(*j.encoding) : KB200_F32, j.retain_misses ? 1 : 0};
            // Every job is checked before any device reads a source.
            if (!kb200_source_job_supported(&full[i]))
                return ProjectionResult::unsupported;
        }
        return run(full, nullptr, false, cancel, sources);
    }

    // The MXFP4 mixture-of-experts layer. The reference's DenseCompute has no
    // virtual for it (its MoeLayer::forward runs routing, gather and combine
    // on the host around batched expert GEMVs, IW/src/models/text/
    // qwen_layers.cpp:378-492), so this is a member of the adapter alone, in
    // DenseCompute's conventions: synchronous host spans; unsupported, with
    // nothing read from a source and nothing of `output` written, when the
    // shapes do not fit or the device operands cannot hold the weights'
    // scales or the activations exactly (the caller then runs its own
    // layer); failures throw. `weights` are device pointers on device
    // `device` (an index into the constructor's list); input [tokens, hidden]
    // and logits [tokens, experts] are the layer's rows and router outputs.
    ProjectionResult moe_mxfp4(const kb200_moe_weights& weights, std::span<const float> input,
                               std::span<const float> logits, std::size_t tokens, std::span<float> output,
                               const std::atomic_bool& cancel, std::size_t device = 0) {
        if (cancel.load())
            throw std::runtime_error(kb200_status_name(KB200_CANCELLED));
        std::lock_guard lock(mutex_);
        const std::size_t hidden = std::size_t(weights.hidden > 0 ? weights.hidden : 0);
        const std::size_t experts = std::size_t(weights.experts > 0 ? weights.experts : 0);
        if (!tokens || device >= devices_.size() || input.size() != tokens * hidden
            || logits.size() != tokens * experts || output.size() != input.size())
            return ProjectionResult::unsupported;
        int result = KB200_RESULT_UNSUPPORTED;
        const int status = kb200_moe_forward_host(devices_[device].ctx, &weights, input.data(), logits.data(), tokens,
                                                  output.data(), cancel_byte(cancel), &result);
        if (status == KB200_UNSUPPORTED)
            return ProjectionResult::unsupported;
        check(status);
        return result == KB200_RESULT_FINITE ? ProjectionResult::finite : ProjectionResult::unvalidated;
    }

    ProjectionResult dense_gguf_source(const WeightIdentity& id, gguf::Encoding encoding,
                                       const GgufWeightSource& source, std::span<const float> bias,
                                       std::span<const float> input, std::size_t in, std::size_t out,
                                       std::span<float> output, const std::atomic_bool& cancel, bool precise,
                                       bool retain_misses) override {
        std::lock_guard lock(mutex_);
        if (!in || input.size() % in || output.size() != input.size() / in * out
            || (!bias.empty() && bias.size() != out))
            return ProjectionResult::unsupported;
        Sources sources;
        Source user{&source, &sources};
        const kb200_weight_identity ident = identity(id);
        const kb200_source_job job{&ident, &read_rows, &user, input.data(), output.data(), std::uint32_t(in),
                                   std::uint32_t(out), std::uint32_t(input.size() / in), std::int32_t(encoding),
                                   retain_misses ? 1 : 0};
        // The reference's fp64 path is not offered: unsupported, before any read.
        if (precise || !kb200_source_job_supported(&job))
            return ProjectionResult::unsupported;
        return run(std::span(&job, 1), bias.empty() ? nullptr : bias.data(), true, cancel, sources);
    }

    void dense(std::span<const float> weights, std::span<const float> bias, std::span<const float> input,
               std::size_t in, std::size_t out, std::span<float> output, const std::atomic_bool& cancel,
               bool precise) override {
        fallback_->dense(weights, bias, input, in, out, output, cancel, precise);
    }

    // -- weight residency: the banks' entries of these tensors retire too.
    Bytes release_weights(std::span<const WeightIdentity> sources) override {
        Bytes released = fallback_->release_weights(sources);
        std::lock_guard lock(mutex_);
        std::vector<kb200_weight_identity> ids;
        for (const auto& w : sources)
            ids.push_back(identity(w));
        for (const auto& d : devices_) {
            std::uint64_t ours = 0;
            check(kb200_bank_release_sources(d.bank, ids.data(), ids.size(), &ours));
            released += ours;
        }
        return released;
    }

    std::vector<DeviceWeightPlacement> weight_placement() const override {
        auto placement = fallback_->weight_placement();
        for (const auto& d : devices_) {
            kb200_bank_state st{};
            if (kb200_bank_state_get(d.bank, &st) == KB200_OK)
                placement.push_back({d.id, Bytes(st.capacity), Bytes(st.allocated)});
        }
        return placement;
    }

    void release_devices() override {
        {
            std::lock_guard lock(mutex_);
            for (const auto& d : devices_)
                check(kb200_bank_release(d.bank));
        }
        fallback_->release_devices();
    }

    // Request boundary: without `keep` the per-layer KV mirrors and recurrent
    // states this adapter holds are released with the wrapped compute's.
    Footprint release_scratch(bool keep) override {
        if (!keep) {
            std::lock_guard lock(mutex_);
            for (const auto& d : devices_)
                check(kb200_context_release_layers(d.ctx));
            delta_layers_.clear();
        }
        return fallback_->release_scratch(keep);
    }

    // Cached attention on the first device (kb200_attend_cached_host); shapes
    // it does not take go to the wrapped compute before anything is read.
    bool attend_cached(std::uint64_t layer, std::span<const float> q, std::span<const float> keys,
                       std::span<const float> values, std::size_t rows, std::size_t position, std::size_t heads,
                       std::size_t kv_heads, std::size_t dim, float scale, std::span<float> output,
                       const std::atomic_bool& cancel, std::span<const std::uint32_t> selected,
                       std::span<const std::uint32_t> offsets) override {
        const std::size_t kv = (position + rows) * kv_heads * dim;
        const bool shaped = rows && q.size() == rows * heads * dim && output.size() == q.size() && keys.size() >= kv
                            && values.size() >= kv && (selected.empty() || offsets.size() == rows + 1)
                            && kb200_attend_supported(heads, kv_heads, dim);
        if (!shaped)
            return fallback_->attend_cached(layer, q, keys, values, rows, position, heads, kv_heads, dim, scale,
                                            output, cancel, selected, offsets);
        if (cancel.load())
            throw std::runtime_error(kb200_status_name(KB200_CANCELLED));
        std::lock_guard lock(mutex_);
        const int status = kb200_attend_cached_host(devices_.front().ctx, layer, q.data(), keys.data(), values.data(),
                                                    rows, position, heads, kv_heads, dim, scale,
                                                    selected.empty() ? nullptr : selected.data(),
                                                    selected.empty() ? nullptr : offsets.data(), output.data(),
                                                    cancel_byte(cancel));
        if (status == KB200_UNSUPPORTED)
            return false;
        check(status);
        return true;
    }

    // Delta-net steps on the first device (kb200_delta_step_host) for the
    // layers whose fresh step it took; other layers stay with the wrapped
    // compute, so a layer's state never moves between the two.
    bool delta_step(const DeltaStep& step, const std::atomic_bool& cancel) override {
        const std::size_t channels = (2 * step.key_heads + step.value_heads) * step.dim;
        const std::size_t inner = step.value_heads * step.dim, rows = step.rows;
        std::unique_lock lock(mutex_);
        const bool ours = delta_layers_.count(step.layer) != 0;
        if (!step.fresh && !ours) {
            lock.unlock();
            return fallback_->delta_step(step, cancel);
        }
        const bool shaped = rows && step.qkv.size() == rows * channels && step.z.size() == rows * inner
                            && step.alpha.size() == rows * step.value_heads
                            && step.beta.size() == rows * step.value_heads
                            && step.conv.size() == channels * step.kernel && step.dt.size() == step.value_heads
                            && step.a.size() == step.value_heads && step.norm.size() == step.dim
                            && step.output.size() == rows * inner
                            && (step.initial_state.empty()
                                || step.initial_state.size() == step.value_heads * step.dim * step.dim)
                            && (step.initial_history.empty()
                                || step.initial_history.size() == (step.kernel - 1) * channels)
                            && kb200_delta_supported(std::uint32_t(step.key_heads), std::uint32_t(step.value_heads),
                                                     std::uint32_t(step.dim), std::uint32_t(step.kernel));
        if (step.fresh && !shaped) {
            delta_layers_.erase(step.layer);
            lock.unlock();
            return fallback_->delta_step(step, cancel);
        }
        if (!shaped)
            throw std::runtime_error("gguf_text_recurrent_device_lost");
        if (cancel.load())
            throw std::runtime_error(kb200_status_name(KB200_CANCELLED));
        const kb200_delta_host host{step.layer, step.fresh ? 1 : 0, step.qkv.data(), step.z.data(),
                                    step.alpha.data(), step.beta.data(), step.conv.data(), step.dt.data(),
                                    step.a.data(), step.norm.data(), std::uint32_t(rows),
                                    std::uint32_t(step.key_heads), std::uint32_t(step.value_heads),
                                    std::uint32_t(step.dim), std::uint32_t(step.kernel), step.eps,
                                    step.sigmoid_gate ? 1 : 0, step.output.data(),
                                    step.initial_state.empty() ? nullptr : step.initial_state.data(),
                                    step.initial_history.empty() ? nullptr : step.initial_history.data()};
        const int status = kb200_delta_step_host(devices_.front().ctx, &host, cancel_byte(cancel));
        if (status == KB200_UNSUPPORTED && step.fresh) {
            delta_layers_.erase(step.layer);
            lock.unlock();
            return fallback_->delta_step(step, cancel);
        }
        check(status);
        delta_layers_.insert(step.layer);
        return true;
    }

    void copy_recurrent_state(std::uint64_t layer, std::span<float> state, std::span<float> history) override {
        {
            std::lock_guard lock(mutex_);
            if (delta_layers_.count(layer)) {
                check(kb200_recurrent_state_get(devices_.front().ctx, layer, state.data(), state.size(),
                                                history.data(), history.size()));
                return;
            }
        }
        fallback_->copy_recurrent_state(layer, state, history);
    }

    // -- everything else is the wrapped compute's.
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

private:
    struct Device {
        int id = 0;
        kb200_context* ctx = nullptr;
        kb200_bank* bank = nullptr;
    };

    // The first exception a source threw during one call.
    struct Sources {
        std::mutex mutex;
        std::exception_ptr error;
    };
    struct Source {
        const GgufWeightSource* fn = nullptr;
        Sources* sources = nullptr;
    };

    // One job's columns on one device: the source shifted to the slice's
    // first row and the slice's outputs staged for the scatter.
    struct Slice {
        std::size_t job = 0;
        kb200_partition part{};
        kb200_row_source fn = nullptr;
        void* user = nullptr;
        std::vector<float> staged;
    };
    struct Part {
        std::vector<Slice> slices;
        std::vector<kb200_source_job> jobs;
        int status = KB200_OK, result = KB200_RESULT_UNSUPPORTED;
        std::string error;
    };

    static int shifted_rows(void* user, std::uint64_t first_row, void* dst, std::uint64_t bytes) {
        const auto* s = static_cast<const Slice*>(user);
        return s->fn(s->user, s->part.first + first_row, dst, bytes);
    }

    void close() noexcept {
        for (auto& d : devices_) {
            kb200_bank_destroy(d.bank);
            kb200_context_destroy(d.ctx);
        }
        devices_.clear();
    }

    // Runs supported jobs (one job with an optional bias when `single`), on
    // one device directly, or split over the devices: each device's slices
    // run on a thread of their own, every thread is joined, and only then are
    // failures reported and outputs scattered (h3_compute.cu's device threads
    // likewise finish before the call returns or throws).
    ProjectionResult run(std::span<const kb200_source_job> jobs, const float* bias, bool single,
                         const std::atomic_bool& cancel, Sources& sources) {
        if (devices_.size() == 1) {
            const Device& d = devices_[0];
            int result = KB200_RESULT_UNSUPPORTED;
            const int s = single ? kb200_dense_gguf_source(d.ctx, d.bank, jobs.data(), bias, scratch_, 0,
                                                           cancel_byte(cancel), &result)
                                 : kb200_dense_gguf_source_batch(d.ctx, d.bank, jobs.data(), jobs.size(), scratch_,
                                                                 cancel_byte(cancel), &result);
            return finish(s, result, sources);
        }
        std::vector<std::uint64_t> capacities;
        for (const auto& d : devices_) {
            kb200_bank_state st{};
            check(kb200_bank_state_get(d.bank, &st));
            capacities.push_back(st.capacity);
        }
        std::vector<Part> parts(devices_.size());
        for (std::size_t d = 0; d < devices_.size(); ++d) {
            Part& part = parts[d];
            part.slices.reserve(jobs.size());  // slices are pointed at: no reallocation
            for (std::size_t j = 0; j < jobs.size(); ++j) {
                const auto& job = jobs[j];
                Slice slice{j, {}, job.source, job.source_user, {}};
                check(kb200_gguf_batch_partition(job.in, job.out, job.encoding, capacities.data(), capacities.size(),
                                                 d, scratch_, &slice.part));
                if (!slice.part.count)
                    continue;
                slice.staged.resize(std::size_t(job.rows) * slice.part.count);
                part.slices.push_back(std::move(slice));
                Slice& placed = part.slices.back();
                kb200_source_job shifted = job;
                shifted.source = &shifted_rows;
                shifted.source_user = &placed;
                shifted.output = placed.staged.data();
                shifted.out = std::uint32_t(placed.part.count);
                part.jobs.push_back(shifted);
            }
        }
        std::vector<std::thread> threads;
        std::exception_ptr spawn_error;
        try {
            for (std::size_t d = 0; d < devices_.size(); ++d) {
                if (parts[d].jobs.empty())
                    continue;
                threads.emplace_back([&, d] {
                    Part& part = parts[d];
                    const Device& dev = devices_[d];
                    const float* slice_bias = bias ? bias + part.slices[0].part.first : nullptr;
                    part.status = single ? kb200_dense_gguf_source(dev.ctx, dev.bank, part.jobs.data(), slice_bias,
                                                                   scratch_, 0, cancel_byte(cancel), &part.result)
                                         : kb200_dense_gguf_source_batch(dev.ctx, dev.bank, part.jobs.data(),
                                                                         part.jobs.size(), scratch_,
                                                                         cancel_byte(cancel), &part.result);
                    if (part.status != KB200_OK)
                        part.error = kb200_last_error();
                });
            }
        } catch (...) {
            // A thread that could not start: the started ones finish first.
            spawn_error = std::current_exception();
        }
        for (auto& t : threads)
            t.join();
        if (spawn_error)
            std::rethrow_exception(spawn_error);
        if (sources.error)
            std::rethrow_exception(sources.error);
        bool finite = true;
        for (const auto& part : parts) {
            if (part.jobs.empty())
                continue;
            if (part.status != KB200_OK)
                throw std::runtime_error(message(part.status, part.error.c_str()));
            finite = finite && part.result == KB200_RESULT_FINITE;
        }
        for (const auto& part : parts)
            for (const auto& slice : part.slices) {
                const auto& job = jobs[slice.job];
                kb200_partition_scatter(&slice.part, slice.staged.data(), job.rows, job.output, job.out);
            }
        return finite ? ProjectionResult::finite : ProjectionResult::unvalidated;
    }

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

    // Statuses that stand for one of the reference's exception messages throw
    // exactly that message (callers compare it); others carry the library's text.
    static std::string message(int status, const char* detail) {
        switch (status) {
        case KB200_NONFINITE_WEIGHT:
        case KB200_NONFINITE_INPUT:
        case KB200_NONFINITE_BIAS:
        case KB200_NONFINITE_OUTPUT:
        case KB200_ALIAS:
        case KB200_CANCELLED:
        case KB200_QUARANTINED:
            return kb200_status_name(status);
        default:
            return detail;
        }
    }

    static void check(int status) {
        if (status != KB200_OK)
            throw std::runtime_error(message(status, kb200_last_error()));
    }

    std::shared_ptr<DenseCompute> fallback_;
    std::uint64_t scratch_;
    std::vector<Device> devices_;
    std::set<std::uint64_t> delta_layers_;  // layers whose recurrent state this adapter holds
    mutable std::mutex mutex_;  // the reference serialises DenseCompute calls (h3_compute.cu:1639)
};

}  // namespace kadan::b200
