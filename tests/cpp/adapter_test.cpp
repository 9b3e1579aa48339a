// The worker-side adapter (include/kadan_b200_dense_compute.hpp) driven
// through the reference's DenseCompute interface, with the library's device
// entry points played by host fakes and its host code (support predicate,
// column partition, scatter, status names) the real libkadan_b200.so. Checks
// what the adapter itself decides: the column split over devices in
// proportion to the banks' envelopes and the scatter back, the source rows
// shifted to each slice, the bias slice, unsupported before any read, the
// reference's exception messages, a source's exception rethrown, the
// finite/unvalidated result over devices, and the residency virtuals over
// the wrapped compute plus the banks. Prints "ok".
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "kadan_b200_dense_compute.hpp"

#define CHECK(c)                                                                        \
    do {                                                                                \
        if (!(c)) {                                                                     \
            std::fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #c);  \
            std::exit(1);                                                               \
        }                                                                               \
    } while (0)

namespace {

// One fake device: its bank's envelope, the status and result it answers
// with, and what it was asked to do.
struct FakeDevice {
    int id = 0;
    std::uint64_t capacity = 0;
    int status = KB200_OK;
    int result = KB200_RESULT_FINITE;
    std::string error;
    int calls = 0;
    std::vector<std::uint32_t> outs;  // out of every job it ran
    const float* bias = nullptr;
    bool saw_cancel = false;
    std::uint64_t released = 0;
    int layer_calls = 0, layers_released = 0;
    std::vector<int> fresh;  // fresh flag of every delta step it ran
};

std::mutex fake_mutex;
std::map<int, FakeDevice> devices;
thread_local std::string last_error;

struct kb200_context_fake {
    int device;
};
struct kb200_bank_fake {
    int device;
};

float half_to_float(std::uint16_t h) {
    const int sign = h >> 15, exponent = (h >> 10) & 31, mantissa = h & 1023;
    const float v = exponent ? std::ldexp(float(1024 + mantissa), exponent - 25) : std::ldexp(float(mantissa), -24);
    return sign ? -v : v;
}

// Row n of a packed matrix decoded to `in` floats (F32 rows or Q8_0 blocks).
std::vector<float> decode_row(const std::uint8_t* row, std::uint32_t in, int encoding) {
    std::vector<float> w(in);
    if (encoding == KB200_F32) {
        std::memcpy(w.data(), row, in * sizeof(float));
        return w;
    }
    CHECK(encoding == KB200_Q8_0);
    for (std::uint32_t b = 0; b < in / 32; ++b) {
        std::uint16_t d;
        std::memcpy(&d, row + b * 34, 2);
        for (int j = 0; j < 32; ++j)
            w[b * 32 + j] = half_to_float(d) * float(std::int8_t(row[b * 34 + 2 + j]));
    }
    return w;
}

std::uint32_t row_bytes(std::uint32_t in, int encoding) {
    return encoding == KB200_F32 ? in * 4 : in / 32 * 34;
}

// y[r, n] = sum_k w[n, k] * x[r, k] in double, rounded once.
void project(const std::vector<std::uint8_t>& packed, std::uint32_t in, std::uint32_t out, int encoding,
             const float* x, std::uint32_t rows, float* y) {
    const std::uint32_t rb = row_bytes(in, encoding);
    for (std::uint32_t n = 0; n < out; ++n) {
        const auto w = decode_row(packed.data() + std::size_t(n) * rb, in, encoding);
        for (std::uint32_t r = 0; r < rows; ++r) {
            double s = 0;
            for (std::uint32_t k = 0; k < in; ++k)
                s += double(w[k]) * double(x[std::size_t(r) * in + k]);
            y[std::size_t(r) * out + n] = float(s);
        }
    }
}

FakeDevice& device_of(int id) {
    std::lock_guard lock(fake_mutex);
    return devices.at(id);
}

}  // namespace

// -- the device entry points, played on the host.
extern "C" {

const char* kb200_last_error(void) {
    return last_error.c_str();
}

int kb200_context_create(int device, kb200_context** out) {
    std::lock_guard lock(fake_mutex);
    if (!devices.count(device)) {
        last_error = "no such device";
        return KB200_CUDA;
    }
    *out = reinterpret_cast<kb200_context*>(new kb200_context_fake{device});
    return KB200_OK;
}

void kb200_context_destroy(kb200_context* ctx) {
    delete reinterpret_cast<kb200_context_fake*>(ctx);
}

int kb200_bank_create_cuda(int device, std::uint64_t, std::uint64_t, kb200_bank** out) {
    *out = reinterpret_cast<kb200_bank*>(new kb200_bank_fake{device});
    return KB200_OK;
}

void kb200_bank_destroy(kb200_bank* bank) {
    delete reinterpret_cast<kb200_bank_fake*>(bank);
}

int kb200_bank_state_get(const kb200_bank* bank, kb200_bank_state* state) {
    const auto& d = device_of(reinterpret_cast<const kb200_bank_fake*>(bank)->device);
    *state = {};
    state->capacity = state->maximum_capacity = d.capacity;
    state->allocated = d.capacity / 4;
    return KB200_OK;
}

int kb200_bank_release_sources(kb200_bank* bank, const kb200_weight_identity*, std::size_t count,
                               std::uint64_t* released) {
    auto& d = device_of(reinterpret_cast<kb200_bank_fake*>(bank)->device);
    d.released += count;
    if (released)
        *released = 100 * count;
    return KB200_OK;
}

int kb200_bank_release(kb200_bank*) {
    return KB200_OK;
}

int kb200_dense_gguf_source_batch(kb200_context* ctx, kb200_bank*, const kb200_source_job* jobs, std::size_t count,
                                  std::uint64_t, const volatile std::uint8_t* cancel, int* result) {
    auto& d = device_of(reinterpret_cast<kb200_context_fake*>(ctx)->device);
    *result = KB200_RESULT_UNSUPPORTED;
    ++d.calls;
    for (std::size_t j = 0; j < count; ++j)
        CHECK(kb200_source_job_supported(&jobs[j]));
    if (cancel && *cancel) {
        d.saw_cancel = true;
        last_error = "cancelled";
        return KB200_CANCELLED;
    }
    for (std::size_t j = 0; j < count; ++j) {
        const auto& job = jobs[j];
        d.outs.push_back(job.out);
        std::vector<std::uint8_t> packed(std::size_t(job.out) * row_bytes(job.in, job.encoding));
        // Two reads, as the library's chunked staging would make them.
        const std::uint32_t half = job.out / 2;
        const std::size_t rb = row_bytes(job.in, job.encoding);
        if (half && job.source(job.source_user, 0, packed.data(), half * rb) != KB200_OK) {
            last_error = "source failed";
            return KB200_INVALID;
        }
        if (job.source(job.source_user, half, packed.data() + half * rb, (job.out - half) * rb) != KB200_OK) {
            last_error = "source failed";
            return KB200_INVALID;
        }
        project(packed, job.in, job.out, job.encoding, job.input, job.rows, job.output);
    }
    // The library reads the caller's flag between chunks too.
    if (cancel && *cancel) {
        d.saw_cancel = true;
        last_error = "cancelled";
        return KB200_CANCELLED;
    }
    if (d.status != KB200_OK) {
        last_error = d.error;
        return d.status;
    }
    *result = d.result;
    return KB200_OK;
}

int kb200_dense_gguf_source(kb200_context* ctx, kb200_bank* bank, const kb200_source_job* job, const float* bias,
                            std::uint64_t scratch, int precise, const volatile std::uint8_t* cancel, int* result) {
    CHECK(!precise);
    const int s = kb200_dense_gguf_source_batch(ctx, bank, job, 1, scratch, cancel, result);
    auto& d = device_of(reinterpret_cast<kb200_context_fake*>(ctx)->device);
    d.bias = bias;
    if (s == KB200_OK && bias)
        for (std::uint32_t r = 0; r < job->rows; ++r)
            for (std::uint32_t n = 0; n < job->out; ++n)
                job->output[std::size_t(r) * job->out + n] += bias[n];
    return s;
}

// The MoE layer on a fake device: out = 2 * x when it answers OK.
int kb200_moe_forward_host(kb200_context* ctx, const kb200_moe_weights* w, const float* x, const float*,
                           std::size_t tokens, float* out, const volatile std::uint8_t* cancel, int* result) {
    auto& d = device_of(reinterpret_cast<kb200_context_fake*>(ctx)->device);
    ++d.calls;
    d.saw_cancel = cancel != nullptr;
    *result = KB200_RESULT_UNSUPPORTED;
    if (d.status != KB200_OK) {
        last_error = d.error;
        return d.status;
    }
    for (std::size_t i = 0; i < tokens * std::size_t(w->hidden); ++i)
        out[i] = 2.f * x[i];
    *result = d.result;
    return KB200_OK;
}

// Attention on a fake device: out = q when it answers OK.
int kb200_attend_cached_host(kb200_context* ctx, std::uint64_t, const float* q, const float*, const float*,
                             std::size_t rows, std::size_t, std::size_t heads, std::size_t, std::size_t dim, float,
                             const std::uint32_t*, const std::uint32_t*, float* out,
                             const volatile std::uint8_t*) {
    auto& d = device_of(reinterpret_cast<kb200_context_fake*>(ctx)->device);
    ++d.layer_calls;
    if (d.status != KB200_OK) {
        last_error = d.error;
        return d.status;
    }
    std::copy(q, q + rows * heads * dim, out);
    return KB200_OK;
}

// A delta-net step on a fake device: every output 1.
int kb200_delta_step_host(kb200_context* ctx, const kb200_delta_host* st, const volatile std::uint8_t*) {
    auto& d = device_of(reinterpret_cast<kb200_context_fake*>(ctx)->device);
    ++d.layer_calls;
    d.fresh.push_back(st->fresh);
    if (d.status != KB200_OK) {
        last_error = d.error;
        return d.status;
    }
    std::fill(st->output, st->output + std::size_t(st->rows) * st->value_heads * st->dim, 1.f);
    return KB200_OK;
}

int kb200_recurrent_state_get(kb200_context* ctx, std::uint64_t, float* state, std::size_t n, float* history,
                              std::size_t m) {
    ++device_of(reinterpret_cast<kb200_context_fake*>(ctx)->device).layer_calls;
    std::fill(state, state + n, 5.f);
    std::fill(history, history + m, 6.f);
    return KB200_OK;
}

int kb200_context_release_layers(kb200_context* ctx) {
    ++device_of(reinterpret_cast<kb200_context_fake*>(ctx)->device).layers_released;
    return KB200_OK;
}

}  // extern "C"

namespace {

using kadan::DenseCompute;
using kadan::ProjectionResult;
using kadan::WeightIdentity;

// The worker's own compute: what the adapter forwards the other virtuals to.
struct Fallback final : DenseCompute {
    int dense_calls = 0, release_devices_calls = 0;
    void dense(std::span<const float>, std::span<const float>, std::span<const float>, std::size_t, std::size_t,
               std::span<float>, const std::atomic_bool&, bool) override {
        ++dense_calls;
    }
    kadan::Bytes release_weights(std::span<const WeightIdentity> w) override {
        return 7 * w.size();
    }
    std::vector<kadan::DeviceWeightPlacement> weight_placement() const override {
        return {{9, 1, 2}};
    }
    void release_devices() override {
        ++release_devices_calls;
    }
    int layer_calls = 0;
    bool attend_cached(std::uint64_t, std::span<const float>, std::span<const float>, std::span<const float>,
                       std::size_t, std::size_t, std::size_t, std::size_t, std::size_t, float, std::span<float>,
                       const std::atomic_bool&, std::span<const std::uint32_t>,
                       std::span<const std::uint32_t>) override {
        ++layer_calls;
        return false;
    }
    bool delta_step(const DeltaStep&, const std::atomic_bool&) override {
        ++layer_calls;
        return true;
    }
    void copy_recurrent_state(std::uint64_t, std::span<float> state, std::span<float>) override {
        ++layer_calls;
        std::fill(state.begin(), state.end(), 7.f);
    }
};

// A packed matrix and the GgufWeightSource over it, recording every row read.
struct Matrix {
    std::uint32_t in, out;
    int encoding;
    std::vector<std::uint8_t> bytes;
    WeightIdentity id{};
    std::mutex mutex;
    std::multiset<std::size_t> rows_read;
    bool throw_on_read = false;
    std::atomic_bool* cancel_on_read = nullptr;
    DenseCompute::GgufWeightSource source;

    Matrix(std::uint32_t in_, std::uint32_t out_, int encoding_, unsigned seed)
        : in(in_), out(out_), encoding(encoding_), bytes(std::size_t(out_) * row_bytes(in_, encoding_)) {
        id.inode = seed;
        id.payload_end = bytes.size();
        unsigned s = seed * 2654435761u + 1;
        auto next = [&] { return s = s * 1664525u + 1013904223u; };
        const std::size_t rb = row_bytes(in, encoding);
        for (std::uint32_t n = 0; n < out; ++n) {
            std::uint8_t* row = bytes.data() + n * rb;
            if (encoding == KB200_F32) {
                for (std::uint32_t k = 0; k < in; ++k) {
                    const float v = float(int(next() >> 24) - 128) / 64.0f;
                    std::memcpy(row + 4 * k, &v, 4);
                }
            } else {
                for (std::uint32_t b = 0; b < in / 32; ++b) {
                    const std::uint16_t d = std::uint16_t(0x3000 + (next() >> 28));  // 2^-3 .. 2^-3 * (1 + 15/1024)
                    std::memcpy(row + b * 34, &d, 2);
                    for (int j = 0; j < 32; ++j)
                        row[b * 34 + 2 + j] = std::uint8_t(next() >> 24);
                }
            }
        }
        source = [this](std::size_t first, std::span<std::byte> dst) {
            if (throw_on_read)
                throw std::out_of_range("source_row_missing");
            if (cancel_on_read)
                *cancel_on_read = true;
            const std::size_t rb = row_bytes(in, encoding);
            CHECK(dst.size() % rb == 0 && first + dst.size() / rb <= out);
            std::memcpy(dst.data(), bytes.data() + first * rb, dst.size());
            std::lock_guard lock(mutex);
            for (std::size_t r = 0; r < dst.size() / rb; ++r)
                rows_read.insert(first + r);
        };
    }

    std::optional<kadan::gguf::Encoding> gguf_encoding() const {
        if (encoding == KB200_F32)
            return std::nullopt;
        return kadan::gguf::Encoding(encoding);
    }

    std::vector<float> expect(const std::vector<float>& x) const {
        const std::uint32_t rows = std::uint32_t(x.size() / in);
        std::vector<float> y(std::size_t(rows) * out);
        project(bytes, in, out, encoding, x.data(), rows, y.data());
        return y;
    }

    // Every row read exactly once.
    bool read_once() const {
        if (rows_read.size() != out)
            return false;
        std::size_t want = 0;
        for (const auto r : rows_read)
            if (r != want++)
                return false;
        return true;
    }
};

std::vector<float> activations(std::size_t n, unsigned seed) {
    std::vector<float> x(n);
    unsigned s = seed;
    for (auto& v : x) {
        s = s * 1664525u + 1013904223u;
        v = float(int(s >> 24) - 128) / 32.0f;
    }
    return x;
}

void reset(std::map<int, std::uint64_t> capacities) {
    std::lock_guard lock(fake_mutex);
    devices.clear();
    for (const auto& [id, cap] : capacities) {
        devices[id].id = id;
        devices[id].capacity = cap;
    }
}

template <class F>
std::string thrown(F&& f) {
    try {
        f();
    } catch (const std::exception& e) {
        return e.what();
    }
    return "";
}

void batch_over_two_devices() {
    reset({{0, 3ull << 30}, {1, 1ull << 30}});
    auto fallback = std::make_shared<Fallback>();
    kadan::b200::Compute adapter(fallback, {0, 1}, 1ull << 30, 1ull << 30);
    DenseCompute& compute = adapter;
    Matrix a(256, 37, KB200_Q8_0, 1), b(64, 20, KB200_F32, 2), c(96, 1, KB200_Q8_0, 3);
    const auto xa = activations(3 * 256, 11), xb = activations(3 * 64, 12), xc = activations(2 * 96, 13);
    std::vector<float> ya(3 * 37, -1), yb(3 * 20, -1), yc(2 * 1, -1);
    const std::vector<DenseCompute::GgufBatchJob> jobs{
        {&a.id, a.gguf_encoding(), &a.source, xa, 256, 37, ya, true},
        {&b.id, b.gguf_encoding(), &b.source, xb, 64, 20, yb, false},
        {&c.id, c.gguf_encoding(), &c.source, xc, 96, 1, yc, true},
    };
    std::atomic_bool cancel = false;
    CHECK(compute.dense_gguf_batch(jobs, cancel) == ProjectionResult::finite);
    CHECK(ya == a.expect(xa) && yb == b.expect(xb) && yc == c.expect(xc));
    CHECK(a.read_once() && b.read_once() && c.read_once());
    // 3:1 envelopes: each job's columns split at weight_boundary; the one-column
    // job lands wholly on one device.
    const std::uint64_t caps[2] = {3ull << 30, 1ull << 30};
    std::vector<std::uint32_t> want0, want1;
    for (const std::uint32_t out : {37u, 20u, 1u}) {
        const auto cut = std::uint32_t(kb200_weight_boundary(out, caps, 2, 1));
        if (cut)
            want0.push_back(cut);
        if (out - cut)
            want1.push_back(out - cut);
    }
    CHECK(device_of(0).outs == want0 && device_of(1).outs == want1);
    CHECK(device_of(0).calls == 1 && device_of(1).calls == 1);
    CHECK(want0.size() + want1.size() == 5);  // only the one-column job is not split
    std::vector<WeightIdentity> ids{a.id, b.id};
    CHECK(compute.release_weights(ids) == 14 + 200 + 200);
    const auto placement = compute.weight_placement();
    CHECK(placement.size() == 3 && placement[0].device == 9 && placement[1].device == 0 && placement[2].device == 1);
    CHECK(placement[1].planned_bytes == (3ull << 30) && placement[2].allocated_bytes == (1ull << 28));
    compute.release_devices();
    CHECK(fallback->release_devices_calls == 1);
    std::vector<float> w(8), y(1);
    compute.dense(w, {}, w, 8, 1, y, cancel, false);
    CHECK(fallback->dense_calls == 1);
}

void source_with_bias_over_two_devices() {
    reset({{0, 1ull << 30}, {1, 1ull << 30}});
    kadan::b200::Compute adapter(std::make_shared<Fallback>(), {0, 1}, 1ull << 30, 1ull << 30);
    DenseCompute& compute = adapter;
    Matrix a(128, 29, KB200_Q8_0, 4);
    const auto x = activations(5 * 128, 21);
    std::vector<float> bias(29), y(5 * 29, -1);
    for (std::size_t n = 0; n < bias.size(); ++n)
        bias[n] = float(n) - 10.5f;
    std::atomic_bool cancel = false;
    CHECK(compute.dense_gguf_source(a.id, *a.gguf_encoding(), a.source, bias, x, 128, 29, y, cancel)
          == ProjectionResult::finite);
    auto want = a.expect(x);
    for (std::size_t r = 0; r < 5; ++r)
        for (std::size_t n = 0; n < 29; ++n)
            want[r * 29 + n] += bias[n];
    CHECK(y == want && a.read_once());
    const std::uint64_t caps[2] = {1ull << 30, 1ull << 30};
    const auto cut = kb200_weight_boundary(29, caps, 2, 1);
    CHECK(device_of(0).bias == bias.data() && device_of(1).bias == bias.data() + cut);
    CHECK(device_of(0).outs == std::vector<std::uint32_t>{std::uint32_t(cut)});
}

void unsupported_before_any_read() {
    reset({{0, 1ull << 30}});
    kadan::b200::Compute adapter(std::make_shared<Fallback>(), {0}, 1ull << 30, 1ull << 30);
    DenseCompute& compute = adapter;
    Matrix good(64, 8, KB200_Q8_0, 5), odd(36, 8, KB200_F32, 6);
    const auto xg = activations(64, 1), xo = activations(36, 2);
    std::vector<float> yg(8, -1), yo(8, -1);
    std::atomic_bool cancel = false;
    // in % 8 != 0 in the second job: nothing read, nothing written, no device call.
    const std::vector<DenseCompute::GgufBatchJob> jobs{
        {&good.id, good.gguf_encoding(), &good.source, xg, 64, 8, yg, true},
        {&odd.id, odd.gguf_encoding(), &odd.source, xo, 36, 8, yo, true},
    };
    CHECK(compute.dense_gguf_batch(jobs, cancel) == ProjectionResult::unsupported);
    // Too many input rows for one job (gguf_batch_max_rows).
    const auto big = activations(4097 * 64, 3);
    std::vector<float> ybig(4097 * 8);
    const std::vector<DenseCompute::GgufBatchJob> tall{{&good.id, good.gguf_encoding(), &good.source, big, 64, 8,
                                                        ybig, true}};
    CHECK(compute.dense_gguf_batch(tall, cancel) == ProjectionResult::unsupported);
    // The fp64 path, a bias of the wrong length and an output of the wrong size.
    CHECK(compute.dense_gguf_source(good.id, *good.gguf_encoding(), good.source, {}, xg, 64, 8, yg, cancel, true)
          == ProjectionResult::unsupported);
    std::vector<float> short_bias(7);
    CHECK(compute.dense_gguf_source(good.id, *good.gguf_encoding(), good.source, short_bias, xg, 64, 8, yg, cancel)
          == ProjectionResult::unsupported);
    CHECK(compute.dense_gguf_source(good.id, *good.gguf_encoding(), good.source, {}, xg, 64, 8,
                                    std::span(yg).first(7), cancel)
          == ProjectionResult::unsupported);
    // The grid-coded encodings were enabled with the worker's own grids; their
    // blocks are 256 values, so a 64-column input is still unsupported.
    CHECK(kb200_encoding_supported(KB200_IQ2_S) && kb200_encoding_supported(KB200_IQ3_XXS)
          && kb200_encoding_supported(KB200_IQ3_S));
    CHECK(compute.dense_gguf_source(good.id, kadan::gguf::Encoding::iq2_s, good.source, {}, xg, 64, 8, yg, cancel)
          == ProjectionResult::unsupported);
    CHECK(good.rows_read.empty() && odd.rows_read.empty() && device_of(0).calls == 0);
    for (const float v : yg)
        CHECK(v == -1);
}

void failures() {
    std::atomic_bool cancel = false;
    Matrix a(64, 16, KB200_Q8_0, 7);
    const auto x = activations(64, 4);
    std::vector<float> y(16);
    const std::vector<DenseCompute::GgufBatchJob> jobs{{&a.id, a.gguf_encoding(), &a.source, x, 64, 16, y, true}};
    // A status that stands for one of the reference's messages throws exactly it,
    // on one device and over two.
    for (const auto& ids : {std::vector<int>{0}, std::vector<int>{0, 1}}) {
        reset({{0, 1ull << 30}, {1, 1ull << 30}});
        kadan::b200::Compute adapter(std::make_shared<Fallback>(), ids, 1ull << 30, 1ull << 30);
        DenseCompute& compute = adapter;
        device_of(ids.back()).status = KB200_NONFINITE_WEIGHT;
        device_of(ids.back()).error = "a weight decoded to a non-finite value";
        CHECK(thrown([&] { compute.dense_gguf_batch(jobs, cancel); }) == "h3_cuda_nonfinite_weight");
        device_of(ids.back()).status = KB200_CUDA;
        device_of(ids.back()).error = "cudaMemcpyAsync: out of memory";
        CHECK(thrown([&] { compute.dense_gguf_batch(jobs, cancel); }) == "cudaMemcpyAsync: out of memory");
        device_of(ids.back()).status = KB200_OK;
        device_of(ids.back()).result = KB200_RESULT_UNVALIDATED;
        CHECK(compute.dense_gguf_batch(jobs, cancel) == ProjectionResult::unvalidated);
        device_of(ids.back()).result = KB200_RESULT_FINITE;
        // Cancelled on entry: thrown before any device call (h3_compute.cu:3966),
        // also for an empty batch; an empty batch is otherwise unsupported.
        const int calls = device_of(0).calls;
        cancel = true;
        CHECK(thrown([&] { compute.dense_gguf_batch(jobs, cancel); }) == "h3_cuda_cancelled");
        CHECK(thrown([&] { compute.dense_gguf_batch({}, cancel); }) == "h3_cuda_cancelled");
        CHECK(device_of(0).calls == calls && !device_of(0).saw_cancel);
        cancel = false;
        CHECK(compute.dense_gguf_batch({}, cancel) == ProjectionResult::unsupported);
        // Cancelled while the sources are read: the devices see the caller's flag.
        a.cancel_on_read = &cancel;
        CHECK(thrown([&] { compute.dense_gguf_batch(jobs, cancel); }) == "h3_cuda_cancelled");
        CHECK(device_of(0).saw_cancel);
        a.cancel_on_read = nullptr;
        cancel = false;
        // A source's own exception comes back as itself, after every device finished.
        a.throw_on_read = true;
        bool caught = false;
        try {
            compute.dense_gguf_batch(jobs, cancel);
        } catch (const std::out_of_range& e) {
            caught = std::string(e.what()) == "source_row_missing";
        }
        CHECK(caught);
        a.throw_on_read = false;
        CHECK(compute.dense_gguf_batch(jobs, cancel) == ProjectionResult::finite && y == a.expect(x));
    }
    // A device that cannot be opened: the constructor throws the library's text.
    reset({{0, 1ull << 30}});
    CHECK(thrown([] { kadan::b200::Compute(std::make_shared<Fallback>(), {0, 5}, 1, 1); }) == "no such device");
    CHECK(thrown([] { kadan::b200::Compute(std::make_shared<Fallback>(), {}, 1, 1); }) == "b200_devices");
}

}  // namespace

// The adapter's MoE member: shapes that do not fit are unsupported before
// the device is asked, the device's unsupported stays unsupported with the
// output untouched, its failures throw the reference's messages, and a
// success returns the device's result on the chosen device.
void moe_layer() {
    reset({{0, 1ull << 30}, {1, 1ull << 30}});
    kadan::b200::Compute compute(std::make_shared<Fallback>(), {0, 1}, 1ull << 30, 1ull << 20);
    kb200_moe_weights w{};
    w.hidden = 8, w.experts = 4, w.top_k = 2;
    std::vector<float> x(3 * 8), logits(3 * 4), y(3 * 8, -1.f);
    for (std::size_t i = 0; i < x.size(); ++i)
        x[i] = float(i);
    std::atomic_bool cancel{false};
    CHECK(compute.moe_mxfp4(w, x, logits, 3, std::span(y).first(8), cancel) == ProjectionResult::unsupported);
    CHECK(compute.moe_mxfp4(w, x, std::span(logits).first(4), 3, y, cancel) == ProjectionResult::unsupported);
    CHECK(compute.moe_mxfp4(w, x, logits, 3, y, cancel, 2) == ProjectionResult::unsupported);
    CHECK(device_of(0).calls == 0 && device_of(1).calls == 0);
    CHECK(compute.moe_mxfp4(w, x, logits, 3, y, cancel, 1) == ProjectionResult::finite);
    CHECK(device_of(1).calls == 1 && device_of(0).calls == 0 && y[5] == 10.f && device_of(1).saw_cancel);
    device_of(0).status = KB200_UNSUPPORTED;
    std::vector<float> untouched(y.size(), -1.f);
    CHECK(compute.moe_mxfp4(w, x, logits, 3, untouched, cancel) == ProjectionResult::unsupported);
    CHECK(untouched[5] == -1.f);
    device_of(0).status = KB200_NONFINITE_INPUT;
    CHECK(thrown([&] { compute.moe_mxfp4(w, x, logits, 3, y, cancel); }) == "h3_cuda_nonfinite_input");
    device_of(0).status = KB200_CUDA;
    device_of(0).error = "h3_cuda: launch failed (moe)";
    CHECK(thrown([&] { compute.moe_mxfp4(w, x, logits, 3, y, cancel); }) == "h3_cuda: launch failed (moe)");
    cancel = true;
    CHECK(thrown([&] { compute.moe_mxfp4(w, x, logits, 3, y, cancel); }) == "h3_cuda_cancelled");
}

// Attention and delta-net: shapes the library does not take, and layers
// whose fresh step it did not take, stay with the wrapped compute; the
// library's layers keep every later step and the snapshot; release_scratch
// without keep drops them.
void layer_math() {
    reset({{0, 1ull << 30}});
    auto fallback = std::make_shared<Fallback>();
    kadan::b200::Compute compute(fallback, {0}, 1ull << 30, 1ull << 20);
    std::atomic_bool cancel{false};
    std::vector<float> q(2 * 8 * 128, 0.5f), kv(6 * 2 * 128), out(q.size());
    CHECK(compute.attend_cached(1, q, kv, kv, 2, 1, 8, 2, 128, 1.f, out, cancel, {}, {}));
    CHECK(device_of(0).layer_calls == 1 && out[7] == 0.5f && fallback->layer_calls == 0);
    std::vector<float> q96(8 * 96), kv96(2 * 96), out96(q96.size());
    CHECK(!compute.attend_cached(1, q96, kv96, kv96, 1, 0, 8, 2, 96, 1.f, out96, cancel, {}, {}));
    CHECK(fallback->layer_calls == 1 && device_of(0).layer_calls == 1);
    device_of(0).status = KB200_CUDA;
    device_of(0).error = "h3_cuda: launch failed (attention)";
    CHECK(thrown([&] { compute.attend_cached(1, q, kv, kv, 2, 1, 8, 2, 128, 1.f, out, cancel, {}, {}); })
          == "h3_cuda: launch failed (attention)");
    device_of(0).status = KB200_OK;

    const std::size_t kh = 2, vh = 4, dim = 64, kernel = 4, rows = 1, channels = (2 * kh + vh) * dim;
    std::vector<float> qkv(rows * channels), z(rows * vh * dim), ab(rows * vh), conv(channels * kernel), dt(vh),
        a(vh), norm(dim), y(rows * vh * dim);
    auto step = [&](std::uint64_t layer, bool fresh, std::size_t d) {
        return DenseCompute::DeltaStep{layer, fresh, qkv, z, ab, ab, conv, dt, a, std::span(norm).first(d), rows, kh,
                                       vh, d, kernel, 1e-6f, true, y};
    };
    const int before = device_of(0).layer_calls;
    // Layer 5: its fresh step does not fit (norm of 32 for dim 64), so the
    // wrapped compute keeps it, later steps included.
    CHECK(compute.delta_step(step(5, true, 32), cancel) && fallback->layer_calls == 2);
    CHECK(compute.delta_step(step(5, false, dim), cancel) && fallback->layer_calls == 3);
    // Layer 6: the library's from its fresh step on.
    CHECK(compute.delta_step(step(6, true, dim), cancel) && y[3] == 1.f);
    CHECK(compute.delta_step(step(6, false, dim), cancel));
    CHECK(device_of(0).layer_calls == before + 2 && device_of(0).fresh == std::vector<int>({1, 0}));
    std::vector<float> st(vh * dim * dim), hist((kernel - 1) * channels);
    compute.copy_recurrent_state(6, st, hist);
    CHECK(st[0] == 5.f && hist[0] == 6.f);
    compute.copy_recurrent_state(5, st, hist);
    CHECK(st[0] == 7.f && fallback->layer_calls == 4);
    compute.release_scratch(true);
    CHECK(device_of(0).layers_released == 0);
    compute.release_scratch(false);
    CHECK(device_of(0).layers_released == 1);
    // After the release layer 6 is no longer the library's.
    CHECK(compute.delta_step(step(6, false, dim), cancel) && fallback->layer_calls == 5);
}

int main() {
    layer_math();
    moe_layer();
    batch_over_two_devices();
    source_with_bias_over_two_devices();
    unsupported_before_any_read();
    failures();
    std::puts("ok");
    return 0;
}
