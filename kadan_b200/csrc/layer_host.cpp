// Attention and delta-net from host spans: the DenseCompute virtuals
// attend_cached, delta_step and copy_recurrent_state
// (services/hikari/inference_worker/include/kadan/dense_compute.hpp:275-330)
// over per-layer device state that a context keeps until
// kb200_context_release_layers (the reference's release_scratch).
//
// KV mirror of a layer: [capacity][kv_heads * dim] keys and values on the
// device. A call uploads positions [min(mirrored, position), position + rows)
// (earlier mirrored positions are reused, the call's own positions are
// uploaded again because the caller may have rewritten them) and attends on
// the device. Delta-net state of a layer: the recurrent state and the
// convolution history, created by a fresh step (zero or from the caller's
// snapshot) and carried from step to step on the device.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <new>

#include "context.hpp"
#include "kb200_host.hpp"

namespace kb200 {

struct KvMirror {
    float* keys = nullptr;
    float* values = nullptr;
    size_t capacity = 0;  // positions
    size_t mirrored = 0;  // positions [0, mirrored) hold the caller's data
    size_t width = 0;     // kv_heads * dim
};

struct DeltaState {
    float* state = nullptr;    // [value_heads][dim][dim]
    float* history = nullptr;  // [(kernel - 1)][channels]
    size_t state_floats = 0, history_floats = 0;
    uint32_t key_heads = 0, value_heads = 0, dim = 0, kernel = 0;
};

struct LayerStore {
    std::map<uint64_t, KvMirror> kv;
    std::map<uint64_t, DeltaState> delta;
};

namespace {

void free_mirror(KvMirror& m) {
    cudaFree(m.keys);
    cudaFree(m.values);
    m = KvMirror{};
}

void free_state(DeltaState& d) {
    cudaFree(d.state);
    cudaFree(d.history);
    d = DeltaState{};
}

LayerStore* store_of(kb200_context* c) {
    if (!c->layers)
        c->layers = new (std::nothrow) LayerStore;
    return c->layers;
}

size_t up256(size_t v) {
    return (v + 255) / 256 * 256;
}

// Grows the mirror to hold `positions` (keeping the mirrored prefix); a new
// row width starts the mirror over.
int reserve(KvMirror& m, size_t positions, size_t width, cudaStream_t stream) {
    if (m.width != width) {
        free_mirror(m);
        m.width = width;
    }
    if (positions <= m.capacity)
        return KB200_OK;
    const size_t cap = std::max(positions, m.capacity + m.capacity / 2);
    float *k = nullptr, *v = nullptr;
    if (cudaMalloc(&k, cap * width * sizeof(float)) != cudaSuccess
        || cudaMalloc(&v, cap * width * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(k);
        return fail(KB200_NO_MEMORY, "KV mirror");
    }
    if (m.mirrored) {
        const size_t bytes = m.mirrored * width * sizeof(float);
        cudaError_t e = cudaMemcpyAsync(k, m.keys, bytes, cudaMemcpyDeviceToDevice, stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(v, m.values, bytes, cudaMemcpyDeviceToDevice, stream);
        if (e == cudaSuccess)
            e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) {
            cudaFree(k);
            cudaFree(v);
            return cuda_fail(e, "KV mirror growth");
        }
    }
    cudaFree(m.keys);
    cudaFree(m.values);
    m.keys = k, m.values = v, m.capacity = cap;
    return KB200_OK;
}

}  // namespace

void release_layers(LayerStore* store) {
    if (!store)
        return;
    for (auto& [layer, m] : store->kv)
        free_mirror(m);
    for (auto& [layer, d] : store->delta)
        free_state(d);
    delete store;
}

}  // namespace kb200

using namespace kb200;

extern "C" {

int kb200_attend_cached_host(kb200_context* c, uint64_t layer, const float* q, const float* keys, const float* values,
                             size_t rows, size_t position, size_t heads, size_t kv_heads, size_t dim, float scale,
                             const uint32_t* selected, const uint32_t* offsets, float* output,
                             const volatile uint8_t* cancel) {
    if (!c || !kb200_attend_supported(heads, kv_heads, dim))
        return fail(KB200_UNSUPPORTED, "attention shape");
    if (cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled before start");
    if (!rows)
        return KB200_OK;
    if (!q || !keys || !values || !output || (selected && !offsets))
        return fail(KB200_INVALID, "null pointer");
    if (rows > 65535 || position + rows > 0x7FFFFFFFu)
        return fail(KB200_UNSUPPORTED, "too many rows or positions");
    const size_t width = kv_heads * dim, qn = rows * heads * dim;
    size_t picks = 0;
    if (selected) {
        if (offsets[0] != 0)
            return fail(KB200_INVALID, "offsets must start at 0");
        for (size_t r = 0; r < rows; ++r) {
            if (offsets[r + 1] < offsets[r] || offsets[r + 1] - offsets[r] > position + rows)
                return fail(KB200_INVALID, "bad selection offsets");
            for (uint32_t t = offsets[r]; t < offsets[r + 1]; ++t)
                if (selected[t] > position + r)
                    return fail(KB200_INVALID, "gguf_text_sparse_future");
        }
        picks = offsets[rows];
    }
    DeviceScope scope(c->device);
    LayerStore* store = store_of(c);
    if (!store)
        return fail(KB200_NO_MEMORY, "layer store");
    KvMirror& m = store->kv[layer];
    if (const int s = reserve(m, position + rows, width, c->stream))
        return s;
    // Device workspace: [q][out][selected][offsets][attention partials];
    // pinned staging: the same without the partials.
    const size_t q_bytes = qn * sizeof(float), o_at = up256(q_bytes), s_at = o_at + up256(q_bytes);
    const size_t f_at = s_at + up256(picks * 4), w_at = f_at + up256((rows + 1) * 4);
    const size_t need = kb200_attend_workspace_bytes(rows, position, heads, dim);
    if (const int s = context_ensure(c, w_at + need, w_at))
        return s;
    auto* dev = static_cast<uint8_t*>(c->workspace);
    auto* host = static_cast<uint8_t*>(c->pinned);
    std::memcpy(host, q, q_bytes);
    if (selected) {
        std::memcpy(host + s_at, selected, picks * 4);
        std::memcpy(host + f_at, offsets, (rows + 1) * 4);
    }
    ++c->counters.calls;
    const size_t from = std::min(m.mirrored, position), count = position + rows - from;
    cudaError_t e = cudaMemcpyAsync(m.keys + from * width, keys + from * width, count * width * sizeof(float),
                                    cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m.values + from * width, values + from * width, count * width * sizeof(float),
                            cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(dev, host, w_at, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) {
        m.mirrored = std::min(m.mirrored, from);
        return cuda_fail(e, "attention upload");
    }
    m.mirrored = position + rows;
    const int s = kb200_attend_cached(reinterpret_cast<const float*>(dev), m.keys, m.values, rows, position, heads,
                                      kv_heads, dim, scale,
                                      selected ? reinterpret_cast<const uint32_t*>(dev + s_at) : nullptr,
                                      selected ? reinterpret_cast<const uint32_t*>(dev + f_at) : nullptr,
                                      reinterpret_cast<float*>(dev + o_at), dev + w_at, need, c->stream);
    if (s) {
        cudaStreamSynchronize(c->stream);
        return s;
    }
    e = cudaMemcpyAsync(host + o_at, dev + o_at, q_bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "attention download");
    if (cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled after download");
    std::memcpy(output, host + o_at, q_bytes);
    return KB200_OK;
}

int kb200_delta_step_host(kb200_context* c, const kb200_delta_host* st, const volatile uint8_t* cancel) {
    if (!c || !st)
        return fail(KB200_INVALID, "null context or step");
    DeltaState* have = nullptr;
    if (c->layers) {
        auto it = c->layers->delta.find(st->layer);
        if (it != c->layers->delta.end())
            have = &it->second;
    }
    if (!st->fresh) {
        // A later step must not lose the state the device holds.
        if (!have)
            return fail(KB200_INVALID, "recurrent_state_lost");
        if (have->key_heads != st->key_heads || have->value_heads != st->value_heads || have->dim != st->dim
            || have->kernel != st->kernel)
            return fail(KB200_INVALID, "recurrent state shape changed");
    } else if (!kb200_delta_supported(st->key_heads, st->value_heads, st->dim, st->kernel)) {
        return fail(KB200_UNSUPPORTED, "delta-net shape");
    }
    if (cancelled(cancel))
        return fail(KB200_CANCELLED, "cancelled before start");
    if (!st->rows)
        return KB200_OK;
    if (!st->qkv || !st->z || !st->alpha || !st->beta || !st->conv || !st->dt || !st->a || !st->norm || !st->output)
        return fail(KB200_INVALID, "null pointer");
    const size_t VH = st->value_heads, dim = st->dim, rows = st->rows;
    const size_t channels = (2 * size_t(st->key_heads) + VH) * dim, inner = VH * dim;
    const size_t state_floats = VH * dim * dim, history_floats = size_t(st->kernel - 1) * channels;
    DeviceScope scope(c->device);
    LayerStore* store = store_of(c);
    if (!store)
        return fail(KB200_NO_MEMORY, "layer store");
    DeltaState& d = store->delta[st->layer];
    if (st->fresh) {
        if (d.state_floats != state_floats || d.history_floats != history_floats) {
            free_state(d);
            if (cudaMalloc(&d.state, state_floats * sizeof(float)) != cudaSuccess
                || (history_floats && cudaMalloc(&d.history, history_floats * sizeof(float)) != cudaSuccess)) {
                cudaGetLastError();
                free_state(d);
                store->delta.erase(st->layer);
                return fail(KB200_NO_MEMORY, "recurrent state");
            }
            d.state_floats = state_floats, d.history_floats = history_floats;
        }
        d.key_heads = st->key_heads, d.value_heads = st->value_heads, d.dim = st->dim, d.kernel = st->kernel;
        cudaError_t e = st->initial_state ? cudaMemcpyAsync(d.state, st->initial_state, state_floats * 4,
                                                            cudaMemcpyHostToDevice, c->stream)
                                          : cudaMemsetAsync(d.state, 0, state_floats * 4, c->stream);
        if (e == cudaSuccess && history_floats)
            e = st->initial_history ? cudaMemcpyAsync(d.history, st->initial_history, history_floats * 4,
                                                      cudaMemcpyHostToDevice, c->stream)
                                    : cudaMemsetAsync(d.history, 0, history_floats * 4, c->stream);
        if (e != cudaSuccess) {
            free_state(d);
            store->delta.erase(st->layer);
            return cuda_fail(e, "recurrent state set-up");
        }
    }
    // Device workspace: [qkv][z][alpha][beta][conv][dt][a][norm][output][step
    // workspace]; pinned staging: all but the step workspace.
    const size_t sizes[9] = {rows * channels, rows * inner, rows * VH, rows * VH, channels * st->kernel,
                             VH, VH, dim, rows * inner};
    const float* srcs[8] = {st->qkv, st->z, st->alpha, st->beta, st->conv, st->dt, st->a, st->norm};
    size_t at[10] = {0};
    for (int i = 0; i < 9; ++i)
        at[i + 1] = at[i] + up256(sizes[i] * sizeof(float));
    kb200_delta_args args{};
    args.rows = st->rows, args.key_heads = st->key_heads, args.value_heads = st->value_heads, args.dim = st->dim;
    args.kernel = st->kernel, args.eps = st->eps, args.sigmoid_gate = st->sigmoid_gate;
    const size_t need = kb200_delta_workspace_bytes(&args);
    if (const int s = context_ensure(c, at[9] + need, at[9]))
        return s;
    auto* dev = static_cast<uint8_t*>(c->workspace);
    auto* host = static_cast<uint8_t*>(c->pinned);
    for (int i = 0; i < 8; ++i)
        std::memcpy(host + at[i], srcs[i], sizes[i] * sizeof(float));
    ++c->counters.calls;
    cudaError_t e = cudaMemcpyAsync(dev, host, at[8], cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "delta-net upload");
    auto F = [&](int i) { return reinterpret_cast<float*>(dev + at[i]); };
    args.qkv = F(0), args.z = F(1), args.alpha = F(2), args.beta = F(3), args.conv = F(4), args.dt = F(5);
    args.a = F(6), args.norm = F(7), args.output = F(8), args.state = d.state, args.history = d.history;
    if (const int s = kb200_delta_step(&args, dev + at[9], need, c->stream)) {
        cudaStreamSynchronize(c->stream);
        return s;
    }
    e = cudaMemcpyAsync(host + at[8], dev + at[8], sizes[8] * sizeof(float), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "delta-net download");
    std::memcpy(st->output, host + at[8], sizes[8] * sizeof(float));
    return KB200_OK;
}

int kb200_recurrent_state_get(kb200_context* c, uint64_t layer, float* state, size_t state_floats, float* history,
                              size_t history_floats) {
    if (!c)
        return fail(KB200_INVALID, "null context");
    if (!c->layers || !c->layers->delta.count(layer))
        return fail(KB200_INVALID, "recurrent_snapshot_unsupported");
    const DeltaState& d = c->layers->delta.at(layer);
    if (state_floats != d.state_floats || history_floats != d.history_floats || (state_floats && !state)
        || (history_floats && !history))
        return fail(KB200_INVALID, "recurrent snapshot size");
    DeviceScope scope(c->device);
    cudaError_t e = cudaMemcpyAsync(state, d.state, state_floats * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess && history_floats)
        e = cudaMemcpyAsync(history, d.history, history_floats * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(c->stream);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "recurrent snapshot download");
}

int kb200_context_release_layers(kb200_context* c) {
    if (!c)
        return fail(KB200_INVALID, "null context");
    DeviceScope scope(c->device);
    cudaStreamSynchronize(c->stream);
    release_layers(c->layers);
    c->layers = nullptr;
    return KB200_OK;
}

}  // extern "C"
