/* Test infrastructure only (see oracle.h): the CPU checker for the layer math
 * around the quantized path (RMSNorm, L2 norm, RoPE, cached attention, the
 * gated delta-net step).
 *
 * A restatement, in plain C, of the reference worker's host code, which the
 * worker runs when its DenseCompute declines attend_cached / delta_step.
 * Paths are relative to services/hikari/inference_worker/ of the reference.
 * Built with -ffp-contract=off like oracle.c, so each float operation rounds
 * on its own as the reference's host code does.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* src/models/text/gguf_weights.cpp:627-637 */
static float f_sigmoid(float x) {
    return 1.f / (1.f + expf(-x));
}

static float f_silu(float x) {
    return x / (1.f + expf(-x));
}

static float f_softplus(float x) {
    return x > 20.f ? x : log1pf(expf(x));
}

/* rms_norm(x, weight, eps) and rms_norm(x, width, eps), gguf_weights.cpp:
 * 639-666: the sum of squares in double, the scale in float, then x * scale
 * (* weight). weight NULL: the unweighted form. Returns 0, or -1 when an
 * output is not finite (the weighted form's gguf_text_norm_nonfinite). */
int orc_rms_norm(float* x, const float* weight, size_t rows, size_t width, float eps) {
    int finite = 1;
    for (size_t r = 0; r < rows; ++r) {
        float* v = x + r * width;
        double sum = 0;
        for (size_t i = 0; i < width; ++i)
            sum += (double)v[i] * v[i];
        const float scale = 1.f / sqrtf((float)(sum / (double)width) + eps);
        for (size_t i = 0; i < width; ++i) {
            v[i] = weight ? v[i] * scale * weight[i] : v[i] * scale;
            if (!isfinite(v[i]))
                finite = 0;
        }
    }
    return weight && !finite ? -1 : 0;
}

/* l2_norm, gguf_weights.cpp:667-674: x / sqrt(sum(x^2) + eps) per width. */
void orc_l2_norm(float* x, size_t rows, size_t width, float eps) {
    orc_rms_norm(x, NULL, rows, width, eps / (float)width);
    const float scale = 1.f / sqrtf((float)width);
    for (size_t i = 0; i < rows * width; ++i)
        x[i] *= scale;
}

/* rope, gguf_weights.cpp:676-700, applied to `rows` rows of `row_width`
 * values (heads of `width` values each) at positions position, position+1,
 * ... (AttentionLayer::forward, qwen_layers.cpp:242-256): per head, pairs
 * (i, i + rotary/2) rotate by theta_i = position * base^(-2i/rotary), theta
 * formed by repeated float multiplication. */
void orc_rope(float* x, size_t rows, size_t row_width, size_t width, size_t rotary, size_t position, float base) {
    const float theta_scale = powf(base, -2.0f / (float)rotary);
    const size_t half = rotary / 2;
    for (size_t r = 0; r < rows; ++r)
        for (size_t at = r * row_width; at < (r + 1) * row_width; at += width) {
            float theta = (float)(position + r);
            for (size_t i = 0; i < half; ++i) {
                const float c = cosf(theta), s = sinf(theta);
                const float a = x[at + i], b = x[at + i + half];
                x[at + i] = a * c - b * s;
                x[at + i + half] = a * s + b * c;
                theta *= theta_scale;
            }
        }
}

/* Host attention of one query row over `count` keys (attend,
 * gguf_weights.cpp:700-777, queries = 1): float dot products accumulated in
 * key order, the max-subtracted exponentials summed in double, weights
 * p = float(e / total), outputs accumulated in float in key order. The
 * row's t-th key sits at cache position chosen[t] (t without a selection). */
static void attend_row(const float* q, const float* keys, const float* values, const uint32_t* chosen, size_t count,
                       size_t heads, size_t kv_heads, size_t dim, float scale, float* scores, float* out) {
    for (size_t h = 0; h < heads; ++h) {
        const size_t kv = h / (heads / kv_heads);
        const float* query = q + h * dim;
        float maximum = -INFINITY;
        for (size_t t = 0; t < count; ++t) {
            const size_t pos = chosen ? chosen[t] : t;
            const float* key = keys + (pos * kv_heads + kv) * dim;
            float dot = 0;
            for (size_t d = 0; d < dim; ++d)
                dot += query[d] * key[d];
            scores[t] = dot * scale;
            if (scores[t] > maximum)
                maximum = scores[t];
        }
        double total = 0;
        for (size_t t = 0; t < count; ++t) {
            scores[t] = expf(scores[t] - maximum);
            total += scores[t];
        }
        float* y = out + h * dim;
        for (size_t d = 0; d < dim; ++d)
            y[d] = 0.f;
        for (size_t t = 0; t < count; ++t) {
            const float p = (float)(scores[t] / total);
            const size_t pos = chosen ? chosen[t] : t;
            const float* value = values + (pos * kv_heads + kv) * dim;
            for (size_t d = 0; d < dim; ++d)
                y[d] += p * value[d];
        }
    }
}

/* AttentionLayer::forward's cached attention (qwen_layers.cpp:259-330):
 * q [rows][heads][dim], keys/values [positions][kv_heads][dim]; row r sits at
 * position + r and attends every position up to its own, or, with
 * `selected`, the positions selected[offsets[r] .. offsets[r + 1]) in that
 * order. out [rows][heads][dim]. Returns -1 on a bad shape. */
int orc_attend_cached(const float* q, const float* keys, const float* values, size_t rows, size_t position,
                      size_t heads, size_t kv_heads, size_t dim, float scale, const uint32_t* selected,
                      const uint32_t* offsets, float* out) {
    if (!rows || !heads || !kv_heads || heads % kv_heads || !dim)
        return -1;
    size_t most = position + rows;
    if (selected)
        for (size_t r = 0; r < rows; ++r)
            if (offsets[r + 1] - offsets[r] > most)
                most = offsets[r + 1] - offsets[r];
    float* scores = (float*)malloc((most ? most : 1) * sizeof(float));
    if (!scores)
        return -1;
    for (size_t r = 0; r < rows; ++r) {
        const uint32_t* chosen = selected ? selected + offsets[r] : NULL;
        const size_t count = selected ? offsets[r + 1] - offsets[r] : position + r + 1;
        attend_row(q + r * heads * dim, keys, values, chosen, count, heads, kv_heads, dim, scale, scores,
                   out + r * heads * dim);
    }
    free(scores);
    return 0;
}

/* delta_rule, gguf_weights.cpp:778-818: the decayed state recomputed in both
 * passes with the same rounding. decay holds one factor (decays == 1) or one
 * per key row (decays == dim). dim <= 256. */
void orc_delta_rule(float* state, const float* q, const float* k, const float* v, const float* decay, size_t decays,
                    float beta, size_t dim, float* out) {
    float delta[256];
    for (size_t j = 0; j < dim; ++j)
        delta[j] = v[j];
    for (size_t i = 0; i < dim; ++i) {
        const float g = decay[decays == 1 ? 0 : i];
        const float* row = state + i * dim;
        for (size_t j = 0; j < dim; ++j)
            delta[j] -= row[j] * g * k[i];
    }
    for (size_t j = 0; j < dim; ++j)
        delta[j] *= beta;
    for (size_t j = 0; j < dim; ++j)
        out[j] = 0.f;
    for (size_t i = 0; i < dim; ++i) {
        const float g = decay[decays == 1 ? 0 : i];
        float* row = state + i * dim;
        for (size_t j = 0; j < dim; ++j) {
            row[j] = row[j] * g + k[i] * delta[j];
            out[j] += row[j] * q[i];
        }
    }
}

/* DeltaNetLayer::forward's host path (qwen_layers.cpp:131-180) for `rows`
 * rows in order. qkv [rows][channels] with channels = 2 key_heads dim +
 * value_heads dim (q, k, v), z [rows][value_heads dim], alpha/beta
 * [rows][value_heads], conv [channels][kernel], dt/a [value_heads], norm
 * [dim]. history [(kernel - 1)][channels] (oldest first) and state
 * [value_heads][dim][dim] are updated in place. out [rows][value_heads dim]. */
int orc_delta_step(const float* qkv, const float* z, const float* alpha, const float* beta, const float* conv,
                   const float* dt, const float* a, const float* norm, size_t rows, size_t key_heads,
                   size_t value_heads, size_t dim, size_t kernel, float eps, int sigmoid_gate, float* history,
                   float* state, float* out) {
    if (!rows || !key_heads || !value_heads || !dim || dim > 256 || kernel < 1)
        return -1;
    const size_t channels = 2 * key_heads * dim + value_heads * dim, inner = value_heads * dim, past = kernel - 1;
    const float scale = 1.f / sqrtf((float)dim);
    float* mixed = (float*)malloc(channels * sizeof(float));
    if (!mixed)
        return -1;
    float query[256], head[256];
    for (size_t r = 0; r < rows; ++r) {
        const float* x = qkv + r * channels;
        for (size_t c = 0; c < channels; ++c) {
            const float* w = conv + c * kernel;
            float sum = 0;
            for (size_t k = 0; k < past; ++k)
                sum += history[k * channels + c] * w[k];
            sum += x[c] * w[past];
            mixed[c] = f_silu(sum);
        }
        if (past) {
            memmove(history, history + channels, (past - 1) * channels * sizeof(float));
            memcpy(history + (past - 1) * channels, x, channels * sizeof(float));
        }
        float* qv = mixed;
        float* kv = mixed + key_heads * dim;
        const float* vv = mixed + 2 * key_heads * dim;
        orc_l2_norm(qv, key_heads, dim, eps);
        orc_l2_norm(kv, key_heads, dim, eps);
        for (size_t h = 0; h < value_heads; ++h) {
            const size_t kh = h % key_heads;
            const float decay = expf(f_softplus(alpha[r * value_heads + h] + dt[h]) * a[h]);
            for (size_t d = 0; d < dim; ++d)
                query[d] = qv[kh * dim + d] * scale;
            orc_delta_rule(state + h * dim * dim, query, kv + kh * dim, vv + h * dim, &decay, 1,
                           f_sigmoid(beta[r * value_heads + h]), dim, head);
            orc_rms_norm(head, norm, 1, dim, eps);
            for (size_t d = 0; d < dim; ++d) {
                const float gate = z[r * inner + h * dim + d];
                out[r * inner + h * dim + d] = head[d] * (sigmoid_gate ? f_sigmoid(gate) : f_silu(gate));
            }
        }
    }
    free(mixed);
    return 0;
}

/* The reference MoE's shared expert (MoeLayer::forward, qwen_layers.cpp:
 * 390-395 and 477-490): the activation silu(gate) * up between its gate/up
 * and down projections, and the gated add of its down projection to the
 * routed experts' sum, gate = sigmoid(shared_gate . x) with the dot product
 * accumulated in float in column order. */
void orc_silu_mul(const float* gate, const float* up, size_t n, float* out) {
    for (size_t j = 0; j < n; ++j)
        out[j] = f_silu(gate[j]) * up[j];
}

void orc_moe_add_shared(const float* x, const float* shared_gate, const float* down, size_t tokens, size_t hidden,
                        float* out) {
    for (size_t t = 0; t < tokens; ++t) {
        float gate = 0;
        for (size_t c = 0; c < hidden; ++c)
            gate += shared_gate[c] * x[t * hidden + c];
        gate = f_sigmoid(gate);
        for (size_t d = 0; d < hidden; ++d)
            out[t * hidden + d] = out[t * hidden + d] + down[t * hidden + d] * gate;
    }
}
