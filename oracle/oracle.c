/* Test infrastructure only (see oracle.h): the CPU checker for kadan_b200.
 *
 * A restatement, in plain C, of the reference worker's arithmetic on the
 * quantized-linear path. Paths below are relative to
 * services/hikari/inference_worker/ of the reference (ghalrym/Kadan).
 *
 * Built with -ffp-contract=off: every product and difference is rounded to
 * float on its own, as detail::multiply/subtract do in
 * include/kadan/gguf_quantization.hpp:597-621.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static float bits_to_float(uint32_t bits) {
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

static uint32_t float_to_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, sizeof b);
    return b;
}

/* IEEE binary16 -> binary32, exact for every pattern including subnormals,
 * infinities and NaN payloads (gguf_quantization.hpp:576-593). */
float orc_half(uint16_t bits) {
    const uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
    uint32_t exponent = (bits >> 10) & 31u, fraction = bits & 1023u;
    if (exponent == 31)
        return bits_to_float(sign | 0x7f800000u | (fraction << 13));
    if (exponent)
        return bits_to_float(sign | ((exponent + 112u) << 23) | (fraction << 13));
    if (!fraction)
        return bits_to_float(sign);
    /* Subnormal half: normalise the fraction. */
    int e = 113;
    while (!(fraction & 1024u)) {
        fraction <<= 1;
        --e;
    }
    return bits_to_float(sign | ((uint32_t)e << 23) | ((fraction & 1023u) << 13));
}

static float half_at(const uint8_t* p) {
    return orc_half((uint16_t)(p[0] | (p[1] << 8)));
}

static int s8(unsigned byte) {
    return byte < 128 ? (int)byte : (int)byte - 256;
}

/* Block geometry (gguf_quantization.hpp:65-95). */
size_t orc_block_values(int e) {
    switch (e) {
    case ORC_BF16: return 1;
    case ORC_Q8_0:
    case ORC_IQ4_NL: return 32;
    case ORC_Q3_K:
    case ORC_Q4_K:
    case ORC_Q6_K:
    case ORC_IQ4_XS:
    case ORC_IQ3_XXS:
    case ORC_IQ2_S:
    case ORC_IQ3_S: return 256;
    default: return 0;
    }
}

size_t orc_block_bytes(int e) {
    switch (e) {
    case ORC_Q3_K: return 110;
    case ORC_Q4_K: return 144;
    case ORC_Q8_0: return 34;
    case ORC_Q6_K: return 210;
    case ORC_IQ4_NL: return 18;
    case ORC_IQ4_XS: return 136;
    case ORC_IQ3_XXS: return 98;
    case ORC_IQ2_S: return 82;
    case ORC_IQ3_S: return 110;
    case ORC_BF16: return 2;
    default: return 0;
    }
}

/* The IQ4_NL non-linear code book (ggml-common.h kvalues_iq4nl). */
static const int8_t iq4nl_book[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                      1,    13,   25,  38,  53,  69,  89,  113};

/* Six-bit scale and minimum of sub-block g of a Q4_K block: 12 packed bytes,
 * groups 0-3 in the low six bits of bytes 0-7, groups 4-7 split between the
 * nibbles of bytes 8-11 and the top two bits of bytes 0-7
 * (gguf_quantization.hpp:749-756). */
static void q4k_scale_min(const uint8_t* s, unsigned g, unsigned* sc, unsigned* m) {
    if (g < 4) {
        *sc = s[g] & 63u;
        *m = s[g + 4] & 63u;
    } else {
        *sc = (s[g + 4] & 15u) | ((unsigned)(s[g - 4] >> 6) << 4);
        *m = (unsigned)(s[g + 4] >> 4) | ((unsigned)(s[g] >> 6) << 4);
    }
}

/* Code grids of the three grid-coded formats: each entry packs four (IQ3_XXS,
 * IQ3_S) or eight (IQ2_S) unsigned magnitudes, one per byte, low byte first. */
static uint32_t grid_iq3xxs[256], grid_iq3s[512];
static uint64_t grid_iq2s[1024];
static int grids_set;

void orc_set_iq_grids(const uint32_t* iq3xxs, const uint64_t* iq2s, const uint32_t* iq3s) {
    memcpy(grid_iq3xxs, iq3xxs, sizeof grid_iq3xxs);
    memcpy(grid_iq2s, iq2s, sizeof grid_iq2s);
    memcpy(grid_iq3s, iq3s, sizeof grid_iq3s);
    grids_set = 1;
}

static uint32_t le32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* Sign of lane j of an 8-value run: bit j of `signs`. The product with -1 or
 * +1 is kept as a product, as the reference writes it. */
static float signed_by(float magnitude, unsigned signs, unsigned j) {
    return magnitude * ((signs >> j) & 1u ? -1.0f : 1.0f);
}

/* One value of one block (gguf_quantization.hpp:631-762). */
float orc_decode(int e, const uint8_t* b, size_t element) {
    const unsigned el = (unsigned)element;
    switch (e) {
    case ORC_BF16:
        return bits_to_float((uint32_t)(b[0] | (b[1] << 8)) << 16);
    case ORC_Q8_0: {
        const float d = half_at(b);
        return d * (float)s8(b[2 + el]);
    }
    case ORC_Q4_K: {
        unsigned sc, m;
        const unsigned g = el / 32;
        q4k_scale_min(b + 4, g, &sc, &m);
        const unsigned packed = b[16 + (el / 64) * 32 + el % 32];
        const unsigned code = (g & 1u) ? packed >> 4 : packed & 15u;
        const float scaled = half_at(b) * (float)sc;
        const float offset = half_at(b + 2) * (float)m;
        const float product = scaled * (float)code;
        return product - offset;
    }
    case ORC_Q6_K: {
        /* 128-value halves: ql[128] low nibbles, qh[64] two high bits,
         * int8 scales[16] per 16 values, half d at byte 208. */
        const unsigned h = el / 128, o = el % 128, quarter = o / 32, lane = o % 32;
        const unsigned packed = b[h * 64 + lane + (quarter & 1u) * 32];
        const unsigned low = quarter < 2 ? packed & 15u : packed >> 4;
        const unsigned high = (b[128 + h * 32 + lane] >> (2 * quarter)) & 3u;
        const int code = (int)(low | (high << 4)) - 32;
        const int scale = s8(b[192 + h * 8 + lane / 16 + 2 * quarter]);
        const float factor = half_at(b + 208) * (float)scale;
        return factor * (float)code;
    }
    case ORC_Q3_K: {
        /* hmask[32], qs[64] two-bit codes, 12 bytes of six-bit scales, half d. */
        const unsigned g = el / 16;
        const uint8_t* s = b + 96;
        const unsigned low = g < 8 ? s[g] & 15u : (unsigned)s[g - 8] >> 4;
        const unsigned high = (s[8 + g % 4] >> (2 * (g / 4))) & 3u;
        const int scale = (int)(low | (high << 4)) - 32;
        const unsigned lane = el % 32, shift = 2 * ((el % 128) / 32);
        const unsigned two = (b[32 + (el / 128) * 32 + lane] >> shift) & 3u;
        const int code = (int)two - ((b[lane] & (1u << (el / 32))) ? 0 : 4);
        const float factor = half_at(b + 108) * (float)scale;
        return factor * (float)code;
    }
    case ORC_IQ4_NL: {
        const unsigned packed = b[2 + el % 16];
        return half_at(b) * (float)iq4nl_book[el < 16 ? packed & 15u : packed >> 4];
    }
    case ORC_IQ4_XS: {
        const unsigned g = el / 32, w = el % 32;
        const unsigned hs = (unsigned)b[2] | ((unsigned)b[3] << 8);
        const int scale =
            (int)(((b[4 + g / 2] >> (4 * (g % 2))) & 15u) | (((hs >> (2 * g)) & 3u) << 4))
            - 32;
        const unsigned packed = b[8 + g * 16 + w % 16];
        const float factor = half_at(b) * (float)scale;
        return factor * (float)iq4nl_book[w < 16 ? packed & 15u : packed >> 4];
    }
    case ORC_IQ3_XXS: {
        /* 98 bytes: half d, 64 grid indices (two per 8-value run), then per
         * 32 values a little-endian word: scale nibble in bits 28-31 and four
         * 7-bit sign sets, whose eighth sign makes the set's parity even
         * (gguf_quantization.hpp:674-694). */
        if (!grids_set)
            return NAN;
        const unsigned g = el / 32, run = (el % 32) / 8, j = el % 8;
        const uint32_t word = le32(b + 66 + 4 * g);
        const float scale = (half_at(b) * (0.5f + (float)(word >> 28))) * 0.5f;
        unsigned signs = (word >> (7 * run)) & 127u, ones = 0;
        for (unsigned t = signs; t; t &= t - 1)
            ++ones;
        signs |= (ones & 1u) << 7;
        const uint32_t entry = grid_iq3xxs[b[2 + 8 * g + 2 * run + j / 4]];
        return signed_by(scale * (float)((entry >> (8 * (j % 4))) & 255u), signs, j);
    }
    case ORC_IQ2_S: {
        /* 82 bytes: half d, 32 low index bytes (one per 8-value run), 32 sign
         * bytes, 8 bytes of two high index bits per run, 8 scale bytes of two
         * nibbles (runs 0-1, runs 2-3) (gguf_quantization.hpp:702-717). */
        if (!grids_set)
            return NAN;
        const unsigned g = el / 32, run = (el % 32) / 8, j = el % 8;
        const unsigned nibble = run < 2 ? b[74 + g] & 15u : (unsigned)b[74 + g] >> 4;
        const float scale = (half_at(b) * (0.5f + (float)nibble)) * 0.25f;
        const unsigned index = b[2 + 4 * g + run] | ((((unsigned)b[66 + g] >> (2 * run)) & 3u) << 8);
        const unsigned magnitude = (unsigned)(grid_iq2s[index] >> (8 * j)) & 255u;
        return signed_by(scale * (float)magnitude, b[34 + 4 * g + run], j);
    }
    case ORC_IQ3_S: {
        /* 110 bytes: half d, 64 low index bytes (two per run), 8 bytes of one
         * high index bit each, 32 sign bytes, 4 scale bytes of two nibbles
         * (odd scale 1 + 2n per 32 values) (gguf_quantization.hpp:719-734). */
        if (!grids_set)
            return NAN;
        const unsigned g = el / 32, run = (el % 32) / 8, j = el % 8, k = 2 * run + j / 4;
        const unsigned nibble = g & 1u ? (unsigned)b[106 + g / 2] >> 4 : b[106 + g / 2] & 15u;
        const float scale = half_at(b) * (float)(1 + 2 * (int)nibble);
        const unsigned index = b[2 + 8 * g + k] | ((((unsigned)b[66 + g] >> k) & 1u) << 8);
        const unsigned magnitude = (grid_iq3s[index] >> (8 * (j % 4))) & 255u;
        return signed_by(scale * (float)magnitude, b[74 + 4 * g + run], j);
    }
    default:
        return NAN;
    }
}

void orc_decode_stream(int e, const uint8_t* packed, size_t count, float* out) {
    const size_t values = orc_block_values(e), bytes = orc_block_bytes(e);
    for (size_t i = 0; i < count; ++i)
        out[i] = orc_decode(e, packed + i / values * bytes, i % values);
}

/* Decode-then-double-dot, the reference's own GEMV check
 * (tests/gguf_text.cpp:200-254 compares against exactly this). */
void orc_gemv_f64(
    int e,
    const uint8_t* weights,
    size_t row_bytes,
    size_t in,
    size_t out,
    const float* x,
    size_t rows,
    double* y,
    size_t y_stride
) {
    float* w = malloc(in * sizeof(float));
    for (size_t c = 0; c < out; ++c) {
        orc_decode_stream(e, weights + c * row_bytes, in, w);
        for (size_t r = 0; r < rows; ++r) {
            double s = 0;
            const float* xr = x + r * in;
            for (size_t k = 0; k < in; ++k)
                s += (double)w[k] * (double)xr[k];
            y[r * y_stride + c] = s;
        }
    }
    free(w);
}

/* E2M1: sign, two exponent bits, one mantissa bit (quantization.cpp:102-110). */
float orc_e2m1(unsigned code) {
    static const float magnitude[8] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    const float v = magnitude[code & 7u];
    return (code & 8u) ? -v : v;
}

/* w = e2m1(code) * 2^(E-127) computed exactly in double
 * (quantization.cpp:89-96); E = 255 is rejected (:47-56). */
int orc_mxfp4_decode_rows(
    size_t rows,
    size_t cols,
    const uint8_t* weights,
    const uint8_t* scales,
    size_t first,
    size_t count,
    float* out
) {
    if (!rows || !cols || cols % 32 || first > rows || count > rows - first)
        return -1;
    for (size_t r = 0; r < count; ++r) {
        const size_t row = first + r;
        for (size_t c = 0; c < cols; ++c) {
            const unsigned exponent = scales[row * (cols / 32) + c / 32];
            if (exponent == 255)
                return -2;
            const unsigned code = (weights[row * (cols / 2) + c / 2] >> (4 * (c % 2))) & 15u;
            const double v = ldexp((double)orc_e2m1(code), (int)exponent - 127);
            if (!isfinite(v) || fabs(v) > 3.4028234663852886e38)
                return -3;
            out[r * cols + c] = (float)v;
        }
    }
    return 0;
}

/* GGUF block_mxfp4: element j is the low nibble of qs[j], element j+16 its
 * high nibble; value = doubled-E2M1 integer * 2^(E-128)
 * (third_party/ggml/src/ggml-quants.c:569-585). The doubled values are
 * integers, so code 8 decodes to +0 here, unlike the signed zero of the
 * checkpoint-layout decoder above. */
static const int8_t e2m1_doubled[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

void orc_mxfp4_gguf_decode(const uint8_t* blocks, size_t nblocks, float* out) {
    for (size_t i = 0; i < nblocks; ++i) {
        const uint8_t* b = blocks + 17 * i;
        for (unsigned j = 0; j < 16; ++j) {
            out[32 * i + j] = (float)ldexp((double)e2m1_doubled[b[1 + j] & 15u], (int)b[0] - 128);
            out[32 * i + j + 16] = (float)ldexp((double)e2m1_doubled[b[1 + j] >> 4], (int)b[0] - 128);
        }
    }
}

float orc_bf16_round(float v) {
    /* Round to nearest even on the upper 16 bits; NaN stays NaN. */
    uint32_t b = float_to_bits(v);
    if ((b & 0x7f800000u) == 0x7f800000u)
        return v;
    b += 0x7fffu + ((b >> 16) & 1u);
    return bits_to_float(b & 0xffff0000u);
}

/* Router of MoeLayer::forward (src/models/text/qwen_layers.cpp:397-424):
 * max-subtracted softmax with a double sum, top-k by probability (ties go to
 * the lower expert index), renormalised by max(sum, 2^-14). */
void orc_moe_route(
    size_t tokens,
    size_t experts,
    size_t top_k,
    const float* logits,
    int32_t* chosen,
    float* weight
) {
    float* p = malloc(experts * sizeof(float));
    char* taken = malloc(experts);
    for (size_t t = 0; t < tokens; ++t) {
        const float* l = logits + t * experts;
        float mx = l[0];
        for (size_t e = 1; e < experts; ++e)
            if (l[e] > mx)
                mx = l[e];
        double total = 0;
        for (size_t e = 0; e < experts; ++e) {
            p[e] = expf(l[e] - mx);
            total += p[e];
        }
        for (size_t e = 0; e < experts; ++e)
            p[e] = (float)(p[e] / total);
        memset(taken, 0, experts);
        float sum = 0;
        for (size_t i = 0; i < top_k; ++i) {
            size_t best = experts;
            for (size_t e = 0; e < experts; ++e)
                if (!taken[e] && (best == experts || p[e] > p[best]))
                    best = e;
            taken[best] = 1;
            chosen[t * top_k + i] = (int32_t)best;
            weight[t * top_k + i] = p[best];
            sum += p[best];
        }
        if (sum < 6.103515625e-5f)
            sum = 6.103515625e-5f;
        for (size_t i = 0; i < top_k; ++i)
            weight[t * top_k + i] /= sum;
    }
    free(p);
    free(taken);
}

/* sum_c decode(w, s)[c] * x[c] in double; each weight is exactly
 * e2m1(code) * 2^(E-127), applied per 32-value block. */
static double mx_dot(const uint8_t* w, const uint8_t* s, size_t cols, const float* x) {
    double acc = 0;
    for (size_t b = 0; b < cols / 32; ++b) {
        const double scale = ldexp(1.0, (int)s[b] - 127);
        double part = 0;
        for (size_t c = 32 * b; c < 32 * b + 32; ++c) {
            const unsigned code = (w[c / 2] >> (4 * (c % 2))) & 15u;
            part += (double)orc_e2m1(code) * (double)x[c];
        }
        acc += part * scale;
    }
    return acc;
}

/* MXFP4 MoE layer. Routing and the selection-order combine follow
 * MoeLayer::forward (qwen_layers.cpp:397-491); the gpt-oss SwiGLU has no
 * counterpart in the reference and follows the public gpt-oss definition. */
int orc_moe_forward(
    size_t tokens,
    size_t hidden,
    size_t inter,
    size_t experts,
    size_t top_k,
    const float* x,
    const float* logits,
    const uint8_t* gu_w,
    const uint8_t* gu_s,
    const float* gu_bias,
    const uint8_t* dn_w,
    const uint8_t* dn_s,
    const float* dn_bias,
    int activation,
    int interleaved,
    float limit,
    float alpha,
    int round_act,
    float* out
) {
    if (hidden % 32 || inter % 32 || !top_k || top_k > experts)
        return -1;
    int32_t* chosen = malloc(tokens * top_k * sizeof(int32_t));
    float* weight = malloc(tokens * top_k * sizeof(float));
    float* act = malloc(inter * sizeof(float));
    double* acc = malloc(hidden * sizeof(double));
    orc_moe_route(tokens, experts, top_k, logits, chosen, weight);
    const size_t gu_row = hidden / 2, gu_srow = hidden / 32;
    const size_t dn_row = inter / 2, dn_srow = inter / 32;
    for (size_t t = 0; t < tokens; ++t) {
        const float* xt = x + t * hidden;
        for (size_t d = 0; d < hidden; ++d)
            acc[d] = 0;
        for (size_t i = 0; i < top_k; ++i) {
            const size_t e = (size_t)chosen[t * top_k + i];
            const uint8_t* gw = gu_w + e * 2 * inter * gu_row;
            const uint8_t* gs = gu_s + e * 2 * inter * gu_srow;
            for (size_t j = 0; j < inter; ++j) {
                const size_t gr = interleaved ? 2 * j : j;
                const size_t ur = interleaved ? 2 * j + 1 : inter + j;
                double g = mx_dot(gw + gr * gu_row, gs + gr * gu_srow, hidden, xt);
                double u = mx_dot(gw + ur * gu_row, gs + ur * gu_srow, hidden, xt);
                if (gu_bias) {
                    g += gu_bias[e * 2 * inter + gr];
                    u += gu_bias[e * 2 * inter + ur];
                }
                float a;
                if (activation == ORC_SWIGLU_OAI) {
                    const double gc = g > limit ? limit : g;
                    const double uc = u > limit ? limit : (u < -limit ? -limit : u);
                    a = (float)(gc / (1.0 + exp(-alpha * gc)) * (uc + 1.0));
                } else {
                    a = (float)(g / (1.0 + exp(-g)) * u);
                }
                act[j] = round_act == 1 ? orc_bf16_round(a) : round_act == 2 ? (float)(_Float16)a : a;
            }
            const uint8_t* dw = dn_w + e * hidden * dn_row;
            const uint8_t* ds = dn_s + e * hidden * dn_srow;
            const double wgt = weight[t * top_k + i];
            for (size_t d = 0; d < hidden; ++d) {
                double v = mx_dot(dw + d * dn_row, ds + d * dn_srow, inter, act);
                if (dn_bias)
                    v += dn_bias[e * hidden + d];
                acc[d] += wgt * v; /* selection order */
            }
        }
        for (size_t d = 0; d < hidden; ++d)
            out[t * hidden + d] = (float)acc[d];
    }
    free(chosen);
    free(weight);
    free(act);
    free(acc);
    return 0;
}
