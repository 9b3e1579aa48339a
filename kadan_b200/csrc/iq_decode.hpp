// The grid-coded GGUF formats IQ3_XXS, IQ2_S and IQ3_S: one value of one
// block, from device code (the dequant and generic GEMV kernels) and from
// host-only C++ (so the same source can be checked against the reference's
// decoder without a GPU).
//
// Each value is d (fp16, widened exactly) times a per-32-value scale, times
// an unsigned magnitude taken from a code grid, times +1 or -1, every product
// rounded on its own as the reference's gguf::decode does
// (services/hikari/inference_worker/include/kadan/gguf_quantization.hpp:674-734).
// The grids themselves (ggml's iq3xxs_grid, iq2s_grid and iq3s_grid) are data
// of the caller's tree, not of this library: the caller registers them with
// kb200_set_iq_grids. The byte layouts are GGUF's and are read as written.
#pragma once

#include <cstdint>
#include <cstring>

#include "gguf_geometry.hpp"

namespace kb200 {

// Code grids: entries pack four (IQ3_XXS, IQ3_S) or eight (IQ2_S) unsigned
// magnitudes, one per byte, lowest byte first.
struct IqGrids {
    const uint32_t* iq3xxs;          // 256 entries
    const unsigned long long* iq2s;  // 1024 entries
    const uint32_t* iq3s;            // 512 entries
};

KB200_HD constexpr bool grid_coded(int e) {
    return e == KB200_IQ3_XXS || e == KB200_IQ2_S || e == KB200_IQ3_S;
}

namespace iq {

KB200_HD inline float float_from_bits(uint32_t bits) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(bits);
#else
    float f;
    std::memcpy(&f, &bits, sizeof f);
    return f;
#endif
}

// binary16 at p (little endian) -> binary32, exact for every pattern.
KB200_HD inline float half_at(const uint8_t* p) {
    const uint32_t h = uint32_t(p[0]) | (uint32_t(p[1]) << 8);
    const uint32_t sign = (h & 0x8000u) << 16, exponent = (h >> 10) & 31u;
    uint32_t fraction = h & 1023u;
    if (exponent == 31)
        return float_from_bits(sign | 0x7f800000u | (fraction << 13));
    if (exponent)
        return float_from_bits(sign | ((exponent + 112u) << 23) | (fraction << 13));
    if (!fraction)
        return float_from_bits(sign);
    // Subnormal: shift the leading one up to bit 10 (at most ten steps).
    uint32_t biased = 113;
    while (!(fraction & 1024u)) {
        fraction <<= 1;
        --biased;
    }
    return float_from_bits(sign | (biased << 23) | ((fraction & 1023u) << 13));
}

// One rounding per operation, never fused.
KB200_HD inline float mul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    volatile float r = a * b;
    return r;
#endif
}

KB200_HD inline float add(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fadd_rn(a, b);
#else
    volatile float r = a + b;
    return r;
#endif
}

KB200_HD inline uint32_t word_at(const uint8_t* p) {
    return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

// magnitude * (+1 or -1) as a product, bit j of `signs` selecting -1.
KB200_HD inline float with_sign(float magnitude, unsigned signs, unsigned j) {
    return mul(magnitude, (signs >> j) & 1u ? -1.0f : 1.0f);
}

// Value `el` (0..255) of one block of encoding `e`; NaN for other encodings.
KB200_HD inline float value(int e, const uint8_t* b, unsigned el, const IqGrids& grids) {
    const unsigned group = el / 32, run = (el % 32) / 8, j = el % 8;
    switch (e) {
    case KB200_IQ3_XXS: {
        // d, 64 grid indices (two per 8-value run), then per group a word:
        // scale nibble on top, four 7-bit sign sets below; each set's eighth
        // sign is its parity bit (an even count of minus signs).
        const uint32_t word = word_at(b + 66 + 4 * group);
        const float scale = mul(mul(half_at(b), add(0.5f, float(word >> 28))), 0.5f);
        uint32_t signs = (word >> (7 * run)) & 127u, parity = signs;
        parity ^= parity >> 4;
        parity ^= parity >> 2;
        parity ^= parity >> 1;
        signs |= (parity & 1u) << 7;
        const uint32_t entry = grids.iq3xxs[b[2 + 8 * group + 2 * run + j / 4]];
        return with_sign(mul(scale, float((entry >> (8 * (j % 4))) & 255u)), signs, j);
    }
    case KB200_IQ2_S: {
        // d, 32 low index bytes (one per run), 32 sign bytes, 8 bytes of
        // two high index bits per run, 8 bytes of two scale nibbles.
        const unsigned nibble = run < 2 ? b[74 + group] & 15u : unsigned(b[74 + group]) >> 4;
        const float scale = mul(mul(half_at(b), add(0.5f, float(nibble))), 0.25f);
        const unsigned index = b[2 + 4 * group + run] | (((unsigned(b[66 + group]) >> (2 * run)) & 3u) << 8);
        const unsigned magnitude = unsigned(grids.iq2s[index] >> (8 * j)) & 255u;
        return with_sign(mul(scale, float(magnitude)), b[34 + 4 * group + run], j);
    }
    case KB200_IQ3_S: {
        // d, 64 low index bytes (two per run), 8 bytes of one high index bit
        // each, 32 sign bytes, 4 bytes of two scale nibbles (scale 1 + 2n).
        const unsigned k = 2 * run + j / 4;
        const unsigned nibble = group & 1u ? unsigned(b[106 + group / 2]) >> 4 : b[106 + group / 2] & 15u;
        const float scale = mul(half_at(b), float(int(1 + 2 * nibble)));
        const unsigned index = b[2 + 8 * group + k] | (((unsigned(b[66 + group]) >> k) & 1u) << 8);
        const unsigned magnitude = (grids.iq3s[index] >> (8 * (j % 4))) & 255u;
        return with_sign(mul(scale, float(magnitude)), b[74 + 4 * group + run], j);
    }
    default:
        return float_from_bits(0x7fc00000u);
    }
}

}  // namespace iq
}  // namespace kb200
