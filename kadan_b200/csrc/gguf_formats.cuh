// GGUF block formats on the device: geometry and the exact per-value decode.
//
// The decode of every value is the reference worker's gguf::decode
// (services/hikari/inference_worker/include/kadan/gguf_quantization.hpp:631-762):
// the fp16 scales are widened exactly and every product/difference is rounded
// on its own (__fmul_rn/__fsub_rn), so results are bit-identical to the
// reference and to ggml's to_float. These byte layouts are GGUF's and must be
// read exactly as written; the arithmetic around them is this file's own.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda_fp16.h>
#include <mutex>

#include "gguf_geometry.hpp"
#include "iq_decode.hpp"
#include "kadan_b200.h"
#include "kb200_host.hpp"

namespace kb200 {

// The caller's IQ code grids (kb200_set_iq_grids), or null before they are set.
const IqGrids* registered_iq_grids();

namespace {

// This translation unit's device copies of the IQ code grids.
__device__ uint32_t iq3xxs_grid_device[256];
__device__ unsigned long long iq2s_grid_device[1024];
__device__ uint32_t iq3s_grid_device[512];

// Before the first launch that decodes a grid-coded encoding on the current
// device: copies the registered grids into this translation unit's arrays
// there (three synchronous copies, once per device). KB200_UNSUPPORTED while
// no grids are registered.
inline int ensure_iq_grids(int encoding) {
    if (!grid_coded(encoding))
        return KB200_OK;
    const IqGrids* grids = registered_iq_grids();
    if (!grids)
        return fail(KB200_UNSUPPORTED, "IQ code grids are not registered (kb200_set_iq_grids)");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64)
        return fail(KB200_UNSUPPORTED, "device index above 63");
    static std::atomic<unsigned long long> uploaded{0};
    const unsigned long long bit = 1ull << dev;
    if (uploaded.load(std::memory_order_acquire) & bit)
        return KB200_OK;
    static std::mutex lock;
    std::lock_guard<std::mutex> guard(lock);
    if (uploaded.load(std::memory_order_relaxed) & bit)
        return KB200_OK;
    e = cudaMemcpyToSymbol(iq3xxs_grid_device, grids->iq3xxs, sizeof(iq3xxs_grid_device));
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbol(iq2s_grid_device, grids->iq2s, sizeof(iq2s_grid_device));
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbol(iq3s_grid_device, grids->iq3s, sizeof(iq3s_grid_device));
    if (e != cudaSuccess)
        return cuda_fail(e, "cudaMemcpyToSymbol (IQ code grids)");
    uploaded.fetch_or(bit, std::memory_order_release);
    return KB200_OK;
}

}  // namespace

// binary16 -> binary32 by integer operations, exact for every pattern
// including subnormals and NaN payloads.
__device__ __forceinline__ float half_exact(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t exponent = (h >> 10) & 31u, fraction = h & 1023u;
    if (exponent == 31)
        return __uint_as_float(sign | 0x7f800000u | (fraction << 13));
    if (exponent)
        return __uint_as_float(sign | ((exponent + 112u) << 23) | (fraction << 13));
    if (!fraction)
        return __uint_as_float(sign);
    // Subnormal: the leading one sits at bit 31 - clz; shift it to bit 10.
    const int lead = 31 - __clz(fraction);
    const uint32_t normal = (fraction << (10 - lead)) & 1023u;
    return __uint_as_float(sign | (uint32_t(103 + lead) << 23) | (normal << 13));
}

__device__ __forceinline__ float half_at(const uint8_t* p) {
    return half_exact(uint32_t(p[0]) | (uint32_t(p[1]) << 8));
}

__device__ __forceinline__ int as_s8(uint32_t b) {
    return int(int8_t(uint8_t(b)));
}

__constant__ const int8_t iq4nl_book[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                            1,    13,   25,  38,  53,  69,  89,  113};

// One value of one block. Grids = true: the grid-coded IQ3_XXS, IQ2_S and
// IQ3_S, in kernel instantiations of their own, so the kernels of the other
// formats compile as if these did not exist.
template <bool Grids = false>
__device__ __forceinline__ float decode_value(int e, const uint8_t* b, unsigned el) {
    if constexpr (Grids)
        return iq::value(e, b, el, IqGrids{iq3xxs_grid_device, iq2s_grid_device, iq3s_grid_device});
    switch (e) {
    case KB200_BF16:
        return __uint_as_float((uint32_t(b[0]) | (uint32_t(b[1]) << 8)) << 16);
    case KB200_Q8_0:
        return __fmul_rn(half_at(b), float(as_s8(b[2 + el])));
    case KB200_Q4_K: {
        // 6-bit scale/min pairs of eight sub-blocks packed into 12 bytes.
        const unsigned g = el / 32, gi = g & 3u;
        const uint8_t* s = b + 4;
        unsigned sc, m;
        if (g < 4) {
            sc = s[gi] & 63u;
            m = s[gi + 4] & 63u;
        } else {
            sc = (s[gi + 8] & 15u) | ((unsigned(s[gi]) >> 6) << 4);
            m = (unsigned(s[gi + 8]) >> 4) | ((unsigned(s[gi + 4]) >> 6) << 4);
        }
        const unsigned packed = b[16 + (el / 64) * 32 + el % 32];
        const unsigned code = (g & 1u) ? packed >> 4 : packed & 15u;
        const float scaled = __fmul_rn(half_at(b), float(sc));
        const float offset = __fmul_rn(half_at(b + 2), float(m));
        return __fsub_rn(__fmul_rn(scaled, float(code)), offset);
    }
    case KB200_Q6_K: {
        const unsigned h = el / 128, o = el % 128, q = o / 32, lane = o % 32;
        const unsigned packed = b[h * 64 + lane + (q & 1u) * 32];
        const unsigned low = q < 2 ? packed & 15u : packed >> 4;
        const unsigned high = (b[128 + h * 32 + lane] >> (2 * q)) & 3u;
        const int code = int(low | (high << 4)) - 32;
        const int scale = as_s8(b[192 + h * 8 + lane / 16 + 2 * q]);
        return __fmul_rn(__fmul_rn(half_at(b + 208), float(scale)), float(code));
    }
    case KB200_Q3_K: {
        const unsigned g = el / 16;
        const uint8_t* s = b + 96;
        const unsigned low = g < 8 ? s[g] & 15u : unsigned(s[g - 8]) >> 4;
        const unsigned high = (s[8 + g % 4] >> (2 * (g / 4))) & 3u;
        const int scale = int(low | (high << 4)) - 32;
        const unsigned lane = el % 32, shift = 2 * ((el % 128) / 32);
        const unsigned two = (b[32 + (el / 128) * 32 + lane] >> shift) & 3u;
        const int code = int(two) - ((b[lane] & (1u << (el / 32))) ? 0 : 4);
        return __fmul_rn(__fmul_rn(half_at(b + 108), float(scale)), float(code));
    }
    case KB200_IQ4_NL: {
        const unsigned packed = b[2 + el % 16];
        return __fmul_rn(half_at(b), float(iq4nl_book[el < 16 ? packed & 15u : packed >> 4]));
    }
    case KB200_IQ4_XS: {
        const unsigned g = el / 32, w = el % 32;
        const unsigned hs = unsigned(b[2]) | (unsigned(b[3]) << 8);
        const int scale =
            int(((b[4 + g / 2] >> (4 * (g % 2))) & 15u) | (((hs >> (2 * g)) & 3u) << 4)) - 32;
        const unsigned packed = b[8 + g * 16 + w % 16];
        return __fmul_rn(
            __fmul_rn(half_at(b), float(scale)), float(iq4nl_book[w < 16 ? packed & 15u : packed >> 4])
        );
    }
    default:
        return __int_as_float(0x7fc00000);
    }
}

}  // namespace kb200
