// GGUF block geometry (values and bytes per block) of the encodings the
// library knows, usable from host-only C++ and from device code. The sizes are
// the GGUF format's (the reference's gguf::block_values / block_bytes,
// services/hikari/inference_worker/include/kadan/gguf_quantization.hpp:64-90).
#pragma once

#include "kadan_b200.h"

#if defined(__CUDACC__)
#define KB200_HD __host__ __device__
#else
#define KB200_HD
#endif

namespace kb200 {

KB200_HD constexpr int block_values(int e) {
    return e == KB200_BF16 ? 1 : (e == KB200_Q8_0 || e == KB200_IQ4_NL) ? 32 : e == KB200_F32 ? 1 : 256;
}

KB200_HD constexpr int block_bytes(int e) {
    switch (e) {
    case KB200_Q3_K: return 110;
    case KB200_Q4_K: return 144;
    case KB200_Q8_0: return 34;
    case KB200_Q6_K: return 210;
    case KB200_IQ4_NL: return 18;
    case KB200_IQ4_XS: return 136;
    case KB200_IQ3_XXS: return 98;  // decoded once the caller registers the code grids
    case KB200_IQ2_S: return 82;
    case KB200_IQ3_S: return 110;
    case KB200_BF16: return 2;
    case KB200_F32: return 4;
    default: return 0;
    }
}

// Encodings GGUF geometry is known for (the reference's gguf::supported set).
KB200_HD constexpr bool gguf_geometry(int e) {
    return e >= KB200_Q3_K && e <= KB200_BF16;
}

// Encodings with a device decoder here that needs no caller data (the
// grid-coded IQ3_XXS, IQ2_S and IQ3_S also decode once their grids are
// registered: kb200_encoding_supported).
KB200_HD constexpr bool decodable(int e) {
    return e == KB200_Q3_K || e == KB200_Q4_K || e == KB200_Q8_0 || e == KB200_Q6_K || e == KB200_IQ4_NL
           || e == KB200_IQ4_XS || e == KB200_BF16;
}

}  // namespace kb200
