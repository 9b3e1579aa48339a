// GGUF MXFP4 (ggml type 39) on the device: exact decode and conversion into
// the MXFP4 expert layout the MoE layer reads.
//
// ggml's block_mxfp4 (IW/third_party/ggml/src/ggml-common.h:214-219) is one
// E8M0 byte e and 16 code bytes for 32 values: value j (j < 16) is the low
// nibble of byte j, value j + 16 its high nibble, and a value is
// kvalues_fp4[c] * 2^(e - 128) with the doubled E2M1 table {0, 1, 2, 3, 4, 6,
// 8, 12, 0, -1, ..., -12} (dequantize_row_mxfp4, ggml-quants.c:569-585;
// ggml_e8m0_to_fp32_half, ggml-impl.h:489-500). The checkpoint layout of the
// MoE layer (Shard::load_mxfp4_expert_rows, IW/src/weights/checkpoint.cpp:
// 669-730) holds value 2i in the low nibble and 2i + 1 in the high nibble of
// byte i, with the undoubled table and scale 2^(e - 127): the same value for
// the same code and byte, except that code 8 is -0 there and +0 in ggml, so
// the conversion writes ggml's code 8 as code 0.
#include <cstdint>

#include "kb200_host.hpp"

namespace kb200 {
namespace {

constexpr int kMxBlock = 17;

// 2^(e - 128) as ggml forms it: subnormal for e < 2, exponent e - 1 above.
__device__ __forceinline__ float e8m0_half(uint32_t e) {
    return __uint_as_float(e < 2u ? 0x00200000u << e : (e - 1u) << 23);
}

__device__ __forceinline__ float fp4_doubled(uint32_t c) {
    const float mag[8] = {0.f, 1.f, 2.f, 3.f, 4.f, 6.f, 8.f, 12.f};
    const float m = mag[c & 7u];
    return (c & 8u) && m != 0.f ? -m : m;  // ggml's table has +0 for code 8
}

// One warp per block: lane j writes value j (coalesced 128-byte stores).
__global__ void __launch_bounds__(256) mxfp4_ggml_dequant_kernel(const uint8_t* blocks, size_t count, float* out) {
    const size_t warps = size_t(gridDim.x) * (blockDim.x / 32);
    const uint32_t lane = threadIdx.x & 31u;
    for (size_t b = size_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32; b < count; b += warps) {
        const uint8_t* blk = blocks + b * kMxBlock;
        const uint32_t byte = blk[1 + (lane & 15u)];
        const uint32_t code = lane < 16u ? byte & 15u : byte >> 4;
        out[b * 32 + lane] = __fmul_rn(fp4_doubled(code), e8m0_half(blk[0]));
    }
}

// One thread per block: source block (expert x, row r, block k) of
// [experts][rows][cols/32] becomes code bytes [x][first + r][16 k .. 16 k + 15]
// and scale [x][first + r][k] of the destination's [experts][dst_rows][...].
__global__ void __launch_bounds__(256) mxfp4_from_ggml_kernel(const uint8_t* blocks, size_t experts, size_t rows,
                                                              size_t nblk, uint8_t* codes, uint8_t* scales,
                                                              size_t dst_rows, size_t first) {
    const size_t total = experts * rows * nblk;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const size_t k = i % nblk, r = (i / nblk) % rows, x = i / (nblk * rows);
        const uint8_t* blk = blocks + i * kMxBlock;
        uint32_t q[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            q[j] = blk[1 + j];
            // ggml code 8 (+0) -> code 0 (+0) in either nibble.
            if ((q[j] & 15u) == 8u)
                q[j] &= 0xF0u;
            if ((q[j] >> 4) == 8u)
                q[j] &= 0x0Fu;
        }
        // Checkpoint byte i: values 2i (low) and 2i + 1 (high); values below
        // 16 are ggml's low nibbles, the rest its high nibbles.
        uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2) {
            const uint32_t lo = i2 < 8 ? q[2 * i2] & 15u : q[2 * i2 - 16] >> 4;
            const uint32_t hi = i2 < 8 ? q[2 * i2 + 1] & 15u : q[2 * i2 - 15] >> 4;
            w[i2 / 4] |= (lo | hi << 4) << (8 * (i2 % 4));
        }
        const size_t row = x * dst_rows + first + r;
        *reinterpret_cast<uint4*>(codes + (row * nblk + k) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        scales[row * nblk + k] = blk[0];
    }
}

int grid_for(size_t work, int per_cta) {
    const size_t g = (work + size_t(per_cta) - 1) / size_t(per_cta);
    return int(g < size_t(sm_count()) * 16 ? (g ? g : 1) : size_t(sm_count()) * 16);
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

int kb200_mxfp4_ggml_dequant(const void* blocks, size_t count, float* out, void* stream) {
    if (!count)
        return KB200_OK;
    if (!blocks || !out)
        return fail(KB200_INVALID, "null blocks or output");
    if (overlap(out, count * 32 * sizeof(float), blocks, count * kMxBlock))
        return fail(KB200_ALIAS, "output overlaps the blocks");
    TraceScope trace(KB200_KERNEL_MXFP4_GGML_DEQUANT, static_cast<cudaStream_t>(stream));
    mxfp4_ggml_dequant_kernel<<<grid_for(count, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(blocks), count, out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "mxfp4_ggml_dequant_kernel launch");
}

int kb200_mxfp4_from_ggml(const void* blocks, size_t experts, size_t rows, size_t cols, void* codes, void* scales,
                          size_t dst_rows, size_t first_row, void* stream) {
    if (!experts || !rows)
        return KB200_OK;
    if (!blocks || !codes || !scales)
        return fail(KB200_INVALID, "null blocks, codes or scales");
    if (!cols || cols % 32)
        return fail(KB200_INVALID, "columns must be whole 32-value blocks");
    if (first_row > dst_rows || rows > dst_rows - first_row)
        return fail(KB200_INVALID, "rows beyond the destination's rows per expert");
    if (!aligned(codes, 16))
        return fail(KB200_INVALID, "codes must be 16-byte aligned");
    const size_t nblk = cols / 32, total = experts * rows * nblk;
    const size_t code_bytes = experts * dst_rows * nblk * 16, scale_bytes = experts * dst_rows * nblk;
    if (overlap(codes, code_bytes, blocks, total * kMxBlock) || overlap(scales, scale_bytes, blocks, total * kMxBlock)
        || overlap(codes, code_bytes, scales, scale_bytes))
        return fail(KB200_ALIAS, "source and destinations overlap");
    TraceScope trace(KB200_KERNEL_MXFP4_FROM_GGML, static_cast<cudaStream_t>(stream));
    mxfp4_from_ggml_kernel<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(blocks), experts, rows, nblk, static_cast<uint8_t*>(codes),
        static_cast<uint8_t*>(scales), dst_rows, first_row);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "mxfp4_from_ggml_kernel launch");
}

}  // extern "C"
