/* Test infrastructure only: a plain-C restatement of the reference worker's
 * quantized-linear arithmetic, used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py as the CHECKER of the CUDA path. Nothing in the
 * kadan_b200 product links, loads or calls this library.
 *
 * Encoding numbers follow kadan::gguf::Encoding
 * (services/hikari/inference_worker/include/kadan/gguf_quantization.hpp:16-27).
 */
#ifndef KADAN_ORACLE_H
#define KADAN_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum orc_encoding {
    ORC_Q3_K = 0,
    ORC_Q4_K = 1,
    ORC_Q8_0 = 2,
    ORC_Q6_K = 3,
    ORC_IQ3_XXS = 4,
    ORC_IQ4_NL = 5,
    ORC_IQ4_XS = 6,
    ORC_IQ2_S = 7,
    ORC_IQ3_S = 8,
    ORC_BF16 = 9
};

float orc_half(uint16_t bits);
size_t orc_block_values(int encoding);
size_t orc_block_bytes(int encoding);
float orc_decode(int encoding, const uint8_t* block, size_t element);
/* The IQ3_XXS, IQ2_S and IQ3_S code grids (256, 1024 and 512 entries; ggml's
 * iq3xxs_grid, iq2s_grid and iq3s_grid, the reference's
 * gguf_quantization.hpp:99-495), copied; until set, those encodings decode to NaN. */
void orc_set_iq_grids(const uint32_t* iq3xxs, const uint64_t* iq2s, const uint32_t* iq3s);
void orc_decode_stream(int encoding, const uint8_t* packed, size_t count, float* out);

/* y[r*y_stride + c] = sum_k decode(W[c,k]) * x[r*in + k], double accumulation. */
void orc_gemv_f64(
    int encoding,
    const uint8_t* weights,
    size_t row_bytes,
    size_t in,
    size_t out,
    const float* x,
    size_t rows,
    double* y,
    size_t y_stride
);

/* MXFP4, safetensors expert layout: weights [rows, cols/2] low nibble first,
 * scales [rows, cols/32] E8M0 (255 invalid). */
float orc_e2m1(unsigned code);
int orc_mxfp4_decode_rows(
    size_t rows,
    size_t cols,
    const uint8_t* weights,
    const uint8_t* scales,
    size_t first,
    size_t count,
    float* out
);
/* GGUF block_mxfp4 (17-byte blocks: E8M0 then 16 code bytes). */
void orc_mxfp4_gguf_decode(const uint8_t* blocks, size_t nblocks, float* out);

/* Softmax router, top-k, renormalize (MoeLayer::forward semantics). */
void orc_moe_route(
    size_t tokens,
    size_t experts,
    size_t top_k,
    const float* logits,
    int32_t* chosen,
    float* weight
);

enum orc_moe_activation {
    ORC_SWIGLU_OAI = 0,   /* gate<=limit, up in [-limit,limit], gate*sigmoid(alpha*gate)*(up+1) */
    ORC_SILU_MUL = 1      /* silu(gate)*up (the reference's MoeLayer) */
};

/* Full MXFP4 MoE layer. gate_up rows: 2*inter per expert; with interleaved=1
 * gate is row 2i and up row 2i+1, else gate rows [0,inter) and up [inter,2inter).
 * gu_bias [E,2*inter] and down_bias [E,hidden] may be NULL. round_act rounds
 * the activation fed to the down projection: 0 no, 1 to bf16, 2 to fp16. */
int orc_moe_forward(
    size_t tokens,
    size_t hidden,
    size_t inter,
    size_t experts,
    size_t top_k,
    const float* x,
    const float* logits,
    const uint8_t* gu_weights,
    const uint8_t* gu_scales,
    const float* gu_bias,
    const uint8_t* down_weights,
    const uint8_t* down_scales,
    const float* down_bias,
    int activation,
    int interleaved,
    float limit,
    float alpha,
    int round_act,
    float* out
);

float orc_bf16_round(float v);

/* Layer math around the path (layer.c): the reference worker's host RMSNorm,
 * L2 norm, RoPE, cached attention and gated delta-net step. */
int orc_rms_norm(float* x, const float* weight, size_t rows, size_t width, float eps);
void orc_l2_norm(float* x, size_t rows, size_t width, float eps);
void orc_rope(float* x, size_t rows, size_t row_width, size_t width, size_t rotary, size_t position, float base);
int orc_attend_cached(const float* q, const float* keys, const float* values, size_t rows, size_t position,
                      size_t heads, size_t kv_heads, size_t dim, float scale, const uint32_t* selected,
                      const uint32_t* offsets, float* out);
void orc_silu_mul(const float* gate, const float* up, size_t n, float* out);
void orc_moe_add_shared(const float* x, const float* shared_gate, const float* down, size_t tokens, size_t hidden,
                        float* out);
void orc_delta_rule(float* state, const float* q, const float* k, const float* v, const float* decay, size_t decays,
                    float beta, size_t dim, float* out);
int orc_delta_step(const float* qkv, const float* z, const float* alpha, const float* beta, const float* conv,
                   const float* dt, const float* a, const float* norm, size_t rows, size_t key_heads,
                   size_t value_heads, size_t dim, size_t kernel, float eps, int sigmoid_gate, float* history,
                   float* state, float* out);

#ifdef __cplusplus
}
#endif
#endif
