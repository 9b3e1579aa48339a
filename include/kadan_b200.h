/* kadan_b200 — B200 (sm_100a) quantized-weight linear path, C ABI.
 *
 * This is the drop-in boundary under the Hikari inference worker's
 * kadan::DenseCompute operator interface
 * (services/hikari/inference_worker/include/kadan/dense_compute.hpp:60-342 in
 * ghalrym/Kadan; "IW/" below abbreviates services/hikari/inference_worker/).
 * Every entry point takes plain pointers and sizes, returns a kb200_status,
 * throws nothing, and is asynchronous on the given CUDA stream unless it says
 * otherwise. Pointers marked "device" must address memory of the current
 * CUDA device. A DenseCompute subclass in the worker maps these status codes
 * back onto the reference's ProjectionResult / std::runtime_error conventions.
 */
#ifndef KADAN_B200_H
#define KADAN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KB200_API __attribute__((visibility("default")))
#else
#define KB200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The reference throws std::runtime_error with "h3_cuda_*"
 * messages for the execution failures (IW/src/cuda/h3_compute.cu:34-51);
 * kb200_status_name() returns the matching message text. */
typedef enum kb200_status {
    KB200_OK = 0,
    KB200_UNSUPPORTED = 1,       /* ProjectionResult::unsupported: nothing read or written */
    KB200_INVALID = 2,           /* bad shape/pointer/alignment argument */
    KB200_CUDA = 3,              /* a CUDA runtime call failed ("h3_cuda: ...") */
    KB200_NONFINITE_WEIGHT = 4,  /* "h3_cuda_nonfinite_weight" */
    KB200_NONFINITE_INPUT = 5,   /* "h3_cuda_nonfinite_input" */
    KB200_ALIAS = 6,             /* "h3_cuda_alias": output overlaps an input */
    KB200_CANCELLED = 7,         /* "h3_cuda_cancelled" */
    KB200_TIMEOUT = 8,           /* a bounded device-side wait ran out */
    KB200_NO_MEMORY = 9,
    KB200_QUARANTINED = 10,      /* "weight_cleanup_unconfirmed": a weight bank's cleanup failed */
    KB200_IO = 11,               /* a checkpoint file could not be opened or read */
    KB200_NONFINITE_BIAS = 12,   /* "h3_cuda_nonfinite_bias" */
    KB200_NONFINITE_OUTPUT = 13  /* "h3_cuda_nonfinite_output" */
} kb200_status;

/* Weight encodings: the numbering of kadan::gguf::Encoding
 * (IW/include/kadan/gguf_quantization.hpp:16-27), plus F32 rows, which the
 * reference expresses as an empty std::optional<gguf::Encoding>. */
typedef enum kb200_encoding {
    KB200_F32 = -1,
    KB200_Q3_K = 0,
    KB200_Q4_K = 1,
    KB200_Q8_0 = 2,
    KB200_Q6_K = 3,
    KB200_IQ3_XXS = 4,
    KB200_IQ4_NL = 5,
    KB200_IQ4_XS = 6,
    KB200_IQ2_S = 7,
    KB200_IQ3_S = 8,
    KB200_BF16 = 9
} kb200_encoding;

/* Input rows one packed GEMV pass reduces, and the most rows a batch job may
 * carry: DenseCompute::gguf_batch_rows / gguf_batch_max_rows
 * (IW/include/kadan/dense_compute.hpp:197-201). */
#define KB200_BATCH_ROWS 8
#define KB200_BATCH_MAX_ROWS 4096

KB200_API const char* kb200_status_name(int status);
/* Text of the last failure on the calling thread. */
KB200_API const char* kb200_last_error(void);
KB200_API int kb200_version(void);
/* 1 if `encoding` has a device decoder (gguf::supported, gguf_quantization.hpp:57-63):
 * IQ3_XXS, IQ2_S and IQ3_S only once their code grids are registered. */
KB200_API int kb200_encoding_supported(int encoding);
/* Registers the code grids of IQ3_XXS, IQ2_S and IQ3_S (copied): 256, 1024 and
 * 512 entries, ggml's iq3xxs_grid, iq2s_grid and iq3s_grid, which the worker
 * holds as kadan::gguf::detail::iq3xxs_grid_host, iq2s_grid_host and
 * iq3s_grid_host (IW/include/kadan/gguf_quantization.hpp:501-504). Until this
 * call those encodings are unsupported. Registering the same grids again is a
 * no-op; other values fail with KB200_INVALID. The first dequant or GEMV of
 * one of these encodings on a device copies the grids to it synchronously
 * (once per device), so make that first call outside any stream capture. */
KB200_API int kb200_set_iq_grids(const uint32_t* iq3xxs_grid, const uint64_t* iq2s_grid, const uint32_t* iq3s_grid);
KB200_API size_t kb200_block_values(int encoding);
KB200_API size_t kb200_block_bytes(int encoding);

/* ---------------------------------------------------------------------------
 * Dequantisation. Replaces gguf_decode_kernel (IW/src/cuda/h3_compute.cu:76-95):
 * out[i] = gguf::decode(encoding, packed + i/values*bytes, i%values) for
 * i < count, bit-exact, with *status |= 1 when a decoded value is not finite.
 * packed, out: device. status: device or NULL. */
KB200_API int kb200_gguf_dequant(
    int encoding,
    const void* packed,
    size_t count,
    float* out,
    unsigned* status,
    void* stream
);

/* ---------------------------------------------------------------------------
 * Packed GEMV. One job is the reference's MatvecJob (h3_compute.cu:110-121):
 *   output[r*stride + c] = sum_k decode(W[c,k]) * input[r*in + k]
 * for r < rows, c < columns; W has `columns` packed rows of row_bytes each.
 * status: device word or NULL; bit 0 is set when a decoded weight of the job
 * is not finite (NULL skips the check, as for bank-validated chunks). */
typedef struct kb200_gemv_job {
    const void* weights; /* device */
    const float* input;  /* device, rows * in floats */
    float* output;       /* device */
    unsigned* status;    /* device or NULL */
    size_t row_bytes;
    size_t stride;
    uint32_t in;
    uint32_t columns;
    uint32_t rows;
    int32_t encoding; /* kb200_encoding */
} kb200_gemv_job;

/* Every job of the batch, one launch per encoding: the job table travels in
 * the launch parameters. Replaces plan_matvec + launch_matvec +
 * gguf_matvec_batch_kernel (h3_compute.cu:243-257, :325-382) and, for one job,
 * gguf_matvec_kernel (:238-240, :294-307). Rows above KB200_BATCH_ROWS are
 * processed as successive groups of rows, as append_row_groups does (:311-319).
 * jobs: host array. The Q4_K kernel splits large launches evenly over its
 * CTAs and keeps, per (device, stream), a small device buffer for the tiles
 * it cuts (allocated by the first call on the stream outside graph capture;
 * inside capture without one it deals whole tiles instead). Launches on one
 * stream share it in stream order; a graph captured on a stream must not be
 * replayed concurrently with other work of that stream's Q4_K launches. */
KB200_API int kb200_gguf_gemv_batch(const kb200_gemv_job* jobs, size_t count, void* stream);

/* Which kernel kb200_gguf_gemv_batch selects for a job: 2 = tensor-pipe Q4_K
 * kernel (TMA tiles + mma.sync), 1 = bulk-copy staged CUDA-core kernel,
 * 0 = generic kernel (unaligned rows), -1 = unsupported. */
KB200_API int kb200_gemv_path(const kb200_gemv_job* job);

/* Prefill projection of many input rows on the tensor cores: the reference
 * decodes the packed chunk to an fp32 tile in scratch and runs an FP32
 * cublasSgemm (Compute::project, h3_compute.cu:1781-2480; decode :2201-2218,
 * SGEMM :2435-2468). Here: Y[t, n] = sum_k decode(W[n, k]) * X[t, k] for all
 * job.rows input rows in one pass over the weights, decoded in shared memory
 * to fp16 operands (each input row scaled by a power of two first, undone
 * exactly on output) with fp32 accumulation. Q4_K, Q6_K and Q8_0
 * (KB200_UNSUPPORTED otherwise, or when kb200_gguf_gemm_supported is 0);
 * `workspace`: device, 256-byte aligned, at least
 * kb200_gguf_gemm_workspace_bytes(rows, in). Asynchronous on `stream`.
 * job.status (optional) receives bit 0 (1) when a decoded weight is not finite
 * and bit 1 (2) when a block's scales could put a weight beyond the fp16
 * operand range (|w| > 65504): that job's outputs are then not valid and the
 * GEMV path (kb200_gguf_gemv_batch) must compute it. The same condition sets
 * the 32-bit word at workspace + kb200_gguf_gemm_range_offset(rows, in),
 * cleared by every call. */
KB200_API size_t kb200_gguf_gemm_workspace_bytes(uint32_t rows, uint32_t in);
KB200_API size_t kb200_gguf_gemm_range_offset(uint32_t rows, uint32_t in);
/* 1 when the GEMM takes the job's weights: one of its encodings, job.in a
 * multiple of 256, 16-byte aligned weights, row_bytes a multiple of 16 (Q6_K
 * rows of K values are 210 K / 256 bytes: a multiple of 16 when K is a
 * multiple of 2048). */
KB200_API int kb200_gguf_gemm_supported(const kb200_gemv_job* job);
KB200_API int kb200_gguf_gemm(const kb200_gemv_job* job, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Multi-device column partition (host only). The reference splits every
 * projection's output columns across devices in proportion to their weight
 * capacity and chunks each device's slice as a single projection on that
 * device would (weight_boundary, IW/include/kadan/device_placement.hpp:341-357;
 * gguf_batch_partition, IW/include/kadan/gguf_batch_partition.hpp:44-83, with
 * the plans of device_placement.hpp:76-142); these return the same geometry.
 * encoding: kb200_encoding, KB200_F32 for fp32 rows. Failures are the
 * reference's std::invalid_argument cases (KB200_INVALID with its message). */
typedef struct kb200_partition {
    size_t first, count, chunk_columns;
} kb200_partition;

KB200_API size_t kb200_weight_boundary(size_t units, const uint64_t* capacities, size_t devices, size_t index);
KB200_API int kb200_gguf_batch_partition(size_t in, size_t out, int encoding, const uint64_t* capacities,
                                         size_t devices, size_t device, uint64_t scratch_limit,
                                         kb200_partition* result);
/* output[r*out + first + c] = local[r*count + c] for r < rows, c < count
 * (GgufBatchPartition::scatter, gguf_batch_partition.hpp:53-66). */
KB200_API void kb200_partition_scatter(const kb200_partition* partition, const float* local, size_t rows,
                                       float* output, size_t out);

/* ---------------------------------------------------------------------------
 * Host-span boundary. A context owns one device, one CUDA stream, a device
 * workspace and pinned staging that grow on demand; calls on one context must
 * not overlap (the reference serialises DenseCompute with a mutex,
 * IW/src/cuda/h3_compute.cu:1639). */
typedef struct kb200_context kb200_context;

KB200_API int kb200_context_create(int device, kb200_context** out);
KB200_API void kb200_context_destroy(kb200_context* ctx);
/* The context's cudaStream_t. */
KB200_API void* kb200_context_stream(kb200_context* ctx);
/* Host threads that read packed-row sources in kb200_dense_gguf_source_batch,
 * the caller included (1..64; default 4, the reference's PackedReadTeam of
 * three workers and the caller, IW/include/kadan/packed_read_team.hpp:22-275).
 * Sources may then run concurrently on disjoint rows. */
KB200_API int kb200_context_set_read_lanes(kb200_context* ctx, int lanes);

/* Work the context's calls have issued so far (cumulative; for tests and
 * telemetry). A projection of more than KB200_BATCH_ROWS input rows runs on
 * the tensor-core GEMM when kb200_gguf_gemm_supported takes its weights (one
 * GEMM launch per job or bank/staging chunk: the reference's switch from the
 * batched GEMV to decode + GEMM, h3_compute.cu:1863-1865); everything else
 * runs as GEMV batches. gemm_fallbacks counts GEMM jobs recomputed on the GEMV
 * path because a block's scales could exceed the fp16 operand range. */
typedef struct kb200_context_counters {
    uint64_t calls;          /* kb200_dense_gguf_batch / _source_batch calls that reached the device */
    uint64_t gemm_launches;  /* kb200_gguf_gemm launches */
    uint64_t gemv_batches;   /* kb200_gguf_gemv_batch calls (one launch per encoding each) */
    uint64_t gemm_fallbacks; /* GEMM jobs recomputed on the GEMV path */
} kb200_context_counters;
KB200_API int kb200_context_counters_get(kb200_context* ctx, kb200_context_counters* out);

/* Caller-managed device-resident packed rows for kb200_dense_gguf_batch: a
 * synchronous upload of `bytes` host bytes into a 256-byte aligned device
 * allocation. (kb200_bank_* keeps resident rows with the reference's
 * DeviceWeights rules instead; kb200_dense_gguf_source_batch uses it.) */
KB200_API int kb200_weights_upload(kb200_context* ctx, const void* host, size_t bytes, void** device);
KB200_API int kb200_weights_free(kb200_context* ctx, void* device);

/* One projection of DenseCompute::GgufBatchJob
 * (IW/include/kadan/dense_compute.hpp:205-213) over resident weights. */
typedef struct kb200_host_job {
    const void* weights; /* device (from kb200_weights_upload or any device buffer) */
    const float* input;  /* host, rows * in floats */
    float* output;       /* host, rows * out floats */
    size_t row_bytes;
    uint32_t in;
    uint32_t out;
    uint32_t rows;
    int32_t encoding;  /* kb200_encoding */
    int32_t validated; /* 1: these weights were already checked finite */
} kb200_host_job;

/* Result codes of kb200_dense_gguf_batch: ProjectionResult
 * (IW/include/kadan/dense_compute.hpp:44-48). */
#define KB200_RESULT_UNSUPPORTED 0
#define KB200_RESULT_UNVALIDATED 1
#define KB200_RESULT_FINITE 2

/* DenseCompute::dense_gguf_batch (IW/src/cuda/h3_compute.cu:3963-4375):
 * synchronous. A cancel byte already set fails the call with KB200_CANCELLED
 * first; then an empty batch or any unsupported job returns KB200_UNSUPPORTED
 * (result UNSUPPORTED) before any read or write; identical input spans upload once;
 * non-finite inputs fail with KB200_NONFINITE_INPUT, outputs overlapping any
 * input with KB200_ALIAS; then one input upload, one launch per encoding, one
 * download of outputs plus the weight status word, and KB200_NONFINITE_WEIGHT
 * when an unvalidated weight decoded non-finite. *cancel (may be NULL) is
 * polled between stages (KB200_CANCELLED).
 *
 * Every `cancel` of this ABI is one byte, nonzero once the call should stop:
 * the storage of the worker's std::atomic_bool (lock-free and one byte on its
 * platforms) can be passed as is. */
KB200_API int kb200_dense_gguf_batch(
    kb200_context* ctx,
    const kb200_host_job* jobs,
    size_t count,
    const volatile uint8_t* cancel,
    int* result
);

/* ---------------------------------------------------------------------------
 * MXFP4 mixture-of-experts layer (gpt-oss style), device pointers.
 *
 * The reference has no device path for this layer: its MoE semantics are
 * MoeLayer::forward (IW/src/models/text/qwen_layers.cpp:378-492: softmax
 * router, top-k, renormalise by max(sum, 2^-14), per-expert gather,
 * gate/up, activation, down, weighted sum in selection order) and its MXFP4
 * format is kadan::quantization (IW/src/weights/quantization.cpp:79-99) with
 * the expert-row layout of Shard::load_mxfp4_expert_rows
 * (IW/src/weights/checkpoint.cpp:669-730):
 *   blocks [E, rows, cols/32, 16] (low nibble first), scales [E, rows, cols/32]
 *   E8M0, value = e2m1(code) * 2^(scale - 127).
 * Expert weights are used in fp16 on the tensor cores, exact for scale bytes
 * 104..140; kb200_moe_forward flags others in *status (bit 1). */
#define KB200_MOE_SWIGLU_OAI 0 /* gate<=limit, up in [-limit,limit], gate*sigmoid(alpha*gate)*(up+1) */
#define KB200_MOE_SILU 1       /* silu(gate) * up (the reference MoeLayer) */

typedef struct kb200_moe_weights {
    const uint8_t* gate_up_blocks; /* device [E, 2*inter, hidden/2] */
    const uint8_t* gate_up_scales; /* device [E, 2*inter, hidden/32] */
    const float* gate_up_bias;     /* device [E, 2*inter] or NULL */
    const uint8_t* down_blocks;    /* device [E, hidden, inter/2] */
    const uint8_t* down_scales;    /* device [E, hidden, inter/32] */
    const float* down_bias;        /* device [E, hidden] or NULL */
    int32_t hidden, inter, experts, top_k;
    int32_t activation;  /* KB200_MOE_* */
    int32_t interleaved; /* 1: gate = row 2i, up = row 2i+1; 0: gate rows [0,inter), up [inter,2*inter) */
    float limit, alpha;
} kb200_moe_weights;

/* GGUF MXFP4 (ggml type 39, block_mxfp4: IW/third_party/ggml/src/ggml-common.h:
 * 214-219): one E8M0 byte e and 16 code bytes per 32 values; value j < 16 is
 * the low nibble of byte j, value j + 16 its high nibble; value =
 * kvalues_fp4[c] * 2^(e - 128) (dequantize_row_mxfp4, ggml-quants.c:569-585).
 * The reference decodes it on the host only (ggml-cpu); these put it on the
 * device. Pointers are device memory; asynchronous on `stream`. */
#define KB200_MXFP4_GGML_BLOCK_BYTES 17
/* out[32 count] = the values of `count` consecutive blocks, bit for bit as
 * ggml's dequantize_row_mxfp4 gives them. */
KB200_API int kb200_mxfp4_ggml_dequant(const void* blocks, size_t count, float* out, void* stream);
/* GGUF MXFP4 rows [experts][rows][cols/32 blocks] (a GGUF expert tensor such
 * as ffn_gate_exps, or one matrix with experts = 1) into the MXFP4 expert
 * layout of kb200_moe_weights: rows [first_row, first_row + rows) of each
 * expert of codes [experts][dst_rows][cols/2] (16-byte aligned) and E8M0
 * scales [experts][dst_rows][cols/32]. Same values (ggml's code 8, +0, is
 * written as code 0; the expert layout's code 8 is -0); scale bytes are kept,
 * so kb200_moe_forward's scale-range flag applies to them. Separate gate and
 * up tensors go to first_row 0 and `inter` of a gate_up destination of
 * dst_rows = 2 * inter, used with interleaved = 0. */
KB200_API int kb200_mxfp4_from_ggml(const void* blocks, size_t experts, size_t rows, size_t cols, void* codes,
                                    void* scales, size_t dst_rows, size_t first_row, void* stream);

/* Device scratch that kb200_moe_forward needs for `tokens` input rows. */
KB200_API size_t kb200_moe_workspace_bytes(const kb200_moe_weights* w, size_t tokens);

/* out[t, :] = sum_i weight[t,i] * down_e(act(gate_up_e(x[t]))) for the top_k
 * experts e of logits[t] (fp32 [tokens, experts]); x is bf16 [tokens, hidden],
 * out fp32 [tokens, hidden]. workspace: device, at least
 * kb200_moe_workspace_bytes. status: device word or NULL (bit 1: a scale byte
 * outside 104..140; bit 2: an activation outside the fp16 range). Calls that
 * overlap on one workspace race. */
KB200_API int kb200_moe_forward(
    const kb200_moe_weights* w,
    const uint16_t* x_bf16,
    const float* logits,
    size_t tokens,
    float* out,
    void* workspace,
    size_t workspace_bytes,
    unsigned* status,
    void* stream
);

/* kb200_moe_forward over fp32 token rows x [tokens, hidden] (device), each
 * value rounded once to the fp16 operand (status bit 2 when beyond its range). */
KB200_API int kb200_moe_forward_f32(const kb200_moe_weights* w, const float* x, const float* logits, size_t tokens,
                                    float* out, void* workspace, size_t workspace_bytes, unsigned* status,
                                    void* stream);

/* The MoE layer with host spans on a context, synchronous, in the
 * conventions of DenseCompute::dense_gguf_batch (IW/include/kadan/
 * dense_compute.hpp:215-221): x fp32 [tokens, hidden] and router logits fp32
 * [tokens, experts] on the host, out fp32 [tokens, hidden] on the host; the
 * weights stay device-resident (kb200_moe_weights). KB200_UNSUPPORTED (and
 * *result KB200_RESULT_UNSUPPORTED) with nothing of `out` written when the
 * call is outside the layer's contract or when the weights' scales or the
 * activations fall outside what the fp16 operands hold exactly: the caller's
 * host path then takes the layer (MoeLayer::forward, IW/src/models/text/
 * qwen_layers.cpp:378-492). Non-finite inputs fail with
 * KB200_NONFINITE_INPUT before any device work, a non-finite output with
 * KB200_NONFINITE_OUTPUT; on success *result is KB200_RESULT_FINITE. */
KB200_API int kb200_moe_forward_host(kb200_context* ctx, const kb200_moe_weights* w, const float* x,
                                     const float* logits, size_t tokens, float* out, const volatile uint8_t* cancel,
                                     int* result);

/* kb200_moe_forward without a caller workspace and without any allocation.
 * No counterpart in the reference: it exists for callers that cannot
 * allocate device memory per call — workers whose device memory is fully
 * admitted to a budget ledger before use, as the Hikari worker's resource
 * accounting does, so an unplanned cudaMalloc would break their accounting,
 * and callers that must not stall other streams (cudaMalloc and cudaFree can
 * synchronise the whole device). The scratch is one file-scope
 * device array of KB200_MOE_STATIC_SCRATCH_BYTES (16 MiB) that every GPU
 * loading the library holds until the process exits; calls whose
 * kb200_moe_workspace_bytes exceeds it fail with KB200_NO_MEMORY before any
 * work. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress), so make that first call before any stream capture.
 * All calls on a device share the array and its contents persist between
 * calls: calls that overlap on the GPU (other streams, other threads) race
 * and must be serialised by the caller. */
#define KB200_MOE_STATIC_SCRATCH_BYTES (16u << 20)
KB200_API int kb200_moe_forward_noalloc(
    const kb200_moe_weights* w,
    const uint16_t* x_bf16,
    const float* logits,
    size_t tokens,
    float* out,
    unsigned* status,
    void* stream
);

/* ---------------------------------------------------------------------------
 * The MoE layer in stages, for expert parallelism: experts split over the
 * ranks of a node, tokens sent to the rank that holds their expert and back
 * (an all-to-all each way, issued by the caller between the stages).
 * kb200_moe_forward == dispatch_rows -> experts -> combine on one device.
 *
 * Dispatch: route each token (the steps of MoeLayer::forward,
 * qwen_layers.cpp:397-431), sort the tokens * top_k (token, choice) slots
 * stably by expert and gather their rows as fp16 into expert-major order.
 * The result points into `workspace` (at least
 * kb200_moe_dispatch_workspace_bytes): rows of expert e are
 * [offsets[e], offsets[e+1]); pos[t * top_k + i] is the row of choice i of
 * token t; weight the renormalised routing weights. Experts are contiguous
 * per rank, so rank r's rows are one contiguous range. */
typedef struct kb200_moe_dispatch {
    int32_t* offsets; /* device [experts + 1] */
    int32_t* pos;     /* device [tokens * top_k] */
    float* weight;    /* device [tokens * top_k] */
    uint16_t* rows;   /* device fp16 [tokens * top_k, hidden] */
    size_t count;     /* tokens * top_k */
} kb200_moe_dispatch;

KB200_API size_t kb200_moe_dispatch_workspace_bytes(size_t tokens, int32_t hidden, int32_t experts, int32_t top_k);
KB200_API int kb200_moe_dispatch_rows(
    const float* logits, const uint16_t* x_bf16, size_t tokens, int32_t hidden, int32_t experts, int32_t top_k,
    void* workspace, size_t workspace_bytes, kb200_moe_dispatch* result, unsigned* status, void* stream
);

/* Expert stage: y[r] = down_e(act(gate_up_e(rows[r]))) for rows grouped by
 * expert, offsets device [w->experts + 1] (w describes the experts this
 * device holds; its top_k is not used). rows fp16 [rows, hidden], y fp32
 * [rows, hidden], workspace at least kb200_moe_experts_workspace_bytes. */
KB200_API size_t kb200_moe_experts_workspace_bytes(const kb200_moe_weights* w, size_t rows);
KB200_API int kb200_moe_experts(
    const kb200_moe_weights* w, const uint16_t* rows_f16, const int32_t* offsets, size_t rows, float* y,
    void* workspace, size_t workspace_bytes, unsigned* status, void* stream
);

/* Combine: out[t] = sum_i weight[t, i] * y[pos[t, i]] in selection order
 * (qwen_layers.cpp:466-491), fp32. */
KB200_API int kb200_moe_combine(
    const float* y, const float* weight, const int32_t* pos, size_t tokens, int32_t top_k, int32_t hidden,
    float* out, void* stream
);

/* The reference MoE's sigmoid-gated shared expert (MoeLayer::forward,
 * IW/src/models/text/qwen_layers.cpp:383-396, :477-490): a dense FFN beside
 * the routed experts whose gate/up/down projections are ordinary GGUF
 * matrices (kb200_gguf_gemv_batch / kb200_gguf_gemm or the host-span batch).
 * kb200_silu_mul: out[j] = silu(gate[j]) * up[j] (the activation between its
 * gate/up and down projections, :390-395), n values; out may equal gate.
 * kb200_moe_add_shared: per token t, out[t][d] += down[t][d] *
 * sigmoid(sum_c shared_gate[c] * x[t][c]) (:477-490); x [tokens][hidden]
 * fp32, shared_gate [hidden], down and out [tokens][hidden]. Applied to
 * kb200_moe_forward's output this gives the reference layer's output. */
KB200_API int kb200_silu_mul(const float* gate, const float* up, size_t n, float* out, void* stream);
KB200_API int kb200_moe_add_shared(const float* x, const float* shared_gate, const float* down, size_t tokens,
                                   size_t hidden, float* out, void* stream);

/* Row permutation by segments: dst rows [d, d+n) = src rows [s, s+n) for
 * each {s, d, n} of `segments` (device int64 [count][3]); row_bytes a
 * multiple of 16; max_rows the longest segment (sizes the grid). Used to
 * regroup rows received from each rank (source-major) into expert-major
 * order and back. */
KB200_API int kb200_rows_regroup(const void* src, void* dst, size_t row_bytes, const int64_t* segments, size_t count,
                                 size_t max_rows, void* stream);

/* ---------------------------------------------------------------------------
 * Peer-memory all-reduce for tensor parallelism (one process per GPU).
 *
 * The reference adds nothing across devices: its column slices are gathered
 * on the host (gguf_batch_partition.hpp:48-59). Row-parallel projections
 * here leave each GPU a partial sum of the whole output, which
 * kb200_peer_allreduce_f32 adds over the ranks in one kernel: every rank
 * stores its values, each tagged with the call's epoch in one 64-bit word,
 * into every peer's buffer over NVLink, reads the peers' words for the same
 * elements until their tags match (bounded by timeout_s) and sums in rank
 * order, so all ranks hold the same bits. count: even; data 8-byte aligned.
 *
 * Setup: each rank allocates kb200_peer_buffer_bytes(world, max_count) with
 * kb200_device_alloc (zeroed), exports it with kb200_ipc_handle, sends the
 * handle to the others, opens theirs with kb200_ipc_open and passes all
 * buffer addresses (its own at [rank]) as `peers`. Every rank must make the
 * same sequence of calls. A wait that runs out sets bit 16 of the device
 * watchdog word (kb200_take_device_error) and leaves data unreduced. */
#define KB200_IPC_HANDLE_BYTES 64
KB200_API size_t kb200_peer_buffer_bytes(int world, size_t max_count);
KB200_API int kb200_device_alloc(size_t bytes, void** ptr);
KB200_API int kb200_device_free(void* ptr);
KB200_API int kb200_ipc_handle(const void* ptr, void* handle);
KB200_API int kb200_ipc_open(const void* handle, void** ptr);
KB200_API int kb200_ipc_close(void* ptr);
KB200_API int kb200_peer_allreduce_f32(float* data, size_t count, void* const* peers, int world, int rank,
                                       size_t max_count, double timeout_s, void* stream);

/* A row-parallel projection plus the all-reduce of its output in one call
 * (tensor parallelism): job as for kb200_gguf_gemv_batch with contiguous
 * output rows (stride == columns, rows * columns even and <= max_count);
 * peers/world/rank/max_count/timeout_s as for kb200_peer_allreduce_f32, whose
 * call sequence it shares. On the tensor-pipe path (kb200_gemv_path == 2)
 * the GEMV stores each finished output straight into every peer's buffer
 * and a gather kernel adds them; otherwise the GEMV is followed by the full
 * all-reduce. On return (stream order) every rank's output holds the sum over
 * the ranks, the same bits on each. */
KB200_API int kb200_gguf_gemv_allreduce(const kb200_gemv_job* job, void* const* peers, int world, int rank,
                                        size_t max_count, double timeout_s, void* stream);

/* ---------------------------------------------------------------------------
 * Expert-parallel exchange over NVLink peer memory (one process per GPU),
 * with no count read-back on the host. Each rank allocates
 * kb200_ep_buffer_bytes(world, experts, hidden, capacity, local_capacity)
 * with kb200_device_alloc, exchanges it by CUDA IPC (kb200_ipc_handle /
 * kb200_ipc_open) and passes all buffers as `peers` (its own at [rank]).
 * capacity: rows any rank can receive (at most the group's tokens * top_k);
 * local_capacity: this rank's tokens * top_k at most.
 *
 * kb200_ep_dispatch: after kb200_moe_dispatch_rows (offsets and rows of its
 * result), stores every row into its expert owner's receive area
 * (kb200_ep_rows_area of the owner's buffer), expert-major (for each local
 * expert, the rows of source 0..N-1), and writes local_offsets (device
 * [experts/world + 1]) for kb200_moe_experts on that area with
 * rows = capacity. kb200_ep_return: stores the expert results (fp32
 * [capacity, hidden] in receive order) into each source's return area
 * (kb200_ep_return_area) in the source's dispatch order, for
 * kb200_moe_combine. Every rank makes the same calls in the same order;
 * waits are bounded by timeout_s and report watchdog bit 32. */
KB200_API size_t kb200_ep_buffer_bytes(int world, int experts, int hidden, size_t capacity, size_t local_capacity);
KB200_API void* kb200_ep_rows_area(void* buffer);
KB200_API void* kb200_ep_return_area(void* buffer, size_t capacity, int hidden);
KB200_API int kb200_ep_dispatch(const int32_t* offsets, const uint16_t* rows, int hidden, int experts, int world,
                                int rank, void* const* peers, size_t capacity, size_t local_capacity,
                                int32_t* local_offsets, double timeout_s, void* stream);
KB200_API int kb200_ep_return(const float* results, int hidden, int experts, int world, int rank,
                              void* const* peers, size_t capacity, size_t local_capacity, double timeout_s,
                              void* stream);

/* The routing stage alone (for tests): chosen [tokens, top_k] int32,
 * weight [tokens, top_k] fp32, device. */
KB200_API int kb200_moe_route(
    const float* logits,
    size_t tokens,
    int32_t experts,
    int32_t top_k,
    int32_t* chosen,
    float* weight,
    void* stream
);

/* Device-side watchdog word: nonzero when a bounded wait inside a kernel gave up
 * since the last call of this function, which also clears it. Synchronous.
 * Bits: 1 a stage never arrived, 2 a stage was never released, 4 the final
 * copies never landed, 8 a cut tile's other pieces never arrived (Q4_K GEMV),
 * 16 a peer's chunk never arrived (peer all-reduce), 32 a peer's counts or
 * rows never arrived (expert-parallel exchange). */
KB200_API int kb200_take_device_error(unsigned* value);

/* ---------------------------------------------------------------------------
 * Resident weight bank: kadan::DeviceWeights
 * (IW/include/kadan/device_weights.hpp:35-486). One bank per device, owned by
 * one thread (calls must not overlap). Entries are immutable packed tiles keyed
 * by the tensor's file identity and a block range; a miss is admitted only
 * inside the bank's byte envelope and the device's free memory, copied in
 * 1 MiB pieces with the cancel word polled before each, synchronised, and only
 * then published. A failed admission rolls back; a rollback or a release whose
 * synchronise or free fails quarantines the bank (KB200_QUARANTINED from every
 * later call except kb200_bank_state and kb200_bank_destroy). */

/* kadan::WeightIdentity (IW/include/kadan/weight_identity.hpp:7-19). */
typedef struct kb200_weight_identity {
    uint64_t device, inode, file_size;
    uint64_t modified_seconds, modified_nanoseconds;
    uint64_t changed_seconds, changed_nanoseconds;
    uint64_t payload_begin, payload_end;
} kb200_weight_identity;

/* DeviceWeights::Key (device_weights.hpp:40-44): `count` blocks of `width`
 * bytes from block `first` of the tensor. */
typedef struct kb200_weight_key {
    kb200_weight_identity source;
    uint64_t first, count, width;
} kb200_weight_key;

/* WeightDeviceOperations (device_weights.hpp:19-32) as a table of callbacks;
 * each returns a kb200_status. `allocate` returning KB200_OK with *out NULL is a
 * confirmed out-of-memory refusal. Both copies write dst + offset from
 * src + offset. */
typedef struct kb200_weight_ops {
    void* user;
    int (*available)(void* user, uint64_t* bytes);
    int (*allocate)(void* user, uint64_t bytes, void** out);
    int (*copy_host)(void* user, void* dst, uint64_t offset, const void* src, uint64_t bytes);
    int (*copy_device)(void* user, void* dst, uint64_t offset, const void* src, uint64_t bytes);
    int (*release)(void* user, void* ptr);
    int (*synchronize)(void* user);
} kb200_weight_ops;

/* Why kb200_bank_retain returned no pointer with KB200_OK (the reference's
 * trace_refusal reasons, device_weights.hpp:199-231). */
#define KB200_BANK_ADMITTED 0
#define KB200_BANK_EMPTY 1
#define KB200_BANK_ENVELOPE 2
#define KB200_BANK_PHYSICAL 3
#define KB200_BANK_ALLOCATION 4

typedef struct kb200_bank_state {
    uint64_t capacity;         /* current envelope (DeviceWeights::capacity) */
    uint64_t maximum_capacity; /* envelope given at creation */
    uint64_t allocated;        /* bytes held by entries */
    uint64_t reserved;         /* envelope charged since the first admission, else 0 */
    uint64_t entries;
    int32_t quarantined;
} kb200_bank_state;

typedef struct kb200_bank kb200_bank;

/* A bank over caller-supplied operations (copied; `user` must outlive the bank). */
KB200_API int kb200_bank_create(uint64_t limit, const kb200_weight_ops* ops, kb200_bank** out);
/* A bank over CUDA memory of `device`: cudaMalloc'd entries, copies on a
 * stream of the bank's own, available = free device memory minus `scratch`. */
KB200_API int kb200_bank_create_cuda(int device, uint64_t limit, uint64_t scratch, kb200_bank** out);
/* Releases every entry (best effort when quarantined) and frees the bank. */
KB200_API void kb200_bank_destroy(kb200_bank* bank);
KB200_API int kb200_bank_state_get(const kb200_bank* bank, kb200_bank_state* state);
/* DeviceWeights::find: *ptr = the published entry or NULL. */
KB200_API int kb200_bank_find(kb200_bank* bank, const kb200_weight_key* key, void** ptr);
/* DeviceWeights::retain / retain_device: `bytes` must equal count * width.
 * A hit returns the entry without a copy; a refusal returns KB200_OK with
 * *ptr NULL and *refusal set (refusal may be NULL). `src` is host memory for
 * kb200_bank_retain and device memory for kb200_bank_retain_device. */
KB200_API int kb200_bank_retain(kb200_bank* bank, const kb200_weight_key* key, const void* src, uint64_t bytes,
                                const volatile uint8_t* cancel, void** ptr, int* refusal);
KB200_API int kb200_bank_retain_device(kb200_bank* bank, const kb200_weight_key* key, const void* src,
                                       uint64_t bytes, const volatile uint8_t* cancel, void** ptr, int* refusal);
/* DeviceWeights::release_sources: drop every entry of these tensors, keep the
 * envelope; *released = bytes freed (may be NULL). Not cancellable. */
KB200_API int kb200_bank_release_sources(kb200_bank* bank, const kb200_weight_identity* sources, size_t count,
                                         uint64_t* released);
/* DeviceWeights::release: drop every entry and the envelope's charge. */
KB200_API int kb200_bank_release(kb200_bank* bank);
/* DeviceWeights::bound: envelope = min(maximum, bytes); KB200_INVALID once
 * anything was admitted since the last release. */
KB200_API int kb200_bank_bound(kb200_bank* bank, uint64_t bytes);

/* ---------------------------------------------------------------------------
 * Host-span batch over packed-row sources and the bank.
 *
 * GgufWeightSource (IW/include/kadan/dense_compute.hpp:172): write `bytes`
 * bytes of whole packed rows, starting at row `first_row`, to `dst`; return a
 * kb200_status (nonzero fails the call with that status). */
typedef int (*kb200_row_source)(void* user, uint64_t first_row, void* dst, uint64_t bytes);

/* DenseCompute::GgufBatchJob (dense_compute.hpp:205-213). */
typedef struct kb200_source_job {
    const kb200_weight_identity* identity;
    kb200_row_source source;
    void* source_user;
    const float* input; /* host, rows * in floats */
    float* output;      /* host, rows * out floats */
    uint32_t in;
    uint32_t out;
    uint32_t rows;
    int32_t encoding; /* kb200_encoding, KB200_F32 for fp32 rows */
    int32_t retain_misses;
} kb200_source_job;

/* 1 if kb200_dense_gguf_source_batch accepts `job` (gguf_batch_supported,
 * IW/include/kadan/gguf_batch_partition.hpp:14-37, for one job: sizes within
 * an int, rows within KB200_BATCH_MAX_ROWS, `in` a multiple of 8 and of the
 * block, a row within one staging half, and an encoding with a decoder here);
 * host only. A caller that splits a batch over several devices checks every
 * job first, so that unsupported still precedes any source read. */
KB200_API int kb200_source_job_supported(const kb200_source_job* job);

/* Staging of kb200_dense_gguf_source_batch: two halves of this many bytes,
 * pinned on the host and on the device. */
#define KB200_SOURCE_STAGING_HALF (16u * 1024u * 1024u)

/* DenseCompute::dense_gguf_batch with packed sources on one device
 * (IW/src/cuda/h3_compute.cu:3963-4375). Each job's columns are cut into the
 * reference's chunks (kb200_gguf_batch_partition for one device and
 * `scratch_limit` bytes of projection scratch) and keyed like the reference's
 * bank entries ({identity, first block, blocks, block bytes}). Chunks found in
 * `bank` run from it; the others are read through their source into pinned
 * staging, one group per staging half (the next group is read while the device
 * multiplies the previous one), multiplied with a finite check, and then,
 * for jobs with retain_misses, admitted into `bank` (a refusal is not an
 * error). `bank` may be NULL: every chunk streams and nothing is kept. The
 * bank must hold memory of the context's device. Unsupported, input, alias,
 * cancel and result rules are those of kb200_dense_gguf_batch; sources are
 * called on the calling thread. */
KB200_API int kb200_dense_gguf_source_batch(kb200_context* ctx, kb200_bank* bank, const kb200_source_job* jobs,
                                            size_t count, uint64_t scratch_limit, const volatile uint8_t* cancel,
                                            int* result);

/* DenseCompute::dense_gguf_source (IW/include/kadan/dense_compute.hpp:180-194,
 * IW/src/cuda/h3_compute.cu:3503-3536): one projection of a packed source with
 * an optional fp32 bias [out]. Unsupported jobs (as for the batch, and every
 * `precise` call: the reference widens to an fp64 GEMM there, which is not
 * offered here) return KB200_UNSUPPORTED before any read or write; a
 * non-finite bias fails with KB200_NONFINITE_BIAS before any source read; then
 * the job runs as a one-job kb200_dense_gguf_source_batch, the bias is added
 * (one fp32 addition per output, as the reference's add_bias), and every
 * output is checked finite: KB200_NONFINITE_OUTPUT (outputs to be discarded)
 * or *result = KB200_RESULT_FINITE. */
KB200_API int kb200_dense_gguf_source(kb200_context* ctx, kb200_bank* bank, const kb200_source_job* job,
                                      const float* bias, uint64_t scratch_limit, int precise,
                                      const volatile uint8_t* cancel, int* result);

/* ---------------------------------------------------------------------------
 * GGUF checkpoint reader: kadan::checkpoint::GgufCheckpoint
 * (IW/include/kadan/gguf_checkpoint.hpp:53-103, IW/src/weights/gguf_checkpoint.cpp).
 * `root` is a directory holding one unsplit GGUF v3 file or a numbered split
 * set (<prefix>-00001-of-0000N.gguf ...). Opening reads bounded metadata only
 * and accepts what the reference accepts: F32 tensors and every
 * kadan::gguf::Encoding, ranks 1-3, tensors laid out contiguously at the
 * file's alignment. Failures return KB200_INVALID (or KB200_IO for open/read
 * errors, KB200_CANCELLED) with the reference's message ("gguf_version",
 * "gguf_missing_tensor", "gguf_row_range", "gguf_checkpoint_changed", ...). */
typedef struct kb200_gguf kb200_gguf;

typedef struct kb200_gguf_tensor {
    uint64_t shape[3];  /* ggml order: values per row, rows, experts; absent dimensions are 1 */
    uint32_t rank;
    uint32_t ggml_type;
    int32_t encoding;   /* kb200_encoding, KB200_F32 for F32 */
    uint32_t file;      /* index of the split file holding it */
    uint64_t bytes;     /* all rows of all experts */
    uint64_t row_bytes;
    uint64_t offset;    /* absolute byte offset of the payload in its file */
} kb200_gguf_tensor;

KB200_API int kb200_gguf_open(const char* root, const volatile uint8_t* cancel, kb200_gguf** out);
/* kb200_gguf_open with options. KB200_GGUF_ACCEPT_MXFP4: also accept tensors
 * of ggml type 39 (GGUF MXFP4, block_mxfp4: IW/third_party/ggml/src/
 * ggml-common.h:214-219), which the reference's reader refuses
 * ("gguf_tensor_type", gguf_checkpoint.cpp:229-230, gguf::encoding has no
 * MXFP4); they report encoding KB200_GGUF_MXFP4, 32 values per 17-byte block,
 * and read as packed rows like any other tensor. Without flags the reader
 * accepts and refuses exactly what the reference's does. */
#define KB200_GGUF_ACCEPT_MXFP4 1u
#define KB200_GGUF_MXFP4 (-3)
KB200_API int kb200_gguf_open_flags(const char* root, const volatile uint8_t* cancel, uint32_t flags, kb200_gguf** out);
KB200_API void kb200_gguf_close(kb200_gguf* file);
KB200_API size_t kb200_gguf_tensor_count(const kb200_gguf* file);
/* Tensors in name order; *name stays valid until kb200_gguf_close. */
KB200_API int kb200_gguf_tensor_at(const kb200_gguf* file, size_t index, kb200_gguf_tensor* info, const char** name);
KB200_API int kb200_gguf_find_tensor(const kb200_gguf* file, const char* name, kb200_gguf_tensor* info);
/* GgufCheckpoint::identity: the file's identity and the payload interval of
 * one expert of the tensor (expert 0 for ordinary matrices). */
KB200_API int kb200_gguf_identity(const kb200_gguf* file, const char* name, uint64_t expert,
                                  kb200_weight_identity* identity);
/* "gguf_checkpoint_changed" when a file's size, mtime or ctime moved since opening. */
KB200_API int kb200_gguf_check_unchanged(const kb200_gguf* file);
/* GgufCheckpoint::read_packed_rows: `bytes` (whole rows) of expert `expert`
 * from row `first_row`, copied without decoding, in 1 MiB preads with the
 * cancel byte polled before each. Safe to call concurrently on disjoint outputs. */
KB200_API int kb200_gguf_read_packed_rows(const kb200_gguf* file, const char* name, uint64_t expert,
                                          uint64_t first_row, void* output, uint64_t bytes,
                                          const volatile uint8_t* cancel);
/* GgufCheckpoint::read_vector: a whole F32 tensor of any rank (`count` its
 * element count), every value finite ("gguf_vector_shape",
 * "gguf_nonfinite_weight"); the output is to be discarded after a failure. */
KB200_API int kb200_gguf_read_vector(const kb200_gguf* file, const char* name, float* output, uint64_t count,
                                     const volatile uint8_t* cancel);
/* Metadata of the first file (GgufCheckpoint::has / integer / number /
 * boolean / string / integers / numbers). `integers` and `numbers` copy at
 * most `capacity` values and report the array's length in *count. */
KB200_API int kb200_gguf_has(const kb200_gguf* file, const char* key);
KB200_API int kb200_gguf_integer(const kb200_gguf* file, const char* key, uint64_t* value);
KB200_API int kb200_gguf_number(const kb200_gguf* file, const char* key, double* value);
KB200_API int kb200_gguf_boolean(const kb200_gguf* file, const char* key, int* value);
KB200_API int kb200_gguf_string(const kb200_gguf* file, const char* key, const char** value, size_t* length);
KB200_API int kb200_gguf_integers(const kb200_gguf* file, const char* key, int64_t* values, size_t capacity,
                                  size_t* count);
KB200_API int kb200_gguf_numbers(const kb200_gguf* file, const char* key, double* values, size_t capacity,
                                 size_t* count);

/* One tensor (and expert) of an open checkpoint as a kb200_row_source:
 * bind it, then pass kb200_gguf_rows_source as a source job's `source` and
 * the bound struct as its `source_user` (rows are whole packed rows of that
 * expert). The struct must outlive the calls; the file must stay open. */
typedef struct kb200_gguf_rows {
    const kb200_gguf* file;
    uint64_t tensor;
    uint64_t expert;
} kb200_gguf_rows;

KB200_API int kb200_gguf_rows_bind(const kb200_gguf* file, const char* name, uint64_t expert, kb200_gguf_rows* rows);
KB200_API int kb200_gguf_rows_source(void* rows, uint64_t first_row, void* dst, uint64_t bytes);

/* ---------------------------------------------------------------------------
 * Safetensors shard reader: kadan::checkpoint::Shard
 * (IW/include/kadan/checkpoint.hpp:91-178, IW/src/weights/checkpoint.cpp:449-730)
 * for the gpt-oss MXFP4 expert tensors. `name` is one file basename in the
 * directory `root`. The header must tile the payload exactly; failures return
 * KB200_INVALID (KB200_IO for open/read errors) with the reference's message
 * ("header_size", "json_syntax", "tensor_gap_or_overlap", "missing_tensor",
 * "mxfp4_expert_shape", "invalid_block_scale", "checkpoint_changed", ...). */
typedef struct kb200_shard kb200_shard;

/* checkpoint::Dtype, in its order. */
#define KB200_DTYPE_U8 0
#define KB200_DTYPE_F8_E4M3 1
#define KB200_DTYPE_F32 2
#define KB200_DTYPE_BF16 3
#define KB200_DTYPE_F16 4
#define KB200_DTYPE_I8 5
#define KB200_DTYPE_U32 6

/* checkpoint::Limits; a NULL pointer means the reference's defaults
 * (16 MiB of header, 65536 tensors, 512-byte metadata values). */
typedef struct kb200_shard_limits {
    uint64_t header_bytes, tensors, metadata_value_bytes;
} kb200_shard_limits;

typedef struct kb200_shard_tensor {
    uint64_t shape[8];
    uint32_t rank;
    int32_t dtype;   /* KB200_DTYPE_* */
    uint64_t bytes;
    uint64_t offset; /* absolute byte offset of the payload in the file */
} kb200_shard_tensor;

KB200_API int kb200_shard_open(const char* root, const char* name, const kb200_shard_limits* limits,
                               kb200_shard** out);
KB200_API void kb200_shard_close(kb200_shard* shard);
KB200_API size_t kb200_shard_tensor_count(const kb200_shard* shard);
/* Tensors in name order; *name stays valid until kb200_shard_close. */
KB200_API int kb200_shard_tensor_at(const kb200_shard* shard, size_t index, kb200_shard_tensor* info,
                                    const char** name);
KB200_API int kb200_shard_find_tensor(const kb200_shard* shard, const char* name, kb200_shard_tensor* info);
KB200_API int kb200_shard_identity(const kb200_shard* shard, const char* name, kb200_weight_identity* identity);
KB200_API int kb200_shard_check_unchanged(const kb200_shard* shard);
/* Shard::read_tensor: `bytes` bytes of the tensor from byte `offset`. */
KB200_API int kb200_shard_read_tensor(const kb200_shard* shard, const char* name, uint64_t offset, void* output,
                                      uint64_t bytes);
/* Shard::load_mxfp4_expert_rows: rows [first, first + count) of one expert
 * of <prefix>_blocks (U8 [experts, rows, groups, 16]) and <prefix>_scales
 * (U8 [experts, rows, groups]), still packed: `weights` receives
 * count * groups * 16 code bytes and `scales` count * groups E8M0 bytes, the
 * per-expert layout kb200_moe_weights takes. *columns = groups * 32. The
 * reads are checked against payload_budget (code + scale bytes) first; after a
 * failure ("invalid_block_scale" included) the outputs must be discarded. */
KB200_API int kb200_shard_load_mxfp4_expert_rows(const kb200_shard* shard, const char* prefix, uint64_t expert,
                                                 uint64_t first, uint64_t count, uint64_t payload_budget,
                                                 void* weights, uint64_t weights_capacity, void* scales,
                                                 uint64_t scales_capacity, uint64_t* columns);

/* ---------------------------------------------------------------------------
 * Layer math around the path on the device (device pointers, stream order).
 * The reference runs it on the host: rms_norm / l2_norm / rope / attend /
 * delta_rule (IW/src/models/text/gguf_weights.cpp:639-818) from
 * AttentionLayer::forward and DeltaNetLayer::forward (qwen_layers.cpp:74-330),
 * unless its DenseCompute takes attend_cached / delta_step
 * (IW/include/kadan/dense_compute.hpp:275-330). */

/* rms_norm (gguf_weights.cpp:639-666): each row of `width` values times
 * 1 / sqrt(float(sum of squares in double / width) + eps), then times weight
 * (NULL: the unweighted form). out may equal x. Bit 0 of *status (when not
 * NULL) is set if an output is not finite (gguf_text_norm_nonfinite). */
KB200_API int kb200_rms_norm(const float* x, const float* weight, size_t rows, size_t width, float eps, float* out,
                             unsigned* status, void* stream);
/* l2_norm (gguf_weights.cpp:667-674): x / sqrt(sum x^2 + eps) per row. */
KB200_API int kb200_l2_norm(const float* x, size_t rows, size_t width, float eps, float* out, void* stream);
/* rope (gguf_weights.cpp:676-700) in place over `rows` rows of row_width
 * values, each a run of heads of `width` values; row r is at position + r
 * (AttentionLayer::forward, qwen_layers.cpp:242-256). Pairs (i, i + rotary/2)
 * of each head turn by (position + r) * base^(-2i/rotary). */
KB200_API int kb200_rope(float* x, size_t rows, size_t row_width, size_t width, size_t rotary, size_t position,
                         float base, void* stream);

/* Cached attention (attend_cached, dense_compute.hpp:275-300; the host's
 * attend, gguf_weights.cpp:700-777): q [rows][heads][dim]; keys and values
 * [positions][kv_heads][dim] (16-byte aligned) with at least position + rows
 * positions; row r is at position + r and attends every position up to its
 * own, or with `selected` the positions selected[offsets[r] ..
 * offsets[r + 1]) (offsets has rows + 1 entries; at most position + rows per
 * row, none after the row's own position). out [rows][heads][dim]. The
 * softmax is over scale * q.k. Supported: head dim 64, 128 or 256, at most 16
 * query heads per KV head and heads/kv_heads * dim <= 2048
 * (kb200_attend_supported); otherwise KB200_UNSUPPORTED before any work. */
KB200_API int kb200_attend_supported(size_t heads, size_t kv_heads, size_t dim);
KB200_API size_t kb200_attend_workspace_bytes(size_t rows, size_t position, size_t heads, size_t dim);
KB200_API int kb200_attend_cached(const float* q, const float* keys, const float* values, size_t rows,
                                  size_t position, size_t heads, size_t kv_heads, size_t dim, float scale,
                                  const uint32_t* selected, const uint32_t* offsets, float* out, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* One gated delta-net step over `rows` rows in order (delta_step,
 * dense_compute.hpp:302-330; the host's DeltaNetLayer::forward,
 * qwen_layers.cpp:131-180): causal depthwise convolution with SiLU over qkv
 * (channels = (2 key_heads + value_heads) dim: q, k, v), L2-normalised q and
 * k heads, then per value head the decayed delta rule (delta_rule,
 * gguf_weights.cpp:778-818) with decay exp(softplus(alpha + dt) a) and
 * sigmoid(beta), RMSNorm by `norm` and the sigmoid (sigmoid_gate) or SiLU
 * gate of z. history [(kernel - 1)][channels] (oldest first) and state
 * [value_heads][dim][dim] are read and updated. */
typedef struct kb200_delta_args {
    const float* qkv;    /* [rows][channels] */
    const float* z;      /* [rows][value_heads * dim] */
    const float* alpha;  /* [rows][value_heads] */
    const float* beta;   /* [rows][value_heads] */
    const float* conv;   /* [channels][kernel] */
    const float* dt;     /* [value_heads] */
    const float* a;      /* [value_heads] */
    const float* norm;   /* [dim] */
    float* history;      /* [(kernel - 1)][channels], updated */
    float* state;        /* [value_heads][dim][dim], updated */
    float* output;       /* [rows][value_heads * dim] */
    uint32_t rows, key_heads, value_heads, dim, kernel;
    float eps;
    int32_t sigmoid_gate;
} kb200_delta_args;
/* dim a multiple of 32 up to 256, value_heads a multiple of key_heads,
 * kernel 1..64. */
KB200_API int kb200_delta_supported(uint32_t key_heads, uint32_t value_heads, uint32_t dim, uint32_t kernel);
KB200_API size_t kb200_delta_workspace_bytes(const kb200_delta_args* args);
KB200_API int kb200_delta_step(const kb200_delta_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* Host-span forms on a context (synchronous; calls on one context must not
 * overlap). The context keeps per-layer device state, keyed by the caller's
 * `layer` id, until kb200_context_release_layers (the reference's
 * release_scratch) or kb200_context_destroy.
 *
 * attend_cached (dense_compute.hpp:275-300): keys / values hold at least
 * position + rows positions of [kv_heads][dim]. The context mirrors the
 * layer's KV cache: positions mirrored by earlier calls below `position` are
 * reused, positions from min(mirrored, position) to position + rows are
 * uploaded. selected / offsets (host, may be NULL) as for kb200_attend_cached;
 * a selected position after its row's own fails with KB200_INVALID.
 * KB200_UNSUPPORTED (nothing read or written) when kb200_attend_supported
 * rejects the shape: the caller's own attention then runs. */
KB200_API int kb200_attend_cached_host(kb200_context* ctx, uint64_t layer, const float* q, const float* keys,
                                       const float* values, size_t rows, size_t position, size_t heads,
                                       size_t kv_heads, size_t dim, float scale, const uint32_t* selected,
                                       const uint32_t* offsets, float* output, const volatile uint8_t* cancel);

/* delta_step (dense_compute.hpp:302-330, its DeltaStep fields): host spans of
 * the step's inputs; the layer's recurrent state and convolution history stay
 * on the device. `fresh` starts them at zero, or at initial_state
 * ([value_heads][dim][dim]) / initial_history ([(kernel - 1)][channels]) when
 * those are not NULL. A fresh step with an unsupported shape returns
 * KB200_UNSUPPORTED before any output write; a later step of a layer without
 * device state fails with KB200_INVALID ("recurrent_state_lost"). */
typedef struct kb200_delta_host {
    uint64_t layer;
    int32_t fresh;
    const float* qkv;    /* [rows][channels] */
    const float* z;      /* [rows][value_heads * dim] */
    const float* alpha;  /* [rows][value_heads] */
    const float* beta;   /* [rows][value_heads] */
    const float* conv;   /* [channels][kernel] */
    const float* dt;     /* [value_heads] */
    const float* a;      /* [value_heads] */
    const float* norm;   /* [dim] */
    uint32_t rows, key_heads, value_heads, dim, kernel;
    float eps;
    int32_t sigmoid_gate;
    float* output;                /* [rows][value_heads * dim] */
    const float* initial_state;   /* NULL or [value_heads][dim][dim] */
    const float* initial_history; /* NULL or [(kernel - 1)][channels] */
} kb200_delta_host;
KB200_API int kb200_delta_step_host(kb200_context* ctx, const kb200_delta_host* step,
                                    const volatile uint8_t* cancel);
/* copy_recurrent_state (dense_compute.hpp:323-326): the layer's device state
 * and history into host arrays of exactly state_floats / history_floats. */
KB200_API int kb200_recurrent_state_get(kb200_context* ctx, uint64_t layer, float* state, size_t state_floats,
                                        float* history, size_t history_floats);
/* Frees every layer's KV mirror and recurrent state (release_scratch). */
KB200_API int kb200_context_release_layers(kb200_context* ctx);

/* ---------------------------------------------------------------------------
 * Per-kernel telemetry (the reference's CudaPhaseScope / cuda_trace::kernel,
 * IW/include/kadan/cuda_phase_metrics.hpp:9-87, IW/src/cuda/cuda_telemetry.cuh:
 * 101-160). A phase collects, for every launch the library issues on a
 * thread while the phase is that thread's current one: the call count and
 * host seconds of the launch call per kernel id, and the device seconds
 * between CUDA events recorded around the launch on its stream. Events are
 * read without waiting (at later launches, at kb200_phase_snapshot and when
 * the thread leaves the phase); a pair still running when the thread leaves
 * the phase counts as dropped, one that cannot be recorded or read as
 * unavailable, and launches into a stream under graph capture are counted
 * without events. Telemetry never fails a launch. Ids are a fixed protocol
 * order: new kernels are added before KB200_KERNEL_COUNT. */
typedef enum kb200_kernel {
    KB200_KERNEL_GGUF_DEQUANT = 0,      /* dequant_kernel (gguf_decode_kernel) */
    KB200_KERNEL_GEMV_STAGED = 1,       /* gemv_staged_kernel (Q8_0 and the staged formats) */
    KB200_KERNEL_GEMV_GENERIC = 2,      /* gemv_generic_kernel (every encoding) */
    KB200_KERNEL_GEMV_Q4K_MMA = 3,      /* gemv_q4k_mma_kernel */
    KB200_KERNEL_GEMV_Q6K_MMA = 4,      /* gemv_q6k_mma_kernel (3-8 input rows) */
    KB200_KERNEL_GEMV_Q6K_PAIR = 5,     /* gemv_q6k_pair_kernel (1-2 input rows) */
    KB200_KERNEL_GEMM_PREFILL_ROWS = 6, /* prefill_rows_kernel (GEMM activation rows) */
    KB200_KERNEL_GEMM_GGUF = 7,         /* gemm_gguf_kernel (tcgen05 prefill GEMM) */
    KB200_KERNEL_MOE_ROUTE = 8,
    KB200_KERNEL_MOE_SORT = 9,
    KB200_KERNEL_MOE_GATHER = 10,
    KB200_KERNEL_MOE_MTILE = 11,
    KB200_KERNEL_MOE_GEMM = 12,         /* grouped tcgen05 GEMM (gate/up or down) */
    KB200_KERNEL_MOE_GEMV = 13,         /* grouped GEMV (decode-sized batches) */
    KB200_KERNEL_MOE_COMBINE = 14,
    KB200_KERNEL_ROWS_REGROUP = 15,
    KB200_KERNEL_MXFP4_GGML_DEQUANT = 16,
    KB200_KERNEL_MXFP4_FROM_GGML = 17,
    KB200_KERNEL_PEER_ALLREDUCE = 18,   /* peer all-reduce / row-parallel gather */
    KB200_KERNEL_EP_EXCHANGE = 19,      /* expert-parallel peer exchange */
    KB200_KERNEL_RMS_NORM = 20,         /* rms_norm_kernel (RMSNorm and L2 norm) */
    KB200_KERNEL_ROPE = 21,
    KB200_KERNEL_ATTEND = 22,           /* attend_kernel (cached attention, per segment) */
    KB200_KERNEL_ATTEND_COMBINE = 23,
    KB200_KERNEL_DELTA_CONV = 24,
    KB200_KERNEL_DELTA_L2 = 25,
    KB200_KERNEL_DELTA_HEADS = 26,
    KB200_KERNEL_SILU_MUL = 27,
    KB200_KERNEL_MOE_SHARED = 28,       /* moe_shared_kernel (shared expert's gated add) */
    KB200_KERNEL_MOE_DECODE = 29,       /* moe_decode_kernel (the whole layer for at most 8 tokens) */
    KB200_KERNEL_PAIR_QUANT = 30,       /* pair_quant_kernel (a Q6_K decode launch's activations, once) */
    KB200_KERNEL_Q4K_QUANT = 31,        /* q4k_quant_kernel (a Q4_K decode launch's activations, once) */
    KB200_KERNEL_COUNT = 32
} kb200_kernel;

typedef struct kb200_kernel_metrics {
    uint64_t calls;       /* launches issued */
    double host_seconds;  /* time inside the launch calls */
    uint64_t measured;    /* launches with a device interval read back */
    double gpu_seconds;   /* sum of those intervals */
} kb200_kernel_metrics;

typedef struct kb200_phase_metrics {
    kb200_kernel_metrics kernels[KB200_KERNEL_COUNT];
    uint64_t dropped;           /* event pairs not finished when collected for the last time, or over capacity */
    uint64_t unavailable;       /* event pairs that could not be created, recorded or read */
    uint64_t shared_batch_size; /* as given to kb200_phase_create */
    int32_t observed;           /* nonzero once anything was counted */
} kb200_phase_metrics;

typedef struct kb200_phase kb200_phase;

KB200_API int kb200_phase_create(uint64_t shared_batch_size, kb200_phase** out);
/* Makes `phase` (or none, NULL) the calling thread's current phase; the
 * previous one is returned in *previous when that is not NULL (it stays
 * referenced by the thread until then: pass it to kb200_phase_release). Event
 * pairs of the previous phase are collected first. */
KB200_API int kb200_phase_enter(kb200_phase* phase, kb200_phase** previous);
/* The phase's counters; collects the calling thread's finished event pairs
 * first (without waiting). */
KB200_API int kb200_phase_snapshot(kb200_phase* phase, kb200_phase_metrics* out);
/* Drops one reference (the creator's, or one returned by kb200_phase_enter). */
KB200_API void kb200_phase_release(kb200_phase* phase);
/* Stable name of a kernel id ("moe_gemm_kernel", ...); NULL when out of range. */
KB200_API const char* kb200_kernel_name(int kernel);

#ifdef __cplusplus
}
#endif
#endif
