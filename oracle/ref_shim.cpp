// Test infrastructure only. A C entry layer over the reference worker's own
// CPU code, compiled in place from the read-only reference tree (see Makefile),
// so Python tests and bench.py's CPU baseline can call it through ctypes.
//
// Wrapped reference functions:
//   kadan::gguf::decode / decode_run     IW/include/kadan/gguf_quantization.hpp:631-916
//   ggml to_float / quantize_chunk       IW/third_party/ggml/src/ggml.c (type traits)
//   kadan::quantization::decode_rows     IW/src/weights/quantization.cpp:193-205
//   kadan::quantization::matvec          IW/src/weights/quantization.cpp:208-247
//   kadan::text::CpuMatvec               IW/src/models/text/cpu_matvec.cpp:18-66
//   kadan::checkpoint::GgufCheckpoint    IW/src/weights/gguf_checkpoint.cpp:441-674
//   kadan::checkpoint::Shard             IW/src/weights/checkpoint.cpp:449-730
// (IW = services/hikari/inference_worker). The 64-column work units of
// ref_cpu_matvec_parallel follow GgufWeights::project's host split
// (IW/src/models/text/gguf_weights.cpp:400-446).
#include <atomic>
#include <cstdint>
#include <cstring>
#include <exception>
#include <span>
#include <thread>
#include <vector>

#include "cpu_matvec.hpp"
#include "kadan/gguf_batch_partition.hpp"
#include "kadan/checkpoint.hpp"
#include "kadan/gguf_checkpoint.hpp"
#include "kadan/gguf_quantization.hpp"
#include "kadan/quantization.hpp"
#include <ggml-cpu.h>
#include <ggml.h>

namespace {
thread_local char last_error[256];

int fail(const std::exception& e) {
    std::strncpy(last_error, e.what(), sizeof(last_error) - 1);
    return -1;
}
}  // namespace

extern "C" {

const char* ref_last_error() {
    return last_error;
}

// kadan::gguf::Encoding numbering (q3_k=0, q4_k, q8_0, q6_k, iq3_xxs, iq4_nl,
// iq4_xs, iq2_s, iq3_s, bf16=9).
float ref_gguf_decode(int encoding, const unsigned char* block, size_t element) {
    return kadan::gguf::decode(kadan::gguf::Encoding(encoding), block, element);
}

// The reference's own code grids of IQ3_XXS, IQ2_S and IQ3_S
// (gguf_quantization.hpp:501-504), as a caller passes them to kb200_set_iq_grids.
void ref_iq_grids(const uint32_t** iq3xxs, const uint64_t** iq2s, const uint32_t** iq3s) {
    *iq3xxs = kadan::gguf::detail::iq3xxs_grid_host;
    *iq2s = kadan::gguf::detail::iq2s_grid_host;
    *iq3s = kadan::gguf::detail::iq3s_grid_host;
}

size_t ref_gguf_block_values(int encoding) {
    return kadan::gguf::block_values(kadan::gguf::Encoding(encoding));
}

size_t ref_gguf_block_bytes(int encoding) {
    return kadan::gguf::block_bytes(kadan::gguf::Encoding(encoding));
}

int ref_gguf_encoding(uint32_t ggml_type) {
    const auto e = kadan::gguf::encoding(ggml_type);
    return e ? int(*e) : -1;
}

// Elementwise decode of `count` values of a packed stream, as the reference's
// gguf_decode_kernel does per thread (IW/src/cuda/h3_compute.cu:76-95).
void ref_gguf_decode_stream(
    int encoding, const unsigned char* packed, size_t count, float* out
) {
    const auto e = kadan::gguf::Encoding(encoding);
    const auto values = kadan::gguf::block_values(e), bytes = kadan::gguf::block_bytes(e);
    for (size_t i = 0; i < count; ++i)
        out[i] = kadan::gguf::decode(e, packed + i / values * bytes, i % values);
}

// decode_run over every aligned run of eight of a packed stream.
void ref_gguf_decode_run_stream(
    int encoding, const unsigned char* packed, size_t count, float* out
) {
    const auto e = kadan::gguf::Encoding(encoding);
    const auto values = kadan::gguf::block_values(e), bytes = kadan::gguf::block_bytes(e);
    for (size_t i = 0; i < count; i += 8)
        kadan::gguf::decode_run(e, packed + i / values * bytes, i % values, out + i);
}

float ref_fp16_to_fp32(uint16_t bits) {
    return ggml_fp16_to_fp32(ggml_fp16_t(bits));
}

int64_t ref_ggml_blck_size(uint32_t type) {
    return ggml_blck_size(ggml_type(type));
}

size_t ref_ggml_type_size(uint32_t type) {
    return ggml_type_size(ggml_type(type));
}

size_t ref_ggml_row_size(uint32_t type, int64_t n) {
    return ggml_row_size(ggml_type(type), n);
}

void ref_ggml_to_float(uint32_t type, const void* src, float* dst, int64_t n) {
    ggml_get_type_traits(ggml_type(type))->to_float(src, dst, n);
}

size_t ref_ggml_quantize(
    uint32_t type, const float* src, void* dst, int64_t rows, int64_t per_row
) {
    return ggml_quantize_chunk(ggml_type(type), src, dst, 0, rows, per_row, nullptr);
}

// kadan::quantization MXFP4 view over the safetensors expert layout.
int ref_mxfp4_decode_rows(
    size_t rows,
    size_t columns,
    const uint8_t* weights,
    const uint8_t* scales,
    size_t first,
    size_t count,
    float* out
) {
    try {
        using namespace kadan::quantization;
        Matrix m{
            Encoding::mxfp4,
            rows,
            columns,
            std::span(weights, rows * columns / 2),
            std::span(scales, rows * columns / 32),
            {}
        };
        const auto decoded = decode_rows(m, first, count, count * columns * sizeof(float));
        std::memcpy(out, decoded.data(), decoded.size() * sizeof(float));
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_mxfp4_matvec(
    size_t rows,
    size_t columns,
    const uint8_t* weights,
    const uint8_t* scales,
    const float* input,
    float* out
) {
    try {
        using namespace kadan::quantization;
        Matrix m{
            Encoding::mxfp4,
            rows,
            columns,
            std::span(weights, rows * columns / 2),
            std::span(scales, rows * columns / 32),
            {}
        };
        matvec(m, std::span(input, columns), std::span(out, rows));
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_cpu_matvec_supported(uint32_t type, size_t in) {
    return kadan::text::CpuMatvec::supported(type, in) ? 1 : 0;
}

void* ref_cpu_matvec_create(uint32_t type, const float* input, size_t in, size_t rows) {
    try {
        return new kadan::text::CpuMatvec(type, std::span(input, in * rows), in);
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void ref_cpu_matvec_destroy(void* handle) {
    delete static_cast<kadan::text::CpuMatvec*>(handle);
}

int ref_cpu_matvec_run(
    void* handle,
    const void* weights,
    size_t row_bytes,
    size_t first,
    size_t end,
    float* output,
    size_t out
) {
    try {
        const auto* p = static_cast<const kadan::text::CpuMatvec*>(handle);
        p->run(
            static_cast<const std::byte*>(weights),
            row_bytes,
            first,
            end,
            std::span(output, p->rows() * out),
            out
        );
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// The worker's host split: 64-column units claimed by `threads` workers.
int ref_cpu_matvec_parallel(
    void* handle,
    const void* weights,
    size_t row_bytes,
    float* output,
    size_t out,
    int threads
) {
    constexpr size_t unit_columns = 64;
    const auto* p = static_cast<const kadan::text::CpuMatvec*>(handle);
    const size_t units = (out + unit_columns - 1) / unit_columns;
    std::atomic<size_t> next{0};
    std::atomic<int> status{0};
    auto work = [&] {
        for (size_t u; (u = next.fetch_add(1)) < units;) {
            const size_t first = u * unit_columns;
            const size_t end = first + unit_columns < out ? first + unit_columns : out;
            try {
                p->run(
                    static_cast<const std::byte*>(weights),
                    row_bytes,
                    first,
                    end,
                    std::span(output, p->rows() * out),
                    out
                );
            } catch (const std::exception& e) {
                status = fail(e);
            }
        }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < threads; ++t)
        pool.emplace_back(work);
    work();
    for (auto& t : pool)
        t.join();
    return status.load();
}

// Column partition (IW/include/kadan/gguf_batch_partition.hpp, device_placement.hpp).
size_t ref_weight_boundary(size_t units, const uint64_t* capacities, size_t devices, size_t index) {
    return kadan::weight_boundary(units, std::span<const kadan::Bytes>(capacities, devices), index);
}

int ref_gguf_batch_partition(size_t in, size_t out, int encoding, const uint64_t* capacities, size_t devices,
                             size_t device, uint64_t scratch_limit, size_t* result) {
    try {
        std::optional<kadan::gguf::Encoding> enc;
        if (encoding >= 0)
            enc = static_cast<kadan::gguf::Encoding>(encoding);
        const auto p = kadan::gguf_batch_partition(in, out, enc, std::span<const kadan::Bytes>(capacities, devices),
                                                   device, scratch_limit);
        result[0] = p.first, result[1] = p.count, result[2] = p.chunk_columns;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// gguf_batch_supported (IW/include/kadan/gguf_batch_partition.hpp:14-37) for
// one job with `rows` input rows; encoding < 0 means F32 rows.
int ref_gguf_batch_supported(size_t in, size_t out, size_t rows, int encoding) {
    static const kadan::WeightIdentity identity{};
    static const kadan::DenseCompute::GgufWeightSource source = [](size_t, std::span<std::byte>) {};
    std::vector<float> input(in * rows), output(out * rows);
    kadan::DenseCompute::GgufBatchJob job{&identity, std::nullopt, &source, input, in, out, output, true};
    if (encoding >= 0)
        job.encoding = static_cast<kadan::gguf::Encoding>(encoding);
    return kadan::gguf_batch_supported(std::span(&job, 1), 1) ? 1 : 0;
}

// GGUF checkpoint reader (IW/include/kadan/gguf_checkpoint.hpp:53-103).
void* ref_gguf_checkpoint_open(const char* root) {
    try {
        static const std::atomic_bool never{false};
        return new kadan::checkpoint::GgufCheckpoint(root, never);
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void ref_gguf_checkpoint_close(void* checkpoint) {
    delete static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint);
}

size_t ref_gguf_checkpoint_tensor_count(void* checkpoint) {
    return static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->tensor_count();
}

// info: shape[3], rank, type, bytes.
int ref_gguf_checkpoint_tensor(void* checkpoint, const char* name, uint64_t* info) {
    try {
        const auto& t = static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->tensor(name);
        info[0] = t.shape[0], info[1] = t.shape[1], info[2] = t.shape[2];
        info[3] = t.rank, info[4] = t.type, info[5] = t.bytes;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

const char* ref_gguf_checkpoint_tensor_name(void* checkpoint, size_t index) {
    try {
        return static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->tensor_at(index).name.c_str();
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

// identity: the nine WeightIdentity fields in declaration order.
int ref_gguf_checkpoint_identity(void* checkpoint, const char* name, uint64_t expert, uint64_t* identity) {
    try {
        const auto id = static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->identity(name, expert);
        const uint64_t v[9] = {id.device, id.inode, id.file_size, id.modified_seconds, id.modified_nanoseconds,
                               id.changed_seconds, id.changed_nanoseconds, id.payload_begin, id.payload_end};
        std::memcpy(identity, v, sizeof(v));
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_gguf_checkpoint_read_packed_rows(void* checkpoint, const char* name, uint64_t expert, uint64_t first_row,
                                         void* output, size_t bytes) {
    try {
        static const std::atomic_bool never{false};
        static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->read_packed_rows(
            name, expert, first_row, std::span<std::byte>(static_cast<std::byte*>(output), bytes), never);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_gguf_checkpoint_read_vector(void* checkpoint, const char* name, float* output, size_t count) {
    try {
        static const std::atomic_bool never{false};
        static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->read_vector(
            name, std::span<float>(output, count), never);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_gguf_checkpoint_check_unchanged(void* checkpoint) {
    try {
        static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->check_unchanged();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_gguf_checkpoint_integer(void* checkpoint, const char* key, uint64_t* value) {
    try {
        *value = static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->integer(key);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_gguf_checkpoint_number(void* checkpoint, const char* key, double* value) {
    try {
        *value = static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->number(key);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_gguf_checkpoint_boolean(void* checkpoint, const char* key, int* value) {
    try {
        *value = static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->boolean(key) ? 1 : 0;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// Copies the string (NUL-terminated, truncated to capacity - 1); returns its full length or -1.
int64_t ref_gguf_checkpoint_string(void* checkpoint, const char* key, char* buffer, size_t capacity) {
    try {
        const auto s = static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->string(key);
        if (capacity) {
            const size_t n = s.size() < capacity - 1 ? s.size() : capacity - 1;
            std::memcpy(buffer, s.data(), n);
            buffer[n] = '\0';
        }
        return int64_t(s.size());
    } catch (const std::exception& e) {
        fail(e);
        return -1;
    }
}

int ref_gguf_checkpoint_has(void* checkpoint, const char* key) {
    return static_cast<kadan::checkpoint::GgufCheckpoint*>(checkpoint)->has(key) ? 1 : 0;
}

// Safetensors shard (IW/include/kadan/checkpoint.hpp:91-178), default Limits,
// a 1 GiB metadata budget.
void* ref_shard_open(const char* root, const char* name) {
    try {
        return new kadan::checkpoint::Shard(root, name, std::make_shared<kadan::checkpoint::MemoryBudget>(1ull << 30));
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void ref_shard_close(void* shard) {
    delete static_cast<kadan::checkpoint::Shard*>(shard);
}

size_t ref_shard_tensor_count(void* shard) {
    return static_cast<kadan::checkpoint::Shard*>(shard)->tensor_count();
}

// info: dtype, rank, bytes, shape[8]; *name: the tensor's name (valid while the shard lives).
int ref_shard_tensor_at(void* shard, size_t index, uint64_t* info, const char** name, size_t* name_length) {
    try {
        const auto t = static_cast<kadan::checkpoint::Shard*>(shard)->tensor_at(index);
        info[0] = uint64_t(t.dtype), info[1] = t.rank, info[2] = t.bytes;
        for (int d = 0; d < 8; ++d)
            info[3 + d] = t.shape[d];
        *name = t.name.data();
        *name_length = t.name.size();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_shard_identity(void* shard, const char* name, uint64_t* identity) {
    try {
        const auto id = static_cast<kadan::checkpoint::Shard*>(shard)->tensor_identity(name);
        const uint64_t v[9] = {id.device, id.inode, id.file_size, id.modified_seconds, id.modified_nanoseconds,
                               id.changed_seconds, id.changed_nanoseconds, id.payload_begin, id.payload_end};
        std::memcpy(identity, v, sizeof(v));
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_shard_read_tensor(void* shard, const char* name, size_t offset, void* output, size_t bytes) {
    try {
        static_cast<kadan::checkpoint::Shard*>(shard)->read_tensor(
            name, offset, std::span<uint8_t>(static_cast<uint8_t*>(output), bytes));
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_shard_check_unchanged(void* shard) {
    try {
        static_cast<kadan::checkpoint::Shard*>(shard)->check_unchanged();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// Shard::load_mxfp4_expert_rows; copies the projection's packed codes and
// E8M0 scales out (capacities in bytes) and returns rows and columns in shape[2].
int ref_shard_load_mxfp4_expert_rows(void* shard, const char* prefix, size_t expert, size_t first, size_t count,
                                     size_t budget, uint8_t* weights, size_t weights_capacity, uint8_t* scales,
                                     size_t scales_capacity, uint64_t* shape) {
    try {
        const auto p = static_cast<kadan::checkpoint::Shard*>(shard)->load_mxfp4_expert_rows(prefix, expert, first,
                                                                                            count, budget);
        const auto v = p.view();
        if (v.weights.size() > weights_capacity || v.block_scales.size() > scales_capacity)
            throw std::length_error("shim_capacity");
        std::memcpy(weights, v.weights.data(), v.weights.size());
        std::memcpy(scales, v.block_scales.data(), v.block_scales.size());
        shape[0] = v.rows, shape[1] = v.columns;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}
}  // extern "C"
