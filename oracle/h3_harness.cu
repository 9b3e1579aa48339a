// Test infrastructure only: the reference worker's own device GEMV path
// (services/hikari/inference_worker/src/cuda/h3_compute.cu: MatvecJob :110-121,
// append_row_groups :311-319, plan_matvec / launch_matvec :321-382, the
// gguf_matvec_batch_kernel it launches :243-257), compiled in place from the
// reference tree for sm_100a by oracle/Makefile (target ref-gpu) as the GPU
// baseline the product's kernels are measured against. Never part of the
// product; only the benchmark's reference-kernel case loads it.
#include <cstring>
#include <exception>
#include <vector>

#include "h3_compute.cu"

namespace {
thread_local char h3_error[256];
}

extern "C" {

const char* h3ref_last_error() {
    return h3_error;
}

// Device bytes one launch's job table needs per row group of 8 input rows.
size_t h3ref_job_bytes() {
    return sizeof(kadan::video::MatvecJob);
}

// One dependency group as the reference launches it: every job split into
// groups of 8 input rows, the table copied to `table` (device), one launch
// per encoding on the legacy stream. Pointers are device memory; encoding is
// kadan::gguf::Encoding's number, or -1 for F32 rows. Returns 0, or -1 with
// h3ref_last_error().
int h3ref_matvec_batch(const void* const* weights, const float* const* inputs, float* const* outputs,
                       const size_t* row_bytes, const unsigned* in, const unsigned* columns, const unsigned* rows,
                       const int* encodings, size_t count, void* table) {
    try {
        std::vector<kadan::video::MatvecJob> chunks;
        for (size_t i = 0; i < count; ++i) {
            const bool f32 = encodings[i] < 0;
            const kadan::video::MatvecJob job{static_cast<const unsigned char*>(weights[i]),
                                              inputs[i],
                                              outputs[i],
                                              nullptr,
                                              row_bytes[i],
                                              columns[i],
                                              in[i],
                                              columns[i],
                                              rows[i],
                                              0,
                                              f32 ? kadan::gguf::Encoding::q8_0
                                                  : static_cast<kadan::gguf::Encoding>(encodings[i]),
                                              f32};
            kadan::video::append_row_groups(job, chunks);
        }
        kadan::video::launch_matvec(chunks, static_cast<kadan::video::MatvecJob*>(table));
        return 0;
    } catch (const std::exception& e) {
        std::strncpy(h3_error, e.what(), sizeof(h3_error) - 1);
        return -1;
    }
}

}  // extern "C"
