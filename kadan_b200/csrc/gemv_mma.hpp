// Tensor-pipe GEMV kernels (host entry points used by the batch dispatcher).
#pragma once

#include <vector>

#include "kadan_b200.h"

namespace kb200 {

// Q4_K job that the mma.sync kernel can take: 16-byte aligned rows of whole
// super-blocks, and the driver's tensor-map encoder is available.
bool q4k_mma_eligible(const kb200_gemv_job& job);
// One launch per 32 jobs; rows above KB200_BATCH_ROWS become row groups.
int launch_q4k_mma(const std::vector<const kb200_gemv_job*>& jobs, cudaStream_t stream);

}  // namespace kb200
