// Tensor-pipe GEMV kernels (host entry points used by the batch dispatcher).
#pragma once

#include <vector>

#include "kadan_b200.h"

namespace kb200 {

// Q4_K or Q6_K job that the mma.sync kernels can take: 16-byte aligned rows
// of whole super-blocks, and the driver's tensor-map encoder is available.
bool mma_eligible(const kb200_gemv_job& job);
// Jobs of one encoding: one launch per 32 jobs; rows above the kernel's rows
// per pass (8 for Q4_K, 4 for Q6_K) become row groups.
int launch_mma(const std::vector<const kb200_gemv_job*>& jobs, cudaStream_t stream);

}  // namespace kb200
