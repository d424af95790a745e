// TMA tensor maps of the parameter gradients (host side).
#pragma once
#include <cuda_runtime.h>

#include "../../include/scao_b200.h"

// Two maps per bf16 Kronecker gradient (row-major rows x cols) into
// P->tmaps: [2i] boxes of 128 rows x 64 columns, [2i+1] boxes of 64 x 64;
// 128-byte swizzle, zero fill out of bounds.  A parameter that is not bf16,
// not 16-byte aligned, or has no gradient this step gets a zeroed map (the
// kernels never read it: their eligibility test is the same).  Returns
// false when the driver entry point is missing or an encode fails.
bool scao_build_tensor_maps(const ScaoPlanDev* P, const ScaoParam* params_host,
                            const ScaoParamStep* step_host, cudaStream_t st);

// same eligibility test as scao_build_tensor_maps, for the device
__host__ __device__ inline bool scao_tmap_ok(const ScaoParam& pr, const ScaoParamStep& s) {
    return pr.mode == 1 && pr.dtype == SCAO_BF16 && s.phase != 0 && s.g_ptr != 0 &&
           (pr.cols % 8) == 0 && (s.g_ptr & 15) == 0;
}

int scao_sm_count();
