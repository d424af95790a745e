// TMA tensor maps of the parameter gradients (host side).
#pragma once
#include <cuda_runtime.h>

#include "../../include/scao_b200.h"

// TMA_PER_PARAM maps per bf16 Kronecker parameter (all 2-D row-major
// rows x cols views) into P->tmaps, slot TM_* of parameter i at
// (i * TMA_PER_PARAM + TM_*) * 128 bytes:
//   TM_G128 / TM_G64   gradient, 128 x 64 and 64 x 64 boxes, 128-byte swizzle
//                      (tensor-core operands)
//   TM_GS, TM_PS, TM_US  gradient, parameter, bf16 update arena;
//   TM_M, TM_V, TM_D, TM_PV  exp_avg, exp_avg_sq, exp_avg_diff, prev_grad
//                      arenas: 16-row x 128-column boxes, no swizzle (state
//                      streaming of the apply kernel);
//   TM_MG              the gradient filter's magnitude EMA (when it is on).
// Zero fill out of bounds.  A parameter that is not bf16, not 16-byte
// aligned, or has no gradient this step gets zeroed maps (the kernels never
// read them: their eligibility tests are the same).  Returns false when the
// driver entry point is missing or an encode fails.
enum { TM_G128 = 0, TM_G64, TM_GS, TM_PS, TM_US, TM_M, TM_V, TM_D, TM_PV, TM_MG, TMA_PER_PARAM };
constexpr int TMA_STATE_ROWS = 16;
bool scao_build_tensor_maps(const ScaoPlanDev* P, const ScaoParam* params_host,
                            const ScaoParamStep* step_host, cudaStream_t st);

// same eligibility test as scao_build_tensor_maps, for the device
__host__ __device__ inline bool scao_tmap_ok(const ScaoParam& pr, const ScaoParamStep& s) {
    return pr.mode == 1 && pr.dtype == SCAO_BF16 && s.phase != 0 && s.g_ptr != 0 &&
           (pr.cols % 8) == 0 && (s.g_ptr & 15) == 0;
}

// the state-streaming maps (TM_PS .. TM_PV) of a parameter are valid
__host__ __device__ inline bool scao_tmap_state_ok(const ScaoParam& pr, const ScaoParamStep& s) {
    return scao_tmap_ok(pr, s) && s.p_ptr != 0 && (s.p_ptr & 15) == 0 && (pr.offset % 8) == 0;
}

__host__ __device__ inline const void* scao_tmap(const uint8_t* base, int param, int slot) {
    return base + ((size_t)param * TMA_PER_PARAM + slot) * 128;
}

int scao_sm_count();

// persistent-kernel grid: SMs minus the plan's reservation, at most `work`
inline int scao_persistent_grid(const ScaoPlanDev* P, long long work) {
    int n = scao_sm_count() - (P->sm_reserve > 0 ? P->sm_reserve : 0);
    if (n < 1) n = 1;
    return (int)(work < n ? work : n);
}
