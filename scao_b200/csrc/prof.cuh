// Launch accounting and optional per-kernel CUDA-event timing.
// Every kernel launch in the library sits inside a ProfScope: the launch is
// counted (scao_launch_count) and, when timing is enabled, bracketed by
// events recorded on the launching stream; scao_prof_read reports the summed
// device time per kernel slot.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

enum ScaoSlot {
    SLOT_PROJ = 0, SLOT_DIAG_PRE, SLOT_LEAF_COEF, SLOT_PARAM_PRE, SLOT_APPLY_KRON,
    SLOT_APPLY_FLAT, SLOT_PARAM_POST, SLOT_GLOBAL_NORM, SLOT_APPLY_P, SLOT_LOOKAHEAD,
    SLOT_GRAM_EMA, SLOT_REQUANT, SLOT_DIAG_EMA, SLOT_EIG_PREP, SLOT_EIG_DIAG,
    SLOT_EIG_GEMM, SLOT_EIG_JACOBI, SLOT_EIG_RESIDUAL, SLOT_EIG_CHOLINV, SLOT_EIG_RANK,
    SLOT_QUANT, SLOT_SEAM, SLOT_GRAM_TC, SLOT_TRANSPOSE, SLOT_FILTER, SLOT_EIG_ITER,
    SLOT_COUNT
};

void scao_prof_begin(int slot, cudaStream_t st);
void scao_prof_end(int slot, cudaStream_t st);
// While suspended (this host thread is capturing a CUDA graph), scopes neither
// record events nor count launches.
void scao_prof_suspend(int on);
// Count n kernel launches made by a graph launch.
void scao_prof_add_launches(int64_t n);

struct ProfScope {
    int slot;
    cudaStream_t st;
    ProfScope(int s, cudaStream_t stream) : slot(s), st(stream) { scao_prof_begin(slot, st); }
    ~ProfScope() { scao_prof_end(slot, st); }
};
