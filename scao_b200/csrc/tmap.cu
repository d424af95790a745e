// Host construction of the TMA tensor maps used by the tensor-core kernels
// (cuTensorMapEncodeTiled through the runtime's driver entry point; no
// link-time dependency on libcuda).
#include <cuda.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "tmap.cuh"

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

}  // namespace

bool scao_build_tensor_maps(const ScaoPlanDev* P, const ScaoParam* ph, const ScaoParamStep* sh,
                            cudaStream_t st) {
    static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
    EncodeTiledFn enc = encode_fn();
    if (!enc || !P->tmaps) return false;
    std::vector<CUtensorMap> maps((size_t)P->n_params * TMA_PER_PARAM);
    memset(maps.data(), 0, maps.size() * sizeof(CUtensorMap));
    auto encode = [&](CUtensorMap* m, CUtensorMapDataType t, int es, const void* base, int64_t rows,
                      int64_t cols, cuuint32_t bx, cuuint32_t by, CUtensorMapSwizzle sw) {
        const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
        const cuuint64_t strides[1] = {(cuuint64_t)cols * es};
        const cuuint32_t box[2] = {bx, by};
        const cuuint32_t estr[2] = {1, 1};
        return enc(m, t, 2, (void*)base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
               CUDA_SUCCESS;
    };
    const auto BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, F4 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const auto SW = CU_TENSOR_MAP_SWIZZLE_128B, NS = CU_TENSOR_MAP_SWIZZLE_NONE;
    const cuuint32_t SR = TMA_STATE_ROWS;
    for (int i = 0; i < P->n_params; ++i) {
        if (!scao_tmap_ok(ph[i], sh[i])) continue;
        CUtensorMap* m = &maps[(size_t)i * TMA_PER_PARAM];
        const int64_t r = ph[i].rows, c = ph[i].cols;
        const void* g = (const void*)sh[i].g_ptr;
        if (!encode(m + TM_G128, BF, 2, g, r, c, 64, 128, SW)) return false;
        if (!encode(m + TM_G64, BF, 2, g, r, c, 64, 64, SW)) return false;
        if (!encode(m + TM_GS, BF, 2, g, r, c, 128, SR, NS)) return false;
        if (!scao_tmap_state_ok(ph[i], sh[i])) continue;
        const int64_t o = ph[i].offset;
        if (!encode(m + TM_PS, BF, 2, (const void*)sh[i].p_ptr, r, c, 128, SR, NS)) return false;
        if (!encode(m + TM_US, BF, 2, P->upd + o, r, c, 128, SR, NS)) return false;
        if (!encode(m + TM_M, F4, 4, P->exp_avg + o, r, c, 128, SR, NS)) return false;
        if (!encode(m + TM_V, F4, 4, P->exp_avg_sq + o, r, c, 128, SR, NS)) return false;
        if (!encode(m + TM_D, F4, 4, P->exp_avg_diff + o, r, c, 128, SR, NS)) return false;
        if (!encode(m + TM_PV, F4, 4, P->prev_grad + o, r, c, 128, SR, NS)) return false;
        if (P->filt.mode && P->filt.mag_ema &&
            !encode(m + TM_MG, F4, 4, P->filt.mag_ema + o, r, c, 128, SR, NS))
            return false;
    }
    // pageable source: the copy is staged before cudaMemcpyAsync returns
    return cudaMemcpyAsync(P->tmaps, maps.data(), maps.size() * sizeof(CUtensorMap),
                           cudaMemcpyHostToDevice, st) == cudaSuccess;
}

int scao_sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

extern "C" int scao_plan_tensor_maps(const ScaoPlanDev* P, const ScaoParam* params_host,
                                     const ScaoParamStep* step_host, void* stream) {
    if (!P || !params_host || !step_host) return SCAO_ERR_ARG;
    return scao_build_tensor_maps(P, params_host, step_host, (cudaStream_t)stream) ? SCAO_OK
                                                                                   : SCAO_ERR_LAUNCH;
}
