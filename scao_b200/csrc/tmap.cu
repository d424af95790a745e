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
    std::vector<CUtensorMap> maps((size_t)P->n_params * 2);
    memset(maps.data(), 0, maps.size() * sizeof(CUtensorMap));
    for (int i = 0; i < P->n_params; ++i) {
        if (!scao_tmap_ok(ph[i], sh[i])) continue;
        const cuuint64_t dims[2] = {(cuuint64_t)ph[i].cols, (cuuint64_t)ph[i].rows};
        const cuuint64_t strides[1] = {(cuuint64_t)ph[i].cols * 2};
        const cuuint32_t es[2] = {1, 1};
        const cuuint32_t box0[2] = {64, 128}, box1[2] = {64, 64};
        if (enc(&maps[2 * i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)sh[i].g_ptr, dims,
                strides, box0, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
        if (enc(&maps[2 * i + 1], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)sh[i].g_ptr, dims,
                strides, box1, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
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
