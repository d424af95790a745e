// Known-answer check of the tcgen05 toolkit (tc.cuh): C = A * B^T for one
// 128 x N tile, bf16 inputs, fp32 accumulate in TMEM.  Exposed through the C
// ABI so the GPU tests can compare it with a float64 product.
#include <cuda_bf16.h>

#include "common.cuh"
#include "prof.cuh"
#include "tc.cuh"

namespace {

__global__ void __launch_bounds__(128)
tc_selftest_kernel(const uint16_t* __restrict__ A, const uint16_t* __restrict__ B,
                   float* __restrict__ C, int N, int K, int* err, int mn) {
    extern __shared__ __align__(1024) unsigned char sm[];
    unsigned char* sa = sm;                       // 128 x K
    unsigned char* sb = sm + 128 * K * 2;         // N x K
    __shared__ uint64_t mbar;
    __shared__ uint32_t tslot;
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int e = tid; e < 128 * K; e += 128) {
        const int r = e / K, k = e % K;
        *(uint16_t*)(sa + (mn ? canon_off_mn(r, k, 128) : canon_off(r, k, K))) = A[e];
    }
    for (int e = tid; e < N * K; e += 128) {
        const int r = e / K, k = e % K;
        *(uint16_t*)(sb + (mn ? canon_off_mn(r, k, N) : canon_off(r, k, K))) = B[e];
    }
    uint32_t ncols = 32;
    while ((int)ncols < N) ncols <<= 1;
    if (warp == 0) tc_alloc(&tslot, ncols);
    if (tid == 0) mbar_init(&mbar, 1);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    if (tid == 0) {
        const uint32_t idesc = idesc_bf16(128, N, mn, mn);
        for (int s = 0; s < K / 16; ++s) {
            uint64_t ad, bd;
            if (mn) {   // K step of 16 = two K groups of LBO = 16*M bytes
                ad = smem_desc(smem_u32(sa) + s * 2 * 16 * 128, 16 * 128, 128);
                bd = smem_desc(smem_u32(sb) + s * 2 * 16 * N, 16 * N, 128);
            } else {
                ad = smem_desc(smem_u32(sa) + s * 256, 128, 16 * K);
                bd = smem_desc(smem_u32(sb) + s * 256, 128, 16 * K);
            }
            tc_mma_bf16(tmem, ad, bd, idesc, s > 0);
        }
        tc_commit(&mbar);
    }
    const bool ok = mbar_wait(&mbar, 0);
    if (!ok && err) atomicExch(err, 1);
    tc_fence_after();
    if (ok) {
        const int row = warp * 32 + (tid & 31);
        for (int c0 = 0; c0 < N; c0 += 16) {
            float v[16];
            tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
            for (int c = 0; c < 16; ++c) C[row * N + c0 + c] = v[c];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, ncols);
}

}  // namespace

extern "C" int scao_tc_selftest(const uint16_t* A, const uint16_t* B, float* C, int N, int K,
                                int* err, int mn_major, void* stream) {
    if (!A || !B || !C || N < 16 || N > 256 || N % 16 || K < 16 || K > 128 || K % 16)
        return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t sm = (size_t)(128 + N) * K * 2;
    cudaFuncSetAttribute(tc_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    { ProfScope _ps(SLOT_SEAM, st); tc_selftest_kernel<<<1, 128, sm, st>>>(A, B, C, N, K, err, mn_major); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}

// Check of the division-by-constant rewrite used in the Adan update:
// counts elements where x*r + one FMA correction differs from IEEE x / c.
namespace {
__global__ void divc_check_kernel(const float* x, const float* c, int n, int* mism) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float cc = c[i & 1023];
        const float r = 1.0f / cc;
        const float q = x[i] * r;
        const float e = fmaf(-q, cc, x[i]);
        const float a = fmaf(e, r, q);
        if (__float_as_int(a) != __float_as_int(__fdiv_rn(x[i], cc))) atomicAdd(mism, 1);
    }
}
}  // namespace

extern "C" int scao_divc_check(const float* x, const float* c, int n, int* mismatches,
                               void* stream) {
    if (!x || !c || !mismatches || n <= 0) return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    { ProfScope _ps(SLOT_SEAM, st); divc_check_kernel<<<256, 256, 0, st>>>(x, c, n, mismatches); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}

namespace {

// An mbarrier wait that nobody satisfies: the bounded wait must give up,
// record the error in *err and return (no trap, the context stays usable).
__global__ void wait_timeout_kernel(int* err, uint32_t limit) {
    __shared__ uint64_t mbar;
    if (threadIdx.x == 0) {
        mbar_init(&mbar, 1);
        fence_async_smem();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool ok = mbar_wait(&mbar, 0, limit);
        *err = ok ? 0 : 1;
    }
}

}  // namespace

extern "C" int scao_wait_timeout_check(int* err, unsigned int limit, void* stream) {
    if (!err) return SCAO_ERR_ARG;
    { ProfScope _ps(SLOT_SEAM, (cudaStream_t)stream);
      wait_timeout_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(err, limit); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}
