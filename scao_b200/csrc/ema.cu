// Batched Kronecker curvature EMA (scao/preconditioner.py:341-353):
//   L <- rho * L + (1 - rho) * G G^T      (a x a, K = b)
//   R <- rho * R + (1 - rho) * G^T G      (b x b, K = a)
// for every active leaf block G (a view into the parameter's gradient), with
// the int8 storage of utils.py:170-203 fused: the GEMM epilogue dequantises the
// old code, forms the new fp32 value with the reference's separate roundings
// (x = fl(fl(fl(q*s)*rho) + fl(alpha*gram))), reduces max|x| per factor, and a
// second pass requantises with IEEE division (bit-exact with the CPU path for
// identical fp32 x).
//
// Only the lower triangle of tiles is computed; the epilogue mirrors it.
// This file holds the portable SIMT-FMA tile kernel; see gram_tc.cu for the
// tcgen05 tensor-core path used for 16-bit gradients.
#include "common.cuh"
#include "prof.cuh"

namespace {

constexpr int TM = 64;     // output tile edge
constexpr int TK = 16;     // K chunk
constexpr int NT = 256;    // threads

struct Prob {
    const void* g;     // param gradient base
    int dt;            // gradient dtype
    int n, K;          // output n x n, reduction K
    int side;          // 0: G G^T, 1: G^T G
    int64_t row0, col0, ld;
    int64_t fac_off;   // into fac arena
    float* x;          // fp32 scratch n*n (int8 mode)
    float* am_new;     // new absmax slot
    int pid;           // problem id (2*leaf+side)
};

__device__ Prob get_prob(const ScaoPlanDev& P, const int32_t* ids, int j,
                         float* xbuf, int64_t xstride, float* amnew) {
    Prob p;
    const int leaf = ids[j >> 1];
    const int side = j & 1;
    const ScaoLeaf& L = P.leaves[leaf];
    const ScaoParamStep& S = P.step[L.param];
    p.g = (const void*)S.g_ptr;
    p.dt = P.params[L.param].dtype;
    p.side = side;
    p.n = side ? L.b : L.a;
    p.K = side ? L.a : L.b;
    p.row0 = L.row0;
    p.col0 = L.col0;
    p.ld = L.ld;
    p.fac_off = side ? L.rq_off : L.lq_off;
    p.x = xbuf + (int64_t)j * xstride;
    p.am_new = amnew + j;
    p.pid = 2 * leaf + side;
    return p;
}

// A(i, k) of the factor product: side 0 -> G[i][k], side 1 -> G[k][i]
__device__ __forceinline__ float load_a(const Prob& p, int i, int k) {
    if (i >= p.n || k >= p.K) return 0.f;
    int64_t r = p.side ? k : i, c = p.side ? i : k;
    return load_dt(p.g, (p.row0 + r) * p.ld + p.col0 + c, p.dt);
}

__global__ void __launch_bounds__(NT)
gram_ema_simt_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                     float* xbuf, int64_t xstride, float* amnew, float rho_f,
                     float alpha_f) {
    const Prob p = get_prob(P, ids, blockIdx.y, xbuf, xstride, amnew);
    const int nt = (p.n + TM - 1) / TM;
    int t = blockIdx.x;
    if (t >= nt * (nt + 1) / 2) return;
    int ti = 0;
    while ((ti + 1) * (ti + 2) / 2 <= t) ++ti;
    const int tj = t - ti * (ti + 1) / 2;
    const int i0 = ti * TM, j0 = tj * TM;

    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TM + 4];
    __shared__ float red[32];
    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    float acc[4][4] = {};

    for (int k0 = 0; k0 < p.K; k0 += TK) {
        // 64 x 16 elements per operand, 4 per thread
        for (int e = tid; e < TM * TK; e += NT) {
            int ii, kk;
            if (p.side == 0) { ii = e >> 4; kk = e & 15; }   // contiguous along k
            else { kk = e >> 6; ii = e & 63; }               // contiguous along i
            As[kk][ii] = load_a(p, i0 + ii, k0 + kk);
            Bs[kk][ii] = load_a(p, j0 + ii, k0 + kk);
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            float4 a = *(const float4*)&As[kk][ty * 4];
            float4 b = *(const float4*)&Bs[kk][tx * 4];
            float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
        }
        __syncthreads();
    }

    // epilogue: EMA with the reference's separate roundings
    float mx = 0.f;
    float xv[4][4];
    if (P.int8_ema) {
        const int8_t* q = (const int8_t*)P.fac + p.fac_off;
        const float s_old = quant_scale_f(P.absmax[p.pid]);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
                float x = 0.f;
                if (i < p.n && j < p.n) {
                    const float deq = __fmul_rn((float)q[(int64_t)i * p.n + j], s_old);
                    x = __fadd_rn(__fmul_rn(deq, rho_f), __fmul_rn(alpha_f, acc[r][c]));
                }
                xv[r][c] = x;
                mx = fmaxf(mx, fabsf(x));
            }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
                if (i < p.n && j < p.n) {
                    p.x[(int64_t)i * p.n + j] = xv[r][c];
                    p.x[(int64_t)j * p.n + i] = xv[r][c];
                }
            }
        mx = block_max(mx, red);
        if (tid == 0) atomic_max_nonneg(p.am_new, mx);
    } else {
        float* L = (float*)P.fac + p.fac_off;
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
                float x = 0.f;
                if (i < p.n && j < p.n)
                    x = __fadd_rn(__fmul_rn(L[(int64_t)i * p.n + j], rho_f),
                                  __fmul_rn(alpha_f, acc[r][c]));
                xv[r][c] = x;
            }
        __syncthreads();   // all old values read before any mirrored write
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
                if (i < p.n && j < p.n) {
                    L[(int64_t)i * p.n + j] = xv[r][c];
                    L[(int64_t)j * p.n + i] = xv[r][c];
                }
            }
    }
}

__global__ void requant_batch_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                                     const float* __restrict__ xbuf, int64_t xstride,
                                     const float* __restrict__ amnew) {
    const int j = blockIdx.y;
    const int leaf = ids[j >> 1], side = j & 1;
    const ScaoLeaf& L = P.leaves[leaf];
    const int n = side ? L.b : L.a;
    const int64_t nn = (int64_t)n * n;
    const float am = amnew[j];
    const bool zero = (double)am < 1e-30;
    const float s = quant_scale_f(am);
    int8_t* q = (int8_t*)P.fac + (side ? L.rq_off : L.lq_off);
    const float* x = xbuf + (int64_t)j * xstride;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nn;
         e += (int64_t)gridDim.x * blockDim.x)
        q[e] = quant_one(x[e], s, zero);
    if (blockIdx.x == 0 && threadIdx.x == 0) P.absmax[2 * leaf + side] = am;
}

// Diagonal curvature (preconditioner.py:332-339):
//   diag_ema <- diag_ema * rho + (1 - rho) * g^2   (separately rounded)
__global__ void diag_ema_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                                float rho_f, float alpha_f) {
    const int pi = ids[blockIdx.y];
    const ScaoParam& pr = P.params[pi];
    const ScaoParamStep& S = P.step[pi];
    const void* g = (const void*)S.g_ptr;
    float* d = P.diag_ema + pr.offset;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < pr.numel;
         e += (int64_t)gridDim.x * blockDim.x) {
        const float gv = load_dt(g, e, pr.dtype);
        d[e] = __fadd_rn(__fmul_rn(d[e], rho_f), __fmul_rn(alpha_f, __fmul_rn(gv, gv)));
    }
}

}  // namespace

extern "C" int64_t scao_ema_scratch_bytes(int n_ids, int max_a, int max_b) {
    const int64_t mx = max_a > max_b ? max_a : max_b;
    return 2 * (int64_t)n_ids * (mx * mx * 4 + 256) + 256 * 4;
}

extern "C" int scao_plan_curvature(const ScaoPlanDev* P, const int32_t* leaf_ids,
                                   int n_ids, int max_a, int max_b, double rho,
                                   void* scratch, int64_t scratch_bytes,
                                   void* stream) {
    if (!P || n_ids < 0 || !scratch) return SCAO_ERR_ARG;
    if (n_ids == 0) return SCAO_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t mx = max_a > max_b ? max_a : max_b;
    const int64_t xstride = ((mx * mx + 63) / 64) * 64;          // floats
    const int64_t per_prob = xstride * 4 + 4;                    // bytes
    int64_t cap = (scratch_bytes - 1024) / per_prob;             // problems
    cap &= ~int64_t(1);
    if (cap < 2) return SCAO_ERR_ARG;
    const float rho_f = (float)rho;
    const float alpha_f = (float)(1.0 - rho);   // Python-float 1 - rho, then cast
    const int nt = (int)((mx + TM - 1) / TM);
    const int tiles = nt * (nt + 1) / 2;
    for (int64_t j0 = 0; j0 < 2 * (int64_t)n_ids; j0 += cap) {
        const int np = (int)((2 * (int64_t)n_ids - j0) < cap ? (2 * (int64_t)n_ids - j0) : cap);
        float* xbuf = (float*)scratch;
        float* amnew = (float*)((char*)scratch + cap * xstride * 4);
        if (P->int8_ema && cudaMemsetAsync(amnew, 0, np * sizeof(float), st) != cudaSuccess)
            return SCAO_ERR_LAUNCH;
        const int32_t* ids = leaf_ids + j0 / 2;
        dim3 grid(tiles, np);
        { ProfScope _ps(SLOT_GRAM_EMA, st); gram_ema_simt_kernel<<<grid, NT, 0, st>>>(*P, ids, xbuf, xstride, amnew,
                                                   rho_f, alpha_f); }
        SCAO_CHECK_LAUNCH();
        if (P->int8_ema) {
            dim3 g2((int)((mx * mx + 255) / 256 < 64 ? (mx * mx + 255) / 256 : 64), np);
            { ProfScope _ps(SLOT_REQUANT, st); requant_batch_kernel<<<g2, 256, 0, st>>>(*P, ids, xbuf, xstride, amnew); }
            SCAO_CHECK_LAUNCH();
        }
    }
    return SCAO_OK;
}

extern "C" int scao_plan_curvature_diag(const ScaoPlanDev* P,
                                        const int32_t* param_ids, int n_ids,
                                        double rho, void* stream) {
    if (!P || n_ids < 0) return SCAO_ERR_ARG;
    if (n_ids == 0) return SCAO_OK;
    dim3 grid(32, n_ids);
    { ProfScope _ps(SLOT_DIAG_EMA, (cudaStream_t)stream); diag_ema_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        *P, param_ids, (float)rho, (float)(1.0 - rho)); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}
