// Batched on-device eigen update of the Kronecker factors
// (scao/preconditioner.py:363-451), without cuSOLVER.
//
// For every factor problem (2 per leaf: L a x a, R b x b):
//   A = dequant(q)/bias + eps*I,  eps = max(1e-8, 1e-4 * tr(L/bias) / n)
//                                               (preconditioner.py:383-406)
// and we need its top kmax eigenpairs (descending) plus the total spectral
// mass for rank selection (utils.py:121-151).
//
// * Exactly diagonal A (the int8 EMA stays at q = 127*I for the benchmark
//   gradient scales): LAPACK returns unit vectors ordered by ascending value,
//   flip makes them descending; for an all-equal diagonal that is the reversed
//   identity.  We emit the same basis directly (ties: larger index first).
// * Otherwise: warm-started subspace iteration on an s-column block
//   (s = n for n <= 160, else kpad + oversampling), one Rayleigh-Ritz step per
//   iteration (H = U^T A U solved by parallel cyclic Jacobi in shared memory),
//   residual test on the top kmax Ritz pairs, and a power step with
//   column-normalised CholeskyQR2 re-orthonormalisation.  The Ritz basis is
//   kept as the warm start for the next curvature step.
// All GEMMs here are batched SIMT FP32 tiles.
#include "common.cuh"
#include "prof.cuh"

namespace {

constexpr int NT = 256;
constexpr int TM = 64, TN = 64, TK = 16;
constexpr int SMAX = 160;   // max subspace width handled in shared memory

enum { AUX_SCALE = 0, AUX_BIAS, AUX_EPS, AUX_TOTAL, AUX_FLAGS, AUX_ITERS, AUX_RES };
enum { F_DIAG = 1, F_UNIFORM = 2, F_CONV = 4, F_CHOLFAIL = 8, F_DIRECT = 16 };
enum { BUF_U = 0, BUF_Y, BUF_X, BUF_AX, BUF_H, BUF_V, BUF_FAC };
enum { DIM_N = 0, DIM_S = 1 };

struct PInfo {
    int leaf, side, n, s, kmax;
    int64_t uoff, hoff, evoff, facoff;
    float* aux;
};

__device__ __forceinline__ PInfo pinfo(const ScaoPlanDev& P, const int32_t* ids, int j) {
    PInfo p;
    p.leaf = ids[j >> 1];
    p.side = j & 1;
    const ScaoLeaf& L = P.leaves[p.leaf];
    p.n = p.side ? L.b : L.a;
    p.s = p.side ? L.sr : L.sl;
    p.kmax = L.kmax;
    p.uoff = p.side ? L.ur_off : L.ul_off;
    p.hoff = p.side ? L.hr_off : L.hl_off;
    p.evoff = p.side ? L.evr_off : L.evl_off;
    p.facoff = p.side ? L.rq_off : L.lq_off;
    p.aux = P.eig_aux + (int64_t)(2 * p.leaf + p.side) * 16;
    return p;
}

__device__ __forceinline__ int flags_of(const PInfo& p) { return __float_as_int(p.aux[AUX_FLAGS]); }
__device__ __forceinline__ bool skip_iter(const PInfo& p) {
    return flags_of(p) & (F_DIAG | F_CONV);
}

// Element (i, k) of A = dequant(fac)/bias + eps*I with the reference's
// separate roundings (preconditioner.py:384-406).
__device__ __forceinline__ float fac_elem(const ScaoPlanDev& P, const PInfo& p, int i, int k) {
    const int64_t e = p.facoff + (int64_t)i * p.n + k;
    float x = P.int8_ema ? __fmul_rn((float)((const int8_t*)P.fac)[e], p.aux[AUX_SCALE])
                         : ((const float*)P.fac)[e];
    x = __fdiv_rn(x, p.aux[AUX_BIAS]);
    if (i == k) x = __fadd_rn(x, p.aux[AUX_EPS]);
    return x;
}

__device__ __forceinline__ float* buf_ptr(const ScaoPlanDev& P, const PInfo& p, int b, int* ld) {
    switch (b) {
        case BUF_U: *ld = p.s; return P.u + p.uoff;
        case BUF_Y: *ld = p.s; return P.eig_y + p.uoff;
        case BUF_X: *ld = p.s; return P.eig_x + p.uoff;
        case BUF_AX: *ld = p.s; return P.eig_ax + p.uoff;
        case BUF_H: *ld = p.s; return P.eig_h + p.hoff;
        case BUF_V: *ld = p.s; return P.eig_v + p.hoff;
    }
    *ld = 0;
    return nullptr;
}

struct GemmSpec {
    int a, b, c;         // buffers
    int m, n, k;         // dims (DIM_N / DIM_S)
    int trans_a;         // 1: A stored K x M
    int skip_direct;     // skip problems solved directly (s == n)
};

// ---------------------------------------------------------------------------
// prep: trace, Tikhonov eps, diagonal detection
// ---------------------------------------------------------------------------
__global__ void eig_prep_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                                const float* __restrict__ bias_factor) {
    const PInfo p = pinfo(P, ids, blockIdx.x);
    __shared__ double dred[32];
    __shared__ float fred[32];
    __shared__ int offnz, diffdiag;
    const float scale = P.int8_ema ? quant_scale_f(P.absmax[2 * p.leaf + p.side]) : 1.f;
    const float bias = fmaxf(bias_factor[p.leaf], 1e-8f);
    if (threadIdx.x == 0) { offnz = 0; diffdiag = 0; }
    __syncthreads();
    // trace of L/bias (fp32 values, accumulated in double)
    double tr = 0.0;
    for (int i = threadIdx.x; i < p.n; i += blockDim.x) {
        const int64_t e = p.facoff + (int64_t)i * p.n + i;
        float x = P.int8_ema ? __fmul_rn((float)((const int8_t*)P.fac)[e], scale)
                             : ((const float*)P.fac)[e];
        tr += (double)__fdiv_rn(x, bias);
    }
    tr = warp_sum_d(tr);
    if ((threadIdx.x & 31) == 0) dred[threadIdx.x >> 5] = tr;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += dred[w];
        const float trf = (float)t;
        double eps = 1e-4 * (double)trf / p.n;
        if (eps < 1e-8) eps = 1e-8;
        p.aux[AUX_SCALE] = scale;
        p.aux[AUX_BIAS] = bias;
        p.aux[AUX_EPS] = (float)eps;
    }
    __syncthreads();
    // diagonal / uniform detection and total = trace(A)
    int nz = 0;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (P.int8_ema) {
        const int8_t* q = (const int8_t*)P.fac + p.facoff;
        if ((p.n & 15) == 0) {
            // 16 codes per load; the diagonal byte is masked out
            const int nc = p.n >> 4;
            for (int i = wid; i < p.n; i += nw) {
                const uint4* row = (const uint4*)(q + (int64_t)i * p.n);
                for (int c = lane; c < nc; c += 32) {
                    uint4 v = row[c];
                    if (c == (i >> 4)) {
                        const int b = i & 15;
                        uint32_t* w = (uint32_t*)&v;
                        w[b >> 2] &= ~(0xFFu << ((b & 3) * 8));
                    }
                    if (v.x | v.y | v.z | v.w) nz = 1;
                }
            }
        } else {
            for (int i = wid; i < p.n; i += nw)
                for (int k = lane; k < p.n; k += 32)
                    if (i != k && q[(int64_t)i * p.n + k] != 0) nz = 1;
        }
    } else {
        const float* q = (const float*)P.fac + p.facoff;
        for (int i = wid; i < p.n; i += nw)
            for (int k = lane; k < p.n; k += 32)
                if (i != k && q[(int64_t)i * p.n + k] != 0.f) nz = 1;
    }
    if (__syncthreads_or(nz) && threadIdx.x == 0) offnz = 1;
    float total = 0.f;
    const float d0 = fac_elem(P, p, 0, 0);
    int dd = 0;
    for (int i = threadIdx.x; i < p.n; i += blockDim.x) {
        const float v = fac_elem(P, p, i, i);
        total += fmaxf(v, 0.f);
        if (v != d0) dd = 1;
    }
    if (__syncthreads_or(dd) && threadIdx.x == 0) diffdiag = 1;
    total = block_sum(total, fred);
    if (threadIdx.x == 0) {
        int fl = 0;
        if (!offnz) fl |= F_DIAG;
        if (!offnz && !diffdiag) fl |= F_UNIFORM;
        if (p.s >= p.n) fl |= F_DIRECT;
        p.aux[AUX_TOTAL] = total;
        p.aux[AUX_FLAGS] = __int_as_float(fl);
        p.aux[AUX_ITERS] = __int_as_float(0);
        p.aux[AUX_RES] = 0.f;
    }
}

// ---------------------------------------------------------------------------
// diagonal A: sorted unit-vector basis (bitonic sort in shared memory)
// ---------------------------------------------------------------------------
__global__ void eig_diag_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids) {
    const PInfo p = pinfo(P, ids, blockIdx.x);
    if (!(flags_of(p) & F_DIAG)) return;
    extern __shared__ unsigned char smem_raw[];
    float* val = (float*)smem_raw;
    int* idx = (int*)(val + 4096);
    int np2 = 1;
    while (np2 < p.n) np2 <<= 1;
    for (int i = threadIdx.x; i < np2; i += blockDim.x) {
        if (i < p.n) { val[i] = fac_elem(P, p, i, i); idx[i] = i; }
        else { val[i] = -INFINITY; idx[i] = -1; }
    }
    __syncthreads();
    // sort descending by (value, index)
    for (int k = 2; k <= np2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < np2; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const bool desc = (i & k) == 0;
                    const bool i_before_l = (val[i] > val[l]) || (val[i] == val[l] && idx[i] > idx[l]);
                    if (desc != i_before_l) {
                        float tv = val[i]; val[i] = val[l]; val[l] = tv;
                        int ti = idx[i]; idx[i] = idx[l]; idx[l] = ti;
                    }
                }
            }
            __syncthreads();
        }
    }
    float* U = P.u + p.uoff;
    const int64_t ns = (int64_t)p.n * p.s;
    for (int64_t e = threadIdx.x; e < ns; e += blockDim.x) U[e] = 0.f;
    __syncthreads();
    float* ev = P.ev + p.evoff;
    for (int c = threadIdx.x; c < p.s; c += blockDim.x) {
        if (c < p.n) {
            U[(int64_t)idx[c] * p.s + c] = 1.f;
            ev[c] = fmaxf(val[c], 0.f);
        } else {
            ev[c] = 0.f;
        }
    }
    if (threadIdx.x == 0) {
        p.aux[AUX_FLAGS] = __int_as_float(flags_of(p) | F_CONV);
        p.aux[AUX_ITERS] = __int_as_float(0);
    }
}

// ---------------------------------------------------------------------------
// batched GEMM  C = op(A) * B  (A may be the transformed factor matrix)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
eig_gemm_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, GemmSpec g) {
    const PInfo p = pinfo(P, ids, blockIdx.y);
    if (skip_iter(p)) return;
    if (g.skip_direct && (flags_of(p) & F_DIRECT)) return;
    const int M = g.m == DIM_N ? p.n : p.s;
    const int N = g.n == DIM_N ? p.n : p.s;
    const int K = g.k == DIM_N ? p.n : p.s;
    const int tn = (N + TN - 1) / TN;
    const int tm = (M + TM - 1) / TM;
    if ((int)blockIdx.x >= tm * tn) return;
    const int i0 = (blockIdx.x / tn) * TM, j0 = (blockIdx.x % tn) * TN;
    int lda = 0, ldb, ldc;
    const float* A = g.a == BUF_FAC ? nullptr : buf_ptr(P, p, g.a, &lda);
    const float* B = buf_ptr(P, p, g.b, &ldb);
    float* C = buf_ptr(P, p, g.c, &ldc);

    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += TK) {
        for (int e = tid; e < TM * TK; e += NT) {
            int ii, kk;
            if (g.trans_a) { kk = e >> 6; ii = e & 63; } else { ii = e >> 4; kk = e & 15; }
            const int i = i0 + ii, k = k0 + kk;
            float v = 0.f;
            if (i < M && k < K) {
                if (g.a == BUF_FAC) v = fac_elem(P, p, i, k);
                else v = g.trans_a ? A[(int64_t)k * lda + i] : A[(int64_t)i * lda + k];
            }
            As[kk][ii] = v;
        }
        for (int e = tid; e < TN * TK; e += NT) {
            const int kk = e >> 6, jj = e & 63;
            const int k = k0 + kk, j = j0 + jj;
            Bs[kk][jj] = (k < K && j < N) ? B[(int64_t)k * ldb + j] : 0.f;
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
    const bool fail = (flags_of(p) & F_CHOLFAIL) && g.c == BUF_U;
    float* X = P.eig_x + p.uoff;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
            if (i < M && j < N)
                C[(int64_t)i * ldc + j] = fail ? X[(int64_t)i * p.s + j] : acc[r][c];
        }
}

// ---------------------------------------------------------------------------
// Rayleigh-Ritz: parallel cyclic Jacobi on H (s x s) -> V, theta (descending)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
eig_jacobi_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, int max_sweeps) {
    const PInfo p = pinfo(P, ids, blockIdx.x);
    if (skip_iter(p)) return;
    extern __shared__ float sm[];
    const int s = p.s;
    const int se = s + (s & 1);          // even size (dummy index if odd)
    const int ld = se + 1;
    float* H = sm;                       // se x ld
    float* V = H + se * ld;              // se x ld
    float* cs = V + se * ld;             // se/2 cos
    float* sn = cs + se / 2;             // se/2 sin
    int* pp = (int*)(sn + se / 2);       // se/2
    int* qq = pp + se / 2;               // se/2
    float* red = (float*)(qq + se / 2);  // 32
    int ldh;
    const float* Hg = buf_ptr(P, p, BUF_H, &ldh);
    for (int e = threadIdx.x; e < se * se; e += blockDim.x) {
        const int i = e / se, j = e % se;
        float h = 0.f;
        if (i < s && j < s) h = 0.5f * (Hg[i * ldh + j] + Hg[j * ldh + i]);
        H[i * ld + j] = h;
        V[i * ld + j] = (i == j) ? 1.f : 0.f;
    }
    __syncthreads();
    const int half = se / 2;
    for (int sweep = 0; sweep < max_sweeps; ++sweep) {
        float off = 0.f, fro = 0.f;
        for (int e = threadIdx.x; e < se * se; e += blockDim.x) {
            const int i = e / se, j = e % se;
            const float h = H[i * ld + j];
            fro += h * h;
            if (i != j) off += h * h;
        }
        off = block_sum(off, red);
        fro = block_sum(fro, red);
        if (off <= 1e-14f * fro || fro == 0.f) break;
        for (int round = 0; round < se - 1; ++round) {
            // round-robin tournament pairing of se players
            for (int t = threadIdx.x; t < half; t += blockDim.x) {
                // circle method: player 0 fixed, players 1..se-1 rotate
                int a, b;
                if (t == 0) { a = 0; b = 1 + round % (se - 1); }
                else {
                    a = 1 + (t + round) % (se - 1);
                    b = 1 + (se - 1 - t + round) % (se - 1);
                }
                const int P0 = a < b ? a : b, Q0 = a < b ? b : a;
                pp[t] = P0; qq[t] = Q0;
                const float apq = H[P0 * ld + Q0];
                float c = 1.f, sv = 0.f;
                if (fabsf(apq) > 1e-30f) {
                    const float app = H[P0 * ld + P0], aqq = H[Q0 * ld + Q0];
                    const float theta = (aqq - app) / (2.f * apq);
                    const float tt = (theta >= 0.f ? 1.f : -1.f) /
                                     (fabsf(theta) + sqrtf(theta * theta + 1.f));
                    c = rsqrtf(tt * tt + 1.f);
                    sv = tt * c;
                }
                cs[t] = c; sn[t] = sv;
            }
            __syncthreads();
            // rows: H <- J^T H
            for (int e = threadIdx.x; e < half * se; e += blockDim.x) {
                const int t = e / se, k = e % se;
                const int P0 = pp[t], Q0 = qq[t];
                const float c = cs[t], sv = sn[t];
                const float hp = H[P0 * ld + k], hq = H[Q0 * ld + k];
                H[P0 * ld + k] = c * hp - sv * hq;
                H[Q0 * ld + k] = sv * hp + c * hq;
            }
            __syncthreads();
            // cols: H <- H J, V <- V J
            for (int e = threadIdx.x; e < half * se; e += blockDim.x) {
                const int t = e / se, k = e % se;
                const int P0 = pp[t], Q0 = qq[t];
                const float c = cs[t], sv = sn[t];
                const float hp = H[k * ld + P0], hq = H[k * ld + Q0];
                H[k * ld + P0] = c * hp - sv * hq;
                H[k * ld + Q0] = sv * hp + c * hq;
                const float vp = V[k * ld + P0], vq = V[k * ld + Q0];
                V[k * ld + P0] = c * vp - sv * vq;
                V[k * ld + Q0] = sv * vp + c * vq;
            }
            __syncthreads();
        }
    }
    // sort eigenvalues descending (ties: lower index first), permute V
    int* rank = (int*)cs;  // reuse: se ints (cs+sn region holds se floats)
    for (int i = threadIdx.x; i < s; i += blockDim.x) {
        const float di = H[i * ld + i];
        int r = 0;
        for (int j = 0; j < s; ++j) {
            const float dj = H[j * ld + j];
            if (dj > di || (dj == di && j < i)) ++r;
        }
        rank[i] = r;
    }
    __syncthreads();
    int ldv;
    float* Vg = buf_ptr(P, p, BUF_V, &ldv);
    float* ev = P.ev + p.evoff;
    for (int e = threadIdx.x; e < s * s; e += blockDim.x) {
        const int i = e / s, j = e % s;   // V[i][j] -> Vg[i][rank[j]]
        Vg[i * ldv + rank[j]] = V[i * ld + j];
    }
    for (int j = threadIdx.x; j < s; j += blockDim.x) ev[rank[j]] = H[j * ld + j];
}

// ---------------------------------------------------------------------------
// residuals of the top kmax Ritz pairs; convergence; column normalisation
// ---------------------------------------------------------------------------
__global__ void eig_residual_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                                    float tol, int iter, int last) {
    const PInfo p = pinfo(P, ids, blockIdx.x);
    if (skip_iter(p)) return;
    __shared__ float red[32];
    __shared__ float colnorm[SMAX];
    const float* X = P.eig_x + p.uoff;
    float* AX = P.eig_ax + p.uoff;
    const float* ev = P.ev + p.evoff;
    const int s = p.s;
    float rmax = 0.f;
    // one warp per column
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int c = wid; c < s; c += nw) {
        const float th = ev[c];
        float r2 = 0.f, a2 = 0.f;
        for (int i = lane; i < p.n; i += 32) {
            const float ax = AX[(int64_t)i * s + c];
            const float d = ax - th * X[(int64_t)i * s + c];
            r2 += d * d;
            a2 += ax * ax;
        }
        r2 = warp_sum(r2);
        a2 = warp_sum(a2);
        if (lane == 0) colnorm[c] = sqrtf(a2);
        if (c < p.kmax) rmax = fmaxf(rmax, sqrtf(r2));
    }
    rmax = block_max(rmax, red);
    const float scale = fmaxf(fabsf(ev[0]), 1e-30f);
    const int fl = flags_of(p);
    const bool conv = (fl & F_DIRECT) || rmax <= tol * scale || last;
    __syncthreads();
    float* U = P.u + p.uoff;
    const int64_t ns = (int64_t)p.n * s;
    if (conv) {
        for (int64_t e = threadIdx.x; e < ns; e += blockDim.x) U[e] = X[e];
    } else {
        for (int64_t e = threadIdx.x; e < ns; e += blockDim.x) {
            const int c = (int)(e % s);
            const float nrm = colnorm[c];
            AX[e] = nrm > 0.f ? AX[e] / nrm : 0.f;
        }
    }
    if (threadIdx.x == 0) {
        int f = fl & ~F_CHOLFAIL;
        if (conv) f |= F_CONV;
        p.aux[AUX_FLAGS] = __int_as_float(f);
        p.aux[AUX_ITERS] = __int_as_float(iter + 1);
        p.aux[AUX_RES] = rmax / scale;
        if (conv && !(fl & F_DIRECT) && rmax > tol * scale)
            p.aux[AUX_ITERS] = __int_as_float(-(iter + 1));   // cap reached
    }
}

// ---------------------------------------------------------------------------
// CholeskyQR helper: H = Gram (s x s) -> H = R^{-1} (upper), G = R^T R
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
eig_cholinv_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids) {
    const PInfo p = pinfo(P, ids, blockIdx.x);
    if (skip_iter(p) || (flags_of(p) & F_DIRECT)) return;
    extern __shared__ float sm[];
    const int s = p.s, ld = s + 1;
    float* R = sm;            // s x ld
    float* X = R + s * ld;    // s x ld
    __shared__ int fail;
    int ldh;
    float* Hg = buf_ptr(P, p, BUF_H, &ldh);
    for (int e = threadIdx.x; e < s * s; e += blockDim.x) {
        const int i = e / s, j = e % s;
        R[i * ld + j] = 0.5f * (Hg[i * ldh + j] + Hg[j * ldh + i]);
    }
    if (threadIdx.x == 0) fail = 0;
    __syncthreads();
    float tr = 0.f;
    for (int i = 0; i < s; ++i) tr += R[i * ld + i];
    // right-looking Cholesky, upper factor R (row k holds R[k][k..])
    for (int k = 0; k < s; ++k) {
        if (threadIdx.x == 0) {
            const float d = R[k * ld + k];
            if (!(d > 1e-12f * tr)) fail = 1;
            R[k * ld + k] = sqrtf(fmaxf(d, 1e-30f));
        }
        __syncthreads();
        const float rkk = R[k * ld + k];
        for (int j = k + 1 + threadIdx.x; j < s; j += blockDim.x) R[k * ld + j] /= rkk;
        __syncthreads();
        for (int e = threadIdx.x; e < (s - k - 1) * (s - k - 1); e += blockDim.x) {
            const int i = k + 1 + e / (s - k - 1), j = k + 1 + e % (s - k - 1);
            if (j >= i) R[i * ld + j] -= R[k * ld + i] * R[k * ld + j];
        }
        __syncthreads();
    }
    // X = R^{-1}: column j solves R x = e_j (back substitution)
    for (int j = threadIdx.x; j < s; j += blockDim.x) {
        for (int i = s - 1; i >= 0; --i) {
            float v = (i == j) ? 1.f : 0.f;
            if (i <= j) {
                for (int k = i + 1; k <= j; ++k) v -= R[i * ld + k] * X[k * ld + j];
                v /= R[i * ld + i];
            } else {
                v = 0.f;
            }
            X[i * ld + j] = v;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < s * s; e += blockDim.x) {
        const int i = e / s, j = e % s;
        Hg[i * ldh + j] = X[i * ld + j];
    }
    if (threadIdx.x == 0 && fail)
        p.aux[AUX_FLAGS] = __int_as_float(flags_of(p) | F_CHOLFAIL);
}

// ---------------------------------------------------------------------------
// rank selection (utils.py:121-151) + hysteresis (preconditioner.py:434-441)
// ---------------------------------------------------------------------------
__device__ int adaptive_rank_dev(const float* ev, int cnt, int n, float total,
                                 float eps_sparse, int kmin, int kmax) {
    if ((double)total < 1e-12) return kmin;
    const float thr = (float)((1.0 - (double)eps_sparse) * (double)total);
    double cum = 0.0;
    int k = -1;
    for (int c = 0; c < cnt; ++c) {
        cum += (double)fmaxf(ev[c], 0.f);
        if ((float)cum >= thr) { k = c + 1; break; }
    }
    if (k < 0) k = (cnt >= n) ? n : cnt + 1;
    return min(kmax, max(kmin, k));
}

__global__ void eig_rank_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, int n_ids,
                                const float* __restrict__ eps_sparse,
                                int32_t* __restrict__ status) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n_ids) return;
    const int leaf = ids[j];
    const ScaoLeaf& L = P.leaves[leaf];
    const float* auxl = P.eig_aux + (int64_t)(2 * leaf) * 16;
    const float* auxr = auxl + 16;
    const int kl = adaptive_rank_dev(P.ev + L.evl_off, min(L.sl, L.a), L.a, auxl[AUX_TOTAL],
                                     eps_sparse[leaf], L.kmin, L.kmax);
    const int kr = adaptive_rank_dev(P.ev + L.evr_off, min(L.sr, L.b), L.b, auxr[AUX_TOTAL],
                                     eps_sparse[leaf], L.kmin, L.kmax);
    const int kprev = P.k[leaf];
    int kn = min(kl, kr);
    kn = max(kn, kprev - 1);
    kn = min(kn, kprev + 4);
    kn = min(L.kmax, max(L.kmin, kn));
    P.k[leaf] = kn;
    if (status) {
        status[2 * j] = __float_as_int(auxl[AUX_ITERS]);
        status[2 * j + 1] = __float_as_int(auxr[AUX_ITERS]);
    }
}

// number of problems that still need the iterative solver
__global__ void eig_count_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, int np) {
    int c = 0;
    for (int j = threadIdx.x; j < np; j += blockDim.x) {
        const PInfo p = pinfo(P, ids, j);
        if (!skip_iter(p)) ++c;
    }
    __shared__ int tot;
    if (threadIdx.x == 0) tot = 0;
    __syncthreads();
    atomicAdd(&tot, c);
    __syncthreads();
    if (threadIdx.x == 0) P.counters[0] = tot;
}

size_t jacobi_smem(int s) {
    const int se = s + (s & 1), ld = se + 1;
    return (size_t)(2 * se * ld + 2 * se) * 4 + 32 * 4 + 64;
}

}  // namespace

// smax / nmax: largest subspace width / factor size among the listed leaves.
extern "C" int scao_plan_eigen(const ScaoPlanDev* P, const int32_t* leaf_ids, int n_ids,
                                  const float* bias_factor, const float* eps_sparse,
                                  int max_iters, float tol, int32_t* status,
                                  int nmax, int smax, void* stream) {
    if (!P || n_ids < 0 || smax > SMAX || nmax > 4096) return SCAO_ERR_ARG;
    if (n_ids == 0) return SCAO_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const int np = 2 * n_ids;
    { ProfScope _ps(SLOT_EIG_PREP, st); eig_prep_kernel<<<np, NT, 0, st>>>(*P, leaf_ids, bias_factor); }
    SCAO_CHECK_LAUNCH();
    const size_t dsm = 4096 * 8;
    { ProfScope _ps(SLOT_EIG_DIAG, st); eig_diag_kernel<<<np, NT, dsm, st>>>(*P, leaf_ids); }
    SCAO_CHECK_LAUNCH();
    // all factors exactly diagonal (the common int8 case): skip the iterations
    int n_iter = 0;
    { ProfScope _ps(SLOT_EIG_PREP, st); eig_count_kernel<<<1, 256, 0, st>>>(*P, leaf_ids, np); }
    SCAO_CHECK_LAUNCH();
    if (cudaMemcpyAsync(&n_iter, P->counters, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return SCAO_ERR_LAUNCH;
    if (n_iter == 0) max_iters = 0;
    const size_t jsm = jacobi_smem(smax);
    const size_t csm = (size_t)2 * smax * (smax + 1) * 4;
    static PerDeviceOnce attr_done;
    if (attr_done.first()) {
        cudaFuncSetAttribute(eig_jacobi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)jacobi_smem(SMAX));
        cudaFuncSetAttribute(eig_cholinv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)((size_t)2 * SMAX * (SMAX + 1) * 4));
    }
    const int tiles_nn = ((nmax + TM - 1) / TM) * ((smax + TN - 1) / TN);
    const int tiles_ss = ((smax + TM - 1) / TM) * ((smax + TN - 1) / TN);
    for (int it = 0; it < max_iters; ++it) {
        const int last = (it == max_iters - 1);
        GemmSpec g;
        // Y = A U
        g = {BUF_FAC, BUF_U, BUF_Y, DIM_N, DIM_S, DIM_N, 0, 0};
        { ProfScope _ps(SLOT_EIG_GEMM, st); eig_gemm_kernel<<<dim3(tiles_nn, np), NT, 0, st>>>(*P, leaf_ids, g); }
        SCAO_CHECK_LAUNCH();
        // H = U^T Y
        g = {BUF_U, BUF_Y, BUF_H, DIM_S, DIM_S, DIM_N, 1, 0};
        { ProfScope _ps(SLOT_EIG_GEMM, st); eig_gemm_kernel<<<dim3(tiles_ss, np), NT, 0, st>>>(*P, leaf_ids, g); }
        SCAO_CHECK_LAUNCH();
        { ProfScope _ps(SLOT_EIG_JACOBI, st); eig_jacobi_kernel<<<np, NT, jsm, st>>>(*P, leaf_ids, 30); }
        SCAO_CHECK_LAUNCH();
        // X = U V, AX = Y V
        g = {BUF_U, BUF_V, BUF_X, DIM_N, DIM_S, DIM_S, 0, 0};
        { ProfScope _ps(SLOT_EIG_GEMM, st); eig_gemm_kernel<<<dim3(tiles_nn, np), NT, 0, st>>>(*P, leaf_ids, g); }
        SCAO_CHECK_LAUNCH();
        g = {BUF_Y, BUF_V, BUF_AX, DIM_N, DIM_S, DIM_S, 0, 0};
        { ProfScope _ps(SLOT_EIG_GEMM, st); eig_gemm_kernel<<<dim3(tiles_nn, np), NT, 0, st>>>(*P, leaf_ids, g); }
        SCAO_CHECK_LAUNCH();
        { ProfScope _ps(SLOT_EIG_RESIDUAL, st); eig_residual_kernel<<<np, NT, 0, st>>>(*P, leaf_ids, tol, it, last); }
        SCAO_CHECK_LAUNCH();
        if (last) break;
        // CholeskyQR2 of the normalised AX: AX -> Y -> U
        g = {BUF_AX, BUF_AX, BUF_H, DIM_S, DIM_S, DIM_N, 1, 1};
        { ProfScope _ps(SLOT_EIG_GEMM, st); eig_gemm_kernel<<<dim3(tiles_ss, np), NT, 0, st>>>(*P, leaf_ids, g); }
        SCAO_CHECK_LAUNCH();
        { ProfScope _ps(SLOT_EIG_CHOLINV, st); eig_cholinv_kernel<<<np, NT, csm, st>>>(*P, leaf_ids); }
        SCAO_CHECK_LAUNCH();
        g = {BUF_AX, BUF_H, BUF_Y, DIM_N, DIM_S, DIM_S, 0, 1};
        { ProfScope _ps(SLOT_EIG_GEMM, st); eig_gemm_kernel<<<dim3(tiles_nn, np), NT, 0, st>>>(*P, leaf_ids, g); }
        SCAO_CHECK_LAUNCH();
        g = {BUF_Y, BUF_Y, BUF_H, DIM_S, DIM_S, DIM_N, 1, 1};
        { ProfScope _ps(SLOT_EIG_GEMM, st); eig_gemm_kernel<<<dim3(tiles_ss, np), NT, 0, st>>>(*P, leaf_ids, g); }
        SCAO_CHECK_LAUNCH();
        { ProfScope _ps(SLOT_EIG_CHOLINV, st); eig_cholinv_kernel<<<np, NT, csm, st>>>(*P, leaf_ids); }
        SCAO_CHECK_LAUNCH();
        g = {BUF_Y, BUF_H, BUF_U, DIM_N, DIM_S, DIM_S, 0, 1};
        { ProfScope _ps(SLOT_EIG_GEMM, st); eig_gemm_kernel<<<dim3(tiles_nn, np), NT, 0, st>>>(*P, leaf_ids, g); }
        SCAO_CHECK_LAUNCH();
    }
    { ProfScope _ps(SLOT_EIG_RANK, st); eig_rank_kernel<<<(n_ids + 127) / 128, 128, 0, st>>>(*P, leaf_ids, n_ids, eps_sparse, status); }
    SCAO_CHECK_LAUNCH();
    return scao_plan_prep_factors(P, leaf_ids, n_ids, stream);
}
