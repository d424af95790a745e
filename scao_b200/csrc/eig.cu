// Batched on-device eigen update of the Kronecker factors
// (scao/preconditioner.py:363-451), without cuSOLVER.
//
// For every factor problem (2 per leaf: L a x a, R b x b):
//   A = dequant(q)/bias + eps*I,  eps = max(1e-8, 1e-4 * tr(L/bias) / n)
//                                               (preconditioner.py:383-406)
// and we need its top eigenpairs (descending) plus the total spectral mass
// for rank selection (utils.py:121-151).
//
// * Exactly diagonal A (the int8 EMA stays at q = 127*I for small gradient
//   scales): LAPACK returns unit vectors ordered by ascending value, flip
//   makes them descending; for an all-equal diagonal that is the reversed
//   identity.  We emit the same basis directly (ties: larger index first).
// * Otherwise: warm-started, Chebyshev-filtered subspace iteration on an
//   s-column block (s = n for n <= 160, else kpad + oversampling; Zhou & Saad,
//   "Self-consistent-field calculations using Chebyshev-filtered subspace
//   iteration", J. Comput. Phys. 219, 2006, scaled three-term recurrence).
//   One outer iteration = a Rayleigh-Ritz step (Y = A U, H = U^T Y solved by
//   parallel cyclic Jacobi in shared memory, X = U V, AX = Y V), a residual
//   test, then a degree-CHEB_M Chebyshev filter that damps [min(0, theta_s),
//   theta_s] (theta_s: the smallest Ritz value of the block) and
//   re-orthonormalisation by column-scaled CholeskyQR2.
// * Convergence is tested only on the Ritz pairs the rank update can use:
//   k_new <= min(kmax, k_prev + 4) (preconditioner.py:437-441), so pairs
//   beyond that never reach the output.  Pairs whose Ritz value lies within
//   CLUSTER_FRAC of theta_s belong to the flat bulk of the spectrum, where
//   individual eigenvectors are not resolvable at any accuracy: they are
//   exempt from the residual test (their Ritz values still converge).
// * Every GEMM runs on the tensor cores (tcgen05.mma kind::f16, fp32
//   accumulators in TMEM): fp32 operands are split into three bf16 parts
//   (x = hi + mid + lo exactly, 24 significant bits), int8 factor codes are
//   exact in bf16, so the products reproduce fp32 GEMMs to ~2^-22.
// * The iteration runs as a CUDA graph with a conditional WHILE node: a
//   control kernel at the end of each outer iteration clears the loop
//   condition once every problem has converged (or the iteration cap is
//   reached), so the host never waits for the device.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "prof.cuh"
#include "tc.cuh"

namespace {

constexpr int NT = 256;
constexpr int SMAX = 160;   // max subspace width handled in shared memory
constexpr int CHEB_M = 3;   // Chebyshev filter degree per outer iteration
constexpr float CLUSTER_FRAC = 0.05f;
constexpr float VAL_TOL = 1e-3f;    // per-pair residual bound (relative to theta_1)
constexpr float GAP_REL = 1e-2f;    // a spectral gap this large (relative) ends a prefix

enum { AUX_SCALE = 0, AUX_BIAS, AUX_EPS, AUX_TOTAL, AUX_FLAGS, AUX_ITERS, AUX_RES,
       AUX_CC, AUX_CE, AUX_CS, AUX_NFAIL, AUX_DEG, AUX_WARM };
enum { F_DIAG = 1, F_UNIFORM = 2, F_CONV = 4, F_CHOLFAIL = 8, F_DIRECT = 16 };
enum { BUF_U = 0, BUF_Y, BUF_X, BUF_AX, BUF_H, BUF_V, BUF_FAC };
enum { DIM_N = 0, DIM_S = 1 };
// device counters (ScaoPlanDev::counters)
enum { CNT_ITER = 2, CNT_ACTIVE = 3 };

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
        p.aux[AUX_NFAIL] = 0.f;
        p.aux[AUX_DEG] = (float)CHEB_M;
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
        p.aux[AUX_WARM] = 0.f;      // U is a unit-vector basis: not a warm start
    }
}

// ---------------------------------------------------------------------------
// start basis.  Direct problems (s >= n) use the reversed identity.  A problem whose
// U is not the result of an earlier iterative
// solve (the initial reversed identity, or the unit-vector basis of the
// diagonal shortcut) starts from a dense orthonormal basis instead.  Unit
// vectors can span an exactly invariant subspace of A (rows the gradient
// signal never reached), which subspace iteration would never leave.  The
// basis: orthonormal DCT-II columns (frequencies 0..s-1) with the rows
// permuted by i -> (a i + b) mod n and random signs -- still orthonormal,
// dense, and in general position.
// ---------------------------------------------------------------------------
SCAO_DEV uint32_t mix32(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352dU; x ^= x >> 15; x *= 0x846ca68bU; x ^= x >> 16;
    return x;
}

__global__ void eig_cold_start_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids) {
    const PInfo p = pinfo(P, ids, blockIdx.y);
    const int fl = flags_of(p);
    if (fl & F_DIAG) return;
    const int n = p.n, s = p.s;
    if (fl & F_DIRECT) {
        // direct solve (s >= n): the basis is the reversed identity, so the
        // Rayleigh-Ritz matrix is A with its index order reversed, formed
        // exactly (products with 1 and 0); with the Jacobi solver's tie rule
        // (lower index first) near-degenerate eigenvalues come out in LAPACK's
        // order (ascending index after the descending flip)
        float* U = P.u + p.uoff;
        for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < (int64_t)n * s;
             e += (int64_t)gridDim.x * blockDim.x)
            U[e] = ((int)(e / s) == n - 1 - (int)(e % s)) ? 1.f : 0.f;
        return;
    }
    if (p.aux[AUX_WARM] != 0.f) return;
    const uint32_t key = mix32(0x9e3779b9U * (uint32_t)(2 * p.leaf + p.side + 1));
    uint32_t a = (mix32(key) % (uint32_t)n) | 1u;
    // a coprime to n (n >= 2): step a up until gcd(a, n) == 1
    for (;;) {
        uint32_t x = a, y = (uint32_t)n;
        while (y) { const uint32_t t = x % y; x = y; y = t; }
        if (x == 1u) break;
        a = (a + 2u) % (uint32_t)n;
        if (a == 0u) a = 1u;
    }
    const uint32_t b = mix32(key ^ 0x5bd1e995U) % (uint32_t)n;
    float* U = P.u + p.uoff;
    const float c0 = rsqrtf((float)n), c1 = sqrtf(2.f / (float)n);
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < (int64_t)n * s;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(e / s), f = (int)(e % s);
        const uint32_t r = (uint32_t)(((uint64_t)a * (uint32_t)i + b) % (uint32_t)n);
        // cos(pi (r + 1/2) f / n) = cospi(((2r + 1) f mod 4n) / 2n)
        const uint32_t m = (uint32_t)(((uint64_t)(2u * r + 1u) * (uint32_t)f) % (4u * (uint32_t)n));
        const float v = (f == 0 ? c0 : c1) * cospif((float)m / (float)(2 * n));
        const float sg = (mix32(key + (uint32_t)i) & 1u) ? -1.f : 1.f;
        U[e] = sg * v;
    }
}

// ---------------------------------------------------------------------------
// batched tensor-core GEMM   C (M x N) = op(A) (M x K) * B (K x N),  N = s
//
// A: the factor (n x n, int8 codes or fp32; EPI_FAC applies scale/bias and
//    the Tikhonov eps), or an n x s / s x s fp32 buffer, row-major; trans_a:
//    A is stored K x M (the Gram products X^T Y).
// B: an fp32 buffer, row-major K x N.
// One CTA = one 128-row tile of C for one problem; K runs in 64-deep chunks
// through two shared-memory stages: all 256 threads load a chunk into
// registers (overlapping the tensor core's work on the previous chunk), split
// fp32 values into three bf16 parts, store them in the canonical no-swizzle
// layouts of tc.cuh (A K-major, or MN-major when transposed; B MN-major), and
// one thread issues the tcgen05.mma products into the TMEM accumulator:
// A exact (int8) x 3 B parts, or the 6 leading products of 3 x 3 parts.
// ---------------------------------------------------------------------------
constexpr int EG_BM = 128, EG_BK = 64;
constexpr int EG_NPMAX = 160;                          // padded N (s <= SMAX)
constexpr uint32_t EG_APART = EG_BM * EG_BK * 2;       // one bf16 A part, 16 KB

enum { EPI_STORE = 0, EPI_FAC = 1, EPI_CHEB = 2 };

struct EgSpec {
    int a, b, c;        // buffers
    int m, k;           // dims of op(A): M x K (DIM_N / DIM_S); N = s always
    int trans_a;        // A stored K x M
    int epi;            // EPI_*
    int prev;           // EPI_CHEB: buffer holding Z_{i-2}
    int cheb_i;         // EPI_CHEB: recurrence index i >= 2
    int fail_x;         // where F_CHOLFAIL is set, store X instead
    int skip_direct;    // skip problems solved directly (s == n)
    int b_img;          // B from its pre-split image (eig_presplit_kernel), not converted here
};

__host__ __device__ constexpr uint32_t eg_bpart(int npad) { return (uint32_t)EG_BK * npad * 2; }
__host__ __device__ constexpr uint32_t eg_stage(int na, int npad) {
    return na * EG_APART + 3 * eg_bpart(npad);
}
// int8 factor products whose factor rows are 16-byte aligned stream both
// operands through a ring of up to EG_MAXST stages (A as raw int8 rows by
// 16-byte asynchronous copies, converted to bf16 in shared memory; B by bulk
// copies of its image): EG_SMEM_STREAM bytes.
constexpr int EG_MAXST = 4;
constexpr size_t EG_SMEM_STREAM = 224 * 1024;
// int8 rows staged 80 bytes apart: the 8-byte reads of 8 rows x 2 column
// groups by a half-warp hit 32 distinct banks
constexpr int EG_SROW = EG_BK + 16;
size_t eg_smem(bool int8_a) {
    const size_t two = 2 * (size_t)eg_stage(int8_a ? 1 : 3, EG_NPMAX) + 1024;
    return int8_a ? (two > EG_SMEM_STREAM ? two : EG_SMEM_STREAM) : two;
}

// x = hi + mid + lo exactly (finite fp32): each part keeps the top 8
// significant bits of what remains (truncation, so every remainder is exact
// in fp32 and the last one fits bf16).  Integer / fp32 ops only.
SCAO_DEV void split3(float x, uint16_t& h, uint16_t& m, uint16_t& l) {
    const uint32_t xb = __float_as_uint(x);
    const float r1 = x - __uint_as_float(xb & 0xFFFF0000u);
    const uint32_t rb = __float_as_uint(r1);
    const float r2 = r1 - __uint_as_float(rb & 0xFFFF0000u);
    h = (uint16_t)(xb >> 16);
    m = (uint16_t)(rb >> 16);
    l = (uint16_t)(__float_as_uint(r2) >> 16);
}

// int8 code -> its exact bf16 bit pattern (|q| <= 127): the bits of
// 1.5 * 2^23 + q as a float, minus the bias, give (float)q exactly
SCAO_DEV uint16_t i8_to_bf16(int q) {
    const float f = __int_as_float(0x4B400000 + q) - 12582912.0f;
    return (uint16_t)(__float_as_uint(f) >> 16);
}

// store 8 fp32 values as 3 x 16 bytes of bf16 parts
SCAO_DEV void put8(unsigned char* base, uint32_t part_bytes, uint32_t off, const float* v) {
    uint16_t h[8], m[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) split3(v[i], h[i], m[i], l[i]);
    uint4 H, M, Lo;
    H.x = h[0] | ((uint32_t)h[1] << 16); H.y = h[2] | ((uint32_t)h[3] << 16);
    H.z = h[4] | ((uint32_t)h[5] << 16); H.w = h[6] | ((uint32_t)h[7] << 16);
    M.x = m[0] | ((uint32_t)m[1] << 16); M.y = m[2] | ((uint32_t)m[3] << 16);
    M.z = m[4] | ((uint32_t)m[5] << 16); M.w = m[6] | ((uint32_t)m[7] << 16);
    Lo.x = l[0] | ((uint32_t)l[1] << 16); Lo.y = l[2] | ((uint32_t)l[3] << 16);
    Lo.z = l[4] | ((uint32_t)l[5] << 16); Lo.w = l[6] | ((uint32_t)l[7] << 16);
    *(uint4*)(base + off) = H;
    *(uint4*)(base + part_bytes + off) = M;
    *(uint4*)(base + 2 * part_bytes + off) = Lo;
}

// 8 consecutive fp32 values of row `row` starting at column `col` of a
// row-major matrix (rows x cols, leading dimension ld); zero outside.
SCAO_DEV void get8(const float* X, int64_t ld, int row, int col, int rows, int cols, bool vec,
                   float* v) {
    if (row < rows && vec && col + 8 <= cols) {
        const float4 a = *(const float4*)(X + row * ld + col);
        const float4 b = *(const float4*)(X + row * ld + col + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        return;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
        v[i] = (row < rows && col + i < cols) ? X[row * ld + col + i] : 0.f;
}

// Chebyshev coefficients of step i (Z_i = al*(A Z_{i-1}) + be*Z_{i-1} + ga*Z_{i-2})
// from the interval centre c, half-width e and sigma_1 = e / (c - theta_1).
SCAO_DEV void cheb_coef(const float* aux, int i, float& al, float& be, float& ga) {
    const float c = aux[AUX_CC], e = aux[AUX_CE], s1 = aux[AUX_CS];
    const float tau = 2.f / s1;
    float sp = s1, s = s1;
    for (int j = 2; j <= i; ++j) { sp = s; s = 1.f / (tau - sp); }
    al = 2.f * s / e;
    be = -c * al;
    ga = -sp * s;
}

// A tile item (8 consecutive K values of one row) -> (row r, first column
// kg): 8 consecutive items take rows 8j..8j+7 at one kg, so their 16-byte
// stores into the canonical K-major tile fill one 128-byte core matrix
// (no shared-memory bank conflicts); a warp covers 8 rows x 32 columns.
SCAO_DEV void a_item(int item, int& r, int& kg) {
    r = (item & 7) + ((item >> 6) << 3);
    kg = ((item >> 3) & 7) * 8;
}

// Pre-split an n x s operand of the factor products (subspace problems) into
// its image: per 64-row chunk the three bf16 parts in the MN-major canonical
// layout the GEMM stages, so the GEMM copies each chunk with one bulk copy
// instead of converting it in every 128-row tile of the product.
__global__ void __launch_bounds__(NT)
eig_presplit_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, int buf) {
    const PInfo p = pinfo(P, ids, blockIdx.y);
    if (skip_iter(p) || (flags_of(p) & F_DIRECT)) return;
    const int n = p.n, N = p.s, npad = (N + 15) & ~15;
    const int k0 = blockIdx.x * EG_BK;
    if (k0 >= n) return;
    int ld;
    const float* X = buf_ptr(P, p, buf, &ld);
    const uint32_t bpart = eg_bpart(npad);
    unsigned char* img = P.eig_img + (int64_t)(2 * p.leaf + p.side) * P.eig_img_stride + (size_t)blockIdx.x * 3 * bpart;
    const int nb8 = npad >> 3, nbi = EG_BK * nb8;
    const bool vec = (ld & 3) == 0;
    for (int item = threadIdx.x; item < nbi; item += blockDim.x) {
        const int kk = (item & 7) + 8 * ((item >> 3) / nb8), ng = ((item >> 3) % nb8) * 8;
        float v[8];
        get8(X, ld, k0 + kk, ng, n, N, vec, v);
        put8(img, bpart, canon_off_mn(ng, kk, npad), v);
    }
}

__global__ void __launch_bounds__(NT, 1)
eig_tc_gemm_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, EgSpec g) {
    const PInfo p = pinfo(P, ids, blockIdx.y);
    if (skip_iter(p)) return;
    if (g.skip_direct && (flags_of(p) & F_DIRECT)) return;
    const int M = g.m == DIM_N ? p.n : p.s;
    const int K = g.k == DIM_N ? p.n : p.s;
    const int N = p.s;
    const int npad = (N + 15) & ~15;
    const int m0 = blockIdx.x * EG_BM;
    if (m0 >= M) return;
    if (g.epi == EPI_CHEB && (float)g.cheb_i > p.aux[AUX_DEG]) {
        // beyond this problem's filter degree: Z_i = Z_{i-1}
        int ldb_, ldc_;
        const float* Bc = buf_ptr(P, p, g.b, &ldb_);
        float* Cc = buf_ptr(P, p, g.c, &ldc_);
        const int rows = min(EG_BM, M - m0);
        for (int e = threadIdx.x; e < rows * N; e += blockDim.x) {
            const int r = m0 + e / N, c = e % N;
            Cc[(int64_t)r * ldc_ + c] = Bc[(int64_t)r * ldb_ + c];
        }
        return;
    }
    const bool fac = g.a == BUF_FAC;
    const bool i8 = fac && P.int8_ema;
    const int na = i8 ? 1 : 3;
    int lda = 0, ldb, ldc;
    const float* A = fac ? nullptr : buf_ptr(P, p, g.a, &lda);
    const float* B = buf_ptr(P, p, g.b, &ldb);
    float* C = buf_ptr(P, p, g.c, &ldc);
    const int8_t* Aq = i8 ? (const int8_t*)P.fac + p.facoff : nullptr;
    const float* Af = (fac && !i8) ? (const float*)P.fac + p.facoff : nullptr;
    if (fac) lda = p.n;

    extern __shared__ __align__(1024) unsigned char eg_smem_raw[];
    unsigned char* sm = (unsigned char*)(((uintptr_t)eg_smem_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t bpart = eg_bpart(npad);
    const uint32_t stage = (uint32_t)na * EG_APART + 3 * bpart;
    __shared__ uint64_t mbar[EG_MAXST], fullb[EG_MAXST];
    __shared__ uint32_t tslot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tcols = npad <= 32 ? 32 : npad <= 64 ? 64 : npad <= 128 ? 128 : 256;
    // B staged by bulk copies of its pre-split image (subspace problems)
    const bool bimg = g.b_img && !(flags_of(p) & F_DIRECT);
    const unsigned char* img = P.eig_img + (int64_t)(2 * p.leaf + p.side) * P.eig_img_stride;
    const uint32_t bbytes = 3 * bpart;
    // both operands by bulk copies (int8 factor, rows 16-byte aligned)
    const bool stream = i8 && bimg && !g.trans_a && (p.n & 15) == 0 && (p.facoff & 15) == 0;
    if (warp == 0) tc_alloc(&tslot, tcols);
    if (tid == 0) {
        for (int i = 0; i < EG_MAXST; ++i) {
            mbar_init(&mbar[i], 1);
            mbar_init(&fullb[i], stream ? NT + 1 : 1);
        }
        fence_async_smem();
        if (bimg && !stream) {
            mbar_expect_tx(&fullb[0], bbytes);
            bulk_g2s(sm + na * EG_APART, img, bbytes, &fullb[0]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    const uint32_t idesc = idesc_bf16(EG_BM, npad, g.trans_a, 1);
    // vector loads need 16-byte aligned rows
    const bool vecA = fac ? (!i8 && (p.n & 3) == 0) : ((lda & 3) == 0);
    const bool vecB = (ldb & 3) == 0;
    const bool vecQ = i8 && (p.n & 7) == 0 && (p.facoff & 7) == 0;
    const int nkb = (K + EG_BK - 1) / EG_BK;
    const int nbi = EG_BK * (npad >> 3);                // B items of 8 values
    constexpr int AIT = EG_BM * EG_BK / 8 / NT;         // 4 A items per thread
    constexpr int BIT = (EG_BK * EG_NPMAX / 8 + NT - 1) / NT;   // <= 5 B items
    float av[AIT][8];
    uint2 aq[AIT];
    float bv[BIT][8];
    bool ok = true;
    // global -> registers for chunk kb (issued one chunk ahead of its use)
    auto load_regs = [&](int kb) {
        const int k0 = kb * EG_BK;
#pragma unroll
        for (int it = 0; it < AIT; ++it) {
            const int item = tid + it * NT;
            if (i8) {
                int r, kg;
                a_item(item, r, kg);
                const int row = m0 + r, col = k0 + kg;
                if (row < M && vecQ && col + 8 <= K) {
                    aq[it] = *(const uint2*)(Aq + (int64_t)row * p.n + col);
                } else {
                    uint32_t w[2] = {0u, 0u};
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int8_t q = (row < M && col + i < K) ? Aq[(int64_t)row * p.n + col + i] : (int8_t)0;
                        w[i >> 2] |= ((uint32_t)(uint8_t)q) << ((i & 3) * 8);
                    }
                    aq[it] = make_uint2(w[0], w[1]);
                }
            } else if (!g.trans_a) {
                int r, kg;
                a_item(item, r, kg);
                get8(fac ? Af : A, lda, m0 + r, k0 + kg, M, K, vecA, av[it]);
            } else {
                // A^T: element (m, k) = X[k][m]; 8 consecutive m of row k
                const int kk = (item & 7) + 8 * (item >> 7), mg = ((item >> 3) & 15) * 8;
                get8(A, lda, k0 + kk, m0 + mg, K, M, vecA, av[it]);
            }
        }
#pragma unroll
        for (int it = 0; it < BIT; ++it) {
            const int item = tid + it * NT;
            if (!bimg && item < nbi) {
                const int nb8 = npad >> 3;   // 8 threads fill one 128-byte core matrix
                const int kk = (item & 7) + 8 * ((item >> 3) / nb8), ng = ((item >> 3) % nb8) * 8;
                get8(B, ldb, k0 + kk, ng, K, N, vecB, bv[it]);
            }
        }
    };
    if (stream) {
        // two bf16 A tiles, then a ring of nst stages [B image chunk | A int8
        // rows]; nst - 1 chunks in flight, all threads convert A into the A
        // tile of the chunk's parity, one thread issues the MMAs and commits
        // them to the stage's empty barrier
        unsigned char* ring = sm + 2 * EG_APART;
        const uint32_t a8 = bbytes;
        const uint32_t stage2 = a8 + EG_BM * EG_SROW;
        int nst = (int)((EG_SMEM_STREAM - 1024 - 2 * EG_APART) / stage2);
        nst = nst > EG_MAXST ? EG_MAXST : nst;
        const int rows_a = min(EG_BM, M - m0);
        // A: 16-byte asynchronous copies by every thread, whose completion
        // arrives on the stage's full barrier (NT arrivals); B: one bulk copy
        // of its image chunk (one arrival with its byte count)
        auto produce_a = [&](int kb) {            // every thread
            const int s_ = kb % nst;
            unsigned char* dst = ring + s_ * stage2 + a8;
            const int k0 = kb * EG_BK;
            // columns past K keep stale int8 codes: finite, and the B image
            // rows past K are zero; rows past M are never stored
            for (int c = tid; c < EG_BM * (EG_BK / 16); c += NT) {
                const int r = c >> 2, seg = (c & 3) * 16;
                if (r < rows_a && k0 + seg < K)
                    cp_async16(dst + r * EG_SROW + seg, Aq + (int64_t)(m0 + r) * p.n + k0 + seg);
            }
            cp_async_arrive_noinc(&fullb[s_]);
        };
        auto produce_b = [&](int kb) {            // thread 0
            const int s_ = kb % nst;
            mbar_expect_tx(&fullb[s_], bbytes);
            bulk_g2s(ring + s_ * stage2, img + (size_t)kb * bbytes, bbytes, &fullb[s_]);
        };
        for (int j = 0; j < nst - 1 && j < nkb; ++j) {
            produce_a(j);
            if (tid == 0) produce_b(j);
        }
        for (int kb = 0; kb < nkb; ++kb) {
            const int st = kb % nst;
            unsigned char* base = ring + st * stage2;
            unsigned char* sa = sm + (kb & 1) * EG_APART;
            ok = mbar_wait(&fullb[st], (kb / nst) & 1) && ok;
            // the A tile of this parity was read by the MMAs of chunk kb - 2
            if (kb >= 2) ok = mbar_wait(&mbar[(kb - 2) % nst], ((kb - 2) / nst) & 1) && ok;
#pragma unroll
            for (int it = 0; it < AIT; ++it) {
                const int item = tid + it * NT;
                int r, kg;
                a_item(item, r, kg);
                const uint2 wq = *(const uint2*)(base + a8 + r * EG_SROW + kg);
                const uint32_t w[2] = {wq.x, wq.y};
                uint16_t h[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    h[i] = i8_to_bf16((int8_t)((w[i >> 2] >> ((i & 3) * 8)) & 0xFF));
                uint4 H;
                H.x = h[0] | ((uint32_t)h[1] << 16); H.y = h[2] | ((uint32_t)h[3] << 16);
                H.z = h[4] | ((uint32_t)h[5] << 16); H.w = h[6] | ((uint32_t)h[7] << 16);
                *(uint4*)(sa + canon_off(r, kg, EG_BK)) = H;
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                const uint32_t a0 = smem_u32(sa), b0 = smem_u32(base);
#pragma unroll
                for (int ks = 0; ks < EG_BK / 16; ++ks) {
                    const uint64_t ad = smem_desc(a0 + ks * 256, 128, 16 * EG_BK);
                    const uint32_t boff = (uint32_t)ks * 2 * 16 * npad;
                    const uint32_t acc0 = (kb > 0 || ks > 0) ? 1u : 0u;
                    tc_mma_bf16(tmem, ad, smem_desc(b0 + boff, 16 * npad, 128), idesc, acc0);
                    tc_mma_bf16(tmem, ad, smem_desc(b0 + bpart + boff, 16 * npad, 128), idesc, 1u);
                    tc_mma_bf16(tmem, ad, smem_desc(b0 + 2 * bpart + boff, 16 * npad, 128), idesc, 1u);
                }
                tc_commit(&mbar[st]);
            }
            // refill the stage of chunk kb - 1: its int8 rows were converted
            // before this iteration's barrier; its B part once its MMAs completed
            if (kb + nst - 1 < nkb) {
                produce_a(kb + nst - 1);
                if (tid == 0) {
                    if (kb >= 1) ok = mbar_wait(&mbar[(kb - 1) % nst], ((kb - 1) / nst) & 1) && ok;
                    produce_b(kb + nst - 1);
                }
            }
        }
        ok = mbar_wait(&mbar[(nkb - 1) % nst], ((nkb - 1) / nst) & 1) && ok;
    } else {
        load_regs(0);
        for (int kb = 0; kb < nkb; ++kb) {
            // ---- wait until the MMAs of chunk kb-2 released this stage ----
            const int st = kb & 1;
            if (kb >= 2) ok = mbar_wait(&mbar[st], ((kb - 2) >> 1) & 1) && ok;
            unsigned char* sa = sm + st * stage;
            unsigned char* sb = sa + na * EG_APART;
    #pragma unroll
            for (int it = 0; it < AIT; ++it) {
                const int item = tid + it * NT;
                if (i8) {
                    int r, kg;
                    a_item(item, r, kg);
                    uint16_t h[8];
                    const uint32_t w[2] = {aq[it].x, aq[it].y};
    #pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int8_t q = (int8_t)((w[i >> 2] >> ((i & 3) * 8)) & 0xFF);
                        h[i] = i8_to_bf16(q);
                    }
                    uint4 H;
                    H.x = h[0] | ((uint32_t)h[1] << 16); H.y = h[2] | ((uint32_t)h[3] << 16);
                    H.z = h[4] | ((uint32_t)h[5] << 16); H.w = h[6] | ((uint32_t)h[7] << 16);
                    *(uint4*)(sa + canon_off(r, kg, EG_BK)) = H;
                } else if (!g.trans_a) {
                    int r, kg;
                    a_item(item, r, kg);
                    put8(sa, EG_APART, canon_off(r, kg, EG_BK), av[it]);
                } else {
                    const int kk = (item & 7) + 8 * (item >> 7), mg = ((item >> 3) & 15) * 8;
                    put8(sa, EG_APART, canon_off_mn(mg, kk, EG_BM), av[it]);
                }
            }
    #pragma unroll
            for (int it = 0; it < BIT; ++it) {
                const int item = tid + it * NT;
                if (!bimg && item < nbi) {
                    const int nb8 = npad >> 3;   // 8 threads fill one 128-byte core matrix
                    const int kk = (item & 7) + 8 * ((item >> 3) / nb8), ng = ((item >> 3) % nb8) * 8;
                    put8(sb, bpart, canon_off_mn(ng, kk, npad), bv[it]);
                }
            }
            // the registers are free again: start the next chunk's loads
            if (kb + 1 < nkb) load_regs(kb + 1);
            if (bimg) ok = mbar_wait(&fullb[st], (kb >> 1) & 1) && ok;
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb);
    #pragma unroll
                for (int ks = 0; ks < EG_BK / 16; ++ks) {
                    const uint32_t aoff = g.trans_a ? (uint32_t)ks * 2 * 16 * EG_BM : (uint32_t)ks * 256;
                    const uint32_t boff = (uint32_t)ks * 2 * 16 * npad;
                    auto adesc = [&](int part) {
                        const uint32_t a = a0 + part * EG_APART + aoff;
                        return g.trans_a ? smem_desc(a, 16 * EG_BM, 128) : smem_desc(a, 128, 16 * EG_BK);
                    };
                    auto bdesc = [&](int part) {
                        return smem_desc(b0 + part * bpart + boff, 16 * npad, 128);
                    };
                    const uint32_t acc0 = (kb > 0 || ks > 0) ? 1u : 0u;
                    if (i8) {
                        tc_mma_bf16(tmem, adesc(0), bdesc(0), idesc, acc0);
                        tc_mma_bf16(tmem, adesc(0), bdesc(1), idesc, 1u);
                        tc_mma_bf16(tmem, adesc(0), bdesc(2), idesc, 1u);
                    } else {
                        tc_mma_bf16(tmem, adesc(0), bdesc(0), idesc, acc0);
                        tc_mma_bf16(tmem, adesc(0), bdesc(1), idesc, 1u);
                        tc_mma_bf16(tmem, adesc(1), bdesc(0), idesc, 1u);
                        tc_mma_bf16(tmem, adesc(0), bdesc(2), idesc, 1u);
                        tc_mma_bf16(tmem, adesc(1), bdesc(1), idesc, 1u);
                        tc_mma_bf16(tmem, adesc(2), bdesc(0), idesc, 1u);
                    }
                }
                tc_commit(&mbar[st]);
                // prefetch chunk kb+1 of B into the other stage once the MMAs of
                // chunk kb-1 have released it
                if (bimg && kb + 1 < nkb) {
                    const int s1 = (kb + 1) & 1;
                    if (kb >= 1) ok = mbar_wait(&mbar[s1], ((kb - 1) >> 1) & 1) && ok;
                    mbar_expect_tx(&fullb[s1], bbytes);
                    bulk_g2s(sm + s1 * stage + na * EG_APART, img + (size_t)(kb + 1) * bbytes, bbytes,
                             &fullb[s1]);
                }
            }
        }
        ok = mbar_wait(&mbar[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1) && ok;
    }
    if (!ok && P.err) atomicExch(P.err, 1);
    tc_fence_after();
    __syncthreads();

    // ---- epilogue: TMEM lane = row of the tile ----
    const int q = warp & 3, half = warp >> 2;
    const bool fail = g.fail_x && (flags_of(p) & F_CHOLFAIL);
    const float* X = P.eig_x + p.uoff;
    float dscale = 1.f, eps = 0.f;
    if (fac) {
        dscale = i8 ? __fdiv_rn(p.aux[AUX_SCALE], p.aux[AUX_BIAS]) : __fdiv_rn(1.f, p.aux[AUX_BIAS]);
        eps = p.aux[AUX_EPS];
    }
    float al = 1.f, be = 0.f, ga = 0.f;
    int ldp = 0;
    const float* Prev = nullptr;
    if (g.epi == EPI_CHEB) {
        cheb_coef(p.aux, g.cheb_i, al, be, ga);
        Prev = buf_ptr(P, p, g.prev, &ldp);
    }
    // TMEM -> shared tile (row stride npad + 4 floats: the float4 stores of
    // 8 consecutive lanes fall in distinct banks), then row-contiguous,
    // coalesced reads of B / Prev and stores of C by all warps.  Every MMA and
    // bulk copy has completed, so the stage memory is free (after a timed-out
    // wait the tile is not read: the output is zero and the error flag set).
    float* T = (float*)sm;
    const int ts = npad + 4;
    const int cw = npad >> 1;                           // columns per warp half (multiple of 8)
    for (int c0 = half * cw; c0 < half * cw + cw; c0 += 8) {
        float v[8];
        tc_ld8(tmem + ((uint32_t)(q * 32) << 16) + c0, v);
        float* t = T + (q * 32 + lane) * ts + c0;
        *(float4*)t = make_float4(v[0], v[1], v[2], v[3]);
        *(float4*)(t + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
    tc_fence_before();
    __syncthreads();
    // EP_R rows per warp step, up to EP_C columns per lane: every load of a
    // step (B, Prev) is issued before its stores, so a warp waits one memory
    // latency per step instead of one per element
    constexpr int EP_R = 8, EP_C = (EG_NPMAX + 31) / 32;
    const int rows = min(EG_BM, M - m0);
    for (int rr0 = warp * EP_R; rr0 < rows; rr0 += EP_R * (NT / 32)) {
        float bc[EP_R][EP_C], pv[EP_R][EP_C];
#pragma unroll
        for (int i = 0; i < EP_R; ++i) {
#pragma unroll
            for (int j = 0; j < EP_C; ++j) {
                const int r = m0 + rr0 + i, c = lane + 32 * j;
                const bool in = rr0 + i < rows && c < N;
                bc[i][j] = (g.epi != EPI_STORE && in) ? B[(int64_t)r * ldb + c] : 0.f;
                pv[i][j] = (g.epi == EPI_CHEB && in) ? Prev[(int64_t)r * ldp + c] : 0.f;
            }
        }
#pragma unroll
        for (int i = 0; i < EP_R; ++i) {
#pragma unroll
            for (int j = 0; j < EP_C; ++j) {
                const int rr = rr0 + i, r = m0 + rr, c = lane + 32 * j;
                if (rr >= rows || c >= N) continue;
                float out = ok ? T[rr * ts + c] : 0.f;
                if (g.epi != EPI_STORE) {
                    out = fmaf(out, dscale, eps * bc[i][j]);
                    if (g.epi == EPI_CHEB) out = fmaf(al, out, fmaf(be, bc[i][j], ga * pv[i][j]));
                }
                if (fail) out = X[(int64_t)r * p.s + c];
                C[(int64_t)r * ldc + c] = out;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, tcols);
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
        // relative off-diagonal Frobenius norm <= 1e-6: Ritz values then
        // carry errors of order 1e-12 relative, vectors 1e-6 (fp32 level)
        if (off <= 1e-12f * fro || fro == 0.f) break;
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
            // H <- J^T H J and V <- V J in one pass: the rotations of a round
            // act on disjoint index pairs, so each 2 x 2 block (rows p1,q1 of
            // pair t1; cols p2,q2 of pair t2) is updated from its own four
            // entries, rows first, then columns
            const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            for (int t1 = warp; t1 < half; t1 += blockDim.x >> 5) {
                const int P1 = pp[t1], Q1 = qq[t1];
                const float c1 = cs[t1], s1 = sn[t1];
                for (int t2 = lane; t2 < half; t2 += 32) {
                    const int P2 = pp[t2], Q2 = qq[t2];
                    const float c2 = cs[t2], s2 = sn[t2];
                    const float hpp = H[P1 * ld + P2], hpq = H[P1 * ld + Q2];
                    const float hqp = H[Q1 * ld + P2], hqq = H[Q1 * ld + Q2];
                    const float rpp = c1 * hpp - s1 * hqp, rqp = s1 * hpp + c1 * hqp;
                    const float rpq = c1 * hpq - s1 * hqq, rqq = s1 * hpq + c1 * hqq;
                    H[P1 * ld + P2] = c2 * rpp - s2 * rpq;
                    H[P1 * ld + Q2] = s2 * rpp + c2 * rpq;
                    H[Q1 * ld + P2] = c2 * rqp - s2 * rqq;
                    H[Q1 * ld + Q2] = s2 * rqp + c2 * rqq;
                }
            }
            for (int k = warp; k < se; k += blockDim.x >> 5) {
                for (int t = lane; t < half; t += 32) {
                    const int P0 = pp[t], Q0 = qq[t];
                    const float c = cs[t], sv = sn[t];
                    const float vp = V[k * ld + P0], vq = V[k * ld + Q0];
                    V[k * ld + P0] = c * vp - sv * vq;
                    V[k * ld + Q0] = sv * vp + c * vq;
                }
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
// residuals of the usable Ritz pairs; convergence; Chebyshev set-up
// ---------------------------------------------------------------------------
__global__ void eig_residual_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                                    float tol, int cap) {
    const PInfo p = pinfo(P, ids, blockIdx.x);
    if (skip_iter(p)) return;
    __shared__ float red[32];
    const int it = P.counters[CNT_ITER];
    const bool last = it >= cap - 1;
    const float* X = P.eig_x + p.uoff;
    const float* AX = P.eig_ax + p.uoff;
    const float* ev = P.ev + p.evoff;
    const int s = p.s;
    // the rank update can only use the top min(kmax, k_prev + 4) pairs
    const int kc = min(s, min(p.kmax, P.k[p.leaf] + 4));
    const float th0 = ev[0], ths = ev[s - 1];
    const float scale = fmaxf(fabsf(th0), 1e-30f);
    const float bulk = ths >= 0.f ? (1.f + CLUSTER_FRAC) * ths : ths;
    __shared__ float rr[SMAX];
    __shared__ int sconv;
    // rows over warps, columns over lanes (row-contiguous, coalesced reads);
    // per-warp partial sums reduced in shared memory
    __shared__ float part[NT / 32][SMAX];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    constexpr int RC = (SMAX + 31) / 32;
    float thc[RC], acc[RC];
#pragma unroll
    for (int j = 0; j < RC; ++j) {
        const int c = lane + 32 * j;
        thc[j] = c < kc ? ev[c] : 0.f;
        acc[j] = 0.f;
    }
    for (int i = wid; i < p.n; i += nw) {
#pragma unroll
        for (int j = 0; j < RC; ++j) {
            const int c = lane + 32 * j;
            if (c < kc) {
                const float d = AX[(int64_t)i * s + c] - thc[j] * X[(int64_t)i * s + c];
                acc[j] = fmaf(d, d, acc[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < RC; ++j) {
        const int c = lane + 32 * j;
        if (c < kc) part[wid][c] = acc[j];
    }
    __syncthreads();
    for (int c = threadIdx.x; c < kc; c += blockDim.x) {
        float r2 = 0.f;
        for (int w = 0; w < nw; ++w) r2 += part[w][c];
        rr[c] = sqrtf(r2);
    }
    __syncthreads();
    // Convergence.  From the third outer iteration on, a pair within
    // CLUSTER_FRAC of theta_s whose residual is below CLUSTER_FRAC * theta_s
    // lies in the flat bulk (exempt).  Every
    // other usable pair needs
    //  * r_j <= VAL_TOL * theta_1 (Ritz values accurate to ~r^2 / gap), and
    //  * for every prefix 0..j that ends at a gap theta_j - theta_{j+1} >=
    //    GAP_REL * theta_1: max_{i<=j} r_i <= tol * gap, so the prefix subspace
    //    is within ~tol rad of the exact one (Davis-Kahan sin(theta) bound).
    const int fl = flags_of(p);
    float rmax = 0.f;
    if (threadIdx.x == 0) {
        bool ok = true;
        for (int j = 0; j < kc; ++j) {
            // (not before the third outer iteration: the Ritz values of an
            // unfiltered block can all sit within CLUSTER_FRAC of each other)
            const bool exempt = it >= 2 && ev[j] <= bulk && rr[j] <= CLUSTER_FRAC * fabsf(ths);
            if (!exempt) {
                rmax = fmaxf(rmax, rr[j]);
                if (rr[j] > VAL_TOL * scale) { ok = false; break; }
            }
            const float gap = (j + 1 < s) ? ev[j] - ev[j + 1] : 0.f;
            if (gap >= GAP_REL * scale && rmax > tol * gap) { ok = false; break; }
        }
        sconv = ok;
        red[0] = rmax;
    }
    __syncthreads();
    rmax = red[0];
    const bool conv = (fl & F_DIRECT) || sconv || last;
    float* U = P.u + p.uoff;
    const int64_t ns = (int64_t)p.n * s;
    if (conv) {
        for (int64_t e = threadIdx.x; e < ns; e += blockDim.x) U[e] = X[e];
    } else {
        // filter interval [a, b] = [min(0, theta_s), theta_s] is damped; the
        // scaled recurrence keeps the component along theta_1 near 1
        const float a = fminf(0.f, ths);
        const float b = fmaxf(ths, a + 1e-6f * scale);
        const float c = 0.5f * (a + b), e = 0.5f * (b - a);
        const float s1 = e / (c - fmaxf(th0, b + 1e-6f * scale));
        // Z_1 = (s1 / e) (A X - c X) -> Y
        float* Y = P.eig_y + p.uoff;
        const float al = s1 / e;
        for (int64_t e_ = threadIdx.x; e_ < ns; e_ += blockDim.x)
            Y[e_] = al * (AX[e_] - c * X[e_]);
        if (threadIdx.x == 0) {
            p.aux[AUX_CC] = c;
            p.aux[AUX_CE] = e;
            p.aux[AUX_CS] = s1;
            atomicAdd(&P.counters[CNT_ACTIVE], 1);
        }
    }
    if (threadIdx.x == 0) {
        int f = fl & ~F_CHOLFAIL;
        if (conv) f |= F_CONV;
        if (conv) p.aux[AUX_WARM] = 1.f;
        p.aux[AUX_FLAGS] = __int_as_float(f);
        p.aux[AUX_ITERS] = __int_as_float(it + 1);
        p.aux[AUX_RES] = rmax / scale;
        if (conv && !(fl & F_DIRECT) && !sconv)
            p.aux[AUX_ITERS] = __int_as_float(-(it + 1));   // cap reached
    }
}

// ---------------------------------------------------------------------------
// CholeskyQR helper: H = Gram (s x s) of Z -> H = D^-1/2 R^{-1} with
// D = diag(Gram), D^-1/2 Gram D^-1/2 = R^T R, so that Z H is orthonormal
// (the column scaling keeps the filtered block's Gram well conditioned)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
eig_cholinv_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids) {
    const PInfo p = pinfo(P, ids, blockIdx.x);
    if (skip_iter(p) || (flags_of(p) & F_DIRECT)) return;
    extern __shared__ float sm[];
    const int s = p.s, ld = s + 1;
    float* R = sm;            // s x ld
    float* X = R + s * ld;    // s x ld
    __shared__ float dinv[SMAX];
    __shared__ int fail;
    int ldh;
    float* Hg = buf_ptr(P, p, BUF_H, &ldh);
    for (int i = threadIdx.x; i < s; i += blockDim.x) {
        const float d = Hg[i * ldh + i];
        dinv[i] = d > 0.f ? rsqrtf(d) : 0.f;
    }
    if (threadIdx.x == 0) fail = 0;
    __syncthreads();
    for (int e = threadIdx.x; e < s * s; e += blockDim.x) {
        const int i = e / s, j = e % s;
        R[i * ld + j] = 0.5f * (Hg[i * ldh + j] + Hg[j * ldh + i]) * dinv[i] * dinv[j];
    }
    __syncthreads();
    // right-looking Cholesky, upper factor R (row k holds R[k][k..]); the
    // scaled Gram has unit diagonal, so trace = s
    for (int k = 0; k < s; ++k) {
        if (threadIdx.x == 0) {
            const float d = R[k * ld + k];
            if (!(d > 1e-12f * s) || dinv[k] == 0.f) fail = 1;
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
        Hg[i * ldh + j] = dinv[i] * X[i * ld + j];
    }
    if (threadIdx.x == 0 && fail) {
        p.aux[AUX_FLAGS] = __int_as_float(flags_of(p) | F_CHOLFAIL);
        p.aux[AUX_NFAIL] += 1.f;
        // a filtered block too ill-conditioned for fp32 CholeskyQR: lower
        // this problem's filter degree for the next outer iterations
        p.aux[AUX_DEG] = fmaxf(1.f, p.aux[AUX_DEG] - 1.f);
    }
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
// loop control of the iteration graph ---------------------------------------
// before the loop: iteration 0, and run the loop only if some problem needs
// the iterative solver
__global__ void eig_loop_init_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, int np,
                                     int cap, cudaGraphConditionalHandle h, int use_h) {
    int c = 0;
    for (int j = threadIdx.x; j < np; j += blockDim.x) {
        const PInfo p = pinfo(P, ids, j);
        if (!skip_iter(p)) ++c;
    }
    c = __syncthreads_count(c > 0);
    if (threadIdx.x == 0) {
        P.counters[CNT_ITER] = 0;
        P.counters[CNT_ACTIVE] = 0;
        if (use_h) cudaGraphSetConditional(h, (c > 0 && cap > 0) ? 1u : 0u);
    }
}

// end of an outer iteration: continue while some problem is still active
__global__ void eig_loop_ctl_kernel(ScaoPlanDev P, int cap, cudaGraphConditionalHandle h,
                                    int use_h) {
    if (threadIdx.x == 0) {
        const int active = P.counters[CNT_ACTIVE];
        const int it = P.counters[CNT_ITER] + 1;
        P.counters[CNT_ACTIVE] = 0;
        P.counters[CNT_ITER] = it;
        if (use_h) cudaGraphSetConditional(h, (active > 0 && it < cap) ? 1u : 0u);
    }
}

size_t jacobi_smem(int s) {
    const int se = s + (s & 1), ld = se + 1;
    return (size_t)(2 * se * ld + 2 * se) * 4 + 32 * 4 + 64;
}

size_t cholinv_smem(int s) { return (size_t)2 * s * (s + 1) * 4; }

// one executable iteration graph per (device, plan arenas, leaf list, sizes)
struct GraphKey {
    int dev, n_ids, nmax, smax, cap;
    float tol;
    const void* ids;
    const void *leaves, *fac, *u, *ev, *k, *y, *x, *ax, *h, *v, *aux, *absmax, *counters, *err;
    int int8_ema;
    bool operator==(const GraphKey& o) const { return memcmp(this, &o, sizeof(GraphKey)) == 0; }
};
struct GraphEntry { GraphKey key; cudaGraphExec_t exec; int64_t kernels; };
std::mutex g_graph_mu;
std::vector<GraphEntry> g_graphs;
cudaStream_t g_capture_stream[64] = {};
constexpr size_t kMaxGraphs = 64;

GraphKey make_key(const ScaoPlanDev* P, const int32_t* ids, int n_ids, int nmax, int smax,
                  int cap, float tol) {
    GraphKey k;
    memset(&k, 0, sizeof(k));
    cudaGetDevice(&k.dev);
    k.n_ids = n_ids; k.nmax = nmax; k.smax = smax; k.cap = cap; k.tol = tol; k.ids = ids;
    k.leaves = P->leaves; k.fac = P->fac; k.u = P->u; k.ev = P->ev; k.k = P->k;
    k.y = P->eig_y; k.x = P->eig_x; k.ax = P->eig_ax; k.h = P->eig_h; k.v = P->eig_v;
    k.aux = P->eig_aux; k.absmax = P->absmax; k.counters = P->counters; k.err = P->err;
    k.int8_ema = P->int8_ema;
    return k;
}

// Launch the body of one outer iteration on stream st (being captured).
// prof: per-kernel timing scopes (the diagnostic launch without a graph,
// SCAO_EIG_NOGRAPH=1); otherwise the launches are being captured.
int64_t launch_iteration(const ScaoPlanDev& P, const int32_t* ids, int np, int nmax, int smax,
                         int cap, float tol, cudaGraphConditionalHandle h, int use_h,
                         cudaStream_t st) {
    const int tiles_n = (nmax + EG_BM - 1) / EG_BM;
    const int tiles_s = (smax + EG_BM - 1) / EG_BM;
    const size_t sm_big = eg_smem(P.int8_ema != 0), sm_small = eg_smem(false);
    const size_t jsm = jacobi_smem(smax), csm = cholinv_smem(smax);
    int64_t n = 0;
    auto gemm = [&](EgSpec g, int tiles, size_t smem) {
        ProfScope _ps(SLOT_EIG_GEMM, st);
        eig_tc_gemm_kernel<<<dim3(tiles, np), NT, smem, st>>>(P, ids, g);
        ++n;
    };
    //            a        b      c       m      k      tA  epi        prev    i  fail skipD
    auto presplit = [&](int buf) {
        ProfScope _ps(SLOT_EIG_GEMM, st);
        eig_presplit_kernel<<<dim3((nmax + EG_BK - 1) / EG_BK, np), NT, 0, st>>>(P, ids, buf);
        ++n;
    };
    // Rayleigh-Ritz: Y = A U, H = U^T Y, Jacobi, X = U V, AX = Y V
    presplit(BUF_U);
    gemm({BUF_FAC, BUF_U, BUF_Y, DIM_N, DIM_N, 0, EPI_FAC, 0, 0, 0, 0, 1}, tiles_n, sm_big);
    gemm({BUF_U, BUF_Y, BUF_H, DIM_S, DIM_N, 1, EPI_STORE, 0, 0, 0, 0}, tiles_s, sm_small);
    { ProfScope _ps(SLOT_EIG_JACOBI, st); eig_jacobi_kernel<<<np, NT, jsm, st>>>(P, ids, 30); ++n; }
    gemm({BUF_U, BUF_V, BUF_X, DIM_N, DIM_S, 0, EPI_STORE, 0, 0, 0, 0}, tiles_n, sm_small);
    gemm({BUF_Y, BUF_V, BUF_AX, DIM_N, DIM_S, 0, EPI_STORE, 0, 0, 0, 0}, tiles_n, sm_small);
    // residuals, convergence; Z_0 = X, Z_1 -> Y
    { ProfScope _ps(SLOT_EIG_RESIDUAL, st); eig_residual_kernel<<<np, NT, 0, st>>>(P, ids, tol, cap); ++n; }
    // Chebyshev filter: Z_i = f(A Z_{i-1}, Z_{i-1}, Z_{i-2}), written over Z_{i-2}
    // (Y and AX alternate; X keeps the Ritz vectors)
    int cur = BUF_Y, prv = BUF_X;
    for (int i = 2; i <= CHEB_M; ++i) {
        const int out = (prv == BUF_X) ? BUF_AX : prv;
        presplit(cur);
        gemm({BUF_FAC, cur, out, DIM_N, DIM_N, 0, EPI_CHEB, prv, i, 0, 0, 1}, tiles_n, sm_big);
        prv = cur;
        cur = out;
    }
    const int other = (cur == BUF_Y) ? BUF_AX : BUF_Y;
    // column-scaled CholeskyQR2 of Z_m: -> other -> U (U = X where it failed)
    gemm({cur, cur, BUF_H, DIM_S, DIM_N, 1, EPI_STORE, 0, 0, 0, 1}, tiles_s, sm_small);
    { ProfScope _ps(SLOT_EIG_CHOLINV, st); eig_cholinv_kernel<<<np, NT, csm, st>>>(P, ids); ++n; }
    gemm({cur, BUF_H, other, DIM_N, DIM_S, 0, EPI_STORE, 0, 0, 0, 1}, tiles_n, sm_small);
    gemm({other, other, BUF_H, DIM_S, DIM_N, 1, EPI_STORE, 0, 0, 0, 1}, tiles_s, sm_small);
    { ProfScope _ps(SLOT_EIG_CHOLINV, st); eig_cholinv_kernel<<<np, NT, csm, st>>>(P, ids); ++n; }
    gemm({other, BUF_H, BUF_U, DIM_N, DIM_S, 0, EPI_STORE, 0, 0, 1, 1}, tiles_n, sm_small);
    { ProfScope _ps(SLOT_EIG_RESIDUAL, st); eig_loop_ctl_kernel<<<1, 32, 0, st>>>(P, cap, h, use_h); ++n; }
    return n;
}

int build_graph(const ScaoPlanDev* P, const int32_t* ids, int np, int nmax, int smax, int cap,
                float tol, cudaGraphExec_t* exec, int64_t* kernels) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (!g_capture_stream[dev] &&
        cudaStreamCreateWithFlags(&g_capture_stream[dev], cudaStreamNonBlocking) != cudaSuccess)
        return SCAO_ERR_LAUNCH;
    cudaGraph_t g = nullptr;
    if (cudaGraphCreate(&g, 0) != cudaSuccess) return SCAO_ERR_LAUNCH;
    int rc = SCAO_ERR_LAUNCH;
    cudaGraphConditionalHandle h;
    cudaGraphNode_t n0, n1;
    alignas(cudaGraphNodeParams) unsigned char cp_raw[sizeof(cudaGraphNodeParams)] = {};
    cudaGraphNodeParams& cp = *reinterpret_cast<cudaGraphNodeParams*>(cp_raw);
    ScaoPlanDev Pc = *P;
    const int32_t* idp = ids;
    int npv = np, capv = cap;
    int use_h = 1;
    void* args[] = {&Pc, &idp, &npv, &capv, &h, &use_h};
    cudaKernelNodeParams kp;
    memset(&kp, 0, sizeof(kp));
    do {
        if (cudaGraphConditionalHandleCreate(&h, g, 0, cudaGraphCondAssignDefault) != cudaSuccess) break;
        kp.func = (void*)eig_loop_init_kernel;
        kp.gridDim = dim3(1);
        kp.blockDim = dim3(256);
        kp.kernelParams = args;
        if (cudaGraphAddKernelNode(&n0, g, nullptr, 0, &kp) != cudaSuccess) break;
        cp.type = cudaGraphNodeTypeConditional;
        cp.conditional.handle = h;
        cp.conditional.type = cudaGraphCondTypeWhile;
        cp.conditional.size = 1;
        if (cudaGraphAddNode(&n1, g, &n0, 1, &cp) != cudaSuccess) break;
        cudaGraph_t body = cp.conditional.phGraph_out[0];
        cudaStream_t cs = g_capture_stream[dev];
        if (cudaStreamBeginCaptureToGraph(cs, body, nullptr, nullptr, 0,
                                          cudaStreamCaptureModeThreadLocal) != cudaSuccess) break;
        scao_prof_suspend(1);
        const int64_t nk = launch_iteration(Pc, ids, np, nmax, smax, cap, tol, h, 1, cs);
        scao_prof_suspend(0);
        const cudaError_t le = cudaGetLastError();
        cudaGraph_t out = nullptr;
        const cudaError_t ce = cudaStreamEndCapture(cs, &out);
        if (le != cudaSuccess || ce != cudaSuccess) break;
        if (cudaGraphInstantiate(exec, g, 0) != cudaSuccess) break;
        *kernels = nk + 1;
        rc = SCAO_OK;
    } while (0);
    cudaGraphDestroy(g);
    return rc;
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
    { ProfScope _ps(SLOT_EIG_DIAG, st); eig_cold_start_kernel<<<dim3(16, np), NT, 0, st>>>(*P, leaf_ids); }
    SCAO_CHECK_LAUNCH();
    static PerDeviceOnce attr_done;
    if (attr_done.first()) {
        cudaFuncSetAttribute(eig_jacobi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)jacobi_smem(SMAX));
        cudaFuncSetAttribute(eig_cholinv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)cholinv_smem(SMAX));
        cudaFuncSetAttribute(eig_tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)std::max(eg_smem(false), eg_smem(true)));
    }
    if (max_iters > 0 && getenv("SCAO_EIG_NOGRAPH")) {
        // diagnostic: the same kernels launched directly, every iteration up
        // to the cap (converged problems return at once), each kernel timed
        { ProfScope _ps(SLOT_EIG_PREP, st);
          eig_loop_init_kernel<<<1, 256, 0, st>>>(*P, leaf_ids, np, max_iters, 0, 0); }
        for (int it = 0; it < max_iters; ++it)
            launch_iteration(*P, leaf_ids, np, nmax, smax, max_iters, tol, 0, 0, st);
        SCAO_CHECK_LAUNCH();
    } else if (max_iters > 0) {
        // the iteration loop: a cached executable graph per plan / leaf list
        const GraphKey key = make_key(P, leaf_ids, n_ids, nmax, smax, max_iters, tol);
        cudaGraphExec_t exec = nullptr;
        int64_t nk = 0;
        {
            std::lock_guard<std::mutex> lk(g_graph_mu);
            for (auto& e : g_graphs)
                if (e.key == key) { exec = e.exec; nk = e.kernels; break; }
            if (!exec) {
                const int rc = build_graph(P, leaf_ids, np, nmax, smax, max_iters, tol, &exec, &nk);
                if (rc != SCAO_OK) return rc;
                if (g_graphs.size() >= kMaxGraphs) {
                    cudaGraphExecDestroy(g_graphs.front().exec);
                    g_graphs.erase(g_graphs.begin());
                }
                g_graphs.push_back({key, exec, nk});
            }
        }
        ProfScope _ps(SLOT_EIG_ITER, st);
        scao_prof_add_launches(nk - 1);
        if (cudaGraphLaunch(exec, st) != cudaSuccess) return SCAO_ERR_LAUNCH;
    }
    { ProfScope _ps(SLOT_EIG_RANK, st); eig_rank_kernel<<<(n_ids + 127) / 128, 128, 0, st>>>(*P, leaf_ids, n_ids, eps_sparse, status); }
    SCAO_CHECK_LAUNCH();
    return scao_plan_prep_factors(P, leaf_ids, n_ids, stream);
}
