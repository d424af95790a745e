// Single-matrix entry points that replace the reference's kernel seam
// ``scao.cuda._scao_cuda`` (scao/cuda/low_rank_ops.cu:388-398):
//   fused_kronecker_precond  (low_rank_ops.cu:118-194, formula of the
//                             fallback scao/cuda/__init__.py:78-99)
//   low_rank_precond_mm      (low_rank_ops.cu:239-296, fallback :102-119;
//                             both left and right application are honoured)
// They run a generic tiled FP32 GEMM in four (resp. two) launches; the
// optimizer itself uses the batched plan kernels in apply.cu.
#include "common.cuh"
#include "prof.cuh"

namespace {

constexpr int NT = 256, TM = 64, TN = 64, TK = 16;

struct Op {            // element (r, c) of a logical matrix
    const void* p;
    int dt;            // SCAO_F32 / BF16 / F16
    int64_t ld;
    int trans;         // 1: stored transposed
    const float* colscale;   // optional per-column scale of the logical matrix
};

__device__ __forceinline__ float op_at(const Op& o, int r, int c) {
    const int64_t e = o.trans ? (int64_t)c * o.ld + r : (int64_t)r * o.ld + c;
    float v = load_dt(o.p, e, o.dt);
    if (o.colscale) v *= o.colscale[c];
    return v;
}

// C (M x N) = A (M x K) * B (K x N); epilogue: store fp32, or add an input
// matrix G (same layout as C, dtype gdt) and round to gdt.
__global__ void __launch_bounds__(NT)
gemm_kernel(Op A, Op B, int M, int N, int K, void* C, int64_t ldc, int cdt,
            const void* Gadd, int gdt) {
    const int tn = (N + TN - 1) / TN;
    const int i0 = (blockIdx.x / tn) * TM, j0 = (blockIdx.x % tn) * TN;
    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += TK) {
        for (int e = tid; e < TM * TK; e += NT) {
            const int ii = e >> 4, kk = e & 15;
            As[kk][ii] = (i0 + ii < M && k0 + kk < K) ? op_at(A, i0 + ii, k0 + kk) : 0.f;
        }
        for (int e = tid; e < TN * TK; e += NT) {
            const int kk = e >> 6, jj = e & 63;
            Bs[kk][jj] = (k0 + kk < K && j0 + jj < N) ? op_at(B, k0 + kk, j0 + jj) : 0.f;
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
    for (int r = 0; r < 4; ++r)
        for (int c = 0; c < 4; ++c) {
            const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
            if (i >= M || j >= N) continue;
            const int64_t e = (int64_t)i * ldc + j;
            float v = acc[r][c];
            if (Gadd) v = round_dt(__fadd_rn(load_dt(Gadd, e, gdt), v), gdt);
            store_dt(C, e, cdt, v);
        }
}

// Delta[a][b] = (s_l[a] * s_r[b] - 1) * P[a][b]   (in place)
__global__ void delta_kernel(float* Pm, const float* sl, const float* sr, int k) {
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < k * k; e += gridDim.x * blockDim.x) {
        const int a = e / k, b = e % k;
        Pm[e] = __fmul_rn(__fsub_rn(__fmul_rn(sl[a], sr[b]), 1.f), Pm[e]);
    }
}

int launch_gemm(Op A, Op B, int M, int N, int K, void* C, int64_t ldc, int cdt,
                const void* Gadd, int gdt, cudaStream_t st) {
    const int tiles = ((M + TM - 1) / TM) * ((N + TN - 1) / TN);
    { ProfScope _ps(SLOT_SEAM, st); gemm_kernel<<<tiles, NT, 0, st>>>(A, B, M, N, K, C, ldc, cdt, Gadd, gdt); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}

int64_t al(int64_t b) { return (b + 255) / 256 * 256; }

}  // namespace

extern "C" int64_t scao_fused_precond_scratch_bytes(int m, int n, int k) {
    return al((int64_t)n * k * 4) + al((int64_t)m * k * 4) + al((int64_t)k * k * 4) +
           al((int64_t)m * k * 4);
}

extern "C" int scao_fused_kronecker_precond(const float* U_l, const float* s_l_inv4,
                                            const float* U_r, const float* s_r_inv4,
                                            const void* G, void* out, int g_dtype,
                                            int m, int n, int k, void* scratch,
                                            void* stream) {
    if (!U_l || !U_r || !s_l_inv4 || !s_r_inv4 || !G || !out || !scratch) return SCAO_ERR_ARG;
    if (m <= 0 || n <= 0 || k <= 0 || k > 256 || g_dtype < 0 || g_dtype > 2) return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    char* s = (char*)scratch;
    float* T = (float*)s;                      s += al((int64_t)m * k * 4);
    float* Pm = (float*)s;                     s += al((int64_t)k * k * 4);
    float* W = (float*)s;
    int rc;
    // T = G U_r  (m x k)
    rc = launch_gemm({G, g_dtype, n, 0, nullptr}, {U_r, SCAO_F32, k, 0, nullptr}, m, k, n,
                     T, k, SCAO_F32, nullptr, 0, st);
    if (rc) return rc;
    // P = U_l^T T  (k x k)
    rc = launch_gemm({U_l, SCAO_F32, k, 1, nullptr}, {T, SCAO_F32, k, 0, nullptr}, k, k, m,
                     Pm, k, SCAO_F32, nullptr, 0, st);
    if (rc) return rc;
    { ProfScope _ps(SLOT_SEAM, st); delta_kernel<<<(k * k + 255) / 256, 256, 0, st>>>(Pm, s_l_inv4, s_r_inv4, k); }
    SCAO_CHECK_LAUNCH();
    // W = U_l Delta  (m x k)
    rc = launch_gemm({U_l, SCAO_F32, k, 0, nullptr}, {Pm, SCAO_F32, k, 0, nullptr}, m, k, k,
                     W, k, SCAO_F32, nullptr, 0, st);
    if (rc) return rc;
    // out = round(G + W U_r^T)
    return launch_gemm({W, SCAO_F32, k, 0, nullptr}, {U_r, SCAO_F32, k, 1, nullptr}, m, n, k,
                       out, n, g_dtype, G, g_dtype, st);
}

extern "C" int64_t scao_low_rank_precond_mm_scratch_bytes(int m, int n, int k, int left) {
    return left ? al((int64_t)k * n * 4) : al((int64_t)m * k * 4);
}

extern "C" int scao_low_rank_precond_mm(const float* U, const float* sv, const float* G,
                                        float* out, int m, int n, int k, int left,
                                        void* scratch, void* stream) {
    if (!U || !sv || !G || !out || !scratch || m <= 0 || n <= 0 || k <= 0) return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    float* T = (float*)scratch;
    int rc;
    if (left) {
        // U diag(s) U^T G:  T = U^T G (k x n), out = (U s) T
        rc = launch_gemm({U, SCAO_F32, k, 1, nullptr}, {G, SCAO_F32, n, 0, nullptr}, k, n, m,
                         T, n, SCAO_F32, nullptr, 0, st);
        if (rc) return rc;
        return launch_gemm({U, SCAO_F32, k, 0, sv}, {T, SCAO_F32, n, 0, nullptr}, m, n, k,
                           out, n, SCAO_F32, nullptr, 0, st);
    }
    // G U diag(s) U^T:  T = G (U s) (m x k), out = T U^T
    rc = launch_gemm({G, SCAO_F32, n, 0, nullptr}, {U, SCAO_F32, k, 0, sv}, m, k, n,
                     T, k, SCAO_F32, nullptr, 0, st);
    if (rc) return rc;
    return launch_gemm({T, SCAO_F32, k, 0, nullptr}, {U, SCAO_F32, k, 1, nullptr}, m, n, k,
                       out, n, SCAO_F32, nullptr, 0, st);
}

extern "C" const char* scao_version(void) { return "scao_b200 0.1.0 sm_100a"; }
