/*
 * scao_b200 -- C ABI of the B200-native SCAO optimizer step.
 *
 * Plain C: device pointers, sizes, a cudaStream_t passed as void*, and an
 * int status (0 = ok, see SCAO_ERR_*).  Nothing here traps on the device;
 * errors are returned.  All pointers are device pointers unless the name says
 * ``host``.  The library never allocates device memory: every scratch buffer
 * is passed in by the caller (its size comes from the *_scratch_bytes query).
 *
 * Two layers:
 *
 *  1. Single-matrix entry points that replace the reference's kernel seam
 *     ``scao.cuda._scao_cuda`` (reference scao/cuda/low_rank_ops.cu:388-398,
 *     dispatched from scao/cuda/__init__.py:149-266).
 *
 *  2. Batched "plan" entry points used by the Python optimizer facade: one
 *     launch per phase per optimizer step covering every parameter, replacing
 *     the per-parameter Python loop of scao/optimizer.py:509-645 and the
 *     per-block loops of scao/preconditioner.py:297-564.
 */
#ifndef SCAO_B200_H
#define SCAO_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SCAO_API __attribute__((visibility("default")))
#else
#define SCAO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SCAO_OK 0
#define SCAO_ERR_ARG 1        /* bad size / pointer / dtype                  */
#define SCAO_ERR_LAUNCH 2     /* a CUDA launch or runtime call failed         */
#define SCAO_ERR_NOCONV 3     /* eigensolver hit its iteration cap (status
                                 per problem is also written to the device)  */

/* parameter dtypes */
#define SCAO_F32 0
#define SCAO_BF16 1
#define SCAO_F16 2

/* ---------------------------------------------------------------------- */
/* Plan tables (layout shared with scao_b200/plan.py, all little-endian)   */
/* ---------------------------------------------------------------------- */

/* One per parameter (static).  mode: 0 diagonal, 1 Kronecker leaf(s).     */
typedef struct {
    int64_t offset;        /* element offset of this param in state arenas */
    int64_t numel;
    int32_t rows, cols;    /* to_2d view (utils.py:208-219)                */
    int32_t mode;
    int32_t dtype;
    int32_t leaf_begin, leaf_end;     /* Kronecker leaves (block order)    */
    int32_t tile_begin, tile_end;     /* apply tiles of those leaves       */
    int32_t chunk_begin, chunk_end;   /* flat chunks of the whole param    */
} ScaoParam;

/* One per parameter per optimizer step (host writes, copies to device).  */
typedef struct {
    uint64_t p_ptr, g_ptr; /* parameter and gradient data                  */
    int32_t phase;         /* 0 no grad, 1 Adam warmup, 2 SCAO             */
    int32_t clip;          /* 1 if tau is not None                         */
    double lr;             /* group lr                                      */
    double alpha1;         /* -(lr / bc1), Phase-1 parameter step           */
    float wd_mult;         /* float(1 - lr*wd)                              */
    float wd;              /* float(weight_decay)                           */
    float beta1, beta2, beta3;
    float c1, c2, c3;      /* float(1 - beta_i)                             */
    float bc1, bc2, bc3;   /* float(1 - beta_i ** step)                     */
    float sqrt_bc2;        /* float(math.sqrt(bc2))                         */
    float eps;
    float blend, one_minus_blend;
    float tau;
    float lars;
    float diag_bias;       /* float(max(1 - rho**precond_step, 1e-8))       */
    float rbc1, rbc2, rbc3;/* reciprocals of bc1..bc3 (division by constant);
                              Phase 1: rbc2 = 1 / sqrt_bc2               */
} ScaoParamStep;

/* One per Kronecker leaf block (static).  Each leaf owns two symmetric
 * "factor problems": side 0 = L (a x a), side 1 = R (b x b); problem id
 * = 2*leaf + side.                                                        */
typedef struct {
    int32_t param;
    int32_t row0, col0;    /* block origin inside the param's 2-D view     */
    int32_t a, b;          /* block rows, cols                             */
    int32_t ld;            /* param cols (row stride of the block)         */
    int32_t kmin, kmax;    /* preconditioner.py:122-124                     */
    int32_t kpad;          /* kmax rounded up to 8                          */
    int32_t sl, sr;        /* eigen subspace widths (kpad <= s <= n)        */
    int32_t tile_begin, tile_end;
    int32_t panel_begin, panel_end;
    int32_t pad0;
    int64_t lq_off, rq_off;/* factor arena offsets (a*a, b*b elements)      */
    int64_t ul_off, ur_off;/* eigenvector arena offsets (a*sl, b*sr floats) */
    int64_t hl_off, hr_off;/* small s x s arena offsets                     */
    int64_t evl_off, evr_off; /* eigenvalue arena offsets (sl, sr floats)   */
    int64_t w_off;         /* W = U_l*Delta scratch: a*kpad floats          */
    /* bf16 hi/lo operand tiles for the tensor-core kernels (byte offsets;
     * Kp = kpad rounded up to 16; tile layouts are the canonical K-major
     * no-swizzle layout of tc.cuh):
     *   ua: U_r rows, per 128-row tile [hi 128 x Kp][lo 128 x Kp]
     *   ut: U_r^T,    per 64-row block of U_r [hi Kp x 64][lo Kp x 64]
     *   wa: W rows,   per 128-row tile [hi 128 x Kp][lo 128 x Kp]          */
    int64_t ua_off, ut_off, wa_off;
} ScaoLeaf;

/* Apply tile of a Kronecker leaf: 64x64 elements.                          */
typedef struct { int32_t leaf, row0, col0, pad0; } ScaoTile;

/* Projection panel of a Kronecker leaf: 64 rows.                           */
typedef struct { int32_t leaf, row0, nrows, pad0; } ScaoPanel;

/* Flat chunk of a parameter (element range).                               */
typedef struct { int32_t param, pad0; int64_t begin, end; } ScaoChunk;

/* Diagonal strip of a block-diagonal parameter: a remainder block of width 1
 * (1 x b or a x 1) of the recursive split, which the reference gives a
 * diagonal sub-preconditioner (preconditioner.py:142-156, 232-236;
 * precondition :506-510, curvature :332-339, natural norm :554-556).  Its
 * elements are begin + j * stride, j < count (stride 1: a row, stride = the
 * parameter's columns: a column).                                           */
typedef struct { int32_t param, count, stride, pad0; int64_t begin; } ScaoStrip;

/* Gradient filter (scao/optimizer.py:40-97, applied at :536-542) and
 * gradient noise (:544-545).  The filtered gradient
 *     grad * (mag_ema >= quantile(mag_ema, sparsity))
 * feeds the moments and prev_grad; the preconditioner keeps the raw grad.
 * The quantile is an exact radix selection of two order statistics on the
 * float32 bit patterns (3 levels: bits 31-20, 19-8, 7-0).                   */
typedef struct {
    double norm_ema;       /* R2 layer-norm EMA (starts at 1.0)              */
    double global_ref;     /* R2 global-norm reference (starts at 1.0)       */
    double sparsity;       /* quantile level of this step                     */
    int64_t rem_lo, rem_hi;/* rank left inside the radix prefix found so far */
    uint32_t pre_lo, pre_hi; /* radix prefixes (float32 bit patterns)        */
    float w;               /* lerp weight: rank - floor(rank)                */
    float thr;             /* threshold of this step                          */
    float gsq;             /* sum of raw grad^2 of this step                  */
    int32_t first;         /* 1 until the parameter's first filter call      */
    int32_t nan;           /* 1 if the magnitude EMA holds a NaN             */
    int32_t sel_begin, sel_end; /* selection chunks of this parameter        */
    int32_t pad0;
} ScaoFilterParam;

typedef struct {
    int32_t mode;          /* 0 off, 1 static sparsity, 2 dynamic (R2)        */
    int32_t n_sel;         /* number of selection chunks                      */
    const ScaoChunk* sel;  /* <= 65536-element pieces of every parameter      */
    float* mag_ema;        /* magnitude EMA, numel total (state arena offsets) */
    ScaoFilterParam* fp;   /* n_params                                        */
    uint32_t* hist;        /* n_params x 2 x 4096 radix histograms            */
    float* sel_part;       /* per selection chunk: sum of raw grad^2          */
    double base, min_s, max_s, norm_coeff; /* sparsity, 0.3, 0.9, 0.95 (R2)   */
    float ema, ema_c;      /* float32(ema), float32(1 - ema)                  */
    int32_t noise_on;      /* 1 if noise_std > 1e-9 this step                 */
    float noise_std;       /* float32(noise_std)                              */
    uint64_t noise_seed;   /* Philox-4x32-10 key                              */
    uint64_t noise_step;   /* counter word: global step                       */
    int32_t gsnr_on;       /* R4: update * (|m| / (sqrt(v) + eps) >= thr)     */
    float gsnr_thr;        /* float32(gsnr_threshold)                         */
} ScaoFilterDev;

/* Device-side plan: pointers to the tables and arenas above.              */
typedef struct {
    int32_t n_params, n_leaves, n_tiles, n_panels, n_chunks;
    int32_t int8_ema;      /* 1: L/R stored int8 + absmax; 0: fp32          */
    int32_t kpad_max;      /* largest leaf kpad (<= 128)                    */
    int32_t p_stride;      /* floats per projection partial: kpad_max^2 + 4 */
    int32_t kron_dtypes;   /* bit mask (1 << dtype) over Kronecker params   */
    int32_t max_leaf_rows_tiles; /* max over leaves of ceil(a / 128)        */
    const ScaoParam* params;
    const ScaoLeaf* leaves;
    const ScaoTile* tiles;
    const ScaoPanel* panels;
    const ScaoChunk* chunks;
    const ScaoParamStep* step;   /* per-step table (n_params)              */
    /* optimizer state arenas (numel total each, fp32)                     */
    float *exp_avg, *exp_avg_sq, *exp_avg_diff, *prev_grad;
    float* diag_ema;             /* numel total (used by diagonal params)   */
    void* fac;                   /* factor arena: int8 or fp32 L and R      */
    float* absmax;               /* per problem max|L| (int8 mode)          */
    float* u;                    /* eigenvector arena (row-major n x s)     */
    float* ev;                   /* eigenvalue arena (descending)           */
    int32_t* k;                  /* per leaf current rank                   */
    /* scratch (caller-owned; sizes computed by the plan builder)          */
    float *eig_y, *eig_x, *eig_ax;  /* same layout as u                     */
    float *eig_h, *eig_v;        /* small s x s arenas                      */
    float* eig_aux;              /* per problem 16 floats                   */
    float* w;                    /* U_l*Delta per leaf                      */
    float* p_part;               /* projection partials n_panels*kpad^2     */
    float* tile_part;            /* per tile partial sums (4 each)          */
    float* chunk_part;           /* per chunk partial sums (4 each)         */
    uint16_t* upd;               /* rounded update, numel (param dtype)     */
    float* upd32;                /* update for fp32 params, numel           */
    float* leaf_nat2;            /* per leaf natural-norm^2                 */
    float* param_scalars;        /* per param: 8 floats                     */
    double* global_norm_ema;     /* 1 double (device)                       */
    uint16_t* slow;              /* lookahead slow weights, 16-bit params   */
    float* slow32;               /* lookahead slow weights, fp32 params     */
    uint8_t *ua, *ut, *wa;       /* operand tile arenas (see ScaoLeaf)      */
    int32_t* counters;           /* 16 device ints of small bookkeeping      */
    /* chunk id lists: diagonal-mode params (static); params whose flat pass
     * runs this step (Phase 1, or Phase 2 diagonal); Phase-2 params        */
    const int32_t *diag_list, *flat_list, *p_list;
    int32_t n_diag, n_flat, n_p;
    int32_t proj_fallback;       /* 1: some Phase-2 bf16 panel needs the
                                    cp.async projection kernel this step   */
    int32_t apply_fallback;      /* 1: some Phase-2 tile needs the register-
                                    streaming apply kernel this step        */
    int32_t sm_reserve;          /* SMs the persistent kernels leave free
                                    (for concurrent collectives)            */
    int32_t la_fused;            /* 1: this step's lookahead of Phase-2 params
                                    runs inside the parameter write (then
                                    scao_plan_lookahead skips them)         */
    int32_t la_init;             /* 1: first lookahead (slow <- p)          */
    float la_alpha;              /* lookahead_alpha                         */
    int32_t pad5_;
    int32_t* err;                /* device error flag: set to 1 when a bounded
                                    wait on the tensor core timed out       */
    uint8_t* tmaps;              /* n_params x 10 TMA tensor maps (128 B each,
                                    written by scao_plan_tensor_maps and
                                    scao_plan_curvature)                    */
    int32_t tmaps_ok;            /* 1: tmaps describe this step's gradients */
    int32_t gnorm_host;          /* 1: the host maintains *global_norm_ema
                                    this step (the kernels only read it)    */
    ScaoFilterDev filt;          /* gradient filter and noise (mode 0: off) */
    const ScaoStrip* strips;     /* diagonal strips of Kronecker params      */
    float* strip_part;           /* per strip: |u|^2, |g|^2, |p_dec|^2, nat^2 */
    int32_t n_strips;
    int32_t pad6_;
    uint8_t* eig_img;            /* eigensolver operand images (bf16 hi/mid/lo
                                    tiles of an n x s block), eig_img_stride
                                    bytes per factor problem 2*leaf+side     */
    int64_t eig_img_stride;
} ScaoPlanDev;

/* ---------------------------------------------------------------------- */
/* 1. Single-matrix entry points (reference kernel seam)                   */
/* ---------------------------------------------------------------------- */

/* Replaces ``fused_kronecker_precond`` (low_rank_ops.cu:118-194,
 * launcher :298-336; fallback formula cuda/__init__.py:78-99):
 *   out = G + U_l ((s_l s_r^T - 1) o (U_l^T G U_r)) U_r^T
 * U_l (m x k), U_r (n x k) row-major fp32, s_* fp32 (k), G (m x n) row-major
 * of dtype g_dtype; out same dtype as G.  k <= 256.  scratch: at least
 * scao_fused_precond_scratch_bytes(m, n, k) bytes.                         */
SCAO_API int scao_fused_kronecker_precond(const float* U_l, const float* s_l_inv4,
                                 const float* U_r, const float* s_r_inv4,
                                 const void* G, void* out, int g_dtype,
                                 int m, int n, int k, void* scratch,
                                 void* stream);
SCAO_API int64_t scao_fused_precond_scratch_bytes(int m, int n, int k);

/* Replaces ``low_rank_precond_mm`` (low_rank_ops.cu:239-296, fallback
 * cuda/__init__.py:102-119): left=1: U diag(s) U^T G, left=0: G U diag(s) U^T.
 * Unlike the reference launcher, left=0 is honoured.  fp32 only.          */
SCAO_API int scao_low_rank_precond_mm(const float* U, const float* s, const float* G,
                             float* out, int m, int n, int k, int left,
                             void* scratch, void* stream);
SCAO_API int64_t scao_low_rank_precond_mm_scratch_bytes(int m, int n, int k, int left);

/* Replaces ``int8_ema_update`` (low_rank_ops.cu:203-231, 342-383) with the
 * semantics the library path actually uses (preconditioner.py:344-350 via
 * utils.py:170-203):  x = float(q)*float(scale)*float(rho) + new_val, then
 * q' = clamp(rint(x / float(s')), +-127), s' = double(max|x|)/127 (1.0 and
 * q'=0 when max|x| < 1e-30).  IEEE division, bit-exact with the CPU path.
 * Writes q_out (may alias q) and scale_out[0] = double s' (device).
 * scratch: scao_int8_ema_scratch_bytes(n) bytes.                           */
SCAO_API int scao_int8_ema_update(const int8_t* q, double scale, const float* new_val,
                         double rho, int64_t n, int8_t* q_out,
                         double* scale_out, void* scratch, void* stream);
SCAO_API int64_t scao_int8_ema_scratch_bytes(int64_t n);

/* Allocation-free form of scao_int8_ema_update, same semantics and results.
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory (a host with its own fixed device-memory pool, or a stream that
 * must not see cudaMalloc/cudaFree): the staging buffer is a file-scope
 * device array of scao_int8_ema_update_noalloc_max_n() = 1,048,576 elements
 * (a 1024 x 1024 factor); larger n returns SCAO_ERR_ARG.  The first call on
 * each device looks up that array's device address (cudaGetSymbolAddress)
 * with the device current -- make that first call before any stream capture.
 * All calls on a device share the one array: calls that overlap on the GPU
 * (different streams without ordering) race and corrupt each other.       */
SCAO_API int scao_int8_ema_update_noalloc(const int8_t* q, double scale,
                                          const float* new_val, double rho,
                                          int64_t n, int8_t* q_out,
                                          double* scale_out, void* stream);
SCAO_API int64_t scao_int8_ema_update_noalloc_max_n(void);

/* Symmetric per-tensor quantisation alone (utils.py:170-189): x (n fp32)
 * -> q (int8), scale_out[0] (double, device).                              */
SCAO_API int scao_quantize_sym_int8(const float* x, int64_t n, int8_t* q,
                           double* scale_out, void* scratch, void* stream);
/* utils.py:192-203: out = float(q) * float(scale).                         */
SCAO_API int scao_dequantize_sym_int8(const int8_t* q, double scale, int64_t n,
                             float* out, void* stream);

/* ---------------------------------------------------------------------- */
/* 2. Batched plan entry points (one optimizer step = a sequence of these) */
/* ---------------------------------------------------------------------- */

/* Curvature EMA for the leaves listed in leaf_ids (device int32, n ids):
 * L <- rho*L + (1-rho) G G^T, R <- rho*R + (1-rho) G^T G
 * (preconditioner.py:341-353), int8 requant fused (utils.py:170-203).
 * scratch: scao_ema_scratch_bytes(...) bytes.  params_host / step_host /
 * leaves_host / leaf_ids_host: host copies of the parameter, step and leaf
 * tables and of leaf_ids (may be NULL); with them the bf16 factor GEMMs run on the TMA-fed persistent
 * tensor-core kernel, whose per-gradient tensor maps are written to
 * plan_host->tmaps, and the fallback kernels launch only when needed.      */
SCAO_API int scao_plan_curvature(const ScaoPlanDev* plan_host, const int32_t* leaf_ids,
                        int n_ids, int max_a, int max_b, double rho,
                        void* scratch, int64_t scratch_bytes,
                        const ScaoParam* params_host, const ScaoParamStep* step_host,
                        const ScaoLeaf* leaves_host, const int32_t* leaf_ids_host,
                        void* stream);
SCAO_API int64_t scao_ema_scratch_bytes(int n_ids, int max_a, int max_b);

/* Diagonal-mode curvature EMA for the params in param_ids
 * (preconditioner.py:332-339).                                             */
SCAO_API int scao_plan_curvature_diag(const ScaoPlanDev* plan_host,
                             const int32_t* param_ids, int n_ids, double rho,
                             void* stream);

/* TMA tensor maps of this step's gradients into plan_host->tmaps (host
 * tables: params_host = the plan's ScaoParam table, step_host = this step's
 * ScaoParamStep table).  The per-step kernels use them only when
 * plan_host->tmaps_ok is 1, which the caller sets after SCAO_OK.           */
SCAO_API int scao_plan_tensor_maps(const ScaoPlanDev* plan_host, const ScaoParam* params_host,
                          const ScaoParamStep* step_host, void* stream);

/* Per-parameter fp32 norm of this step's raw gradient, ||g|| (0 for params
 * without a gradient) into out (device, n_params floats).  Feeds the host
 * logic of the R1 / R3 / R5 extensions (optimizer.py:161-214, 383-401,
 * 439-446).                                                                 */
SCAO_API int scao_plan_grad_norms(const ScaoPlanDev* plan_host, float* out, void* stream);

/* Eigen update of the listed leaves (preconditioner.py:363-451):
 * debias, Tikhonov eps = max(1e-8, 1e-4 tr/m), the top eigenpairs by
 * warm-started Chebyshev-filtered subspace iteration with Rayleigh-Ritz
 * (Jacobi) on the tensor cores -- no cuSOLVER -- and rank selection
 * (utils.py:121-151 + hysteresis :437-441).
 * bias_factor, eps_sparse: per leaf (device float arrays indexed by leaf).
 * max_iters: cap on outer iterations (each: Rayleigh-Ritz + one filter).
 * tol: a leading block of Ritz vectors that ends at a relative spectral gap
 * of 1e-2 is accepted when its largest residual norm is <= tol * gap
 * (subspace angle <~ tol rad); every usable pair also needs residual <=
 * 1e-3 * theta_1, except pairs in the flat bulk at the bottom of the block.
 * nmax / smax: largest factor size / subspace width among the listed leaves
 * (nmax <= 4096, smax <= 160).  status (device, 2*n_ids ints, may be NULL):
 * iterations used per factor problem, negative when the cap was reached.
 * The iteration runs as a cached CUDA graph (conditional WHILE node): the
 * host does not wait for the device.  Workspaces are the plan's eig_*
 * arenas.                                                                   */
SCAO_API int scao_plan_eigen(const ScaoPlanDev* plan_host, const int32_t* leaf_ids,
                    int n_ids, const float* bias_factor,
                    const float* eps_sparse, int max_iters, float tol,
                    int32_t* status, int nmax, int smax, void* stream);

/* One full optimizer step for every parameter whose step-table phase is 1
 * or 2 (optimizer.py:521-645): projection, curvature clip, Adan/Adam
 * moments, LARS trust ratio and the parameter write.  The per-step table
 * plan->step must already be on the device.                                */
SCAO_API int scao_plan_step(const ScaoPlanDev* plan_host, void* stream);

/* Refresh the bf16 hi/lo operand tiles (ua, ut) of the listed leaves from
 * their fp32 eigenvectors; scao_plan_eigen does this itself, the plan
 * builder calls it once after initialising U.                             */
SCAO_API int scao_plan_prep_factors(const ScaoPlanDev* plan_host, const int32_t* leaf_ids,
                                    int n_ids, void* stream);

/* Lookahead (optimizer.py:356-365): slow += alpha (p - slow); p <- slow.
 * init=1 on the first sync copies p into slow first.                      */
SCAO_API int scao_plan_lookahead(const ScaoPlanDev* plan_host, float alpha, int init,
                        void* stream);

/* Instrumentation: number of kernels this library has launched so far, and
 * optional CUDA-event timing of every launch on its own stream (per kernel
 * slot; names from scao_prof_name).                                        */
SCAO_API int64_t scao_launch_count(void);
SCAO_API void scao_prof_enable(int on);
SCAO_API int scao_prof_read(double* ms, int64_t* counts, int nslots);
SCAO_API void scao_prof_reset(void);
SCAO_API const char* scao_prof_name(int slot);
SCAO_API int scao_prof_slots(void);

/* Known-answer check of the tensor-core path: C (128 x N fp32) = A (128 x K
 * bf16, row-major) * B^T (B: N x K bf16, row-major); N, K multiples of 16,
 * N <= 256, K <= 128.  *err set to 1 if the MMA completion wait timed out.
 * mn_major=1 stages both operands in the MN-major shared-memory layout.   */
SCAO_API int scao_tc_selftest(const uint16_t* A, const uint16_t* B, float* C, int N, int K,
                              int* err, int mn_major, void* stream);

/* Check of the division-by-constant rewrite used by the Adan update: counts
 * x[i] / c[i % 1024] where reciprocal-plus-FMA-correction differs from the
 * IEEE quotient (adds into *mismatches).                                   */
/* Self-check of the bounded device waits (no reference counterpart): one
 * kernel waits on an mbarrier nothing arrives at, with an iteration limit;
 * it must give up, write 1 to *err (device int) and return normally.      */
SCAO_API int scao_wait_timeout_check(int* err, unsigned int limit, void* stream);

SCAO_API int scao_divc_check(const float* x, const float* c, int n, int* mismatches,
                             void* stream);

/* Library identification. */
SCAO_API const char* scao_version(void);

#ifdef __cplusplus
}
#endif
#endif /* SCAO_B200_H */
