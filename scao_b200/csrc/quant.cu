// int8 symmetric quantisation and the int8 curvature-EMA requant.
//
// Semantics follow the path the reference library actually runs
// (scao/preconditioner.py:344-350 -> scao/utils.py:170-203):
//   x      = float(q) * float(scale)          (dequantize, utils.py:203)
//   x      = x * float(rho) + new_val         (preconditioner.py:345)
//   s'     = double(max|x|) / 127             (utils.py:184-187, Python float)
//   q'     = clamp(rint(x / float(s')), +-127)  (utils.py:188: true division,
//            round-half-even; the reference CUDA kernel's reciprocal multiply,
//            low_rank_ops.cu:227-228, is NOT bit-exact and is not used here)
//   max|x| < 1e-30 -> q' = 0, s' = 1.0         (utils.py:185-186)
// Every multiply and add is rounded separately (no FMA contraction), as the
// reference evaluates them as separate tensor ops.
#include "common.cuh"
#include "prof.cuh"

#include <mutex>

namespace {

constexpr int kThreads = 256;

__global__ void ema_pass1_kernel(const int8_t* __restrict__ q, float scale_f,
                                 float rho_f, const float* __restrict__ add,
                                 int64_t n, float* __restrict__ x_out,
                                 float* __restrict__ absmax) {
    __shared__ float red[32];
    float m = 0.f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float x = q ? __fmul_rn(__fmul_rn((float)q[i], scale_f), rho_f) : 0.f;
        if (add) x = __fadd_rn(x, add[i]);
        if (x_out) x_out[i] = x;
        m = fmaxf(m, fabsf(x));
    }
    m = block_max(m, red);
    if (threadIdx.x == 0) atomic_max_nonneg(absmax, m);
}

__global__ void requant_kernel(const float* __restrict__ x, int64_t n,
                               const float* __restrict__ absmax,
                               int8_t* __restrict__ q, double* scale_out) {
    const float am = *absmax;
    const bool zero = (double)am < 1e-30;
    const float s = quant_scale_f(am);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        q[i] = quant_one(x[i], s, zero);
    if (scale_out && blockIdx.x == 0 && threadIdx.x == 0)
        *scale_out = zero ? 1.0 : (double)am / 127.0;
}

__global__ void dequant_kernel(const int8_t* __restrict__ q, float scale_f,
                               int64_t n, float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn((float)q[i], scale_f);
}

int grid_for(int64_t n) {
    int64_t g = (n + kThreads - 1) / kThreads;
    if (g > 148 * 16) g = 148 * 16;
    return g < 1 ? 1 : (int)g;
}

}  // namespace

extern "C" int64_t scao_int8_ema_scratch_bytes(int64_t n) {
    return ((n * 4 + 255) / 256) * 256 + 256;
}

extern "C" int scao_int8_ema_update(const int8_t* q, double scale,
                                    const float* new_val, double rho,
                                    int64_t n, int8_t* q_out,
                                    double* scale_out, void* scratch,
                                    void* stream) {
    if (n <= 0 || !q || !new_val || !q_out || !scratch) return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    float* x = (float*)scratch;
    float* am = (float*)((char*)scratch + ((n * 4 + 255) / 256) * 256);
    if (cudaMemsetAsync(am, 0, sizeof(float), st) != cudaSuccess) return SCAO_ERR_LAUNCH;
    { ProfScope _ps(SLOT_QUANT, st); ema_pass1_kernel<<<grid_for(n), kThreads, 0, st>>>(q, (float)scale, (float)rho,
                                                       new_val, n, x, am); }
    SCAO_CHECK_LAUNCH();
    { ProfScope _ps(SLOT_QUANT, st); requant_kernel<<<grid_for(n), kThreads, 0, st>>>(x, n, am, q_out, scale_out); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}

extern "C" int scao_quantize_sym_int8(const float* x, int64_t n, int8_t* q,
                                      double* scale_out, void* scratch,
                                      void* stream) {
    if (n <= 0 || !x || !q || !scratch) return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    float* am = (float*)scratch;
    if (cudaMemsetAsync(am, 0, sizeof(float), st) != cudaSuccess) return SCAO_ERR_LAUNCH;
    // pass 1 with no dequantised term and no output: absmax of x only
    { ProfScope _ps(SLOT_QUANT, st); ema_pass1_kernel<<<grid_for(n), kThreads, 0, st>>>(nullptr, 0.f, 0.f, x, n,
                                                       nullptr, am); }
    SCAO_CHECK_LAUNCH();
    { ProfScope _ps(SLOT_QUANT, st); requant_kernel<<<grid_for(n), kThreads, 0, st>>>(x, n, am, q, scale_out); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}

extern "C" int scao_dequantize_sym_int8(const int8_t* q, double scale, int64_t n,
                                        float* out, void* stream) {
    if (n <= 0 || !q || !out) return SCAO_ERR_ARG;
    { ProfScope _ps(SLOT_QUANT, (cudaStream_t)stream); dequant_kernel<<<grid_for(n), kThreads, 0, (cudaStream_t)stream>>>(q, (float)scale, n, out); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of scao_int8_ema_update.
//
// Some callers cannot allocate device memory at all: code running inside a
// host that owns a fixed memory pool (an inference server or a framework
// plugin whose allocator is not reachable from this library), or a caller
// that must not add cudaMalloc/cudaFree synchronisation points to its stream.
// For them the fp32 staging buffer and the max|x| slot live in this
// file-scope device array, sized for factors up to 1024 x 1024.  Every GPU
// that loads the library holds these 4 MiB until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocMaxN = int64_t(1) << 20;   // elements (a 1024 x 1024 factor)
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMaxN + 64];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  The name of the
// array in host code is only a host-side stand-in, never a device pointer.
int noalloc_scratch(float** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return SCAO_ERR_LAUNCH;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            (void)cudaGetLastError();
            return SCAO_ERR_LAUNCH;
        }
        g_noalloc_ptr[dev] = (float*)p;
    }
    *out = g_noalloc_ptr[dev];
    return SCAO_OK;
}

}  // namespace

extern "C" int64_t scao_int8_ema_update_noalloc_max_n(void) { return kNoAllocMaxN; }

extern "C" int scao_int8_ema_update_noalloc(const int8_t* q, double scale,
                                            const float* new_val, double rho,
                                            int64_t n, int8_t* q_out,
                                            double* scale_out, void* stream) {
    if (n <= 0 || n > kNoAllocMaxN || !q || !new_val || !q_out) return SCAO_ERR_ARG;
    float* x = nullptr;
    const int rc = noalloc_scratch(&x);
    if (rc != SCAO_OK) return rc;
    float* am = x + kNoAllocMaxN;
    cudaStream_t st = (cudaStream_t)stream;
    // the array keeps the previous call's contents: the max slot must restart at 0
    if (cudaMemsetAsync(am, 0, sizeof(float), st) != cudaSuccess) return SCAO_ERR_LAUNCH;
    { ProfScope _ps(SLOT_QUANT, st); ema_pass1_kernel<<<grid_for(n), kThreads, 0, st>>>(q, (float)scale, (float)rho, new_val, n, x, am); }
    SCAO_CHECK_LAUNCH();
    { ProfScope _ps(SLOT_QUANT, st); requant_kernel<<<grid_for(n), kThreads, 0, st>>>(x, n, am, q_out, scale_out); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}
