// Sparse gradient filter of scao/optimizer.py:40-97 for all parameters at
// once, run at the start of scao_plan_step when sparsity > 0.
//
//   mag_ema <- |g|                               (first call, :52-53)
//   mag_ema <- mag_ema*ema + (1-ema)*|g|         (separately rounded, :55)
//   thr     <- torch.quantile(mag_ema, sparsity) (:56)
//   mask    =  mag_ema >= thr                    (:57, applied in apply.cu)
//
// R2 (_DynamicSparseFilter, :59-97) replaces ``sparsity`` per parameter by
// clamp(base + 0.2 (1 - min(norm_ema / global_ref, 2) / 2), 0.3, 0.9) with
// norm_ema an EMA of ||g|| and global_ref the optimizer's global grad-norm
// EMA (set before the call, :464-467), all in double like Python floats.
//
// The quantile is exact.  ATen's linear quantile is
//   rank = float32(q) * (n - 1)     (float32 arithmetic)
//   lo = floor(rank), hi = ceil(rank), w = rank - lo
//   thr = lerp(sorted[lo], sorted[hi], w)
// and any NaN makes it NaN.  Magnitudes are non-negative, so their float32
// bit patterns sort like the values: the two order statistics come from a
// three-level radix selection over the bit patterns (bits 31-20, 19-8, 7-0),
// each level one histogram pass over the parameter and one scan per
// parameter.  No sort, no 2^24 cap (torch.quantile refuses larger inputs;
// beyond that size the rank is formed in float64 here).
#include "filter.cuh"
#include "prof.cuh"

namespace {

constexpr int FB = 4096;    // bins of the 12-bit levels
constexpr int FNT = 512;    // threads of the histogram passes
constexpr int SNT = 1024;   // threads of the scans

SCAO_DEV bool nan_key(uint32_t k) { return (k & 0x7fffffffu) > 0x7f800000u; }

// Level-1 pass: magnitude EMA update, level-1 histogram, sum of raw g^2.
__global__ void __launch_bounds__(FNT)
filt_update_kernel(ScaoPlanDev P) {
    const ScaoChunk ch = P.filt.sel[blockIdx.x];
    const int pi = ch.param;
    const ScaoParamStep& S = P.step[pi];
    if (S.phase == 0) return;
    const ScaoParam& pr = P.params[pi];
    ScaoFilterParam* F = P.filt.fp + pi;
    __shared__ uint32_t h[FB];
    __shared__ float red[32];
    __shared__ int snan;
    for (int i = threadIdx.x; i < FB; i += FNT) h[i] = 0;
    if (threadIdx.x == 0) snan = 0;
    __syncthreads();
    const bool first = F->first != 0;
    const float ema = P.filt.ema, emc = P.filt.ema_c;
    float* mg = P.filt.mag_ema + pr.offset;
    const void* g = (const void*)S.g_ptr;
    const int dt = pr.dtype;
    float gsq = 0.f;
    int nan = 0;
    auto one = [&](float gv, float& m) {
        const float a = fabsf(gv);
        m = first ? a : __fadd_rn(__fmul_rn(m, ema), __fmul_rn(emc, a));
        gsq = fmaf(gv, gv, gsq);
        const uint32_t k = __float_as_uint(m);
        if (nan_key(k)) nan = 1;
        else atomicAdd(&h[k >> 20], 1u);
    };
    const bool vec = ((S.g_ptr & 15) == 0) && ((pr.offset & 3) == 0) && ((ch.begin & 3) == 0);
    int64_t vend = ch.begin;
    if (vec) {
        const int64_t n4 = (ch.end - ch.begin) >> 2;
        vend = ch.begin + n4 * 4;
        for (int64_t q = threadIdx.x; q < n4; q += FNT) {
            const int64_t e = ch.begin + q * 4;
            const float4 g4 = load4_dt(g, e, dt);
            float4 m4 = first ? make_float4(0.f, 0.f, 0.f, 0.f) : *(const float4*)(mg + e);
            one(g4.x, m4.x);
            one(g4.y, m4.y);
            one(g4.z, m4.z);
            one(g4.w, m4.w);
            *(float4*)(mg + e) = m4;
        }
    }
    for (int64_t e = vend + threadIdx.x; e < ch.end; e += FNT) {
        float m = first ? 0.f : mg[e];
        one(load_dt(g, e, dt), m);
        mg[e] = m;
    }
    if (nan) snan = 1;
    gsq = block_sum(gsq, red);      // also orders the shared histogram
    uint32_t* gh = P.filt.hist + (size_t)pi * 2 * FB;
    for (int i = threadIdx.x; i < FB; i += FNT)
        if (h[i]) atomicAdd(gh + i, h[i]);
    if (threadIdx.x == 0) {
        P.filt.sel_part[blockIdx.x] = gsq;
        if (snan) F->nan = 1;
    }
}

// Per parameter: ||g||^2 from the chunk partials.
__global__ void __launch_bounds__(256)
filt_param_kernel(ScaoPlanDev P) {
    const int pi = blockIdx.x;
    if (P.step[pi].phase == 0) return;
    ScaoFilterParam* F = P.filt.fp + pi;
    __shared__ float red[32];
    float s = 0.f;
    for (int c = F->sel_begin + threadIdx.x; c < F->sel_end; c += 256) s += P.filt.sel_part[c];
    s = block_sum(s, red);
    if (threadIdx.x == 0) {
        F->gsq = s;
        P.param_scalars[pi * 8 + PS_GNORM2] = s;
    }
}

// Global grad-norm EMA (optimizer.py:439-446, summed in parameter order like
// Python's sum), then per parameter the quantile level (R2 in double) and
// the two target ranks.
__global__ void __launch_bounds__(256)
filt_global_kernel(ScaoPlanDev P) {
    __shared__ double gema;
    __shared__ float nrm[1024];
    __shared__ int live[1024];
    double s = 0.0;
    int c = 0;
    for (int p0 = 0; p0 < P.n_params; p0 += 1024) {
        const int m = min(1024, P.n_params - p0);
        for (int i = threadIdx.x; i < m; i += blockDim.x) {
            live[i] = P.step[p0 + i].phase != 0;
            // float(p.grad.norm()) of optimizer.py:440: in the gradient's dtype
            nrm[i] = round_dt(sqrtf(P.filt.fp[p0 + i].gsq), P.params[p0 + i].dtype);
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int i = 0; i < m; ++i)
                if (live[i]) { s = __dadd_rn(s, (double)nrm[i]); ++c; }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        double e = *P.global_norm_ema;
        // the host keeps the EMA itself when it needs the norms (R1/R3/R5)
        if (c > 0 && !P.gnorm_host) e = __dadd_rn(__dmul_rn(0.95, e), __dmul_rn(0.05, s / (double)c));
        *P.global_norm_ema = e;
        gema = e;
    }
    __syncthreads();
    const ScaoFilterDev& FD = P.filt;
    for (int pi = threadIdx.x; pi < P.n_params; pi += blockDim.x) {
        if (P.step[pi].phase == 0) continue;
        ScaoFilterParam* F = FD.fp + pi;
        const int64_t n = P.params[pi].numel;
        double q = FD.base;
        if (FD.mode == 2) {
            if (!F->first) F->global_ref = fmax(gema, 1e-8);
            const double layer = (double)sqrtf(F->gsq);   // of p.grad.float() (:531)
            F->norm_ema = __dadd_rn(__dmul_rn(FD.norm_coeff, F->norm_ema),
                                    __dmul_rn(1.0 - FD.norm_coeff, layer));
            const double ratio = F->norm_ema / F->global_ref;
            const double margin = 0.2 * (1.0 - fmin(ratio, 2.0) / 2.0);
            q = fmax(FD.min_s, fmin(FD.max_s, FD.base + margin));
        }
        F->sparsity = q;
        const float qf = (float)q;
        int64_t lo;
        float w;
        if (n <= (int64_t(1) << 24)) {
            const float r = __fmul_rn(qf, (float)(n - 1));
            lo = (int64_t)floorf(r);
            w = __fsub_rn(r, (float)lo);
        } else {
            const double r = (double)qf * (double)(n - 1);
            lo = (int64_t)floor(r);
            w = (float)(r - (double)lo);
        }
        int64_t hi = w > 0.f ? lo + 1 : lo;
        if (hi > n - 1) hi = n - 1;
        F->rem_lo = lo;
        F->rem_hi = hi;
        F->pre_lo = F->pre_hi = 0u;
        F->w = w;
    }
}

// Find the bin holding rank ``rem`` in h[0..nb): block-wide exclusive scan,
// 4 bins per thread.  Writes (bin, count before bin) to shared.
__device__ void find_bin(const uint32_t* __restrict__ h, int nb, int64_t rem,
                         int* out_bin, long long* out_before, long long* wsum) {
    const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
    uint32_t c[4] = {0u, 0u, 0u, 0u};
    long long loc = 0;
    if (t * 4 < nb) {
#pragma unroll
        for (int i = 0; i < 4; ++i) { c[i] = h[t * 4 + i]; loc += c[i]; }
    }
    long long inc = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) wsum[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        long long v = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
        long long x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        wsum[lane] = x - v;     // exclusive prefix of warps
    }
    __syncthreads();
    long long before = wsum[wid] + inc - loc;
    if (t * 4 < nb && rem >= before && rem < before + loc) {
        for (int i = 0; i < 4; ++i) {
            if (rem < before + (long long)c[i]) {
                *out_bin = t * 4 + i;
                *out_before = before;
                break;
            }
            before += c[i];
        }
    }
    __syncthreads();
}

SCAO_DEV float lerp_f(float a, float b, float w) {
    // ATen lerp (Lerp.h) with its multiply-add contracted
    const float d = __fsub_rn(b, a);
    return fabsf(w) < 0.5f ? __fmaf_rn(w, d, a) : __fmaf_rn(-d, __fsub_rn(1.f, w), b);
}

// One radix level for both targets of every parameter.
__global__ void __launch_bounds__(SNT)
filt_scan_kernel(ScaoPlanDev P, int level) {
    const int pi = blockIdx.x;
    if (P.step[pi].phase == 0) return;
    ScaoFilterParam* F = P.filt.fp + pi;
    __shared__ long long wsum[32];
    __shared__ int bin;
    __shared__ long long before;
    const int nb = level == 3 ? 256 : FB;
    const int shift = level == 1 ? 20 : level == 2 ? 8 : 0;
    const int hs = level == 1 ? 32 : level == 2 ? 20 : 8;   // bits of the prefix so far
    const uint32_t plo = F->pre_lo, phi = F->pre_hi;
    const bool split = level > 1 && ((plo ^ phi) >> hs) != 0u;
    const uint32_t* h0 = P.filt.hist + (size_t)pi * 2 * FB;
    uint32_t res[2];
    long long rem[2] = {F->rem_lo, F->rem_hi};
    for (int t = 0; t < 2; ++t) {
        if (threadIdx.x == 0) { bin = -1; before = 0; }
        __syncthreads();
        find_bin((t == 1 && split) ? h0 + FB : h0, nb, rem[t], &bin, &before, wsum);
        const int b = bin;
        const uint32_t pre = t == 0 ? plo : phi;
        res[t] = b >= 0 ? (pre | ((uint32_t)b << shift)) : pre;
        if (b >= 0) rem[t] -= before;
        __syncthreads();
    }
    if (threadIdx.x != 0) return;
    F->pre_lo = res[0];
    F->pre_hi = res[1];
    F->rem_lo = rem[0];
    F->rem_hi = rem[1];
    if (level == 3) {
        const float a = __uint_as_float(res[0]), b = __uint_as_float(res[1]);
        F->thr = F->nan ? __int_as_float(0x7fc00000) : lerp_f(a, b, F->w);
        F->first = 0;
        F->nan = 0;
    }
}

// Levels 2 and 3: histogram of the next bit field over the elements whose
// prefix matches a target's prefix so far.
__global__ void __launch_bounds__(FNT)
filt_hist_kernel(ScaoPlanDev P, int level) {
    const ScaoChunk ch = P.filt.sel[blockIdx.x];
    const int pi = ch.param;
    if (P.step[pi].phase == 0) return;
    const ScaoParam& pr = P.params[pi];
    const ScaoFilterParam* F = P.filt.fp + pi;
    __shared__ uint32_t h[2 * FB];
    const int width = level == 2 ? 12 : 8;
    const int shift = level == 2 ? 8 : 0;
    const int hs = shift + width;
    const uint32_t fmask = (1u << width) - 1u;
    const uint32_t plo = F->pre_lo >> hs, phi = F->pre_hi >> hs;
    const bool split = plo != phi;
    const int nb = 1 << width;
    for (int i = threadIdx.x; i < 2 * nb; i += FNT) h[i] = 0;
    __syncthreads();
    const float* mg = P.filt.mag_ema + pr.offset;
    auto one = [&](float m) {
        const uint32_t k = __float_as_uint(m);
        const uint32_t top = k >> hs;
        if (top == plo) atomicAdd(&h[(k >> shift) & fmask], 1u);
        else if (split && top == phi) atomicAdd(&h[nb + ((k >> shift) & fmask)], 1u);
    };
    const bool vec = ((pr.offset & 3) == 0) && ((ch.begin & 3) == 0);
    int64_t vend = ch.begin;
    if (vec) {
        const int64_t n4 = (ch.end - ch.begin) >> 2;
        vend = ch.begin + n4 * 4;
        for (int64_t q = threadIdx.x; q < n4; q += FNT) {
            const float4 m4 = *(const float4*)(mg + ch.begin + q * 4);
            one(m4.x);
            one(m4.y);
            one(m4.z);
            one(m4.w);
        }
    }
    for (int64_t e = vend + threadIdx.x; e < ch.end; e += FNT) one(mg[e]);
    __syncthreads();
    uint32_t* gh = P.filt.hist + (size_t)pi * 2 * FB;
    for (int i = threadIdx.x; i < nb; i += FNT) {
        if (h[i]) atomicAdd(gh + i, h[i]);
        if (split && h[nb + i]) atomicAdd(gh + FB + i, h[nb + i]);
    }
}

}  // namespace

int scao_filter_run(const ScaoPlanDev* P, cudaStream_t st) {
    if (P->filt.mode == 0 || P->filt.n_sel == 0) return SCAO_OK;
    if (!P->filt.sel || !P->filt.fp || !P->filt.hist || !P->filt.mag_ema || !P->filt.sel_part)
        return SCAO_ERR_ARG;
    const size_t hb = (size_t)P->n_params * 2 * FB * sizeof(uint32_t);
    if (cudaMemsetAsync(P->filt.hist, 0, hb, st) != cudaSuccess) return SCAO_ERR_LAUNCH;
    { ProfScope _ps(SLOT_FILTER, st); filt_update_kernel<<<P->filt.n_sel, FNT, 0, st>>>(*P); }
    { ProfScope _ps(SLOT_FILTER, st); filt_param_kernel<<<P->n_params, 256, 0, st>>>(*P); }
    { ProfScope _ps(SLOT_FILTER, st); filt_global_kernel<<<1, 256, 0, st>>>(*P); }
    { ProfScope _ps(SLOT_FILTER, st); filt_scan_kernel<<<P->n_params, SNT, 0, st>>>(*P, 1); }
    for (int level = 2; level <= 3; ++level) {
        if (cudaMemsetAsync(P->filt.hist, 0, hb, st) != cudaSuccess) return SCAO_ERR_LAUNCH;
        { ProfScope _ps(SLOT_FILTER, st); filt_hist_kernel<<<P->filt.n_sel, FNT, 0, st>>>(*P, level); }
        { ProfScope _ps(SLOT_FILTER, st); filt_scan_kernel<<<P->n_params, SNT, 0, st>>>(*P, level); }
    }
    if (cudaPeekAtLastError() != cudaSuccess) {
        (void)cudaGetLastError();
        return SCAO_ERR_LAUNCH;
    }
    return SCAO_OK;
}
