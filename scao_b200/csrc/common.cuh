// Shared device helpers for the scao_b200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/scao_b200.h"

// Kernel attributes (cudaFuncSetAttribute) belong to the function in the
// current device's context: a launcher sets them once per device.
struct PerDeviceOnce {
    bool done[64] = {};
    // true for the first call on the current device
    bool first() {
        int d = 0;
        if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return true;
        if (done[d]) return false;
        done[d] = true;
        return true;
    }
};

#define SCAO_DEV __device__ __forceinline__

// per-parameter scalar slots of ScaoPlanDev::param_scalars (8 floats each)
enum { PS_CLIPMUL = 0, PS_CLIP, PS_PNORM2, PS_UNORM2, PS_GNORM2, PS_ALPHA, PS_NAT, PS_TRUST };

// ---------------------------------------------------------------------------
// parameter-dtype load / round / store.  All arithmetic is fp32 ("opmath"),
// values are rounded to the parameter dtype where the reference stores a
// parameter-dtype tensor.
// ---------------------------------------------------------------------------
SCAO_DEV float bf16_bits_to_f(uint16_t b) {
    return __uint_as_float(((uint32_t)b) << 16);
}
SCAO_DEV uint16_t f_to_bf16_bits(float x) {  // round to nearest even
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
SCAO_DEV float f16_bits_to_f(uint16_t b) {
    return __half2float(__ushort_as_half(b));
}
SCAO_DEV uint16_t f_to_f16_bits(float x) {
    return __half_as_ushort(__float2half_rn(x));
}

// Round a float to the parameter dtype and return it as float.
SCAO_DEV float round_dt(float x, int dt) {
    if (dt == SCAO_BF16) return bf16_bits_to_f(f_to_bf16_bits(x));
    if (dt == SCAO_F16) return f16_bits_to_f(f_to_f16_bits(x));
    return x;
}

SCAO_DEV float load_dt(const void* base, int64_t i, int dt) {
    if (dt == SCAO_F32) return ((const float*)base)[i];
    uint16_t b = ((const uint16_t*)base)[i];
    return dt == SCAO_BF16 ? bf16_bits_to_f(b) : f16_bits_to_f(b);
}

SCAO_DEV void store_dt(void* base, int64_t i, int dt, float x) {
    if (dt == SCAO_F32) {
        ((float*)base)[i] = x;
    } else {
        ((uint16_t*)base)[i] = dt == SCAO_BF16 ? f_to_bf16_bits(x) : f_to_f16_bits(x);
    }
}

// Load 4 consecutive elements (16-byte aligned for fp32, 8-byte for 16-bit).
SCAO_DEV float4 load4_dt(const void* base, int64_t i, int dt) {
    if (dt == SCAO_F32) return *(const float4*)((const float*)base + i);
    uint2 r = *(const uint2*)((const uint16_t*)base + i);
    float4 o;
    if (dt == SCAO_BF16) {
        o.x = bf16_bits_to_f(r.x & 0xffff); o.y = bf16_bits_to_f(r.x >> 16);
        o.z = bf16_bits_to_f(r.y & 0xffff); o.w = bf16_bits_to_f(r.y >> 16);
    } else {
        o.x = f16_bits_to_f(r.x & 0xffff); o.y = f16_bits_to_f(r.x >> 16);
        o.z = f16_bits_to_f(r.y & 0xffff); o.w = f16_bits_to_f(r.y >> 16);
    }
    return o;
}

SCAO_DEV void store4_dt(void* base, int64_t i, int dt, float4 v) {
    if (dt == SCAO_F32) { *(float4*)((float*)base + i) = v; return; }
    uint16_t a, b, c, d;
    if (dt == SCAO_BF16) {
        a = f_to_bf16_bits(v.x); b = f_to_bf16_bits(v.y);
        c = f_to_bf16_bits(v.z); d = f_to_bf16_bits(v.w);
    } else {
        a = f_to_f16_bits(v.x); b = f_to_f16_bits(v.y);
        c = f_to_f16_bits(v.z); d = f_to_f16_bits(v.w);
    }
    uint2 r;
    r.x = (uint32_t)a | ((uint32_t)b << 16);
    r.y = (uint32_t)c | ((uint32_t)d << 16);
    *(uint2*)((uint16_t*)base + i) = r;
}

// Streaming (evict-first) 128-bit load/store for state arenas touched once.
SCAO_DEV float4 ldg_stream4(const float* p) { return __ldcs((const float4*)p); }
SCAO_DEV void stg_stream4(float* p, float4 v) { __stcs((float4*)p, v); }

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
SCAO_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
SCAO_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
SCAO_DEV double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide sum; `red` must hold >= 32 floats.  Result valid in all threads.
SCAO_DEV float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float r = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
    if (wid == 0) r = warp_sum(r);
    if (threadIdx.x == 0) red[0] = r;
    __syncthreads();
    r = red[0];
    __syncthreads();
    return r;
}
SCAO_DEV float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float r = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
    if (wid == 0) r = warp_max(r);
    if (threadIdx.x == 0) red[0] = r;
    __syncthreads();
    r = red[0];
    __syncthreads();
    return r;
}

// atomicMax on non-negative floats through their integer bit patterns.
SCAO_DEV void atomic_max_nonneg(float* addr, float v) {
    atomicMax((int*)addr, __float_as_int(v));
}

// ---------------------------------------------------------------------------
// int8 symmetric quantisation (utils.py:170-203)
// ---------------------------------------------------------------------------
// float(scale) where scale = double(absmax) / 127 (Python float division).
SCAO_DEV float quant_scale_f(float absmax) {
    return (double)absmax < 1e-30 ? 1.0f : (float)((double)absmax / 127.0);
}
SCAO_DEV int8_t quant_one(float x, float scale_f, bool zero) {
    if (zero) return 0;
    float q = rintf(__fdiv_rn(x, scale_f));  // IEEE division, ties-to-even
    q = fminf(fmaxf(q, -127.f), 127.f);
    return (int8_t)q;
}

#define SCAO_CHECK_LAUNCH()                                   \
    do {                                                      \
        if (cudaPeekAtLastError() != cudaSuccess) {           \
            (void)cudaGetLastError();                         \
            return SCAO_ERR_LAUNCH;                           \
        }                                                     \
    } while (0)
