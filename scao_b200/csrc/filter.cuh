// Gradient filter and gradient noise as the elementwise passes see them
// (scao/optimizer.py:536-545): the moments and prev_grad take
//     grad = p.grad * (mag_ema >= threshold)        (sparse filter, :56)
//     grad = grad + randn * noise_std               (noise, :544-545)
// while the preconditioner keeps the raw p.grad.
#pragma once
#include "common.cuh"

// Philox-4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011): ten rounds of
// two 32x32->64 multiplies with the paper's round multipliers and Weyl key
// increments.
SCAO_DEV uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
        const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
        c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

// Four standard normals for the elements 4*e4 .. 4*e4+3 of parameter
// ``param`` at global step ``step``: one Philox block, two Box-Muller pairs
// (uniforms in (0, 1] from the top 24 bits; the hardware approximations of
// log and sin/cos -- the noise is a distribution, not a value to match).
// The stream depends only on (seed, param, step, element), never on which
// kernel or thread asks.
SCAO_DEV float4 noise_normal4(uint64_t seed, uint32_t param, uint64_t step, int64_t e4) {
    const uint4 r = philox4x32_10(
        make_uint4((uint32_t)e4, (uint32_t)((uint64_t)e4 >> 32), (uint32_t)step, param),
        (uint32_t)seed, (uint32_t)(seed >> 32));
    const float k = 5.9604644775390625e-08f;   // 2^-24
    const float u0 = ((r.x >> 8) + 1) * k, u1 = ((r.y >> 8) + 1) * k;
    const float u2 = ((r.z >> 8) + 1) * k, u3 = ((r.w >> 8) + 1) * k;
    const float ra = sqrtf(-2.f * __logf(u0)), rb = sqrtf(-2.f * __logf(u2));
    const float two_pi = 6.283185307179586f;
    float sa, ca, sb, cb;
    __sincosf(two_pi * u1, &sa, &ca);
    __sincosf(two_pi * u3, &sb, &cb);
    return make_float4(ra * ca, ra * sa, rb * cb, rb * sb);
}

SCAO_DEV float f4_get(const float4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Per-element gradient of the moment updates.  ``mag`` is this element's
// magnitude EMA (ignored when the filter is off), ``z`` its normal draw
// (ignored when noise is off).  grad * mask is a multiply (a NaN or inf
// gradient stays NaN under a zero mask, as in the reference).
SCAO_DEV float filt_grad(const ScaoFilterDev& F, float g, float mag, float thr, float z) {
    if (F.mode) g = __fmul_rn(g, mag >= thr ? 1.f : 0.f);
    if (F.noise_on) g = __fadd_rn(g, __fmul_rn(z, F.noise_std));
    return g;
}

// R4 gSNR clip (optimizer.py:161-175, applied at :637-638): the update is
// multiplied by (|m| / (sqrt(v) + eps) >= thr) with the updated moments.
SCAO_DEV float gsnr_mask(float u, float m, float v, float eps, float thr) {
    const float snr = __fdiv_rn(fabsf(m), __fadd_rn(sqrtf(v), eps));
    return __fmul_rn(u, snr >= thr ? 1.f : 0.f);
}

// Host entry of the filter passes (filter.cu): magnitude EMA, radix
// selection of the quantile, threshold per parameter.
int scao_filter_run(const ScaoPlanDev* P, cudaStream_t st);
