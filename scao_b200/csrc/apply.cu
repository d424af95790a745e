// The every-step optimizer pass (scao/optimizer.py:521-645) for all
// parameters at once, plus the Kronecker precondition
// (scao/preconditioner.py:457-521, fallback formula scao/cuda/__init__.py:95-99)
// and the curvature clip (optimizer.py:667-678, preconditioner.py:527-564).
//
// Kernel sequence of one step (scao_plan_step):
//   filter     (sparsity > 0) magnitude EMA + exact quantile threshold,
//              filter.cu
//   proj       P_panel = U_l[rows]^T (G[rows] U_r)      per 128-row panel
//   diag_pre   natural-norm^2 and p_dec^2 of diagonal-mode params
//   leaf_coef  P = sum of panels; nat^2; Delta = (s_l s_r^T - 1) o P
//   leaf_w     W = U_l Delta as bf16 hi/lo operand tiles
//   param_pre  clip factor tau / nat  per param
//   apply_kron per 128x128 tile: corr = W U_r^T on the tensor core,
//              g_prec = round(G + corr), clip, blend, Adan moments,
//              update u (rounded to param dtype), sum p_dec^2
//   apply_flat Phase-1 Adam (full update) and Phase-2 diagonal params
//   param_post LARS trust ratio -> alpha = -(lr * trust) per param
//   global     global grad-norm EMA (optimizer.py:439-446)
//   apply_p    p = round(round(p * (1 - lr wd)) + alpha * u)   (Phase 2)
//
// Rounding: every op the reference evaluates as a separate tensor op is
// rounded separately here (explicit __fmul_rn/__fadd_rn/__fdiv_rn); the ops
// torch contracts to a fused multiply-add on CPU (add_ with alpha, addcmul_)
// use fmaf.  Parameter-dtype roundings are reproduced exactly.
#include "common.cuh"
#include "prof.cuh"
#include "tc.cuh"
#include "filter.cuh"
#include "tmap.cuh"

namespace {

constexpr int NT = 256;
constexpr int TC_T = 128;    // tensor-core tile edge (rows and columns)


__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// S^(-1/4) and S^(-1/2) with the clamp of utils.py:113 / preconditioner.py:558
__device__ __forceinline__ float s_inv4(float s) { return powf(fmaxf(s, 1e-8f), -0.25f); }
__device__ __forceinline__ float s_inv2(float s) { return powf(fmaxf(s, 1e-8f), -0.5f); }

// ---------------------------------------------------------------------------
// diagonal-mode Phase-2 params: natural-norm^2 and p_dec^2 per chunk
// (preconditioner.py:554-556; optimizer.py:373)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
diag_pre_kernel(ScaoPlanDev P) {
    const int cid = P.diag_list[blockIdx.x];
    const ScaoChunk ch = P.chunks[cid];
    const ScaoParam& pr = P.params[ch.param];
    const ScaoParamStep& S = P.step[ch.param];
    if (S.phase != 2 || pr.mode != 0) return;
    __shared__ float red[32];
    const void* g = (const void*)S.g_ptr;
    const void* pp = (const void*)S.p_ptr;
    const float* de = P.diag_ema + pr.offset;
    float nat = 0.f, psq = 0.f;
    const float eps = S.eps;
    for (int64_t e = ch.begin + threadIdx.x; e < ch.end; e += NT) {
        const float gv = load_dt(g, e, pr.dtype);
        const float den = fadd(sqrtf(de[e]), eps);
        nat += fdiv(fmul(gv, gv), den);
        const float pd = round_dt(fmul(load_dt(pp, e, pr.dtype), S.wd_mult), pr.dtype);
        psq = fmaf(pd, pd, psq);
    }
    nat = block_sum(nat, red);
    psq = block_sum(psq, red);
    if (threadIdx.x == 0) {
        P.chunk_part[cid * 4 + 2] = nat;
        P.chunk_part[cid * 4 + 3] = psq;
    }
}

// ---------------------------------------------------------------------------
// diagonal strips of Kronecker params (width-1 blocks of the split): their
// natural-norm^2 sum(g^2 / (sqrt(diag_ema) + eps)) (preconditioner.py:554-556)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
strip_pre_kernel(ScaoPlanDev P) {
    const ScaoStrip sp = P.strips[blockIdx.x];
    const ScaoParam& pr = P.params[sp.param];
    const ScaoParamStep& S = P.step[sp.param];
    if (S.phase != 2) return;
    __shared__ float red[32];
    const void* g = (const void*)S.g_ptr;
    const float* de = P.diag_ema + pr.offset;
    float nat = 0.f;
    for (int j = threadIdx.x; j < sp.count; j += NT) {
        const int64_t e = sp.begin + (int64_t)j * sp.stride;
        const float gv = load_dt(g, e, pr.dtype);
        nat += fdiv(fmul(gv, gv), fadd(sqrtf(de[e]), S.eps));
    }
    nat = block_sum(nat, red);
    if (threadIdx.x == 0) P.strip_part[blockIdx.x * 4 + 3] = nat;
}

// ---------------------------------------------------------------------------
// per leaf: reduce panels, natural norm, Delta, W = U_l Delta
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
leaf_coef_kernel(ScaoPlanDev P) {
    const ScaoLeaf& L = P.leaves[blockIdx.x];
    const ScaoParamStep& S = P.step[L.param];
    if (S.phase != 2) return;
    extern __shared__ float sm[];
    const int kp = L.kpad;
    const int k = P.k[blockIdx.x];
    float* D = sm;                    // kp x kp  (Delta)
    float* s4l = D + kp * kp;
    float* s4r = s4l + kp;
    float* s2l = s4r + kp;
    float* s2r = s2l + kp;
    __shared__ float red[32];
    const float* evl = P.ev + L.evl_off;
    const float* evr = P.ev + L.evr_off;
    for (int a = threadIdx.x; a < kp; a += NT) {
        const bool on = a < k;
        s4l[a] = on ? s_inv4(evl[a]) : 0.f;
        s4r[a] = on ? s_inv4(evr[a]) : 0.f;
        s2l[a] = on ? s_inv2(evl[a]) : 0.f;
        s2r[a] = on ? s_inv2(evr[a]) : 0.f;
    }
    __syncthreads();
    float nat = 0.f;
    for (int e = threadIdx.x; e < kp * kp; e += NT) {
        const int a = e / kp, b = e % kp;
        float pv = 0.f;
        for (int q = L.panel_begin; q < L.panel_end; ++q) pv += P.p_part[(int64_t)q * P.p_stride + e];
        float dv = 0.f;
        if (a < k && b < k) {
            const float gs = fmul(fmul(s2l[a], pv), s2r[b]);
            nat = fmaf(gs, gs, nat);
            dv = fmul(fsub(fmul(s4l[a], s4r[b]), 1.f), pv);
        }
        D[e] = dv;
    }
    nat = block_sum(nat, red);
    if (threadIdx.x == 0) P.leaf_nat2[blockIdx.x] = nat;
    // Delta overwrites the first panel's partial slot (read above by this
    // same thread for the same element, so no other reader remains)
    float* Dg = P.p_part + (int64_t)L.panel_begin * P.p_stride;
    for (int e = threadIdx.x; e < kp * kp; e += NT) Dg[e] = D[e];
}

__device__ __forceinline__ void stage_ls(float* Ls, const float* Ul, int row0, int nrows, int sl,
                                         int kpad, int Kp);

// W = U_l Delta (rows [128 t, 128 t + 128) of the leaf; only the first k
// columns of U_l contribute), written as bf16 hi/lo canonical tiles for the
// tensor-core apply.  4 x 8 register blocks, 16-byte tile stores.
__global__ void __launch_bounds__(256)
leaf_w_kernel(ScaoPlanDev P) {
    const int leaf = blockIdx.y;
    const ScaoLeaf& L = P.leaves[leaf];
    const ScaoParamStep& S = P.step[L.param];
    if (S.phase != 2) return;
    const int r0 = blockIdx.x * TC_T;
    if (r0 >= L.a) return;
    const int kp = L.kpad, Kp = (kp + 15) & ~15;
    const int k = P.k[leaf];
    extern __shared__ float sm[];
    float* Ds = sm;                       // kp x Kp (zero beyond kp)
    float* Ls = Ds + kp * Kp;             // 128 x (Kp+4)
    const float* Dg = P.p_part + (int64_t)L.panel_begin * P.p_stride;
    for (int e = threadIdx.x; e < kp * Kp; e += blockDim.x) {
        const int a = e / Kp, bb = e - a * Kp;
        Ds[e] = bb < kp ? Dg[a * kp + bb] : 0.f;
    }
    stage_ls(Ls, P.u + L.ul_off, r0, min(TC_T, L.a - r0), L.sl, kp, Kp);
    __syncthreads();
    const int64_t tbytes = (int64_t)TC_T * Kp * 2;
    uint8_t* t = P.wa + L.wa_off + (int64_t)blockIdx.x * 2 * tbytes;
    const int nb = Kp / 8;
    for (int blk = threadIdx.x; blk < 32 * nb; blk += blockDim.x) {
        const int rr = (blk / nb) * 4, b0 = (blk % nb) * 8;
        float acc[4][8] = {};
        for (int a = 0; a < k; ++a) {
            const float4 d0 = *(const float4*)&Ds[a * Kp + b0];
            const float4 d1 = *(const float4*)&Ds[a * Kp + b0 + 4];
            const float dv[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float u = Ls[(rr + i) * (Kp + 4) + a];
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(u, dv[j], acc[i][j]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint16_t h0, l0, h1, l1;
                split_bf16(acc[i][2 * j], h0, l0);
                split_bf16(acc[i][2 * j + 1], h1, l1);
                hw[j] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                lw[j] = (uint32_t)l0 | ((uint32_t)l1 << 16);
            }
            const uint32_t o = canon_off(rr + i, b0, Kp);
            *(uint4*)(t + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *(uint4*)(t + tbytes + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
    }
}

// ---------------------------------------------------------------------------
// per param: clip factor (optimizer.py:667-678)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
param_pre_kernel(ScaoPlanDev P) {
    const int pi = blockIdx.x;
    const ScaoParam& pr = P.params[pi];
    const ScaoParamStep& S = P.step[pi];
    if (S.phase != 2) return;
    __shared__ float red[32];
    float nat2 = 0.f, psq = 0.f;
    if (pr.mode == 1) {
        // block-diagonal: sqrt(sum of squared block norms) (preconditioner.py:542-552)
        for (int l = pr.leaf_begin + threadIdx.x; l < pr.leaf_end; l += NT) {
            const float bn = sqrtf(P.leaf_nat2[l]);
            nat2 = fmaf(bn, bn, nat2);
        }
        for (int s = threadIdx.x; s < P.n_strips; s += NT)
            if (P.strips[s].param == pi) {
                const float bn = sqrtf(P.strip_part[s * 4 + 3]);
                nat2 = fmaf(bn, bn, nat2);
            }
    } else {
        for (int c = pr.chunk_begin + threadIdx.x; c < pr.chunk_end; c += NT) {
            nat2 += P.chunk_part[c * 4 + 2];
            psq += P.chunk_part[c * 4 + 3];
        }
    }
    nat2 = block_sum(nat2, red);
    psq = block_sum(psq, red);
    if (threadIdx.x == 0) {
        float* ps = P.param_scalars + pi * 8;
        const float nat = sqrtf(nat2);
        const bool clip = S.clip && nat > S.tau;
        ps[PS_CLIP] = clip ? 1.f : 0.f;
        ps[PS_CLIPMUL] = clip ? fdiv(S.tau, fmaxf(nat, S.eps)) : 1.f;
        if (pr.mode == 0) ps[PS_PNORM2] = psq;   // Kronecker params: from the apply tiles
        ps[PS_NAT] = nat;
    }
}

// Adan moments + update for one element (optimizer.py:608-633).
struct AdanOut { float u; };
// x / c for a per-step constant c (bias corrections) with r = RN(1/c), the
// correctly rounded float32 reciprocal computed on the host: q = x*r, then one
// fused residual correction q + r*(x - c*q) (Markstein, IBM J. Res. Dev. 34,
// 1990).  Markstein's theorem gives the IEEE quotient when r is the correctly
// rounded reciprocal and q lies within one ulp of x/c; the second hypothesis
// can fail only near binade edges of the quotient, where the result may be one
// ulp off.  Sampled against __fdiv_rn over the bias-correction constants
// (tests/test_tc.py) with no mismatch.  An exact per-element check with an IEEE
// fallback costs the HBM-bound apply about 40 % (measured), so it is not used.
__device__ __forceinline__ float div_c(float x, float c, float r) {
    const float q = x * r;
    const float e = fmaf(-q, c, x);
    return fmaf(e, r, q);
}

__device__ __forceinline__ float adan_elem(const ScaoParamStep& S, int dt, float g, float gp,
                                           float& m, float& v, float& d, float& prev,
                                           bool clip, float clipmul) {
    if (clip) gp = round_dt(fmul(gp, clipmul), dt);
    const float geff = fadd(fmul(S.blend, gp), fmul(S.one_minus_blend, g));
    const float delta = fsub(g, prev);
    prev = g;
    m = fmaf(geff, S.c1, fmul(m, S.beta1));
    d = fmaf(delta, S.c3, fmul(d, S.beta3));
    const float gad = fadd(geff, fmul(S.c3, delta));
    v = fmaf(fmul(S.c2, gad), gad, fmul(v, S.beta2));
    const float num = fadd(div_c(m, S.bc1, S.rbc1), fmul(S.c3, div_c(d, S.bc3, S.rbc3)));
    const float den = fadd(sqrtf(div_c(v, S.bc2, S.rbc2)), S.eps);
    return fdiv(num, den);
}

// ---------------------------------------------------------------------------
// flat chunks: Phase-1 Adam (optimizer.py:561-578) and Phase-2 diagonal
// params (preconditioner.py:506-510 + the Adan step)
// ---------------------------------------------------------------------------
template <bool FN>
__global__ void __launch_bounds__(NT)
apply_flat_kernel(ScaoPlanDev P) {
    const int cid = P.flat_list[blockIdx.x];
    const ScaoChunk ch = P.chunks[cid];
    const ScaoParam& pr = P.params[ch.param];
    const ScaoParamStep& S = P.step[ch.param];
    const int phase = S.phase;
    if (phase == 0 || (phase == 2 && pr.mode == 1)) return;
    __shared__ float red[32];
    const int dt = pr.dtype;
    const void* g = (const void*)S.g_ptr;
    void* pp = (void*)S.p_ptr;
    float* M = P.exp_avg + pr.offset;
    float* V = P.exp_avg_sq + pr.offset;
    float* Dd = P.exp_avg_diff + pr.offset;
    float* Pv = P.prev_grad + pr.offset;
    float usq = 0.f, gsq = 0.f;
    const ScaoFilterDev& FD = P.filt;
    const float* MG = FD.mode ? FD.mag_ema + pr.offset : nullptr;
    const float thr = FD.mode ? FD.fp[ch.param].thr : 0.f;
    constexpr bool fl = FN;
    // filtered / noised gradient of element e (optimizer.py:536-545)
    auto gfilt = [&](float g_, int64_t e) {
        return filt_grad(FD, g_, FD.mode ? MG[e] : 0.f, thr,
                         FD.noise_on ? f4_get(noise_normal4(FD.noise_seed, ch.param, FD.noise_step,
                                                            e >> 2), (int)(e & 3)) : 0.f);
    };
    if (phase == 1) {
        const float a1 = round_dt((float)S.alpha1, dt);
        auto adam4 = [&](float graw, float g_, float p_, float& m_, float& v_) {
            const float pd = round_dt(fmul(p_, S.wd_mult), dt);
            m_ = fmaf(g_, S.c1, fmul(m_, S.beta1));
            v_ = fmaf(fmul(S.c2, g_), g_, fmul(v_, S.beta2));
            // Phase-1 rows carry 1 / sqrt_bc2 in rbc2
            const float den = fadd(div_c(sqrtf(v_), S.sqrt_bc2, S.rbc2), S.eps);
            const float u = round_dt(fdiv(m_, den), dt);
            gsq = fmaf(graw, graw, gsq);
            return round_dt(fmaf(a1, u, pd), dt);
        };
        const bool vec = ((S.g_ptr & 15) == 0) && ((S.p_ptr & 15) == 0) &&
                         ((pr.offset & 3) == 0) && ((ch.begin & 3) == 0);
        int64_t vend = ch.begin;
        if (vec) {
            const int64_t n4 = (ch.end - ch.begin) >> 2;
            vend = ch.begin + n4 * 4;
            for (int64_t q = threadIdx.x; q < n4; q += NT) {
                const int64_t e = ch.begin + q * 4;
                const float4 g4 = load4_dt(g, e, dt), p4 = load4_dt(pp, e, dt);
                float4 m4 = ldg_stream4(M + e), v4 = ldg_stream4(V + e);
                float4 f4 = g4;
                if (fl) {
                    const float4 mg4 = FD.mode ? *(const float4*)(MG + e) : make_float4(0.f, 0.f, 0.f, 0.f);
                    const float4 z4 = FD.noise_on ? noise_normal4(FD.noise_seed, ch.param, FD.noise_step, e >> 2)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                    f4.x = filt_grad(FD, g4.x, mg4.x, thr, z4.x);
                    f4.y = filt_grad(FD, g4.y, mg4.y, thr, z4.y);
                    f4.z = filt_grad(FD, g4.z, mg4.z, thr, z4.z);
                    f4.w = filt_grad(FD, g4.w, mg4.w, thr, z4.w);
                }
                float4 o;
                o.x = adam4(g4.x, f4.x, p4.x, m4.x, v4.x);
                o.y = adam4(g4.y, f4.y, p4.y, m4.y, v4.y);
                o.z = adam4(g4.z, f4.z, p4.z, m4.z, v4.z);
                o.w = adam4(g4.w, f4.w, p4.w, m4.w, v4.w);
                store4_dt(pp, e, dt, o);
                stg_stream4(M + e, m4);
                stg_stream4(V + e, v4);
                stg_stream4(Pv + e, f4);
            }
        }
        for (int64_t e = vend + threadIdx.x; e < ch.end; e += NT) {
            const float graw = load_dt(g, e, dt);
            const float gv = fl ? gfilt(graw, e) : graw;
            const float pd = round_dt(fmul(load_dt(pp, e, dt), S.wd_mult), dt);
            float m = fmaf(gv, S.c1, fmul(M[e], S.beta1));
            float v = fmaf(fmul(S.c2, gv), gv, fmul(V[e], S.beta2));
            const float den = fadd(div_c(sqrtf(v), S.sqrt_bc2, S.rbc2), S.eps);
            const float u = round_dt(fdiv(m, den), dt);
            store_dt(pp, e, dt, round_dt(fmaf(a1, u, pd), dt));
            M[e] = m; V[e] = v; Pv[e] = gv;
            gsq = fmaf(graw, graw, gsq);
        }
    } else {
        // Phase 2, diagonal mode
        const float* de = P.diag_ema + pr.offset;
        const float* ps = P.param_scalars + ch.param * 8;
        const bool clip = ps[PS_CLIP] != 0.f;
        const float clipmul = ps[PS_CLIPMUL];
        for (int64_t e = ch.begin + threadIdx.x; e < ch.end; e += NT) {
            const float gv = load_dt(g, e, dt);
            const float den = fadd(powf(fdiv(de[e], S.diag_bias), 0.25f), 1e-8f);
            const float gp = round_dt(fdiv(gv, den), dt);
            float m = M[e], v = V[e], d = Dd[e], pv = Pv[e];
            float u = adan_elem(S, dt, fl ? gfilt(gv, e) : gv, gp, m, v, d, pv, clip, clipmul);
            if (FN && FD.gsnr_on) u = gsnr_mask(u, m, v, S.eps, FD.gsnr_thr);
            usq = fmaf(u, u, usq);
            gsq = fmaf(gv, gv, gsq);
            M[e] = m; V[e] = v; Dd[e] = d; Pv[e] = pv;
            if (dt == SCAO_F32) P.upd32[pr.offset + e] = u;
            else store_dt(P.upd + pr.offset, e, dt, u);
        }
    }
    usq = block_sum(usq, red);
    gsq = block_sum(gsq, red);
    if (threadIdx.x == 0) {
        P.chunk_part[cid * 4 + 0] = usq;
        P.chunk_part[cid * 4 + 1] = gsq;
    }
}

// ---------------------------------------------------------------------------
// Phase 2 on the diagonal strips of Kronecker params: the diagonal
// preconditioner g / ((diag_ema / bias)^(1/4) + 1e-8) (preconditioner.py:
// 506-510), rounded to the parameter dtype like every block's output, then
// the same Adan element step as the Kronecker tiles
// ---------------------------------------------------------------------------
template <bool FN>
__global__ void __launch_bounds__(NT)
strip_apply_kernel(ScaoPlanDev P) {
    const ScaoStrip sp = P.strips[blockIdx.x];
    const int pi = sp.param;
    const ScaoParam& pr = P.params[pi];
    const ScaoParamStep& S = P.step[pi];
    if (S.phase != 2) return;
    __shared__ float red[32];
    const int dt = pr.dtype;
    const void* g = (const void*)S.g_ptr;
    const void* pp = (const void*)S.p_ptr;
    float* M = P.exp_avg + pr.offset;
    float* V = P.exp_avg_sq + pr.offset;
    float* Dd = P.exp_avg_diff + pr.offset;
    float* Pv = P.prev_grad + pr.offset;
    const float* de = P.diag_ema + pr.offset;
    const float* ps = P.param_scalars + pi * 8;
    const bool clip = ps[PS_CLIP] != 0.f;
    const float clipmul = ps[PS_CLIPMUL];
    const ScaoFilterDev& FD = P.filt;
    const float thr = (FN && FD.mode) ? FD.fp[pi].thr : 0.f;
    float usq = 0.f, gsq = 0.f, psq = 0.f;
    for (int j = threadIdx.x; j < sp.count; j += NT) {
        const int64_t e = sp.begin + (int64_t)j * sp.stride;
        const float gv = load_dt(g, e, dt);
        const float den = fadd(powf(fdiv(de[e], S.diag_bias), 0.25f), 1e-8f);
        const float gp = round_dt(fdiv(gv, den), dt);
        float gf = gv;
        if (FN)
            gf = filt_grad(FD, gv, FD.mode ? FD.mag_ema[pr.offset + e] : 0.f, thr,
                           FD.noise_on ? f4_get(noise_normal4(FD.noise_seed, pi, FD.noise_step, e >> 2),
                                                (int)(e & 3)) : 0.f);
        float m = M[e], v = V[e], d = Dd[e], pv = Pv[e];
        float u = adan_elem(S, dt, gf, gp, m, v, d, pv, clip, clipmul);
        if (FN && FD.gsnr_on) u = gsnr_mask(u, m, v, S.eps, FD.gsnr_thr);
        usq = fmaf(u, u, usq);
        gsq = fmaf(gv, gv, gsq);
        const float pd = round_dt(fmul(load_dt(pp, e, dt), S.wd_mult), dt);
        psq = fmaf(pd, pd, psq);
        M[e] = m; V[e] = v; Dd[e] = d; Pv[e] = pv;
        if (dt == SCAO_F32) P.upd32[pr.offset + e] = u;
        else store_dt(P.upd + pr.offset, e, dt, u);
    }
    usq = block_sum(usq, red);
    gsq = block_sum(gsq, red);
    psq = block_sum(psq, red);
    if (threadIdx.x == 0) {
        P.strip_part[blockIdx.x * 4 + 0] = usq;
        P.strip_part[blockIdx.x * 4 + 1] = gsq;
        P.strip_part[blockIdx.x * 4 + 2] = psq;
    }
}

// ---------------------------------------------------------------------------
// per param: LARS trust ratio (optimizer.py:371-377) -> alpha
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
param_post_kernel(ScaoPlanDev P) {
    const int pi = blockIdx.x;
    const ScaoParam& pr = P.params[pi];
    const ScaoParamStep& S = P.step[pi];
    if (S.phase == 0) return;
    __shared__ float red[32];
    float usq = 0.f, gsq = 0.f, psq = 0.f;
    const bool kron2 = (S.phase == 2 && pr.mode == 1);
    if (kron2) {
        for (int t = pr.tile_begin + threadIdx.x; t < pr.tile_end; t += NT) {
            usq += P.tile_part[t * 4 + 0];
            gsq += P.tile_part[t * 4 + 1];
            psq += P.tile_part[t * 4 + 2];
        }
        for (int s = threadIdx.x; s < P.n_strips; s += NT)
            if (P.strips[s].param == pi) {
                usq += P.strip_part[s * 4 + 0];
                gsq += P.strip_part[s * 4 + 1];
                psq += P.strip_part[s * 4 + 2];
            }
    } else {
        for (int c = pr.chunk_begin + threadIdx.x; c < pr.chunk_end; c += NT) {
            usq += P.chunk_part[c * 4 + 0];
            gsq += P.chunk_part[c * 4 + 1];
        }
    }
    usq = block_sum(usq, red);
    gsq = block_sum(gsq, red);
    psq = block_sum(psq, red);
    if (threadIdx.x != 0) return;
    float* ps = P.param_scalars + pi * 8;
    if (kron2) ps[PS_PNORM2] = psq;
    ps[PS_GNORM2] = gsq;
    if (S.phase != 2) return;
    ps[PS_UNORM2] = usq;
    const int dt = pr.dtype;
    double trust = 1.0;
    if (S.lars > 0.f) {
        const float pnorm = round_dt(sqrtf(ps[PS_PNORM2]), dt);   // p.data.norm() in param dtype
        const float unorm = sqrtf(usq);
        if (!(pnorm == 0.f || unorm == 0.f)) {
            const float num = round_dt(fmul(S.lars, pnorm), dt);
            const float wdp = round_dt(fmul(S.wd, pnorm), dt);
            const float den = fadd(fadd(unorm, wdp), 1e-8f);
            trust = (double)fdiv(num, den);
        }
    }
    ps[PS_TRUST] = (float)trust;
    ps[PS_ALPHA] = round_dt((float)(-(S.lr * trust)), dt);
}

// global grad-norm EMA (optimizer.py:439-446): mean of the fp32 per-param
// norms, summed in parameter order like Python's sum, then the EMA in
// double without contraction.
__global__ void global_norm_kernel(ScaoPlanDev P) {
    __shared__ float nrm[1024];
    __shared__ int live[1024];
    double s = 0.0;
    int c = 0;
    for (int p0 = 0; p0 < P.n_params; p0 += 1024) {
        const int m = min(1024, P.n_params - p0);
        for (int i = threadIdx.x; i < m; i += blockDim.x) {
            live[i] = P.step[p0 + i].phase != 0;
            // per-parameter norm in the gradient's dtype, as float(p.grad.norm())
            nrm[i] = round_dt(sqrtf(P.param_scalars[(p0 + i) * 8 + PS_GNORM2]),
                              P.params[p0 + i].dtype);
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int i = 0; i < m; ++i)
                if (live[i]) { s = __dadd_rn(s, (double)nrm[i]); ++c; }
        __syncthreads();
    }
    if (threadIdx.x == 0 && c > 0)
        *P.global_norm_ema = __dadd_rn(__dmul_rn(0.95, *P.global_norm_ema),
                                       __dmul_rn(0.05, s / (double)c));
}

// Phase-2 parameter write: p = round(round(p*(1-lr wd)) + alpha*u)
// LA: lookahead step fused (a separate instantiation keeps the plain
// kernel's register count and occupancy)
template <bool LA>
__global__ void __launch_bounds__(NT)
apply_p_kernel(ScaoPlanDev P) {
    const int cid = P.p_list[blockIdx.x];
    const ScaoChunk ch = P.chunks[cid];
    const ScaoParam& pr = P.params[ch.param];
    const ScaoParamStep& S = P.step[ch.param];
    if (S.phase != 2) return;
    const int dt = pr.dtype;
    void* pp = (void*)S.p_ptr;
    const float alpha = P.param_scalars[ch.param * 8 + PS_ALPHA];
    const float wdm = S.wd_mult;
    const bool vec = ((S.p_ptr & 15) == 0) && ((pr.offset & 3) == 0) && ((ch.begin & 3) == 0);
    if (LA) {
        // lookahead step (optimizer.py:356-365) fused into the write:
        //   slow <- slow + a (p_new - slow) (param dtype roundings); p <- slow
        void* sl = dt == SCAO_F32 ? (void*)(P.slow32 + pr.offset) : (void*)(P.slow + pr.offset);
        const float la_a = P.la_alpha;
        const int init = P.la_init;
        auto step1 = [&](int64_t e, float pv, float u, float s) {
            const float pn = round_dt(fmaf(alpha, u, round_dt(fmul(pv, wdm), dt)), dt);
            const float s0 = init ? pn : s;
            const float diff = round_dt(fsub(pn, s0), dt);
            return round_dt(fadd(s0, round_dt(fmul(la_a, diff), dt)), dt);
        };
        int64_t vend = ch.begin;
        if (vec) {
            const int64_t n4 = (ch.end - ch.begin) >> 2;
            vend = ch.begin + n4 * 4;
            for (int64_t q = threadIdx.x; q < n4; q += NT) {
                const int64_t e = ch.begin + q * 4;
                const float4 p4 = load4_dt(pp, e, dt);
                const float4 u4 = dt == SCAO_F32 ? *(const float4*)(P.upd32 + pr.offset + e)
                                                 : load4_dt(P.upd + pr.offset, e, dt);
                const float4 s4 = init ? p4 : load4_dt(sl, e, dt);
                const float4 o = make_float4(step1(e, p4.x, u4.x, s4.x), step1(e, p4.y, u4.y, s4.y),
                                             step1(e, p4.z, u4.z, s4.z), step1(e, p4.w, u4.w, s4.w));
                store4_dt(sl, e, dt, o);
                store4_dt(pp, e, dt, o);
            }
        }
        for (int64_t e = vend + threadIdx.x; e < ch.end; e += NT) {
            const float u = dt == SCAO_F32 ? P.upd32[pr.offset + e] : load_dt(P.upd + pr.offset, e, dt);
            const float pv = load_dt(pp, e, dt);
            const float o = step1(e, pv, u, init ? 0.f : load_dt(sl, e, dt));
            store_dt(sl, e, dt, o);
            store_dt(pp, e, dt, o);
        }
        return;
    }
    if (vec) {
        const int64_t n4 = (ch.end - ch.begin) >> 2;
        for (int64_t q = threadIdx.x; q < n4; q += NT) {
            const int64_t e = ch.begin + q * 4;
            const float4 p4 = load4_dt(pp, e, dt);
            const float4 u4 = dt == SCAO_F32 ? *(const float4*)(P.upd32 + pr.offset + e)
                                             : load4_dt(P.upd + pr.offset, e, dt);
            float4 o;
            o.x = round_dt(fmaf(alpha, u4.x, round_dt(fmul(p4.x, wdm), dt)), dt);
            o.y = round_dt(fmaf(alpha, u4.y, round_dt(fmul(p4.y, wdm), dt)), dt);
            o.z = round_dt(fmaf(alpha, u4.z, round_dt(fmul(p4.z, wdm), dt)), dt);
            o.w = round_dt(fmaf(alpha, u4.w, round_dt(fmul(p4.w, wdm), dt)), dt);
            store4_dt(pp, e, dt, o);
        }
        for (int64_t e = ch.begin + n4 * 4 + threadIdx.x; e < ch.end; e += NT) {
            const float u = dt == SCAO_F32 ? P.upd32[pr.offset + e] : load_dt(P.upd + pr.offset, e, dt);
            store_dt(pp, e, dt, round_dt(fmaf(alpha, u, round_dt(fmul(load_dt(pp, e, dt), wdm), dt)), dt));
        }
    } else {
        for (int64_t e = ch.begin + threadIdx.x; e < ch.end; e += NT) {
            const float u = dt == SCAO_F32 ? P.upd32[pr.offset + e] : load_dt(P.upd + pr.offset, e, dt);
            store_dt(pp, e, dt, round_dt(fmaf(alpha, u, round_dt(fmul(load_dt(pp, e, dt), wdm), dt)), dt));
        }
    }
}

// Lookahead (optimizer.py:356-365), parameter dtype arithmetic:
//   slow = round(slow + round(alpha * round(p - slow))); p = slow
__global__ void __launch_bounds__(NT)
lookahead_kernel(ScaoPlanDev P, float alpha, int init) {
    const ScaoChunk ch = P.chunks[blockIdx.x];
    const ScaoParam& pr = P.params[ch.param];
    const ScaoParamStep& S = P.step[ch.param];
    if (P.la_fused && S.phase == 2) return;     // done inside apply_p_kernel
    const int dt = pr.dtype;
    void* pp = (void*)S.p_ptr;
    void* sl = dt == SCAO_F32 ? (void*)(P.slow32 + pr.offset) : (void*)(P.slow + pr.offset);
    auto la = [&](float p, float s) {
        const float diff = round_dt(fsub(p, s), dt);
        return round_dt(fadd(s, round_dt(fmul(alpha, diff), dt)), dt);
    };
    int64_t vend = ch.begin;
    if (((S.p_ptr & 15) == 0) && ((pr.offset & 3) == 0) && ((ch.begin & 3) == 0)) {
        const int64_t n4 = (ch.end - ch.begin) >> 2;
        vend = ch.begin + n4 * 4;
        for (int64_t q = threadIdx.x; q < n4; q += NT) {
            const int64_t e = ch.begin + q * 4;
            const float4 p4 = load4_dt(pp, e, dt);
            const float4 s4 = init ? p4 : load4_dt(sl, e, dt);
            const float4 o = make_float4(la(p4.x, s4.x), la(p4.y, s4.y), la(p4.z, s4.z),
                                         la(p4.w, s4.w));
            store4_dt(sl, e, dt, o);
            store4_dt(pp, e, dt, o);
        }
    }
    for (int64_t e = vend + threadIdx.x; e < ch.end; e += NT) {
        const float p = load_dt(pp, e, dt);
        float s = init ? p : load_dt(sl, e, dt);
        const float diff = round_dt(fsub(p, s), dt);
        s = round_dt(fadd(s, round_dt(fmul(alpha, diff), dt)), dt);
        store_dt(sl, e, dt, s);
        store_dt(pp, e, dt, s);
    }
}

// ===========================================================================
// Tensor-core (tcgen05) projection and correction.
// fp32 operands (U_r, W) are pre-split into bf16 hi + lo canonical tiles
// (prep_factors_kernel, leaf_coef_kernel) and brought into shared memory by
// TMA bulk copies; products hi*hi + hi*lo + lo*hi keep ~2^-16 relative
// accuracy.  bf16 gradients enter the MMA unsplit (exact); fp16/fp32
// gradients are split while staging.
// ===========================================================================

// Panels whose gradient the cp.async path can stream (bf16, 16-byte rows).
__device__ __forceinline__ bool proj_fast(const ScaoLeaf& L, const ScaoParamStep& S,
                                          const ScaoParam& pr) {
    return pr.dtype == SCAO_BF16 && ((L.ld & 7) == 0) && ((L.col0 & 7) == 0) &&
           ((L.b & 7) == 0) && ((S.g_ptr & 15) == 0);
}

// U_l rows [row0, row0+128) x [0, Kp) -> shared (row stride Kp+4), zero
// padded; 16-byte cp.async chunks when the rows are 16-byte aligned.
__device__ __forceinline__ void stage_ls(float* Ls, const float* Ul, int row0, int nrows, int sl,
                                         int kpad, int Kp) {
    const int q4 = Kp >> 2;
    if ((sl & 3) == 0 && (reinterpret_cast<uintptr_t>(Ul) & 15) == 0) {
        for (int c = threadIdx.x; c < TC_T * q4; c += blockDim.x) {
            const int r = c / q4, a = (c - r * q4) * 4;
            const bool in = r < nrows && a < kpad;
            const float* src = in ? Ul + (int64_t)(row0 + r) * sl + a : Ul;
            asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;"
                         :: "r"(smem_u32(Ls + r * (Kp + 4) + a)), "l"(src), "r"(in ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
    } else {
        for (int e = threadIdx.x; e < TC_T * Kp; e += blockDim.x) {
            const int r = e / Kp, a = e - (e / Kp) * Kp;
            Ls[r * (Kp + 4) + a] = (r < nrows && a < kpad) ? Ul[(int64_t)(row0 + r) * sl + a] : 0.f;
        }
    }
}

// P_part = Ls^T Ts (kp x kp) from two row-major [rows][ld] fp32 tiles in
// shared memory.  Work item = an 8 x 4 output block and one half of the
// rows; the two halves of a block sit in lanes l and l ^ 16 of one warp and
// are added by a shuffle (fixed order: first half + second half).  Per row a
// thread does 32 FMA for three 128-bit shared loads.  t / nthreads: this
// thread among the participating ones (a multiple of 32).
template <class LsRow>
__device__ __forceinline__ void proj_pblock_g(LsRow ls_row, const float* Ts, int ld, int kp,
                                              int nrows, float* out, bool ok, int t, int nthreads) {
    const int nbb = (kp >> 3) * (kp >> 2);           // 8 x 4 blocks (kp is a multiple of 8)
    const int lane = t & 31, w = t >> 5;
    const int ks = lane >> 4;
    const int h = (nrows + 1) >> 1;
    const int r0 = ks ? h : 0, r1 = ks ? nrows : h;
    const int per_it = nthreads >> 1;
    for (int base = 0; base < nbb; base += per_it) {
        const int blk = base + w * 16 + (lane & 15);
        const bool live = blk < nbb;
        const int a0 = live ? (blk / (kp >> 2)) * 8 : 0, b0 = live ? (blk % (kp >> 2)) * 4 : 0;
        float acc[8][4] = {};
        if (live) {
            for (int r = r0; r < r1; ++r) {
                float av[8];
                ls_row(r, a0, av);
                const float4 tb = *(const float4*)&Ts[r * ld + b0];
                const float bv[4] = {tb.x, tb.y, tb.z, tb.w};
#pragma unroll
                for (int i2 = 0; i2 < 8; ++i2)
#pragma unroll
                    for (int j2 = 0; j2 < 4; ++j2) acc[i2][j2] = fmaf(av[i2], bv[j2], acc[i2][j2]);
            }
        }
#pragma unroll
        for (int i2 = 0; i2 < 8; ++i2)
#pragma unroll
            for (int j2 = 0; j2 < 4; ++j2) {
                const float o = __shfl_xor_sync(0xffffffffu, acc[i2][j2], 16);
                acc[i2][j2] = ks ? acc[i2][j2] : __fadd_rn(acc[i2][j2], o);
            }
        if (live && ks == 0)
#pragma unroll
            for (int i2 = 0; i2 < 8; ++i2)
#pragma unroll
                for (int j2 = 0; j2 < 4; ++j2)
                    out[(a0 + i2) * kp + b0 + j2] = ok ? acc[i2][j2] : 0.f;
    }
}

// U_l rows staged in shared memory (row stride ld)
__device__ __forceinline__ void proj_pblock(const float* Ls, const float* Ts, int ld, int kp,
                                            int nrows, float* out, bool ok, int t, int nthreads) {
    proj_pblock_g([&](int r, int a0, float* av) {
        const float4 l0 = *(const float4*)&Ls[r * ld + a0];
        const float4 l1 = *(const float4*)&Ls[r * ld + a0 + 4];
        av[0] = l0.x; av[1] = l0.y; av[2] = l0.z; av[3] = l0.w;
        av[4] = l1.x; av[5] = l1.y; av[6] = l1.z; av[7] = l1.w;
    }, Ts, ld, kp, nrows, out, ok, t, nthreads);
}

// U_r rows -> ua tiles; U_r^T 64-row blocks -> ut tiles
__global__ void __launch_bounds__(256)
prep_factors_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids) {
    const ScaoLeaf& L = P.leaves[ids[blockIdx.y]];
    const int kp = L.kpad, Kp = (kp + 15) & ~15;
    const float* Ur = P.u + L.ur_off;
    const int brows = (L.b + TC_T - 1) / TC_T * TC_T;
    const int64_t tb = (int64_t)TC_T * Kp * 2;
    const int64_t nA = (int64_t)brows * Kp;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nA; e += stride) {
        const int j = (int)(e / Kp), c = (int)(e % Kp);
        const float x = (j < L.b && c < kp) ? Ur[(int64_t)j * L.sr + c] : 0.f;
        uint16_t h, l;
        split_bf16(x, h, l);
        uint8_t* t = P.ua + L.ua_off + (int64_t)(j / TC_T) * 2 * tb;
        const uint32_t o = canon_off(j % TC_T, c, Kp);
        *(uint16_t*)(t + o) = h;
        *(uint16_t*)(t + tb + o) = l;
    }
    // ut: block kb holds B[n][c] = U_r[64 kb + c][n], n < Kp, c < 64
    const int nkb = (L.b + 63) / 64;
    const int64_t bb = (int64_t)Kp * 64 * 2;
    const int64_t nB = (int64_t)nkb * 64 * Kp;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nB; e += stride) {
        const int row = (int)(e / Kp), n = (int)(e % Kp);   // row = 64 kb + c
        const float x = (row < L.b && n < kp) ? Ur[(int64_t)row * L.sr + n] : 0.f;
        uint16_t h, l;
        split_bf16(x, h, l);
        uint8_t* t = P.ut + L.ut_off + (int64_t)(row / 64) * 2 * bb;
        const uint32_t o = canon_off(n, row % 64, 64);
        *(uint16_t*)(t + o) = h;
        *(uint16_t*)(t + bb + o) = l;
    }
}

// corr^T tile on the tensor core, then a row-major streaming epilogue:
// TMEM -> shared (corr[i][j]) -> every thread handles 4 consecutive columns
// of a row (128-bit state accesses, 512 contiguous bytes per warp).  Also
// accumulates ||round(p*(1-lr wd))||^2 for the LARS ratio.
#ifndef SCAO_APPLY_PD
#define SCAO_APPLY_PD 4
#endif
// L2 prefetch of one row segment (128 columns) of every array the apply
// epilogue touches; one request per 128-byte line.
__device__ __forceinline__ void apply_prefetch_row(const ScaoPlanDev& P, const ScaoLeaf& L,
                                                   const ScaoParamStep& S, const ScaoParam& pr,
                                                   int i0, int rr, int nrow, int jcol, int lane) {
    if (rr >= nrow || jcol >= L.b) return;
    const int64_t o = (int64_t)(L.row0 + i0 + rr) * L.ld + L.col0 + jcol;
    if ((lane & 7) == 0) {
        asm volatile("prefetch.global.L2 [%0];" :: "l"(P.exp_avg + pr.offset + o));
        asm volatile("prefetch.global.L2 [%0];" :: "l"(P.exp_avg_sq + pr.offset + o));
        asm volatile("prefetch.global.L2 [%0];" :: "l"(P.exp_avg_diff + pr.offset + o));
        asm volatile("prefetch.global.L2 [%0];" :: "l"(P.prev_grad + pr.offset + o));
    }
    const int es = pr.dtype == SCAO_F32 ? 4 : 2;
    if ((lane & (es == 4 ? 7 : 15)) == 0) {
        asm volatile("prefetch.global.L2 [%0];" :: "l"((const char*)S.g_ptr + o * es));
        asm volatile("prefetch.global.L2 [%0];" :: "l"((const char*)S.p_ptr + o * es));
    }
}

#ifndef SCAO_APPLY_NT
#define SCAO_APPLY_NT 256
#endif
#ifndef SCAO_APPLY_MINB
#define SCAO_APPLY_MINB 3
#endif
// tiles the persistent TMA apply kernel takes (bf16, whole 128 x 128 tiles,
// 16-byte aligned rows, tensor maps valid this step)
__device__ __forceinline__ bool apply_tma_use(const ScaoPlanDev& P, const ScaoLeaf& L) {
    const ScaoParam& pr = P.params[L.param];
    const ScaoParamStep& S = P.step[L.param];
    return P.tmaps_ok && S.phase == 2 && pr.dtype == SCAO_BF16 && (L.a % 128) == 0 &&
           (L.b % 128) == 0 && (L.ld % 8) == 0 && (L.col0 % 8) == 0 && scao_tmap_state_ok(pr, S);
}

// FN: the gradient filter or noise is on this step (a separate
// instantiation keeps the plain epilogue's register budget).
template <bool FN>
__global__ void __launch_bounds__(SCAO_APPLY_NT, SCAO_APPLY_MINB)
apply_kron_tc_kernel(ScaoPlanDev P, int* err) {
    const ScaoTile tl = P.tiles[blockIdx.x];
    const ScaoLeaf& L = P.leaves[tl.leaf];
    const ScaoParamStep& S = P.step[L.param];
    if (S.phase != 2) return;
    if (apply_tma_use(P, L)) return;     // apply_tma_kernel
    const ScaoParam& pr = P.params[L.param];
    const int dt = pr.dtype;
    const int Kp = (L.kpad + 15) & ~15;
    extern __shared__ __align__(1024) unsigned char smx[];
    const uint32_t tb = TC_T * Kp * 2;
    unsigned char* A = smx;            // [hi][lo] of U_r rows j0..
    unsigned char* B = smx + 2 * tb;   // [hi][lo] of W rows i0..
    float* Cs = (float*)smx;           // after the MMA: corr[i][j], 128 x 132
    constexpr int CLD = TC_T + 4;
    __shared__ uint64_t mbar_ld, mbar_mma;
    __shared__ uint32_t tslot;
    __shared__ float red[32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int i0 = tl.row0, j0 = tl.col0;
    if (tid == 0) {
        mbar_init(&mbar_ld, 1);
        mbar_init(&mbar_mma, 1);
        fence_async_smem();
        mbar_expect_tx(&mbar_ld, 4 * tb);
        bulk_g2s(A, P.ua + L.ua_off + (int64_t)(j0 / TC_T) * 2 * tb, 2 * tb, &mbar_ld);
        bulk_g2s(B, P.wa + L.wa_off + (int64_t)(i0 / TC_T) * 2 * tb, 2 * tb, &mbar_ld);
    }
    // start pulling this thread's first state rows into L2 while the
    // correction is built on the tensor core
    for (int d = 0; d < SCAO_APPLY_PD; ++d)
        apply_prefetch_row(P, L, S, pr, i0, (tid >> 5) + d * (SCAO_APPLY_NT / 32),
                           min(TC_T, L.a - i0), j0 + (tid & 31) * 4, lane);
    if (warp == 0) tc_alloc(&tslot, TC_T);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    bool ok = mbar_wait(&mbar_ld, 0);
    if (tid == 0 && ok) {
        const uint32_t idesc = idesc_bf16(TC_T, TC_T);
        const uint32_t sbo = 16 * Kp;
        const uint32_t a0 = smem_u32(A), b0 = smem_u32(B);
        for (int s = 0; s < Kp / 16; ++s) {
            const uint64_t ah = smem_desc(a0 + s * 256, 128, sbo);
            const uint64_t al = smem_desc(a0 + tb + s * 256, 128, sbo);
            const uint64_t bh = smem_desc(b0 + s * 256, 128, sbo);
            const uint64_t bl = smem_desc(b0 + tb + s * 256, 128, sbo);
            tc_mma_bf16(tmem, ah, bh, idesc, s > 0);
            tc_mma_bf16(tmem, ah, bl, idesc, 1);
            tc_mma_bf16(tmem, al, bh, idesc, 1);
        }
        tc_commit(&mbar_mma);
    }
    ok = mbar_wait(&mbar_mma, 0) && ok;
    if (!ok && err) atomicExch(err, 1);
    tc_fence_after();
    // the MMA has consumed A/B: reuse the staging area for corr[i][j]
    {
        constexpr int CPG = TC_T * 4 / (SCAO_APPLY_NT / 32);   // TMEM columns per warp group
        const int q = warp & 3, h = warp >> 2;
        const int jj = q * 32 + lane;
        for (int c0 = h * CPG; c0 < h * CPG + CPG; c0 += 16) {
            float v[16];
            tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + c0, v);
#pragma unroll
            for (int c = 0; c < 16; ++c) Cs[(c0 + c) * CLD + jj] = ok ? v[c] : 0.f;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, TC_T);
    float usq = 0.f, gsq = 0.f, psq = 0.f;
    const float* ps = P.param_scalars + L.param * 8;
    const bool clip = ps[PS_CLIP] != 0.f;
    const float clipmul = ps[PS_CLIPMUL];
    const void* g = (const void*)S.g_ptr;
    const void* pp = (const void*)S.p_ptr;
    float* M = P.exp_avg + pr.offset;
    float* V = P.exp_avg_sq + pr.offset;
    float* Dd = P.exp_avg_diff + pr.offset;
    float* Pv = P.prev_grad + pr.offset;
    const float wdm = S.wd_mult;
    const ScaoFilterDev& FD = P.filt;
    const float* MG = FD.mag_ema + pr.offset;
    const float thr = FD.mode ? FD.fp[L.param].thr : 0.f;
    const int cg = (tid & 31) * 4;          // 4 columns
    const int jcol = j0 + cg;
    const bool vec = ((L.ld & 3) == 0) && ((L.col0 & 3) == 0) && ((S.g_ptr & 15) == 0) &&
                     ((S.p_ptr & 15) == 0) && ((pr.offset & 3) == 0) && (jcol + 3 < L.b);
    const int nrow = min(TC_T, L.a - i0);
    for (int rr = tid >> 5; rr < nrow; rr += SCAO_APPLY_NT / 32) {
        apply_prefetch_row(P, L, S, pr, i0, rr + SCAO_APPLY_PD * (SCAO_APPLY_NT / 32), nrow, jcol, lane);
        const int i = i0 + rr;
        const int64_t o = (int64_t)(L.row0 + i) * L.ld + L.col0 + jcol;
        const float4 cr = *(const float4*)&Cs[rr * CLD + cg];
        const float crv[4] = {cr.x, cr.y, cr.z, cr.w};
        if (vec) {
            const float4 gg = load4_dt(g, o, dt);
            const float4 p4 = load4_dt(pp, o, dt);
            float4 m4 = ldg_stream4(M + o), v4 = ldg_stream4(V + o);
            float4 d4 = ldg_stream4(Dd + o), q4 = ldg_stream4(Pv + o);
            float gv[4] = {gg.x, gg.y, gg.z, gg.w}, pv[4] = {p4.x, p4.y, p4.z, p4.w};
            float mv[4] = {m4.x, m4.y, m4.z, m4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w};
            float dv[4] = {d4.x, d4.y, d4.z, d4.w}, qv[4] = {q4.x, q4.y, q4.z, q4.w};
            float gf[4] = {gv[0], gv[1], gv[2], gv[3]};
            if (FN) {
                const float4 mg4 = FD.mode ? *(const float4*)(MG + o) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 z4 = FD.noise_on ? noise_normal4(FD.noise_seed, L.param, FD.noise_step, o >> 2)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    gf[c] = filt_grad(FD, gv[c], f4_get(mg4, c), thr, f4_get(z4, c));
            }
            float uo[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float gp = round_dt(fadd(gv[c], crv[c]), dt);
                float u = adan_elem(S, dt, gf[c], gp, mv[c], vv[c], dv[c], qv[c], clip, clipmul);
                if (FN && FD.gsnr_on) u = gsnr_mask(u, mv[c], vv[c], S.eps, FD.gsnr_thr);
                usq = fmaf(u, u, usq);
                gsq = fmaf(gv[c], gv[c], gsq);
                const float pd = round_dt(fmul(pv[c], wdm), dt);
                psq = fmaf(pd, pd, psq);
                uo[c] = round_dt(u, dt);
            }
            stg_stream4(M + o, make_float4(mv[0], mv[1], mv[2], mv[3]));
            stg_stream4(V + o, make_float4(vv[0], vv[1], vv[2], vv[3]));
            stg_stream4(Dd + o, make_float4(dv[0], dv[1], dv[2], dv[3]));
            stg_stream4(Pv + o, make_float4(qv[0], qv[1], qv[2], qv[3]));
            if (dt == SCAO_F32) store4_dt(P.upd32 + pr.offset, o, dt, make_float4(uo[0], uo[1], uo[2], uo[3]));
            else store4_dt(P.upd + pr.offset, o, dt, make_float4(uo[0], uo[1], uo[2], uo[3]));
        } else {
            for (int c = 0; c < 4; ++c) {
                if (jcol + c >= L.b) break;
                const int64_t oc = o + c;
                const float gv = load_dt(g, oc, dt);
                float mv = M[oc], vv = V[oc], dv = Dd[oc], qv = Pv[oc];
                const float gp = round_dt(fadd(gv, crv[c]), dt);
                float gf = gv;
                if (FN)
                    gf = filt_grad(FD, gv, FD.mode ? MG[oc] : 0.f, thr,
                                   FD.noise_on ? f4_get(noise_normal4(FD.noise_seed, L.param,
                                                                      FD.noise_step, oc >> 2), (int)(oc & 3))
                                               : 0.f);
                float u = adan_elem(S, dt, gf, gp, mv, vv, dv, qv, clip, clipmul);
                if (FN && FD.gsnr_on) u = gsnr_mask(u, mv, vv, S.eps, FD.gsnr_thr);
                usq = fmaf(u, u, usq);
                gsq = fmaf(gv, gv, gsq);
                const float pd = round_dt(fmul(load_dt(pp, oc, dt), wdm), dt);
                psq = fmaf(pd, pd, psq);
                M[oc] = mv; V[oc] = vv; Dd[oc] = dv; Pv[oc] = qv;
                if (dt == SCAO_F32) P.upd32[pr.offset + oc] = u;
                else store_dt(P.upd + pr.offset, oc, dt, u);
            }
        }
    }
    usq = block_sum(usq, red);
    gsq = block_sum(gsq, red);
    psq = block_sum(psq, red);
    if (tid == 0) {
        P.tile_part[blockIdx.x * 4 + 0] = usq;
        P.tile_part[blockIdx.x * 4 + 1] = gsq;
        P.tile_part[blockIdx.x * 4 + 2] = psq;
    }
}

// ---------------------------------------------------------------------------
// Persistent, warp-specialised projection for bf16 gradients with a TMA
// tensor map: one work item per 128-row panel of a Kronecker leaf.
//   warp 0     TMA producer: G panel block (128 rows x 64 columns, 128-byte
//              swizzle) + U_r^T block (bf16 hi/lo, bulk copy) per stage
//   warp 1     TMEM owner + MMA issuer: T = G_panel U_r (hi and lo
//              products, fp32 accumulators, two TMEM buffers)
//   warps 2-5  epilogue: T -> shared, P_part = U_l[rows]^T T (FFMA, U_l
//              rows read through L1), overlapping the next panel's loads
// Panels whose leaf width is not a multiple of 64 stay on proj_bf16_kernel.
// ---------------------------------------------------------------------------
constexpr int PT_MAXST = 4;
constexpr int PT_EPI = 256;                // epilogue threads (8 warps)
constexpr int PT_THREADS = 64 + PT_EPI;

__device__ __forceinline__ bool proj_tma_use(const ScaoPlanDev& P, const ScaoLeaf& L) {
    const ScaoParam& pr = P.params[L.param];
    const ScaoParamStep& S = P.step[L.param];
    return P.tmaps_ok && S.phase == 2 && proj_fast(L, S, pr) && scao_tmap_ok(pr, S) &&
           (L.b % 64) == 0;
}

__host__ __device__ inline int proj_tma_stages(int kpmax) { return kpmax > 64 ? 3 : 4; }
__host__ __device__ inline uint32_t proj_tma_stage_bytes(int kpmax) {
    return 128 * 64 * 2 + 2 * (uint32_t)kpmax * 64 * 2;
}
// U_l panel rows are staged in shared memory when they fit (Kp <= 64)
__host__ __device__ inline bool proj_tma_ls_smem(int kpmax) { return kpmax <= 64; }
size_t proj_tma_smem(int kpad_max) {
    const int Kp = (kpad_max + 15) & ~15;
    return (size_t)proj_tma_stages(Kp) * proj_tma_stage_bytes(Kp) +
           (size_t)(proj_tma_ls_smem(Kp) ? 2 : 1) * 128 * (Kp + 4) * 4 + 1024;
}

__global__ void __launch_bounds__(PT_THREADS, 1)
proj_tma_kernel(ScaoPlanDev P, int* err) {
    extern __shared__ unsigned char psm_raw[];
    unsigned char* psm = (unsigned char*)(((uintptr_t)psm_raw + 1023) & ~(uintptr_t)1023);
    const int Kpm = (P.kpad_max + 15) & ~15;
    const int nst = proj_tma_stages(Kpm);
    const uint32_t SB = proj_tma_stage_bytes(Kpm);
    float* Ts = (float*)(psm + (size_t)nst * SB);
    float* Ls = Ts + 128 * (Kpm + 4);            // used when proj_tma_ls_smem(Kpm)
    const bool ls_sm = proj_tma_ls_smem(Kpm);
    __shared__ uint64_t full[PT_MAXST], empty[PT_MAXST], accf[2], acce[2], fin;
    __shared__ uint32_t tslot;
    __shared__ volatile int abort_flag, ep_go;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < PT_MAXST; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&accf[i], 1); mbar_init(&acce[i], PT_EPI); }
        mbar_init(&fin, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // two accumulators of 2 Kp columns: T_hi = G U_r,hi and T_lo = G U_r,lo
    // side by side (one MMA of N = 2 Kp reads the gradient block once)
    const uint32_t tcols = Kpm > 64 ? 512u : 256u;
    if (warp == 1) tc_alloc(&tslot, tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    const int total = P.n_panels;
    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t ph = 0, issued = 0, last_ph = 0;
            for (int T = blockIdx.x; T < total && !abort_flag; T += gridDim.x) {
                const ScaoPanel pn = P.panels[T];
                const ScaoLeaf& L = P.leaves[pn.leaf];
                if (!proj_tma_use(P, L)) continue;
                const int Kp = (L.kpad + 15) & ~15;
                const uint32_t bb = (uint32_t)Kp * 64 * 2;
                const void* map = scao_tmap(P.tmaps, L.param, TM_G128);
                for (int kb = 0; kb < L.b / 64; ++kb) {
                    if (!mbar_wait(&empty[stage], ph ^ 1)) { abort_flag = 1; atomicExch(err, 2); break; }
                    mbar_expect_tx(&full[stage], 128 * 64 * 2 + 2 * bb);
                    unsigned char* st = psm + (size_t)stage * SB;
                    tma_load_2d(smem_u32(st), map, L.col0 + kb * 64, L.row0 + pn.row0, &full[stage]);
                    bulk_g2s(st + 128 * 64 * 2, P.ut + L.ut_off + (int64_t)kb * 2 * bb, 2 * bb, &full[stage]);
                    issued |= 1u << stage;
                    last_ph = (last_ph & ~(1u << stage)) | (ph << stage);
                    if (++stage == nst) { stage = 0; ph ^= 1; }
                }
            }
            for (int s2 = 0; s2 < nst; ++s2)
                if ((issued >> s2) & 1u)
                    if (!mbar_wait(&full[s2], (last_ph >> s2) & 1u)) atomicExch(err, 2);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0, acc = 0;
            uint32_t ph = 0, aph = 0;
            for (int T = blockIdx.x; T < total && !abort_flag; T += gridDim.x) {
                const ScaoPanel pn = P.panels[T];
                const ScaoLeaf& L = P.leaves[pn.leaf];
                if (!proj_tma_use(P, L)) continue;
                const int Kp = (L.kpad + 15) & ~15;
                if (!mbar_wait(&acce[acc], aph ^ 1)) { abort_flag = 1; atomicExch(err, 2); break; }
                tc_fence_after();
                const uint32_t d = tmem + acc * 2 * Kpm;
                const uint32_t idesc = idesc_bf16(128, 2 * Kp);
                bool ok = true;
                for (int kb = 0; kb < L.b / 64; ++kb) {
                    if (!mbar_wait(&full[stage], ph)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a = smem_u32(psm + (size_t)stage * SB);
                    const uint32_t bh = a + 128 * 64 * 2;     // [hi: Kp rows][lo: Kp rows]
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint64_t ad = smem_desc_sw128(a + s * 32, 16, 1024);
                        tc_mma_bf16(d, ad, smem_desc(bh + s * 256, 128, 16 * 64), idesc,
                                    (kb > 0 || s > 0) ? 1u : 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == nst) { stage = 0; ph ^= 1; }
                }
                if (!ok) { abort_flag = 1; atomicExch(err, 2); break; }
                tc_commit(&accf[acc]);
                acc ^= 1;
                if (acc == 0) aph ^= 1;
            }
            tc_commit(&fin);
            if (!mbar_wait(&fin, 0)) atomicExch(err, 2);
        }
    } else {
        const int et = tid - 64;                 // epilogue thread 0..PT_EPI-1
        const int q = warp & 3;                  // TMEM lane quarter
        const int h = (warp - 2) >> 2;           // which 16-column chunks
        const int r = q * 32 + lane;
        int acc = 0;
        uint32_t aph = 0;
        for (int T = blockIdx.x; T < total; T += gridDim.x) {
            const ScaoPanel pn = P.panels[T];
            const ScaoLeaf& L = P.leaves[pn.leaf];
            if (!proj_tma_use(P, L)) continue;
            // one decision for all four epilogue warps (they meet at named
            // barriers, so none may leave the loop alone); also frees Ts
            if (et == 0) ep_go = !abort_flag;
            named_bar(1, PT_EPI);
            if (!ep_go) break;
            const int Kp = (L.kpad + 15) & ~15;
            const int ld = Kp + 4;
            const float* Ulp = P.u + L.ul_off + (int64_t)pn.row0 * L.sl;
            const bool ls_async = ls_sm && (L.sl & 3) == 0;
            if (ls_async) {
                // U_l panel rows -> shared, overlapping the wait for T
                const int q4 = Kp >> 2;
                for (int c = et; c < 128 * q4; c += PT_EPI) {
                    const int rr = c / q4, a = (c - rr * q4) * 4;
                    const bool in = rr < pn.nrows && a < L.kpad;
                    const float* src = in ? Ulp + (int64_t)rr * L.sl + a : Ulp;
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;"
                                 :: "r"(smem_u32(Ls + rr * ld + a)), "l"(src), "r"(in ? 16 : 0)
                                 : "memory");
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
            }
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&accf[acc], aph));
            if (!ok) { abort_flag = 1; atomicExch(err, 2); }
            if (ok) {
                tc_fence_after();
                const uint32_t tb = tmem + acc * 2 * Kpm + ((uint32_t)(q * 32) << 16);
                for (int c0 = 16 * h; c0 < Kp; c0 += 32) {
                    float vh[16], vl[16];
                    tc_ld16(tb + c0, vh);
                    tc_ld16(tb + Kp + c0, vl);
#pragma unroll
                    for (int c = 0; c < 16; ++c) Ts[r * ld + c0 + c] = __fadd_rn(vh[c], vl[c]);
                }
            }
            tc_fence_before();
            mbar_arrive(&acce[acc]);
            acc ^= 1;
            if (acc == 0) aph ^= 1;
            if (ls_async) asm volatile("cp.async.wait_all;" ::: "memory");
            named_bar(1, PT_EPI);                 // Ts (and Ls) complete
            // P_part = U_l[rows]^T T
            const int kp = L.kpad;
            float* out = P.p_part + (int64_t)T * P.p_stride;
            if (ls_async) {
                proj_pblock(Ls, Ts, ld, kp, pn.nrows, out, ok, et, PT_EPI);
            } else {
                const int sl = L.sl;
                proj_pblock_g([&](int r, int a0, float* av) {
#pragma unroll
                    for (int i2 = 0; i2 < 8; ++i2)
                        av[i2] = a0 + i2 < kp ? __ldg(Ulp + (int64_t)r * sl + a0 + i2) : 0.f;
                }, Ts, ld, kp, pn.nrows, out, ok, et, PT_EPI);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tc_dealloc(tmem, tcols);
}

// ---------------------------------------------------------------------------
// Persistent apply for bf16 parameters (Phase 2, filter and noise off): the
// Kronecker correction of a 128 x 128 tile on the tensor core, and the
// Adan / blend / weight-decay epilogue streaming the tile's gradient,
// parameter and four fp32 moments through shared memory by TMA tensor
// copies in 16-row chunks; the moments and the rounded update go back by
// TMA tensor stores from the same buffers.
//   warp 0      state producer: 6 tensor loads per chunk into a stage ring
//   warp 1      TMEM owner + operand loads (bulk) + MMA issuer, two
//               accumulators (corr^T: lane j, column i)
//   warps 2-9   epilogue: thread = tile column j (its TMEM lane), half the
//               rows of each chunk; an elected thread issues the stores
// ---------------------------------------------------------------------------
#ifndef SCAO_APPLY_EPI
#define SCAO_APPLY_EPI 512
#endif
constexpr int AT_EPI = SCAO_APPLY_EPI;          // epilogue threads (256 or 512)
constexpr int AT_THREADS = 64 + AT_EPI;
#ifndef SCAO_APPLY_ST
#define SCAO_APPLY_ST 4
#endif
constexpr int AT_MAXST = 4;
constexpr int AT_R = TMA_STATE_ROWS;                   // rows per chunk (16)
constexpr int AT_RPT = AT_R * 128 / AT_EPI;           // rows per thread per chunk
constexpr uint32_t AT_G = 0, AT_P = AT_R * 128 * 2, AT_M = 2 * AT_R * 128 * 2;
constexpr uint32_t AT_V = AT_M + AT_R * 128 * 4, AT_D = AT_V + AT_R * 128 * 4;
constexpr uint32_t AT_PV = AT_D + AT_R * 128 * 4;
constexpr uint32_t AT_STAGE = AT_PV + AT_R * 128 * 4;  // 40 KB
constexpr uint32_t AT_MG = AT_STAGE;                   // filter: magnitude EMA chunk
constexpr uint32_t AT_STAGE_FN = AT_STAGE + AT_R * 128 * 4;   // 48 KB


__host__ __device__ inline uint32_t apply_tma_ops_bytes(int kpm) { return 4u * 128 * kpm * 2; }
__host__ __device__ inline uint32_t apply_tma_stage_bytes(bool fn) { return fn ? AT_STAGE_FN : AT_STAGE; }
// as many stages (<= SCAO_APPLY_ST) as fit next to the operand tiles
__host__ __device__ inline int apply_tma_stages(int kpm, bool fn) {
    int s = SCAO_APPLY_ST;
    // 227 KB opt-in per block, less 1 KB for the kernel's static shared data
    while (s > 2 && apply_tma_ops_bytes(kpm) + (uint32_t)s * apply_tma_stage_bytes(fn) + 1024 > 231424u) --s;
    return s;
}
size_t apply_tma_smem(int kpad_max, bool fn) {
    const int Kp = (kpad_max + 15) & ~15;
    return (size_t)apply_tma_ops_bytes(Kp) + (size_t)apply_tma_stages(Kp, fn) * apply_tma_stage_bytes(fn) +
           1024;
}

// FN: the gradient filter, noise or gSNR clip is on this step
template <bool FN>
__global__ void __launch_bounds__(AT_THREADS, 1)
apply_tma_kernel(ScaoPlanDev P, int* err) {
    extern __shared__ unsigned char asm_raw[];
    unsigned char* sm = (unsigned char*)(((uintptr_t)asm_raw + 1023) & ~(uintptr_t)1023);
    const int Kpm = (P.kpad_max + 15) & ~15;
    const int nst = apply_tma_stages(Kpm, FN);
    constexpr uint32_t SBY = FN ? AT_STAGE_FN : AT_STAGE;
    const bool with_mg = FN && P.filt.mode != 0;
    unsigned char* ops = sm;                                  // [A hi|lo][B hi|lo]
    unsigned char* stg = sm + apply_tma_ops_bytes(Kpm);
    __shared__ uint64_t full[AT_MAXST], empty[AT_MAXST], accf[2], acce[2], opfull, opfree, fin;
    __shared__ uint32_t tslot;
    __shared__ volatile int abort_flag, ep_go;
    __shared__ float red[AT_EPI / 32][3];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < AT_MAXST; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&accf[i], 1); mbar_init(&acce[i], AT_EPI); }
        mbar_init(&opfull, 1);
        mbar_init(&opfree, 1);
        mbar_init(&fin, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tc_alloc(&tslot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    const int total = P.n_tiles;
    if (warp == 0) {
        if (lane == 0) {
            // ---------------- state producer ----------------
            int stage = 0;
            uint32_t ph = 0, issued = 0, last_ph = 0;
            constexpr int NCH = 128 / AT_R;
            for (int T = blockIdx.x; T < total && !abort_flag; T += gridDim.x) {
                const ScaoTile tl = P.tiles[T];
                const ScaoLeaf& L = P.leaves[tl.leaf];
                if (!apply_tma_use(P, L)) continue;
                const int x = L.col0 + tl.col0;
                for (int c = 0; c < NCH; ++c) {
                    if (!mbar_wait(&empty[stage], ph ^ 1)) { abort_flag = 1; atomicExch(err, 2); break; }
                    const int y = L.row0 + tl.row0 + c * AT_R;
                    mbar_expect_tx(&full[stage], with_mg ? AT_STAGE_FN : AT_STAGE);
                    const uint32_t s = smem_u32(stg + (size_t)stage * SBY);
#ifdef SCAO_APPLY_EVF
                    const uint64_t pol = l2_policy_evict_first();
#define AT_LOAD(off, slot) tma_load_2d_hint(s + off, scao_tmap(P.tmaps, L.param, slot), x, y, &full[stage], pol)
#else
#define AT_LOAD(off, slot) tma_load_2d(s + off, scao_tmap(P.tmaps, L.param, slot), x, y, &full[stage])
#endif
                    if (with_mg) AT_LOAD(AT_MG, TM_MG);
                    AT_LOAD(AT_G, TM_GS);
                    AT_LOAD(AT_P, TM_PS);
                    AT_LOAD(AT_M, TM_M);
                    AT_LOAD(AT_V, TM_V);
                    AT_LOAD(AT_D, TM_D);
                    AT_LOAD(AT_PV, TM_PV);
#undef AT_LOAD
                    issued |= 1u << stage;
                    last_ph = (last_ph & ~(1u << stage)) | (ph << stage);
                    if (++stage == nst) { stage = 0; ph ^= 1; }
                }
            }
            for (int s2 = 0; s2 < nst; ++s2)
                if ((issued >> s2) & 1u)
                    if (!mbar_wait(&full[s2], (last_ph >> s2) & 1u)) atomicExch(err, 2);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- operands + MMA ----------------
            int acc = 0;
            uint32_t aph = 0, opph = 0, ofph = 0;
            bool any = false;
            const uint32_t tbm = 128u * Kpm * 2;
            for (int T = blockIdx.x; T < total && !abort_flag; T += gridDim.x) {
                const ScaoTile tl = P.tiles[T];
                const ScaoLeaf& L = P.leaves[tl.leaf];
                if (!apply_tma_use(P, L)) continue;
                const int Kp = (L.kpad + 15) & ~15;
                const uint32_t tb = 128u * Kp * 2;
                if (any) {               // the previous tile's MMAs have read the operands
                    if (!mbar_wait(&opfree, opph)) { abort_flag = 1; atomicExch(err, 2); break; }
                    opph ^= 1;
                }
                any = true;
                unsigned char* A = ops;                  // U_r rows j0.. [hi][lo]
                unsigned char* B = ops + 2 * tbm;        // W rows i0..   [hi][lo]
                mbar_expect_tx(&opfull, 4 * tb);
                bulk_g2s(A, P.ua + L.ua_off + (int64_t)(tl.col0 / 128) * 2 * tb, 2 * tb, &opfull);
                bulk_g2s(B, P.wa + L.wa_off + (int64_t)(tl.row0 / 128) * 2 * tb, 2 * tb, &opfull);
                if (!mbar_wait(&opfull, ofph)) { abort_flag = 1; atomicExch(err, 2); break; }
                ofph ^= 1;
                if (!mbar_wait(&acce[acc], aph ^ 1)) { abort_flag = 1; atomicExch(err, 2); break; }
                tc_fence_after();
                const uint32_t d = tmem + acc * 128;
                const uint32_t idesc = idesc_bf16(128, 128);
                const uint32_t sbo = 16 * Kp;
                const uint32_t a0 = smem_u32(A), b0 = smem_u32(B);
                for (int s = 0; s < Kp / 16; ++s) {
                    const uint64_t ah = smem_desc(a0 + s * 256, 128, sbo);
                    const uint64_t al = smem_desc(a0 + tb + s * 256, 128, sbo);
                    const uint64_t bh = smem_desc(b0 + s * 256, 128, sbo);
                    const uint64_t bl = smem_desc(b0 + tb + s * 256, 128, sbo);
                    tc_mma_bf16(d, ah, bh, idesc, s > 0 ? 1u : 0u);
                    tc_mma_bf16(d, ah, bl, idesc, 1u);
                    tc_mma_bf16(d, al, bh, idesc, 1u);
                }
                tc_commit(&accf[acc]);
                tc_commit(&opfree);
                acc ^= 1;
                if (acc == 0) aph ^= 1;
            }
            tc_commit(&fin);
            if (!mbar_wait(&fin, 0)) atomicExch(err, 2);
        }
    } else {
        // ---------------- epilogue ----------------
        const int et = tid - 64;
        const int ew = warp - 2;                  // epilogue warp
        const int q = warp & 3;                   // TMEM lane quarter -> columns 32q..
        const int h = ew >> 2;                    // row group of each chunk
        const int j = q * 32 + lane;              // tile column of this thread
        int acc = 0, stage = 0;
        uint32_t aph = 0, ph = 0;
        for (int T = blockIdx.x; T < total; T += gridDim.x) {
            const ScaoTile tl = P.tiles[T];
            const ScaoLeaf& L = P.leaves[tl.leaf];
            if (!apply_tma_use(P, L)) continue;
            if (et == 0) ep_go = !abort_flag;
            named_bar(1, AT_EPI);
            if (!ep_go) break;
            const ScaoParamStep& S = P.step[L.param];
            const float* ps = P.param_scalars + L.param * 8;
            const bool clip = ps[PS_CLIP] != 0.f;
            const float clipmul = ps[PS_CLIPMUL];
            const float wdm = S.wd_mult;
            const int x = L.col0 + tl.col0;
            bool ok = __all_sync(0xffffffffu, mbar_wait(&accf[acc], aph));
            if (ok) tc_fence_after();
            float usq = 0.f, gsq = 0.f, psq = 0.f;
            for (int c = 0; c < 128 / AT_R; ++c) {
                const bool okc = ok && __all_sync(0xffffffffu, mbar_wait(&full[stage], ph));
                if (!okc) { abort_flag = 1; atomicExch(err, 2); }
                unsigned char* st = stg + (size_t)stage * SBY;
                if (okc) {
                    float corr[AT_RPT];
                    if (AT_RPT == 8) tc_ld8(tmem + acc * 128 + ((uint32_t)(q * 32) << 16) + c * AT_R + h * 8, corr);
                    else tc_ld4(tmem + acc * 128 + ((uint32_t)(q * 32) << 16) + c * AT_R + h * 4, corr);
                    uint16_t* gs = (uint16_t*)(st + AT_G);
                    const uint16_t* pps = (const uint16_t*)(st + AT_P);
                    float* ms = (float*)(st + AT_M);
                    float* vs = (float*)(st + AT_V);
                    float* ds = (float*)(st + AT_D);
                    float* qs = (float*)(st + AT_PV);
                    float zr[AT_RPT];
                    if (FN) {
                        // gradient noise of (row, column j): the Philox block of a
                        // 4-column group is drawn once per row by one lane of the
                        // group and handed to the others by shuffles
                        const int rbase = L.row0 + tl.row0 + c * AT_R + h * AT_RPT;
                        const int64_t cols = P.params[L.param].cols;
                        const int g4 = lane >> 2, t4 = lane & 3;
#pragma unroll
                        for (int rr = 0; rr < AT_RPT; ++rr) zr[rr] = 0.f;
                        if (P.filt.noise_on) {
                            if (AT_RPT == 4) {
                                const int64_t e = (int64_t)(rbase + t4) * cols + x + q * 32 + g4 * 4;
                                const float4 z4 = noise_normal4(P.filt.noise_seed, L.param,
                                                                P.filt.noise_step, e >> 2);
#pragma unroll
                                for (int rr = 0; rr < AT_RPT; ++rr) {
                                    const int src = (lane & ~3) + rr;
                                    const float a0 = __shfl_sync(0xffffffffu, z4.x, src);
                                    const float a1 = __shfl_sync(0xffffffffu, z4.y, src);
                                    const float a2 = __shfl_sync(0xffffffffu, z4.z, src);
                                    const float a3 = __shfl_sync(0xffffffffu, z4.w, src);
                                    zr[rr] = t4 == 0 ? a0 : t4 == 1 ? a1 : t4 == 2 ? a2 : a3;
                                }
                            } else {
#pragma unroll
                                for (int rr = 0; rr < AT_RPT; ++rr) {
                                    const int64_t e = (int64_t)(rbase + rr) * cols + x + j;
                                    zr[rr] = f4_get(noise_normal4(P.filt.noise_seed, L.param,
                                                                  P.filt.noise_step, e >> 2), (int)(e & 3));
                                }
                            }
                        }
                    }
                    const float* mgs = (const float*)(st + AT_MG);
                    const float thr = (FN && P.filt.mode) ? P.filt.fp[L.param].thr : 0.f;
#pragma unroll
                    for (int rr = 0; rr < AT_RPT; ++rr) {
                        const int o = (h * AT_RPT + rr) * 128 + j;
                        const float gv = bf16_bits_to_f(gs[o]);
                        const float pv = bf16_bits_to_f(pps[o]);
                        float mv = ms[o], vv = vs[o], dv = ds[o], qv = qs[o];
                        const float gp = round_dt(fadd(gv, corr[rr]), SCAO_BF16);
                        float gf = gv;
                        if (FN) gf = filt_grad(P.filt, gv, with_mg ? mgs[o] : 0.f, thr, zr[rr]);
                        float u = adan_elem(S, SCAO_BF16, gf, gp, mv, vv, dv, qv, clip, clipmul);
                        if (FN && P.filt.gsnr_on) u = gsnr_mask(u, mv, vv, S.eps, P.filt.gsnr_thr);
                        usq = fmaf(u, u, usq);
                        gsq = fmaf(gv, gv, gsq);
                        const float pd = round_dt(fmul(pv, wdm), SCAO_BF16);
                        psq = fmaf(pd, pd, psq);
                        ms[o] = mv; vs[o] = vv; ds[o] = dv; qs[o] = qv;
                        gs[o] = f_to_bf16_bits(u);
                    }
                }
                fence_async_smem();
                named_bar(1, AT_EPI);
                if (et == 0) {
                    if (okc) {
                        const int y = L.row0 + tl.row0 + c * AT_R;
                        const uint32_t s = smem_u32(st);
#ifdef SCAO_APPLY_EVF
                        const uint64_t pol = l2_policy_evict_first();
#define AT_STORE(slot, off) tma_store_2d_hint(scao_tmap(P.tmaps, L.param, slot), x, y, s + off, pol)
#else
#define AT_STORE(slot, off) tma_store_2d(scao_tmap(P.tmaps, L.param, slot), x, y, s + off)
#endif
                        AT_STORE(TM_US, AT_G);
                        AT_STORE(TM_M, AT_M);
                        AT_STORE(TM_V, AT_V);
                        AT_STORE(TM_D, AT_D);
                        AT_STORE(TM_PV, AT_PV);
#undef AT_STORE
                        bulk_commit();
                        bulk_wait_read0();
                    }
                    mbar_arrive(&empty[stage]);
                }
                if (++stage == nst) { stage = 0; ph ^= 1; }
            }
            tc_fence_before();
            mbar_arrive(&acce[acc]);
            acc ^= 1;
            if (acc == 0) aph ^= 1;
            // per-tile sums (usq, gsq, psq) -> tile_part
            usq = warp_sum(usq);
            gsq = warp_sum(gsq);
            psq = warp_sum(psq);
            if (lane == 0) { red[ew][0] = usq; red[ew][1] = gsq; red[ew][2] = psq; }
            named_bar(1, AT_EPI);
            if (et == 0) {
                float a = 0.f, b = 0.f, cc = 0.f;
                for (int w = 0; w < AT_EPI / 32; ++w) { a += red[w][0]; b += red[w][1]; cc += red[w][2]; }
                P.tile_part[T * 4 + 0] = a;
                P.tile_part[T * 4 + 1] = b;
                P.tile_part[T * 4 + 2] = cc;
            }
        }
        if (et == 0) bulk_wait0();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tc_dealloc(tmem, 256);
}

// bf16 gradients: T = G_panel * U_r with the gradient streamed into shared
// memory by cp.async (16-byte chunks land directly in the canonical layout),
// a 4-stage pipeline, U_r^T blocks by TMA bulk copy.
constexpr int PJ_STAGES = 3;
__global__ void __launch_bounds__(128)
proj_bf16_kernel(ScaoPlanDev P, int* err) {
    const ScaoPanel pn = P.panels[blockIdx.x];
    const ScaoLeaf& L = P.leaves[pn.leaf];
    const ScaoParamStep& S = P.step[L.param];
    if (S.phase != 2) return;
    const ScaoParam& pr = P.params[L.param];
    if (!proj_fast(L, S, pr)) return;        // handled by proj_tc_kernel
    if (proj_tma_use(P, L)) return;          // handled by proj_tma_kernel
    const int Kp = (L.kpad + 15) & ~15;
    constexpr int KB = 64;
    extern __shared__ __align__(1024) unsigned char smx[];
    const uint32_t abytes = TC_T * KB * 2, bbytes = Kp * KB * 2;
    const uint32_t sbytes = abytes + 2 * bbytes;     // [A][B hi][B lo]
    __shared__ uint64_t mbar_b[PJ_STAGES], mbar_m[PJ_STAGES];
    __shared__ uint32_t tslot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint16_t* g = (const uint16_t*)S.g_ptr;
    const float* Ul = P.u + L.ul_off;
    uint32_t ncols = 32;                        // [T_hi | T_lo]: 2 Kp columns
    while ((int)ncols < 2 * Kp) ncols <<= 1;
    if (warp == 0) tc_alloc(&tslot, ncols);
    if (tid == 0) {
        for (int i = 0; i < PJ_STAGES; ++i) { mbar_init(&mbar_b[i], 1); mbar_init(&mbar_m[i], 1); }
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    const uint32_t idesc = idesc_bf16(TC_T, 2 * Kp);
    const int64_t base = (int64_t)(L.row0 + pn.row0) * L.ld + L.col0;
    const int nkb = (L.b + KB - 1) / KB;
    bool ok = true;
    auto issue = [&](int kb) {
        const int buf = kb % PJ_STAGES;
        unsigned char* st = smx + buf * sbytes;
        const int c0 = kb * KB;
        if (tid == 0) {
            mbar_expect_tx(&mbar_b[buf], 2 * bbytes);
            bulk_g2s(st + abytes, P.ut + L.ut_off + (int64_t)kb * 2 * bbytes, 2 * bbytes,
                     &mbar_b[buf]);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int ch = tid + q * 128;
            const int r = ch >> 3, cc = (ch & 7) * 8;
            const uint32_t dst = smem_u32(st + canon_off(r, cc, KB));
            const bool in = r < pn.nrows && c0 + cc + 8 <= L.b;
            const uint16_t* src = g + base + (int64_t)(in ? r : 0) * L.ld + (in ? c0 + cc : 0);
            const int sz = in ? 16 : 0;      // zero-fill rows/cols outside the panel
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                         :: "r"(dst), "l"(src), "r"(sz) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // prologue: always S-1 commit groups (empty ones past the last block) so
    // that "wait_group S-1" in iteration kb means block kb has landed
    for (int kb = 0; kb < PJ_STAGES - 1; ++kb) {
        if (kb < nkb) issue(kb);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int kb = 0; kb < nkb; ++kb) {
        const int buf = kb % PJ_STAGES;
        const int nxt = kb + PJ_STAGES - 1;
        if (nxt < nkb) {
            // buffer of nxt was last used by block nxt - STAGES: wait for its MMA
            if (nxt >= PJ_STAGES)
                ok = mbar_wait(&mbar_m[nxt % PJ_STAGES], ((nxt - PJ_STAGES) / PJ_STAGES) & 1) && ok;
            issue(nxt);
        } else {
            asm volatile("cp.async.commit_group;" ::: "memory");   // keep group count uniform
        }
        asm volatile("cp.async.wait_group %0;" :: "n"(PJ_STAGES - 1) : "memory");
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            ok = mbar_wait(&mbar_b[buf], (kb / PJ_STAGES) & 1) && ok;
            const uint32_t sa = smem_u32(smx + buf * sbytes), sbh = sa + abytes;
            for (int s = 0; s < KB / 16; ++s) {
                const uint64_t a0 = smem_desc(sa + s * 256, 128, 16 * KB);
                // B = [U_r,hi ; U_r,lo] (2 Kp rows): one MMA gives T_hi and T_lo
                tc_mma_bf16(tmem, a0, smem_desc(sbh + s * 256, 128, 16 * KB), idesc, (kb > 0 || s > 0));
            }
            tc_commit(&mbar_m[buf]);
        }
    }
    ok = mbar_wait(&mbar_m[(nkb - 1) % PJ_STAGES], ((nkb - 1) / PJ_STAGES) & 1) && ok;
    if (!ok && err) atomicExch(err, 1);
    tc_fence_after();
    __syncthreads();
    float* Ts = (float*)smx;
    float* Ls = Ts + TC_T * (Kp + 4);
    {
        const int r = warp * 32 + lane;
        for (int c0 = 0; c0 < Kp; c0 += 16) {
            float v[16];
            float vl[16];
            tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
            tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + Kp + c0, vl);
            for (int c = 0; c < 16; ++c) Ts[r * (Kp + 4) + c0 + c] = ok ? __fadd_rn(v[c], vl[c]) : 0.f;
        }
    }
    stage_ls(Ls, Ul, pn.row0, pn.nrows, L.sl, L.kpad, Kp);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, ncols);
    float* out = P.p_part + (int64_t)blockIdx.x * P.p_stride;
    const int kp = L.kpad;
    proj_pblock(Ls, Ts, Kp + 4, kp, pn.nrows, out, true, threadIdx.x, blockDim.x);
}

size_t proj_bf16_smem(int kpad) {
    const int Kp = (kpad + 15) & ~15;
    const size_t stage = (size_t)128 * 64 * 2 + 2 * (size_t)Kp * 64 * 2;
    const size_t epi = (size_t)2 * 128 * (Kp + 4) * 4;
    return PJ_STAGES * stage > epi ? PJ_STAGES * stage : epi;
}

// Load one 128 x 64 block of the gradient panel (8 chunks of 8 elements per
// thread) into registers as fp32, plus the decayed parameter's squares.
struct GChunk { float v[8]; };

__device__ __forceinline__ void load_gblock(const void* g, const void* pp, int dt, int64_t base,
                                            int64_t ld, int nrows, int ncols, int c0, float wdm,
                                            bool vec, GChunk* out, float& psq) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const int ch = threadIdx.x + q * 128;       // 1024 chunks: 128 rows x 8 chunks
        const int r = ch >> 3, cc = (ch & 7) * 8;
        const int64_t off = base + (int64_t)r * ld + c0 + cc;
        float gx[8], px[8];
        if (r < nrows && vec && c0 + cc + 8 <= ncols) {
            if (dt == SCAO_F32) {
                const float4 a = *(const float4*)((const float*)g + off);
                const float4 b = *(const float4*)((const float*)g + off + 4);
                const float4 c = *(const float4*)((const float*)pp + off);
                const float4 d = *(const float4*)((const float*)pp + off + 4);
                gx[0] = a.x; gx[1] = a.y; gx[2] = a.z; gx[3] = a.w;
                gx[4] = b.x; gx[5] = b.y; gx[6] = b.z; gx[7] = b.w;
                px[0] = c.x; px[1] = c.y; px[2] = c.z; px[3] = c.w;
                px[4] = d.x; px[5] = d.y; px[6] = d.z; px[7] = d.w;
            } else {
                const float4 a = load4_dt(g, off, dt), b = load4_dt(g, off + 4, dt);
                const float4 c = load4_dt(pp, off, dt), d = load4_dt(pp, off + 4, dt);
                gx[0] = a.x; gx[1] = a.y; gx[2] = a.z; gx[3] = a.w;
                gx[4] = b.x; gx[5] = b.y; gx[6] = b.z; gx[7] = b.w;
                px[0] = c.x; px[1] = c.y; px[2] = c.z; px[3] = c.w;
                px[4] = d.x; px[5] = d.y; px[6] = d.z; px[7] = d.w;
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const float pd = round_dt(fmul(px[t], wdm), dt);
                psq = fmaf(pd, pd, psq);
            }
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                gx[t] = 0.f;
                if (r < nrows && c0 + cc + t < ncols) {
                    gx[t] = load_dt(g, off + t, dt);
                    const float pd = round_dt(fmul(load_dt(pp, off + t, dt), wdm), dt);
                    psq = fmaf(pd, pd, psq);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) out[q].v[t] = gx[t];
    }
}

// T = G_panel (128 x b) * U_r (b x Kp) on the tensor core (2-stage pipeline:
// registers hold the next gradient block while the MMA consumes the current
// one; U_r^T blocks arrive by TMA bulk copy), then P_part = U_l[rows]^T T
// with FFMA, and sum p_dec^2 over the panel.
__global__ void __launch_bounds__(128)
proj_tc_kernel(ScaoPlanDev P, int* err) {
    const ScaoPanel pn = P.panels[blockIdx.x];
    const ScaoLeaf& L = P.leaves[pn.leaf];
    const ScaoParamStep& S = P.step[L.param];
    if (S.phase != 2) return;
    const ScaoParam& pr = P.params[L.param];
    if (proj_fast(L, S, pr)) return;         // handled by proj_bf16_kernel / proj_tma_kernel
    const int dt = pr.dtype;
    const int Kp = (L.kpad + 15) & ~15;
    constexpr int KB = 64;
    const int gparts = dt == SCAO_BF16 ? 1 : 2;
    extern __shared__ __align__(1024) unsigned char smx[];
    const uint32_t abytes = TC_T * KB * 2, bbytes = Kp * KB * 2;
    const uint32_t sbytes = 2 * abytes + 2 * bbytes;   // [A hi][A lo][B hi][B lo]
    __shared__ uint64_t mbar_b[2], mbar_m[2];
    __shared__ uint32_t tslot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const void* g = (const void*)S.g_ptr;
    const void* pp = (const void*)S.p_ptr;
    const float* Ul = P.u + L.ul_off;
    uint32_t ncols = 32;
    while ((int)ncols < Kp) ncols <<= 1;
    if (warp == 0) tc_alloc(&tslot, ncols);
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) { mbar_init(&mbar_b[i], 1); mbar_init(&mbar_m[i], 1); }
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    const uint32_t idesc = idesc_bf16(TC_T, Kp);
    const float wdm = S.wd_mult;
    const int64_t base = (int64_t)(L.row0 + pn.row0) * L.ld + L.col0;
    const bool vec = ((L.ld & 7) == 0) && ((L.col0 & 7) == 0) && ((S.g_ptr & 15) == 0) &&
                     ((S.p_ptr & 15) == 0);
    float psq = 0.f;
    const int nkb = (L.b + KB - 1) / KB;
    bool ok = true;
    GChunk cur[8];
    load_gblock(g, pp, dt, base, L.ld, pn.nrows, L.b, 0, wdm, vec, cur, psq);
    for (int kb = 0; kb < nkb; ++kb) {
        const int buf = kb & 1;
        unsigned char* st = smx + buf * sbytes;
        if (kb >= 2) ok = mbar_wait(&mbar_m[buf], ((kb - 2) >> 1) & 1) && ok;
        if (tid == 0) {
            mbar_expect_tx(&mbar_b[buf], 2 * bbytes);
            bulk_g2s(st + 2 * abytes, P.ut + L.ut_off + (int64_t)kb * 2 * bbytes, 2 * bbytes,
                     &mbar_b[buf]);
        }
        // registers -> canonical A tile(s): one 16-byte core-matrix row per chunk
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int ch = tid + q * 128;
            const int r = ch >> 3, cc = (ch & 7) * 8;
            const uint32_t o = canon_off(r, cc, KB);
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                uint16_t h0, l0, h1, l1;
                if (gparts == 1) {
                    h0 = f_to_bf16_bits(cur[q].v[2 * t]); h1 = f_to_bf16_bits(cur[q].v[2 * t + 1]);
                    l0 = l1 = 0;
                } else {
                    split_bf16(cur[q].v[2 * t], h0, l0);
                    split_bf16(cur[q].v[2 * t + 1], h1, l1);
                }
                hw[t] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                lw[t] = (uint32_t)l0 | ((uint32_t)l1 << 16);
            }
            *(uint4*)(st + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            if (gparts == 2) *(uint4*)(st + abytes + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        if (kb + 1 < nkb)
            load_gblock(g, pp, dt, base, L.ld, pn.nrows, L.b, (kb + 1) * KB, wdm, vec, cur, psq);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            ok = mbar_wait(&mbar_b[buf], (kb >> 1) & 1) && ok;
            const uint32_t sa = smem_u32(st), sbh = sa + 2 * abytes, sbl = sbh + bbytes;
            for (int s = 0; s < KB / 16; ++s) {
                const uint64_t a0 = smem_desc(sa + s * 256, 128, 16 * KB);
                const uint64_t dh = smem_desc(sbh + s * 256, 128, 16 * KB);
                const uint64_t dl = smem_desc(sbl + s * 256, 128, 16 * KB);
                tc_mma_bf16(tmem, a0, dh, idesc, (kb > 0 || s > 0));
                tc_mma_bf16(tmem, a0, dl, idesc, 1);
                if (gparts == 2) {
                    const uint64_t a1 = smem_desc(sa + abytes + s * 256, 128, 16 * KB);
                    tc_mma_bf16(tmem, a1, dh, idesc, 1);
                }
            }
            tc_commit(&mbar_m[buf]);
        }
    }
    const int lastbuf = (nkb - 1) & 1;
    ok = mbar_wait(&mbar_m[lastbuf], ((nkb - 1) >> 1) & 1) && ok;
    if (!ok && err) atomicExch(err, 1);
    tc_fence_after();
    __syncthreads();
    float* Ts = (float*)smx;                  // 128 x (Kp+1)
    float* Ls = Ts + TC_T * (Kp + 4);         // 128 x (Kp+1)
    if (ok) {
        const int r = warp * 32 + lane;
        for (int c0 = 0; c0 < Kp; c0 += 16) {
            float v[16];
            tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
            for (int c = 0; c < 16; ++c) Ts[r * (Kp + 4) + c0 + c] = v[c];
        }
    }
    stage_ls(Ls, Ul, pn.row0, pn.nrows, L.sl, L.kpad, Kp);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, ncols);
    float* out = P.p_part + (int64_t)blockIdx.x * P.p_stride;
    const int kp = L.kpad;
    proj_pblock(Ls, Ts, Kp + 4, kp, pn.nrows, out, ok, threadIdx.x, blockDim.x);
    (void)psq;
}

size_t apply_tc_smem(int kpad) {
    const int Kp = (kpad + 15) & ~15;
    const size_t st = (size_t)4 * TC_T * Kp * 2, cs = (size_t)TC_T * (TC_T + 4) * 4;
    return st > cs ? st : cs;
}
size_t proj_tc_smem(int kpad) {
    const int Kp = (kpad + 15) & ~15;
    const size_t stage = (size_t)2 * 128 * 64 * 2 + 2 * (size_t)Kp * 64 * 2;
    const size_t epi = (size_t)2 * 128 * (Kp + 4) * 4;
    return 2 * stage > epi ? 2 * stage : epi;
}

}  // namespace

extern "C" int scao_plan_step(const ScaoPlanDev* P, void* stream) {
    if (!P || P->kpad_max > 128 || P->kpad_max < 0) return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    // the gradient filter also folds the global grad-norm EMA (its R2 form
    // reads it before the moments are updated)
    {
        const int rc = scao_filter_run(P, st);
        if (rc != SCAO_OK) return rc;
    }
    const bool fn = P->filt.mode != 0 || P->filt.noise_on != 0 || P->filt.gsnr_on != 0;
    if (P->n_panels > 0) {
        static PerDeviceOnce pattr;
        if (pattr.first()) {
            cudaFuncSetAttribute(proj_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)proj_tc_smem(128));
            cudaFuncSetAttribute(apply_kron_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)apply_tc_smem(128));
            cudaFuncSetAttribute(apply_kron_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)apply_tc_smem(128));
            cudaFuncSetAttribute(apply_kron_tc_kernel<true>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
            cudaFuncSetAttribute(proj_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)proj_bf16_smem(128));
            // full shared-memory carveout so several CTAs fit per SM
            cudaFuncSetAttribute(proj_bf16_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
            cudaFuncSetAttribute(proj_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
            cudaFuncSetAttribute(apply_kron_tc_kernel<false>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        }
        if (P->tmaps_ok) {
            static PerDeviceOnce tattr;
            if (tattr.first()) {
                cudaFuncSetAttribute(proj_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)proj_tma_smem(128));
            }
            const int g = scao_persistent_grid(P, P->n_panels);
            ProfScope _ps(SLOT_PROJ, st);
            proj_tma_kernel<<<g, PT_THREADS, proj_tma_smem(P->kpad_max), st>>>(*P, P->err);
        }
        SCAO_CHECK_LAUNCH();
        { ProfScope _ps(SLOT_PROJ, st);
          if (!P->tmaps_ok || P->proj_fallback)
              proj_bf16_kernel<<<P->n_panels, 128, proj_bf16_smem(P->kpad_max), st>>>(*P, P->err);
          // fp32 / fp16 leaves, and bf16 leaves whose rows are not 16-byte
          // aligned (both outside the TMA / cp.async paths)
          if ((P->kron_dtypes & ~(1 << SCAO_BF16)) || !P->tmaps_ok || P->proj_fallback)
              proj_tc_kernel<<<P->n_panels, 128, proj_tc_smem(P->kpad_max), st>>>(*P, P->err); }
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_chunks > 0) {
        if (P->n_diag > 0) { ProfScope _ps(SLOT_DIAG_PRE, st); diag_pre_kernel<<<P->n_diag, NT, 0, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_leaves > 0) {
        const int kp = P->kpad_max;
        const size_t sm = (size_t)(kp * kp + 4 * kp) * 4;
        static PerDeviceOnce attr;
        if (attr.first()) {
            cudaFuncSetAttribute(leaf_coef_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (128 * 128 + 4 * 128) * 4);
        }
        { ProfScope _ps(SLOT_LEAF_COEF, st); leaf_coef_kernel<<<P->n_leaves, NT, sm, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
        {
            const size_t smw = (size_t)(kp * ((kp + 15) & ~15) + TC_T * (((kp + 15) & ~15) + 4)) * 4;
            static PerDeviceOnce wattr;
            if (wattr.first()) {
                cudaFuncSetAttribute(leaf_w_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)((128 * 128 + 128 * 132) * 4));
            }
            ProfScope _ps(SLOT_LEAF_COEF, st);
            leaf_w_kernel<<<dim3(P->max_leaf_rows_tiles, P->n_leaves), 256, smw, st>>>(*P);
        }
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_strips > 0) {
        { ProfScope _ps(SLOT_DIAG_PRE, st); strip_pre_kernel<<<P->n_strips, NT, 0, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    { ProfScope _ps(SLOT_PARAM_PRE, st); param_pre_kernel<<<P->n_params, NT, 0, st>>>(*P); }
    SCAO_CHECK_LAUNCH();
    if (P->n_tiles > 0) {
        { ProfScope _ps(SLOT_APPLY_KRON, st);
          static PerDeviceOnce aattr;
          if (aattr.first()) {
              // the largest launch size over kpad_max
              size_t m0 = 0, m1 = 0;
              for (int k = 16; k <= 128; k += 16) {
                  m0 = apply_tma_smem(k, false) > m0 ? apply_tma_smem(k, false) : m0;
                  m1 = apply_tma_smem(k, true) > m1 ? apply_tma_smem(k, true) : m1;
              }
              cudaFuncSetAttribute(apply_tma_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m0);
              cudaFuncSetAttribute(apply_tma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m1);
          }
          const int g = scao_persistent_grid(P, P->n_tiles);
          if (P->tmaps_ok) {
              if (fn) apply_tma_kernel<true><<<g, AT_THREADS, apply_tma_smem(P->kpad_max, true), st>>>(*P, P->err);
              else apply_tma_kernel<false><<<g, AT_THREADS, apply_tma_smem(P->kpad_max, false), st>>>(*P, P->err);
          }
          if (!P->tmaps_ok || P->apply_fallback) {
              if (fn) apply_kron_tc_kernel<true><<<P->n_tiles, SCAO_APPLY_NT, apply_tc_smem(P->kpad_max), st>>>(*P, P->err);
              else apply_kron_tc_kernel<false><<<P->n_tiles, SCAO_APPLY_NT, apply_tc_smem(P->kpad_max), st>>>(*P, P->err);
          } }
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_chunks > 0) {
        if (P->n_flat > 0) {
            ProfScope _ps(SLOT_APPLY_FLAT, st);
            if (fn) apply_flat_kernel<true><<<P->n_flat, NT, 0, st>>>(*P);
            else apply_flat_kernel<false><<<P->n_flat, NT, 0, st>>>(*P);
        }
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_strips > 0) {
        { ProfScope _ps(SLOT_APPLY_FLAT, st);
          if (fn) strip_apply_kernel<true><<<P->n_strips, NT, 0, st>>>(*P);
          else strip_apply_kernel<false><<<P->n_strips, NT, 0, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    { ProfScope _ps(SLOT_PARAM_POST, st); param_post_kernel<<<P->n_params, NT, 0, st>>>(*P); }
    SCAO_CHECK_LAUNCH();
    if (P->filt.mode == 0 && !P->gnorm_host) {
        { ProfScope _ps(SLOT_GLOBAL_NORM, st); global_norm_kernel<<<1, 256, 0, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_chunks > 0) {
        if (P->n_p > 0) {
            ProfScope _ps(SLOT_APPLY_P, st);
            if (P->la_fused) apply_p_kernel<true><<<P->n_p, NT, 0, st>>>(*P);
            else apply_p_kernel<false><<<P->n_p, NT, 0, st>>>(*P);
        }
        SCAO_CHECK_LAUNCH();
    }
    return SCAO_OK;
}

namespace {

// sum of raw grad^2 per flat chunk (slot 3 of chunk_part)
__global__ void __launch_bounds__(NT)
grad_sq_kernel(ScaoPlanDev P) {
    const ScaoChunk ch = P.chunks[blockIdx.x];
    const ScaoParamStep& S = P.step[ch.param];
    if (S.phase == 0) return;
    const ScaoParam& pr = P.params[ch.param];
    __shared__ float red[32];
    const void* g = (const void*)S.g_ptr;
    const int dt = pr.dtype;
    float s = 0.f;
    const bool vec = ((S.g_ptr & 15) == 0) && ((ch.begin & 3) == 0);
    int64_t vend = ch.begin;
    if (vec) {
        const int64_t n4 = (ch.end - ch.begin) >> 2;
        vend = ch.begin + n4 * 4;
        for (int64_t q = threadIdx.x; q < n4; q += NT) {
            const float4 v = load4_dt(g, ch.begin + q * 4, dt);
            s = fmaf(v.x, v.x, s); s = fmaf(v.y, v.y, s);
            s = fmaf(v.z, v.z, s); s = fmaf(v.w, v.w, s);
        }
    }
    for (int64_t e = vend + threadIdx.x; e < ch.end; e += NT) {
        const float v = load_dt(g, e, dt);
        s = fmaf(v, v, s);
    }
    s = block_sum(s, red);
    if (threadIdx.x == 0) P.chunk_part[blockIdx.x * 4 + 3] = s;
}

__global__ void __launch_bounds__(NT)
grad_norm_param_kernel(ScaoPlanDev P, float* out) {
    const int pi = blockIdx.x;
    const ScaoParam& pr = P.params[pi];
    __shared__ float red[32];
    if (P.step[pi].phase == 0) {
        if (threadIdx.x == 0) out[pi] = 0.f;
        return;
    }
    float s = 0.f;
    for (int c = pr.chunk_begin + threadIdx.x; c < pr.chunk_end; c += NT) s += P.chunk_part[c * 4 + 3];
    s = block_sum(s, red);
    // float32 norm (of p.grad.float(), optimizer.py:531-532); the host rounds
    // it to the gradient's dtype where the reference does (the average, :440)
    if (threadIdx.x == 0) out[pi] = sqrtf(s);
}

}  // namespace

extern "C" int scao_plan_grad_norms(const ScaoPlanDev* P, float* out, void* stream) {
    if (!P || !out) return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    if (P->n_chunks > 0) {
        { ProfScope _ps(SLOT_GLOBAL_NORM, st); grad_sq_kernel<<<P->n_chunks, NT, 0, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    { ProfScope _ps(SLOT_GLOBAL_NORM, st); grad_norm_param_kernel<<<P->n_params, NT, 0, st>>>(*P, out); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}

extern "C" int scao_plan_lookahead(const ScaoPlanDev* P, float alpha, int init,
                                   void* stream) {
    if (!P) return SCAO_ERR_ARG;
    if (P->n_chunks == 0) return SCAO_OK;
    { ProfScope _ps(SLOT_LOOKAHEAD, (cudaStream_t)stream); lookahead_kernel<<<P->n_chunks, NT, 0, (cudaStream_t)stream>>>(*P, alpha, init); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}

extern "C" int scao_plan_prep_factors(const ScaoPlanDev* P, const int32_t* leaf_ids, int n_ids,
                                      void* stream) {
    if (!P || n_ids < 0) return SCAO_ERR_ARG;
    if (n_ids == 0) return SCAO_OK;
    cudaStream_t st = (cudaStream_t)stream;
    { ProfScope _ps(SLOT_EIG_RANK, st); prep_factors_kernel<<<dim3(16, n_ids), 256, 0, st>>>(*P, leaf_ids); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}
