// The every-step optimizer pass (scao/optimizer.py:521-645) for all
// parameters at once, plus the Kronecker precondition
// (scao/preconditioner.py:457-521, fallback formula scao/cuda/__init__.py:95-99)
// and the curvature clip (optimizer.py:667-678, preconditioner.py:527-564).
//
// Kernel sequence of one step (scao_plan_step):
//   proj       P_panel = U_l[rows]^T (G[rows] U_r)      per 64-row panel
//              + sum p_dec^2 per panel (LARS, optimizer.py:373)
//   diag_pre   natural-norm^2 and p_dec^2 of diagonal-mode params
//   leaf_coef  P = sum of panels; nat^2; Delta = (s_l s_r^T - 1) o P;
//              W = U_l Delta                            per leaf
//   param_pre  clip factor tau / nat  per param
//   apply_kron per 64x64 tile: corr = W U_r^T, g_prec = round(G + corr),
//              clip, blend, Adan moments, update u (rounded to param dtype)
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

namespace {

constexpr int NT = 256;
constexpr int TT = 64;       // apply tile edge
constexpr int CH = 4096;     // flat chunk length (elements), 16 per thread

enum { PS_CLIPMUL = 0, PS_CLIP, PS_PNORM2, PS_UNORM2, PS_GNORM2, PS_ALPHA, PS_NAT, PS_TRUST };

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// S^(-1/4) and S^(-1/2) with the clamp of utils.py:113 / preconditioner.py:558
__device__ __forceinline__ float s_inv4(float s) { return powf(fmaxf(s, 1e-8f), -0.25f); }
__device__ __forceinline__ float s_inv2(float s) { return powf(fmaxf(s, 1e-8f), -0.5f); }

// ---------------------------------------------------------------------------
// projection: T = G_panel * U_r (rows x kpad), P_part = U_l[rows]^T T
// ---------------------------------------------------------------------------
template <int KP>
__global__ void __launch_bounds__(NT)
proj_kernel(ScaoPlanDev P) {
    const ScaoPanel pn = P.panels[blockIdx.x];
    const ScaoLeaf& L = P.leaves[pn.leaf];
    const ScaoParamStep& S = P.step[L.param];
    if (S.phase != 2) return;
    const ScaoParam& pr = P.params[L.param];
    const int dt = pr.dtype;
    const void* g = (const void*)S.g_ptr;
    const void* pp = (const void*)S.p_ptr;
    const int kp = L.kpad;
    const float* Ul = P.u + L.ul_off;
    const float* Ur = P.u + L.ur_off;
    constexpr int TKK = 16;
    constexpr int CPT = KP / 16;         // columns per thread
    extern __shared__ float psm[];
    float (*Gs)[TT + 4] = (float (*)[TT + 4])psm;                  // [TKK][TT+4]
    float (*Us)[KP + 4] = (float (*)[KP + 4])(psm + TKK * (TT + 4)); // [TKK][KP+4]
    float (*Ts)[KP + 4] = Us + TKK;                                 // [TT][KP+4]
    float (*Ls)[KP + 4] = Ts + TT;                                  // [TT][KP+4]
    __shared__ float red[32];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    float acc[4][CPT] = {};
    float psq = 0.f;
    const float wdm = S.wd_mult;
    for (int c0 = 0; c0 < L.b; c0 += TKK) {
        for (int e = tid; e < TT * TKK; e += NT) {
            const int r = e >> 4, c = e & 15;
            float v = 0.f;
            if (r < pn.nrows && c0 + c < L.b) {
                const int64_t off = (int64_t)(L.row0 + pn.row0 + r) * L.ld + L.col0 + c0 + c;
                v = load_dt(g, off, dt);
                const float pd = round_dt(fmul(load_dt(pp, off, dt), wdm), dt);
                psq = fmaf(pd, pd, psq);
            }
            Gs[c][r] = v;
        }
        for (int e = tid; e < TKK * KP; e += NT) {
            const int c = e / KP, b = e % KP;
            Us[c][b] = (c0 + c < L.b && b < kp) ? Ur[(int64_t)(c0 + c) * L.sr + b] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int c = 0; c < TKK; ++c) {
            float4 a = *(const float4*)&Gs[c][ty * 4];
            float av[4] = {a.x, a.y, a.z, a.w};
            float bv[CPT];
#pragma unroll
            for (int q = 0; q < CPT; q += 4) {
                float4 b = *(const float4*)&Us[c][tx * CPT + q];
                bv[q] = b.x; bv[q + 1] = b.y; bv[q + 2] = b.z; bv[q + 3] = b.w;
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < CPT; ++q) acc[r][q] = fmaf(av[r], bv[q], acc[r][q]);
        }
        __syncthreads();
    }
    // second stage: P_part[a][b] = sum_r U_l[row0+r][a] * T[r][b]
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < CPT; ++q) Ts[ty * 4 + r][tx * CPT + q] = acc[r][q];
    for (int e = tid; e < TT * KP; e += NT) {
        const int r = e / KP, a = e % KP;
        Ls[r][a] = (r < pn.nrows && a < kp) ? Ul[(int64_t)(pn.row0 + r) * L.sl + a] : 0.f;
    }
    __syncthreads();
    float* out = P.p_part + (int64_t)blockIdx.x * P.p_stride;
    for (int e = tid; e < kp * kp; e += NT) {
        const int a = e / kp, b = e % kp;
        float s = 0.f;
        for (int r = 0; r < pn.nrows; ++r) s = fmaf(Ls[r][a], Ts[r][b], s);
        out[e] = s;
    }
    psq = block_sum(psq, red);
    if (tid == 0) out[P.p_stride - 4] = psq;
}

// ---------------------------------------------------------------------------
// diagonal-mode Phase-2 params: natural-norm^2 and p_dec^2 per chunk
// (preconditioner.py:554-556; optimizer.py:373)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
diag_pre_kernel(ScaoPlanDev P) {
    const ScaoChunk ch = P.chunks[blockIdx.x];
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
        P.chunk_part[blockIdx.x * 4 + 2] = nat;
        P.chunk_part[blockIdx.x * 4 + 3] = psq;
    }
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
    // W = U_l * Delta  (a x kp), only the first k columns of U_l contribute
    const float* Ul = P.u + L.ul_off;
    float* W = P.w + L.w_off;
    for (int64_t e = threadIdx.x; e < (int64_t)L.a * kp; e += NT) {
        const int i = (int)(e / kp), b = (int)(e % kp);
        float s = 0.f;
        const float* urow = Ul + (int64_t)i * L.sl;
        for (int a = 0; a < k; ++a) s = fmaf(urow[a], D[a * kp + b], s);
        W[e] = s;
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
            const ScaoLeaf& L = P.leaves[l];
            for (int q = L.panel_begin; q < L.panel_end; ++q)
                psq += P.p_part[(int64_t)q * P.p_stride + P.p_stride - 4];
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
        ps[PS_PNORM2] = psq;
        ps[PS_NAT] = nat;
    }
}

// Adan moments + update for one element (optimizer.py:608-633).
struct AdanOut { float u; };
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
    const float num = fadd(fdiv(m, S.bc1), fmul(S.c3, fdiv(d, S.bc3)));
    const float den = fadd(sqrtf(fdiv(v, S.bc2)), S.eps);
    return fdiv(num, den);
}

// ---------------------------------------------------------------------------
// Kronecker Phase-2 tiles
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
apply_kron_kernel(ScaoPlanDev P) {
    const ScaoTile tl = P.tiles[blockIdx.x];
    const ScaoLeaf& L = P.leaves[tl.leaf];
    const ScaoParamStep& S = P.step[L.param];
    if (S.phase != 2) return;
    const ScaoParam& pr = P.params[L.param];
    const int dt = pr.dtype;
    const int kp = L.kpad;
    extern __shared__ float sm[];
    float* Ws = sm;                       // kp x (TT+4): Ws[b][i]
    float* Us = Ws + kp * (TT + 4);       // kp x (TT+4): Us[b][j]
    __shared__ float red[32];
    const float* W = P.w + L.w_off;
    const float* Ur = P.u + L.ur_off;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    for (int e = tid; e < TT * kp; e += NT) {
        const int r = e / kp, b = e % kp;
        const int i = tl.row0 + r, j = tl.col0 + r;
        Ws[b * (TT + 4) + r] = i < L.a ? W[(int64_t)i * kp + b] : 0.f;
        Us[b * (TT + 4) + r] = j < L.b ? Ur[(int64_t)j * L.sr + b] : 0.f;
    }
    __syncthreads();
    float acc[4][4] = {};
    for (int b = 0; b < kp; ++b) {
        const float4 a = *(const float4*)&Ws[b * (TT + 4) + ty * 4];
        const float4 u = *(const float4*)&Us[b * (TT + 4) + tx * 4];
        const float av[4] = {a.x, a.y, a.z, a.w}, uv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(av[r], uv[c], acc[r][c]);
    }
    const float* ps = P.param_scalars + L.param * 8;
    const bool clip = ps[PS_CLIP] != 0.f;
    const float clipmul = ps[PS_CLIPMUL];
    const void* g = (const void*)S.g_ptr;
    float* M = P.exp_avg + pr.offset;
    float* V = P.exp_avg_sq + pr.offset;
    float* Dd = P.exp_avg_diff + pr.offset;
    float* Pv = P.prev_grad + pr.offset;
    float usq = 0.f, gsq = 0.f;
    const bool vec = ((L.ld & 3) == 0) && ((L.col0 & 3) == 0) &&
                     ((S.g_ptr & 15) == 0) && ((pr.offset & 3) == 0);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int i = tl.row0 + ty * 4 + r;
        const int j0 = tl.col0 + tx * 4;
        if (i >= L.a) continue;
        const int64_t off = (int64_t)(L.row0 + i) * L.ld + L.col0 + j0;
        if (vec && j0 + 3 < L.b) {
            const float4 gg = load4_dt(g, off, dt);
            float4 m4 = ldg_stream4(M + off), v4 = ldg_stream4(V + off);
            float4 d4 = ldg_stream4(Dd + off), p4 = ldg_stream4(Pv + off);
            float gv[4] = {gg.x, gg.y, gg.z, gg.w};
            float mv[4] = {m4.x, m4.y, m4.z, m4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w};
            float dv[4] = {d4.x, d4.y, d4.z, d4.w}, pv[4] = {p4.x, p4.y, p4.z, p4.w};
            float uo[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float gp = round_dt(fadd(gv[c], acc[r][c]), dt);
                const float u = adan_elem(S, dt, gv[c], gp, mv[c], vv[c], dv[c], pv[c], clip, clipmul);
                usq = fmaf(u, u, usq);
                gsq = fmaf(gv[c], gv[c], gsq);
                uo[c] = round_dt(u, dt);
            }
            stg_stream4(M + off, make_float4(mv[0], mv[1], mv[2], mv[3]));
            stg_stream4(V + off, make_float4(vv[0], vv[1], vv[2], vv[3]));
            stg_stream4(Dd + off, make_float4(dv[0], dv[1], dv[2], dv[3]));
            stg_stream4(Pv + off, make_float4(pv[0], pv[1], pv[2], pv[3]));
            if (dt == SCAO_F32) store4_dt(P.upd32 + pr.offset, off, dt, make_float4(uo[0], uo[1], uo[2], uo[3]));
            else store4_dt(P.upd + pr.offset, off, dt, make_float4(uo[0], uo[1], uo[2], uo[3]));
        } else {
            for (int c = 0; c < 4; ++c) {
                const int j = j0 + c;
                if (j >= L.b) break;
                const int64_t o = off + c;
                const float gv = load_dt(g, o, dt);
                float mv = M[o], vv = V[o], dv = Dd[o], pv = Pv[o];
                const float gp = round_dt(fadd(gv, acc[r][c]), dt);
                const float u = adan_elem(S, dt, gv, gp, mv, vv, dv, pv, clip, clipmul);
                usq = fmaf(u, u, usq);
                gsq = fmaf(gv, gv, gsq);
                M[o] = mv; V[o] = vv; Dd[o] = dv; Pv[o] = pv;
                if (dt == SCAO_F32) P.upd32[pr.offset + o] = u;
                else store_dt(P.upd + pr.offset, o, dt, u);
            }
        }
    }
    usq = block_sum(usq, red);
    gsq = block_sum(gsq, red);
    if (tid == 0) {
        P.tile_part[blockIdx.x * 4 + 0] = usq;
        P.tile_part[blockIdx.x * 4 + 1] = gsq;
    }
}

// ---------------------------------------------------------------------------
// flat chunks: Phase-1 Adam (optimizer.py:561-578) and Phase-2 diagonal
// params (preconditioner.py:506-510 + the Adan step)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT)
apply_flat_kernel(ScaoPlanDev P) {
    const ScaoChunk ch = P.chunks[blockIdx.x];
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
    if (phase == 1) {
        const float a1 = round_dt((float)S.alpha1, dt);
        for (int64_t e = ch.begin + threadIdx.x; e < ch.end; e += NT) {
            const float gv = load_dt(g, e, dt);
            const float pd = round_dt(fmul(load_dt(pp, e, dt), S.wd_mult), dt);
            float m = fmaf(gv, S.c1, fmul(M[e], S.beta1));
            float v = fmaf(fmul(S.c2, gv), gv, fmul(V[e], S.beta2));
            const float den = fadd(fdiv(sqrtf(v), S.sqrt_bc2), S.eps);
            const float u = round_dt(fdiv(m, den), dt);
            store_dt(pp, e, dt, round_dt(fmaf(a1, u, pd), dt));
            M[e] = m; V[e] = v; Pv[e] = gv;
            gsq = fmaf(gv, gv, gsq);
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
            const float u = adan_elem(S, dt, gv, gp, m, v, d, pv, clip, clipmul);
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
        P.chunk_part[blockIdx.x * 4 + 0] = usq;
        P.chunk_part[blockIdx.x * 4 + 1] = gsq;
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
    float usq = 0.f, gsq = 0.f;
    const bool kron2 = (S.phase == 2 && pr.mode == 1);
    if (kron2) {
        for (int t = pr.tile_begin + threadIdx.x; t < pr.tile_end; t += NT) {
            usq += P.tile_part[t * 4 + 0];
            gsq += P.tile_part[t * 4 + 1];
        }
    } else {
        for (int c = pr.chunk_begin + threadIdx.x; c < pr.chunk_end; c += NT) {
            usq += P.chunk_part[c * 4 + 0];
            gsq += P.chunk_part[c * 4 + 1];
        }
    }
    usq = block_sum(usq, red);
    gsq = block_sum(gsq, red);
    if (threadIdx.x != 0) return;
    float* ps = P.param_scalars + pi * 8;
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

// global grad-norm EMA (optimizer.py:439-446): mean of fp32 per-param norms
__global__ void global_norm_kernel(ScaoPlanDev P) {
    __shared__ double red[32];
    double s = 0.0, c = 0.0;
    for (int pi = threadIdx.x; pi < P.n_params; pi += blockDim.x) {
        if (P.step[pi].phase == 0) continue;
        s += (double)sqrtf(P.param_scalars[pi * 8 + PS_GNORM2]);
        c += 1.0;
    }
    s = warp_sum_d(s);
    c = warp_sum_d(c);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { red[wid] = s; red[16 + wid] = c; }
    __syncthreads();
    if (threadIdx.x == 0) {
        double ts = 0.0, tc = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { ts += red[w]; tc += red[16 + w]; }
        if (tc > 0.0) *P.global_norm_ema = 0.95 * (*P.global_norm_ema) + 0.05 * (ts / tc);
    }
}

// Phase-2 parameter write: p = round(round(p*(1-lr wd)) + alpha*u)
__global__ void __launch_bounds__(NT)
apply_p_kernel(ScaoPlanDev P) {
    const ScaoChunk ch = P.chunks[blockIdx.x];
    const ScaoParam& pr = P.params[ch.param];
    const ScaoParamStep& S = P.step[ch.param];
    if (S.phase != 2) return;
    const int dt = pr.dtype;
    void* pp = (void*)S.p_ptr;
    const float alpha = P.param_scalars[ch.param * 8 + PS_ALPHA];
    const float wdm = S.wd_mult;
    const bool vec = ((S.p_ptr & 15) == 0) && ((pr.offset & 3) == 0) && ((ch.begin & 3) == 0);
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
    const int dt = pr.dtype;
    void* pp = (void*)S.p_ptr;
    void* sl = dt == SCAO_F32 ? (void*)(P.slow32 + pr.offset) : (void*)(P.slow + pr.offset);
    for (int64_t e = ch.begin + threadIdx.x; e < ch.end; e += NT) {
        const float p = load_dt(pp, e, dt);
        float s = init ? p : load_dt(sl, e, dt);
        const float diff = round_dt(fsub(p, s), dt);
        s = round_dt(fadd(s, round_dt(fmul(alpha, diff), dt)), dt);
        store_dt(sl, e, dt, s);
        store_dt(pp, e, dt, s);
    }
}

size_t proj_smem(int kp) {
    return (size_t)(16 * (TT + 4) + (16 + 2 * TT) * (kp + 4)) * 4;
}

}  // namespace

extern "C" int scao_plan_step(const ScaoPlanDev* P, void* stream) {
    if (!P || P->kpad_max > 128 || P->kpad_max < 0) return SCAO_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    if (P->n_panels > 0) {
        static bool pattr = false;
        if (!pattr) {
            cudaFuncSetAttribute(proj_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)proj_smem(128));
            pattr = true;
        }
        ProfScope _ps(SLOT_PROJ, st);
        if (P->kpad_max <= 64) proj_kernel<64><<<P->n_panels, NT, proj_smem(64), st>>>(*P);
        else proj_kernel<128><<<P->n_panels, NT, proj_smem(128), st>>>(*P);
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_chunks > 0) {
        { ProfScope _ps(SLOT_DIAG_PRE, st); diag_pre_kernel<<<P->n_chunks, NT, 0, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_leaves > 0) {
        const int kp = P->kpad_max;
        const size_t sm = (size_t)(kp * kp + 4 * kp) * 4;
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(leaf_coef_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (128 * 128 + 4 * 128) * 4);
            cudaFuncSetAttribute(apply_kron_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 2 * 128 * (TT + 4) * 4);
            attr = true;
        }
        { ProfScope _ps(SLOT_LEAF_COEF, st); leaf_coef_kernel<<<P->n_leaves, NT, sm, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    { ProfScope _ps(SLOT_PARAM_PRE, st); param_pre_kernel<<<P->n_params, NT, 0, st>>>(*P); }
    SCAO_CHECK_LAUNCH();
    if (P->n_tiles > 0) {
        const size_t sm = (size_t)2 * P->kpad_max * (TT + 4) * 4;
        { ProfScope _ps(SLOT_APPLY_KRON, st); apply_kron_kernel<<<P->n_tiles, NT, sm, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    if (P->n_chunks > 0) {
        { ProfScope _ps(SLOT_APPLY_FLAT, st); apply_flat_kernel<<<P->n_chunks, NT, 0, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
    { ProfScope _ps(SLOT_PARAM_POST, st); param_post_kernel<<<P->n_params, NT, 0, st>>>(*P); }
    SCAO_CHECK_LAUNCH();
    { ProfScope _ps(SLOT_GLOBAL_NORM, st); global_norm_kernel<<<1, 512, 0, st>>>(*P); }
    SCAO_CHECK_LAUNCH();
    if (P->n_chunks > 0) {
        { ProfScope _ps(SLOT_APPLY_P, st); apply_p_kernel<<<P->n_chunks, NT, 0, st>>>(*P); }
        SCAO_CHECK_LAUNCH();
    }
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
