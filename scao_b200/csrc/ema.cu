// Batched Kronecker curvature EMA (scao/preconditioner.py:341-353):
//   L <- rho * L + (1 - rho) * G G^T      (a x a, K = b)
//   R <- rho * R + (1 - rho) * G^T G      (b x b, K = a)
// for every active leaf block G (a view into the parameter's gradient), with
// the int8 storage of utils.py:170-203 fused: the GEMM epilogue dequantises the
// old code, forms the new fp32 value with the reference's separate roundings
// (x = fl(fl(fl(q*s)*rho) + fl(alpha*gram))), reduces max|x| per factor, and a
// second pass requantises with IEEE division (bit-exact with the CPU path for
// identical fp32 x).
//
// Only the lower triangle of tiles is computed; the epilogue mirrors it.
// This file holds the portable SIMT-FMA tile kernel; see gram_tc.cu for the
// tcgen05 tensor-core path used for 16-bit gradients.
#include <stdlib.h>

#include "common.cuh"
#include "prof.cuh"
#include "tc.cuh"
#include "tmap.cuh"

namespace {

constexpr int TM = 64;     // output tile edge
constexpr int TK = 16;     // K chunk
constexpr int NT = 256;    // threads

struct Prob {
    const void* g;     // param gradient base
    int dt;            // gradient dtype
    int n, K;          // output n x n, reduction K
    int side;          // 0: G G^T, 1: G^T G
    int64_t row0, col0, ld;
    int64_t fac_off;   // into fac arena
    float* x;          // fp32 scratch n*n (int8 mode)
    float* am_new;     // new absmax slot
    int pid;           // problem id (2*leaf+side)
};

__device__ Prob get_prob(const ScaoPlanDev& P, const int32_t* ids, int j,
                         float* xbuf, int64_t xstride, float* amnew) {
    Prob p;
    const int leaf = ids[j >> 1];
    const int side = j & 1;
    const ScaoLeaf& L = P.leaves[leaf];
    const ScaoParamStep& S = P.step[L.param];
    p.g = (const void*)S.g_ptr;
    p.dt = P.params[L.param].dtype;
    p.side = side;
    p.n = side ? L.b : L.a;
    p.K = side ? L.a : L.b;
    p.row0 = L.row0;
    p.col0 = L.col0;
    p.ld = L.ld;
    p.fac_off = side ? L.rq_off : L.lq_off;
    p.x = xbuf + (int64_t)j * xstride;
    p.am_new = amnew + j;
    p.pid = 2 * leaf + side;
    return p;
}

// A(i, k) of the factor product: side 0 -> G[i][k], side 1 -> G[k][i]
__device__ __forceinline__ float load_a(const Prob& p, int i, int k) {
    if (i >= p.n || k >= p.K) return 0.f;
    int64_t r = p.side ? k : i, c = p.side ? i : k;
    return load_dt(p.g, (p.row0 + r) * p.ld + p.col0 + c, p.dt);
}

// ---------------------------------------------------------------------------
// Tensor-core gram + EMA for bf16 gradients (tcgen05, fp32 accumulators in
// TMEM).  One CTA per lower-triangle 128 x 128 output tile; the gradient is
// streamed by cp.async in 64-deep K blocks (3 stages).  L = G G^T reads
// gradient rows (K-major operands); R = G^T G reads gradient columns, which
// are contiguous along the output index, so both operands use the MN-major
// layout and no transpose is needed.
// ---------------------------------------------------------------------------
constexpr int GT = 128, GKB = 64, GSTAGES = 3;

__device__ __forceinline__ bool gram_tc_ok(const Prob& p, const ScaoLeaf& L) {
    return p.dt == SCAO_BF16 && (L.ld % 8) == 0 && (L.col0 % 8) == 0 && (L.a % 8) == 0 &&
           (L.b % 8) == 0 && ((reinterpret_cast<uintptr_t>(p.g) & 15) == 0);
}

// TMA path (gram_tma_kernel): whole 64-deep K blocks, 16-byte aligned rows
__host__ __device__ inline bool gram_tma_ok(const ScaoLeaf& L, int side, int dt) {
    const int K = side ? L.a : L.b;
    return dt == SCAO_BF16 && (K % 64) == 0 && (L.a % 64) == 0 && (L.b % 64) == 0 &&
           (L.ld % 8) == 0 && (L.col0 % 8) == 0;
}

// the TMA kernel takes a factor problem when the block fits it and the
// parameter's gradient has a tensor map this call
__host__ __device__ inline bool gram_tma_use(const ScaoParam* params, const ScaoParamStep* step,
                                             const ScaoLeaf& L, int side) {
    return gram_tma_ok(L, side, params[L.param].dtype) &&
           scao_tmap_ok(params[L.param], step[L.param]);
}

__global__ void __launch_bounds__(256, 2)
gram_ema_tc_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, float* xbuf, int64_t xstride,
                   float* amnew, float rho_f, float alpha_f, int* err, int tma_on) {
    const Prob p = get_prob(P, ids, blockIdx.y, xbuf, xstride, amnew);
    const ScaoLeaf& L = P.leaves[ids[blockIdx.y >> 1]];
    if (!gram_tc_ok(p, L)) return;
    if (tma_on && gram_tma_use(P.params, P.step, L, p.side)) return;     // gram_tma_kernel
    const int nt = (p.n + GT - 1) / GT;
    const int t = blockIdx.x;
    if (t >= nt * (nt + 1) / 2) return;
    int ti = 0;
    while ((ti + 1) * (ti + 2) / 2 <= t) ++ti;
    const int tj = t - ti * (ti + 1) / 2;
    const int i0 = ti * GT, j0 = tj * GT;
    const bool diag = ti == tj;
    extern __shared__ __align__(1024) unsigned char smx[];
    constexpr uint32_t OPB = GT * GKB * 2;          // one operand block, 16 KB
    constexpr uint32_t SB = 2 * OPB;
    __shared__ uint64_t mbar_m[GSTAGES];
    __shared__ uint32_t tslot;
    __shared__ float red[32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint16_t* g = (const uint16_t*)p.g;
    const int mn = p.side;    // R = G^T G uses MN-major operands
    if (warp == 0) tc_alloc(&tslot, GT);
    if (tid == 0) {
        for (int i = 0; i < GSTAGES; ++i) mbar_init(&mbar_m[i], 1);
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    const uint32_t idesc = idesc_bf16(GT, GT, mn, mn);
    const int nkb = (p.K + GKB - 1) / GKB;
    auto issue = [&](int kb) {
        unsigned char* st = smx + (kb % GSTAGES) * SB;
        const int k0 = kb * GKB;
#pragma unroll
        for (int q = 0; q < 8; ++q) {           // 2 operands x 1024 chunks / 256 threads
            const int cq = tid + q * 256;
            const int ch = cq & 1023;
            const int opnd = cq >> 10;
            const int base = opnd ? j0 : i0;
            int r, k;                           // output index r (< 128), depth k (< 64)
            if (!mn) { r = ch >> 3; k = (ch & 7) * 8; } else { k = ch >> 4; r = (ch & 15) * 8; }
            const bool in = (base + r < p.n) && (k0 + k < p.K);
            int64_t off = 0;
            if (in) off = mn ? (p.row0 + k0 + k) * p.ld + p.col0 + base + r
                             : (p.row0 + base + r) * p.ld + p.col0 + k0 + k;
            const uint32_t o = mn ? canon_off_mn(r, k, GT) : canon_off(r, k, GKB);
            const uint32_t dst = smem_u32(st + opnd * OPB + o);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                         :: "r"(dst), "l"(g + off), "r"(in ? 16 : 0) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int kb = 0; kb < GSTAGES - 1; ++kb) {
        if (kb < nkb) issue(kb);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
        const int nxt = kb + GSTAGES - 1;
        if (nxt < nkb) {
            if (nxt >= GSTAGES)
                ok = mbar_wait(&mbar_m[nxt % GSTAGES], ((nxt - GSTAGES) / GSTAGES) & 1) && ok;
            issue(nxt);
        } else {
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        asm volatile("cp.async.wait_group %0;" :: "n"(GSTAGES - 1) : "memory");
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint32_t sa = smem_u32(smx + (kb % GSTAGES) * SB), sb = sa + OPB;
            for (int s = 0; s < GKB / 16; ++s) {
                uint64_t ad, bd;
                if (mn) {
                    ad = smem_desc(sa + s * 2 * 16 * GT, 16 * GT, 128);
                    bd = smem_desc(sb + s * 2 * 16 * GT, 16 * GT, 128);
                } else {
                    ad = smem_desc(sa + s * 256, 128, 16 * GKB);
                    bd = smem_desc(sb + s * 256, 128, 16 * GKB);
                }
                tc_mma_bf16(tmem, ad, bd, idesc, (kb > 0 || s > 0));
            }
            tc_commit(&mbar_m[kb % GSTAGES]);
        }
    }
    ok = mbar_wait(&mbar_m[(nkb - 1) % GSTAGES], ((nkb - 1) / GSTAGES) & 1) && ok;
    if (!ok && err) atomicExch(err, 1);
    tc_fence_after();
    __syncthreads();
    // TMEM (lane i, column j) -> Cs[i][j]
    constexpr int CLD = GT + 1;
    float* Cs = (float*)smx;
    {
        const int qd = warp & 3, hf = warp >> 2;
        const int r = qd * 32 + lane;
        for (int c0 = hf * 64; c0 < hf * 64 + 64; c0 += 16) {
            float v[16];
            tc_ld16(tmem + ((uint32_t)(qd * 32) << 16) + c0, v);
#pragma unroll
            for (int c = 0; c < 16; ++c) Cs[r * CLD + c0 + c] = ok ? v[c] : 0.f;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, GT);
    // EMA epilogue with the reference's separate roundings; rows i, lanes j
    const int n = p.n;
    float mx = 0.f;
    const int jj = tid & 127;
    const int j = j0 + jj;
    const int rlo = (tid >> 7) * 64, rhi = rlo + 64;   // this thread's row half
    if (P.int8_ema) {
        const int8_t* q = (const int8_t*)P.fac + p.fac_off;
        const float s_old = quant_scale_f(P.absmax[p.pid]);
        for (int ib = rlo; ib < rhi; ib += 16) {
            // 16 independent old-code loads in flight, then the arithmetic
            int8_t qv[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int i = i0 + ib + c;
                qv[c] = (i < n && j < n) ? q[(int64_t)i * n + j] : (int8_t)0;
            }
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int ii = ib + c, i = i0 + ii;
                float x = 0.f;
                if (i < n && j < n && (!diag || ii >= jj)) {
                    const float deq = __fmul_rn((float)qv[c], s_old);
                    x = __fadd_rn(__fmul_rn(deq, rho_f), __fmul_rn(alpha_f, Cs[ii * CLD + jj]));
                    p.x[(int64_t)i * n + j] = x;
                    mx = fmaxf(mx, fabsf(x));
                }
                Cs[ii * CLD + jj] = x;
            }
        }
    } else {
        float* Lm = (float*)P.fac + p.fac_off;
        for (int ii = rlo; ii < rhi; ++ii) {
            const int i = i0 + ii;
            if (i >= n || j >= n) continue;
            float x = 0.f;
            if (!diag || ii >= jj)
                x = __fadd_rn(__fmul_rn(Lm[(int64_t)i * n + j], rho_f),
                              __fmul_rn(alpha_f, Cs[ii * CLD + jj]));
            Cs[ii * CLD + jj] = x;
        }
        __syncthreads();    // every old value read before any write
        for (int ii = rlo; ii < rhi; ++ii) {
            const int i = i0 + ii;
            if (i < n && j < n && (!diag || ii >= jj)) Lm[(int64_t)i * n + j] = Cs[ii * CLD + jj];
        }
    }
    __syncthreads();
    // mirror: element (j, i) = x(i, j) for the strict lower part
    {
        float* dst = P.int8_ema ? p.x : (float*)P.fac + p.fac_off;
        const int ii = tid & 127;
        const int i = i0 + ii;
        for (int jr = rlo; jr < rhi; ++jr) {
            const int jm = j0 + jr;
            if (i >= n || jm >= n) continue;
            if (diag && ii <= jr) continue;
            dst[(int64_t)jm * n + i] = Cs[ii * CLD + jr];
        }
    }
    if (P.int8_ema) {
        mx = block_max(mx, red);
        if (tid == 0) atomic_max_nonneg(p.am_new, mx);
    }
}

size_t gram_tc_smem() {
    const size_t st = (size_t)GSTAGES * 2 * GT * GKB * 2, cs = (size_t)GT * (GT + 1) * 4;
    return st > cs ? st : cs;
}

// ---------------------------------------------------------------------------
// Persistent, warp-specialised tensor-core gram + EMA on SM pairs (bf16
// gradients whose leaf block allows whole 64-deep K blocks).  The grid is made
// of clusters of 2 CTAs (one CTA per SM); a cluster computes 256 x 256 output
// tiles of the lower triangle with tcgen05.mma.cta_group::2 (M = 256): each CTA
// holds its 128 rows of A and 128 of the 256 columns of B in its own shared
// memory and its 128 accumulator rows in its own TMEM, so per SM the operand
// traffic of a 128 x 256 tile is A + B/2 instead of A + B (the 1-SM tile was
// bound by shared-memory bandwidth).  Operands arrive by TMA tensor copies
// (cp.async.bulk.tensor, 128-byte swizzle, no multicast) from one 2-D tensor
// map per parameter gradient; each CTA copies its own halves and the copies
// complete on the pair leader's barrier.  Roles per CTA (320 threads):
//   warp 0      TMA producer over a GST-stage ring (both CTAs)
//   warp 1      TMEM owner (both); MMA issuer (leader, one thread)
//   warps 2-9   epilogue: own TMEM rows -> dequant*rho + alpha*gram -> staging
// The epilogue of tile t overlaps the main loop of tile t+1 (two TMEM
// accumulators).  L = G G^T uses K-major operands (gradient rows); R = G^T G
// uses MN-major operands (gradient columns) -- no transpose.  Every wait is
// bounded; on a timeout the CTA records an error, stops issuing, and both CTAs
// still meet at the final cluster barrier.
// ---------------------------------------------------------------------------
constexpr int GN = 256;                 // output tile: 256 rows x GN columns per pair
constexpr int GST = 6;                  // pipeline stages
constexpr uint32_t GOPB = 128 * 64 * 2; // one 128 x 64 operand block, 16 KB
constexpr uint32_t GSTAGE = 2 * GOPB;   // per CTA: A half + B half
constexpr int GEPI = 256;                // epilogue threads (8 warps)
constexpr int GTHREADS = 64 + GEPI;
constexpr int GTRI = GT * GT;           // floats per staged 128 x 128 sub-tile

// work tiles of one factor problem: row block ti2 (256 rows), column block tc
// (256 columns) for every tc <= ti2 (lower triangle)
__host__ __device__ inline int gram_work_tiles(int n) {
    const int nt2 = (n + 255) / 256;
    return nt2 * (nt2 + 1) / 2;
}

struct GTile {
    int j, leaf, side, n, K, ti2, tc, param;
    int64_t row0, col0;
};

// decode work item T of the persistent loop; false when it is padding
__device__ __forceinline__ bool gram_tile(const ScaoPlanDev& P, const int32_t* ids, int tpp,
                                          int T, GTile& w) {
    w.j = T / tpp;
    int t = T - w.j * tpp;
    w.leaf = ids[w.j >> 1];
    w.side = w.j & 1;
    const ScaoLeaf& L = P.leaves[w.leaf];
    w.param = L.param;
    if (!gram_tma_use(P.params, P.step, L, w.side)) return false;
    w.n = w.side ? L.b : L.a;
    w.K = w.side ? L.a : L.b;
    const int nt2 = (w.n + 255) / 256;
    int ti2 = 0;
    for (; ti2 < nt2; ++ti2) {
        if (t < ti2 + 1) break;
        t -= ti2 + 1;
    }
    if (ti2 >= nt2) return false;
    w.ti2 = ti2;
    w.tc = t;
    w.row0 = L.row0;
    w.col0 = L.col0;
    return true;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GTHREADS, 1)
gram_tma_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, int nprob, int tpp,
                float* xbuf, int64_t xstride, float* amnew, float rho_f, float alpha_f, int* err) {
    extern __shared__ unsigned char gsm_raw[];
    unsigned char* gsm = (unsigned char*)(((uintptr_t)gsm_raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t full[GST], empty[GST], accf[2], acce[2], fin;
    __shared__ uint32_t tslot;
    __shared__ volatile int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    if (tid == 0) {
        // the leader's full barrier counts both CTAs' producers; its acce
        // counts both CTAs' epilogue warps
        for (int i = 0; i < GST; ++i) { mbar_init(&full[i], 2); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&accf[i], 1); mbar_init(&acce[i], 2 * (GEPI / 32)); }
        mbar_init(&fin, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tc_alloc_pair(&tslot, 2 * GN);
    tc_fence_before();
    cluster_sync_all();        // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem = tslot;
    const int total = nprob * tpp;
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    const unsigned char* maps = P.tmaps;
    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            int stage = 0;
            uint32_t ph = 0, issued = 0, last_ph = 0;
            GTile w;
            for (int T = cid; T < total && !abort_flag; T += ncl) {
                if (!gram_tile(P, ids, tpp, T, w)) continue;
                const void* map = scao_tmap(maps, w.param, w.side ? TM_G64 : TM_G128);
                // this CTA's 128 rows of A and 128 columns of B
                const int i0 = w.ti2 * 256 + 128 * (int)rank, j0 = w.tc * GN + 128 * (int)rank;
                const int x0 = (int)w.col0, y0 = (int)w.row0;
                for (int kb = 0; kb < w.K / 64; ++kb) {
                    if (!mbar_wait(&empty[stage], ph ^ 1)) { abort_flag = 1; atomicExch(err, 2); break; }
                    const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
                    mbar_arrive_expect_tx_cl(fb, GSTAGE);
                    const uint32_t a = smem_u32(gsm + (size_t)stage * GSTAGE), b = a + GOPB;
                    const int k0 = kb * 64;
                    if (w.side == 0) {
                        // K-major: x = K (gradient column), y = output index (row)
                        tma_load_2d_pair(a, map, x0 + k0, y0 + i0, fb);
                        tma_load_2d_pair(b, map, x0 + k0, y0 + j0, fb);
                    } else {
                        // MN-major: x = output index (gradient column), y = K (row)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            tma_load_2d_pair(a + h * (GOPB / 2), map, x0 + i0 + 64 * h, y0 + k0, fb);
                            tma_load_2d_pair(b + h * (GOPB / 2), map, x0 + j0 + 64 * h, y0 + k0, fb);
                        }
                    }
                    issued |= 1u << stage;
                    last_ph = (last_ph & ~(1u << stage)) | (ph << stage);
                    if (++stage == GST) { stage = 0; ph ^= 1; }
                }
            }
            // the leader waits until no copy of either CTA is still landing
            // (both CTAs' copies complete on the leader's barriers)
            if (leader)
                for (int s2 = 0; s2 < GST; ++s2)
                    if ((issued >> s2) & 1u)
                        if (!mbar_wait(&full[s2], (last_ph >> s2) & 1u)) atomicExch(err, 2);
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer (leader) ----------------
            int stage = 0, acc = 0;
            uint32_t ph = 0, aph = 0;
            GTile w;
            for (int T = cid; T < total && !abort_flag; T += ncl) {
                if (!gram_tile(P, ids, tpp, T, w)) continue;
                if (!mbar_wait(&acce[acc], aph ^ 1)) { abort_flag = 1; atomicExch(err, 2); break; }
                tc_fence_after();
                const uint32_t d = tmem + acc * GN;
                const uint32_t idesc = idesc_bf16(256, GN, w.side, w.side);
                bool ok = true;
                for (int kb = 0; kb < w.K / 64; ++kb) {
                    if (!mbar_wait(&full[stage], ph)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a = smem_u32(gsm + (size_t)stage * GSTAGE), b = a + GOPB;
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        uint64_t ad, bd;
                        if (w.side == 0) {          // K-major: 16 K = 32 bytes along the row
                            ad = smem_desc_sw128(a + s * 32, 16, 1024);
                            bd = smem_desc_sw128(b + s * 32, 16, 1024);
                        } else {                    // MN-major: 16 K rows = 2 x 1024 bytes
                            ad = smem_desc_sw128(a + s * 2048, GOPB / 2, 1024);
                            bd = smem_desc_sw128(b + s * 2048, GOPB / 2, 1024);
                        }
                        tc_mma_bf16_pair(d, ad, bd, idesc, (kb > 0 || s > 0) ? 1u : 0u);
                    }
                    tc_commit_pair(&empty[stage], 0x3);
                    if (++stage == GST) { stage = 0; ph ^= 1; }
                }
                if (!ok) { abort_flag = 1; atomicExch(err, 2); break; }
                tc_commit_pair(&accf[acc], 0x3);
                acc ^= 1;
                if (acc == 0) aph ^= 1;
            }
            // every issued MMA has completed before either CTA releases TMEM
            tc_commit_pair(&fin, 0x3);
        }
        __syncwarp();
        if (!mbar_wait(&fin, 0)) atomicExch(err, 2);
    } else {
        // ---------------- epilogue (warps 2..9, both CTAs) ----------------
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const int h = (warp - 2) >> 2;          // column half of the tile
        const int r = q * 32 + lane;            // row within this CTA's 128 rows
        const uint32_t acce_cl[2] = {mapa_shared(smem_u32(&acce[0]), 0),
                                     mapa_shared(smem_u32(&acce[1]), 0)};
        int acc = 0;
        uint32_t aph = 0;
        GTile w;
        for (int T = cid; T < total; T += ncl) {
            if (__any_sync(0xffffffffu, abort_flag)) break;
            if (!gram_tile(P, ids, tpp, T, w)) continue;
            // warp-uniform: the TMEM loads below are warp-collective
            if (!__all_sync(0xffffffffu, mbar_wait(&accf[acc], aph))) {
                abort_flag = 1;
                atomicExch(err, 2);
                break;
            }
            tc_fence_after();
            const int n = w.n;
            const int ti = 2 * w.ti2 + (int)rank;           // 128-row block of this CTA
            const int i0 = ti * 128, j0 = w.tc * GN + h * (GN / 2);
            const int i = i0 + r;
            const int pid = 2 * w.leaf + w.side;
            const ScaoLeaf& L = P.leaves[w.leaf];
            const int64_t fo = w.side ? L.rq_off : L.lq_off;
            float mx = 0.f;
            const uint32_t tbase = tmem + acc * GN + h * (GN / 2) + ((uint32_t)(q * 32) << 16);
            int cend = min(GN / 2, n - j0);
            // columns above the diagonal sub-tile are not needed
            cend = min(cend, ((ti + 1) << 7) - j0);
            if (P.int8_ema) {
                const int8_t* qo = (const int8_t*)P.fac + fo;
                const float s_old = quant_scale_f(P.absmax[pid]);
                // all old codes of this thread's row segment in flight at once
                int4 q4[GN / 32];
#pragma unroll
                for (int u = 0; u < GN / 32; ++u)
                    q4[u] = (i < n && u * 16 < cend) ? *(const int4*)(qo + (int64_t)i * n + j0 + u * 16)
                                                    : make_int4(0, 0, 0, 0);
#pragma unroll
                for (int u = 0; u < GN / 32; ++u) {
                    const int c0 = u * 16;
                    if (c0 >= cend) break;
                    const int tj = (j0 + c0) >> 7;          // 128-sub-tile of these columns
                    const bool diag = tj == ti;
                    float v[16];
                    tc_ld16(tbase + c0, v);
                    const int8_t* qv = (const int8_t*)&q4[u];
                    float xo[16];
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const int jc = j0 + c0 + c;
                        float x = 0.f;
                        if (i < n && (!diag || jc <= i)) {
                            const float deq = __fmul_rn((float)qv[c], s_old);
                            x = __fadd_rn(__fmul_rn(deq, rho_f), __fmul_rn(alpha_f, v[c]));
                            mx = fmaxf(mx, fabsf(x));
                        }
                        xo[c] = x;
                    }
                    float* xt = xbuf + (int64_t)w.j * xstride +
                                (int64_t)(ti * (ti + 1) / 2 + tj) * GTRI + r * GT + ((j0 + c0) & 127);
#pragma unroll
                    for (int c = 0; c < 16; c += 4)
                        __stcs((float4*)(xt + c), make_float4(xo[c], xo[c + 1], xo[c + 2], xo[c + 3]));
                }
            } else {
                float* Lm = (float*)P.fac + fo;
                for (int c0 = 0; c0 < cend; c0 += 16) {
                    float v[16];
                    tc_ld16(tbase + c0, v);
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const int jc = j0 + c0 + c;
                        if (i < n && jc <= i) {
                            const int64_t o = (int64_t)i * n + jc;
                            const float x = __fadd_rn(__fmul_rn(Lm[o], rho_f), __fmul_rn(alpha_f, v[c]));
                            Lm[o] = x;
                            if (jc != i) Lm[(int64_t)jc * n + i] = x;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cl(acce_cl[acc]);   // the leader's accumulator is free
            acc ^= 1;
            if (acc == 0) aph ^= 1;
            if (P.int8_ema) {
                mx = warp_max(mx);
                if (lane == 0) atomic_max_nonneg(amnew + w.j, mx);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    // neither CTA leaves while the other may still touch its barriers
    cluster_sync_all();
    tc_fence_after();
    if (warp == 1) tc_dealloc_pair(tmem, 2 * GN);
}

size_t gram_tma_smem() { return (size_t)GST * GSTAGE + 1024; }

// Requantise the tile-major staging of gram_tma_kernel (lower-triangle
// tiles only) into both triangles of the int8 factor (utils.py:170-189).
__global__ void __launch_bounds__(256)
requant_tile_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids, const float* __restrict__ xbuf,
                    int64_t xstride, const float* __restrict__ amnew) {
    const int j = blockIdx.y;
    const int leaf = ids[j >> 1], side = j & 1;
    const ScaoLeaf& L = P.leaves[leaf];
    if (!gram_tma_use(P.params, P.step, L, side)) return;
    const int n = side ? L.b : L.a;
    const int nt = (n + GT - 1) / GT;
    const int t = blockIdx.x;
    if (t >= nt * (nt + 1) / 2) return;
    int ti = 0;
    while ((ti + 1) * (ti + 2) / 2 <= t) ++ti;
    const int tj = t - ti * (ti + 1) / 2;
    const int i0 = ti * GT, j0 = tj * GT;
    const bool diag = ti == tj;
    const float am = amnew[j];
    const bool zero = (double)am < 1e-30;
    const float s = quant_scale_f(am);
    int8_t* qd = (int8_t*)P.fac + (side ? L.rq_off : L.lq_off);
    const float* x = xbuf + (int64_t)j * xstride + (int64_t)t * GTRI;
    __shared__ int8_t tq[GT][GT + 4];
    for (int e = threadIdx.x; e < GTRI / 4; e += 256) {
        const float4 v = __ldcs((const float4*)x + e);
        const int rr = (e * 4) / GT, cc = (e * 4) % GT;
        tq[rr][cc + 0] = quant_one(v.x, s, zero);
        tq[rr][cc + 1] = quant_one(v.y, s, zero);
        tq[rr][cc + 2] = quant_one(v.z, s, zero);
        tq[rr][cc + 3] = quant_one(v.w, s, zero);
    }
    __syncthreads();
    // rows i0+rr, columns j0..j0+127 (diagonal tile: upper part mirrored)
    for (int e = threadIdx.x; e < GT * GT / 4; e += 256) {
        const int rr = (e * 4) / GT, cc = (e * 4) % GT;
        if (i0 + rr >= n || j0 + cc >= n) continue;
        char4 o;
        if (!diag) {
            o = make_char4(tq[rr][cc], tq[rr][cc + 1], tq[rr][cc + 2], tq[rr][cc + 3]);
        } else {
            const int8_t a0 = cc + 0 <= rr ? tq[rr][cc + 0] : tq[cc + 0][rr];
            const int8_t a1 = cc + 1 <= rr ? tq[rr][cc + 1] : tq[cc + 1][rr];
            const int8_t a2 = cc + 2 <= rr ? tq[rr][cc + 2] : tq[cc + 2][rr];
            const int8_t a3 = cc + 3 <= rr ? tq[rr][cc + 3] : tq[cc + 3][rr];
            o = make_char4(a0, a1, a2, a3);
        }
        *(char4*)(qd + (int64_t)(i0 + rr) * n + j0 + cc) = o;
    }
    if (!diag) {
        // transposed copy: rows j0+cc, columns i0..i0+127
        for (int e = threadIdx.x; e < GT * GT / 4; e += 256) {
            const int cc = (e * 4) / GT, rr = (e * 4) % GT;
            if (j0 + cc >= n || i0 + rr >= n) continue;
            *(char4*)(qd + (int64_t)(j0 + cc) * n + i0 + rr) =
                make_char4(tq[rr][cc], tq[rr + 1][cc], tq[rr + 2][cc], tq[rr + 3][cc]);
        }
    }
    if (t == 0 && threadIdx.x == 0) P.absmax[2 * leaf + side] = am;
}

__global__ void __launch_bounds__(NT)
gram_ema_simt_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                     float* xbuf, int64_t xstride, float* amnew, float rho_f,
                     float alpha_f) {
    const Prob p = get_prob(P, ids, blockIdx.y, xbuf, xstride, amnew);
    if (gram_tc_ok(p, P.leaves[ids[blockIdx.y >> 1]])) return;   // tensor-core kernel
    const int nt = (p.n + TM - 1) / TM;
    int t = blockIdx.x;
    if (t >= nt * (nt + 1) / 2) return;
    int ti = 0;
    while ((ti + 1) * (ti + 2) / 2 <= t) ++ti;
    const int tj = t - ti * (ti + 1) / 2;
    const int i0 = ti * TM, j0 = tj * TM;

    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TM + 4];
    __shared__ float red[32];
    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    float acc[4][4] = {};

    for (int k0 = 0; k0 < p.K; k0 += TK) {
        // 64 x 16 elements per operand, 4 per thread
        for (int e = tid; e < TM * TK; e += NT) {
            int ii, kk;
            if (p.side == 0) { ii = e >> 4; kk = e & 15; }   // contiguous along k
            else { kk = e >> 6; ii = e & 63; }               // contiguous along i
            As[kk][ii] = load_a(p, i0 + ii, k0 + kk);
            Bs[kk][ii] = load_a(p, j0 + ii, k0 + kk);
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

    // epilogue: EMA with the reference's separate roundings
    float mx = 0.f;
    float xv[4][4];
    if (P.int8_ema) {
        const int8_t* q = (const int8_t*)P.fac + p.fac_off;
        const float s_old = quant_scale_f(P.absmax[p.pid]);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
                float x = 0.f;
                if (i < p.n && j < p.n) {
                    const float deq = __fmul_rn((float)q[(int64_t)i * p.n + j], s_old);
                    x = __fadd_rn(__fmul_rn(deq, rho_f), __fmul_rn(alpha_f, acc[r][c]));
                }
                xv[r][c] = x;
                mx = fmaxf(mx, fabsf(x));
            }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
                if (i < p.n && j < p.n) {
                    p.x[(int64_t)i * p.n + j] = xv[r][c];
                    p.x[(int64_t)j * p.n + i] = xv[r][c];
                }
            }
        mx = block_max(mx, red);
        if (tid == 0) atomic_max_nonneg(p.am_new, mx);
    } else {
        float* L = (float*)P.fac + p.fac_off;
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
                float x = 0.f;
                if (i < p.n && j < p.n)
                    x = __fadd_rn(__fmul_rn(L[(int64_t)i * p.n + j], rho_f),
                                  __fmul_rn(alpha_f, acc[r][c]));
                xv[r][c] = x;
            }
        __syncthreads();   // all old values read before any mirrored write
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int i = i0 + ty * 4 + r, j = j0 + tx * 4 + c;
                if (i < p.n && j < p.n) {
                    L[(int64_t)i * p.n + j] = xv[r][c];
                    L[(int64_t)j * p.n + i] = xv[r][c];
                }
            }
    }
}

__global__ void requant_batch_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                                     const float* __restrict__ xbuf, int64_t xstride,
                                     const float* __restrict__ amnew, int tma_on) {
    const int j = blockIdx.y;
    const int leaf = ids[j >> 1], side = j & 1;
    const ScaoLeaf& L = P.leaves[leaf];
    if (tma_on && gram_tma_use(P.params, P.step, L, side)) return;   // requant_tile_kernel
    const int n = side ? L.b : L.a;
    const int64_t nn = (int64_t)n * n;
    const float am = amnew[j];
    const bool zero = (double)am < 1e-30;
    const float s = quant_scale_f(am);
    int8_t* q = (int8_t*)P.fac + (side ? L.rq_off : L.lq_off);
    const float* x = xbuf + (int64_t)j * xstride;
    const int64_t n4 = nn >> 2;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n4;
         e += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = __ldcs((const float4*)x + e);
        char4 o;
        o.x = quant_one(v.x, s, zero); o.y = quant_one(v.y, s, zero);
        o.z = quant_one(v.z, s, zero); o.w = quant_one(v.w, s, zero);
        ((char4*)q)[e] = o;
    }
    for (int64_t e = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nn;
         e += (int64_t)gridDim.x * blockDim.x)
        q[e] = quant_one(x[e], s, zero);
    if (blockIdx.x == 0 && threadIdx.x == 0) P.absmax[2 * leaf + side] = am;
}

// Diagonal curvature (preconditioner.py:332-339):
//   diag_ema <- diag_ema * rho + (1 - rho) * g^2   (separately rounded)
__global__ void diag_ema_kernel(ScaoPlanDev P, const int32_t* __restrict__ ids,
                                float rho_f, float alpha_f) {
    const int pi = ids[blockIdx.y];
    const ScaoParam& pr = P.params[pi];
    const ScaoParamStep& S = P.step[pi];
    const void* g = (const void*)S.g_ptr;
    float* d = P.diag_ema + pr.offset;
    if (pr.mode == 1) {
        // a Kronecker param: only its diagonal strips (width-1 blocks)
        for (int s = 0; s < P.n_strips; ++s) {
            const ScaoStrip sp = P.strips[s];
            if (sp.param != pi) continue;
            for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < sp.count;
                 j += gridDim.x * blockDim.x) {
                const int64_t e = sp.begin + (int64_t)j * sp.stride;
                const float gv = load_dt(g, e, pr.dtype);
                d[e] = __fadd_rn(__fmul_rn(d[e], rho_f), __fmul_rn(alpha_f, __fmul_rn(gv, gv)));
            }
        }
        return;
    }
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < pr.numel;
         e += (int64_t)gridDim.x * blockDim.x) {
        const float gv = load_dt(g, e, pr.dtype);
        d[e] = __fadd_rn(__fmul_rn(d[e], rho_f), __fmul_rn(alpha_f, __fmul_rn(gv, gv)));
    }
}

}  // namespace

namespace {

int64_t ntri_tiles(int64_t n) {
    const int64_t nt = (n + GT - 1) / GT;
    return nt * (nt + 1) / 2;
}

// floats of fp32 staging per factor problem: the full n x n square (SIMT
// and cp.async kernels) or the lower-triangle tiles (TMA kernel)
int64_t xstride_floats(int64_t mx) {
    const int64_t a = mx * mx, b = ntri_tiles(mx) * GTRI;
    return ((a > b ? a : b) + 63) / 64 * 64;
}

}  // namespace

extern "C" int64_t scao_ema_scratch_bytes(int n_ids, int max_a, int max_b) {
    const int64_t mx = max_a > max_b ? max_a : max_b;
    return 2 * (int64_t)n_ids * (xstride_floats(mx) * 4 + 256) + 256 * 4;
}

extern "C" int scao_plan_curvature(const ScaoPlanDev* P, const int32_t* leaf_ids,
                                   int n_ids, int max_a, int max_b, double rho,
                                   void* scratch, int64_t scratch_bytes,
                                   const ScaoParam* params_host, const ScaoParamStep* step_host,
                                   const ScaoLeaf* leaves_host, const int32_t* leaf_ids_host,
                                   void* stream) {
    if (!P || n_ids < 0 || !scratch) return SCAO_ERR_ARG;
    if (n_ids == 0) return SCAO_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t mx = max_a > max_b ? max_a : max_b;
    const int64_t xstride = xstride_floats(mx);                   // floats
    const int64_t per_prob = xstride * 4 + 4;                    // bytes
    int64_t cap = (scratch_bytes - 1024) / per_prob;             // problems
    cap &= ~int64_t(1);
    if (cap < 2) return SCAO_ERR_ARG;
    const float rho_f = (float)rho;
    const float alpha_f = (float)(1.0 - rho);   // Python-float 1 - rho, then cast
    const int nt = (int)((mx + TM - 1) / TM);
    const int tiles = nt * (nt + 1) / 2;
    const int tpp = gram_work_tiles((int)mx);   // work tiles per problem (upper bound)
    // SCAO_NO_TMA=1 selects the cp.async kernel for every problem (the
    // tests compare both paths)
    const char* no_tma = getenv("SCAO_NO_TMA");
    const int tma_on = (params_host && step_host && !(no_tma && no_tma[0] == '1') &&
                        scao_build_tensor_maps(P, params_host, step_host, st)) ? 1 : 0;
    // with the host leaf table, the fallback kernels launch only when some
    // listed problem needs them
    bool fallback = true;
    if (tma_on && leaves_host && leaf_ids_host) {
        fallback = false;
        for (int k = 0; k < n_ids && !fallback; ++k) {
            const ScaoLeaf& L = leaves_host[leaf_ids_host[k]];
            if (!gram_tma_use(params_host, step_host, L, 0) || !gram_tma_use(params_host, step_host, L, 1))
                fallback = true;
        }
    }
    for (int64_t j0 = 0; j0 < 2 * (int64_t)n_ids; j0 += cap) {
        const int np = (int)((2 * (int64_t)n_ids - j0) < cap ? (2 * (int64_t)n_ids - j0) : cap);
        float* xbuf = (float*)scratch;
        float* amnew = (float*)((char*)scratch + cap * xstride * 4);
        if (P->int8_ema && cudaMemsetAsync(amnew, 0, np * sizeof(float), st) != cudaSuccess)
            return SCAO_ERR_LAUNCH;
        const int32_t* ids = leaf_ids + j0 / 2;
        dim3 grid(tiles, np);
        if (tma_on) {
            static PerDeviceOnce tattr;
            if (tattr.first()) {
                cudaFuncSetAttribute(gram_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)gram_tma_smem());
            }
            const int64_t work = (int64_t)np * tpp;
            // clusters of 2 CTAs: an even grid of at most one CTA per SM
            int g = scao_persistent_grid(P, 2 * work) & ~1;
            if (g < 2) g = 2;
            ProfScope _ps(SLOT_GRAM_TC, st);
            gram_tma_kernel<<<g, GTHREADS, gram_tma_smem(), st>>>(*P, ids, np, tpp, xbuf, xstride,
                                                                  amnew, rho_f, alpha_f, P->err);
        }
        SCAO_CHECK_LAUNCH();
        if (fallback) {
            static PerDeviceOnce attr;
            if (attr.first()) {
                cudaFuncSetAttribute(gram_ema_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)gram_tc_smem());
                cudaFuncSetAttribute(gram_ema_tc_kernel,
                                     cudaFuncAttributePreferredSharedMemoryCarveout, 100);
            }
            const int nt2 = (int)((mx + GT - 1) / GT);
            ProfScope _ps2(SLOT_GRAM_EMA, st);
            gram_ema_tc_kernel<<<dim3(nt2 * (nt2 + 1) / 2, np), 256, gram_tc_smem(), st>>>(
                *P, ids, xbuf, xstride, amnew, rho_f, alpha_f, P->err, tma_on);
        }
        SCAO_CHECK_LAUNCH();
        if (fallback) {
            ProfScope _ps(SLOT_GRAM_EMA, st);
            gram_ema_simt_kernel<<<grid, NT, 0, st>>>(*P, ids, xbuf, xstride, amnew, rho_f, alpha_f);
        }
        SCAO_CHECK_LAUNCH();
        if (P->int8_ema) {
            dim3 g2((int)((mx * mx + 255) / 256 < 64 ? (mx * mx + 255) / 256 : 64), np);
            if (fallback) {
                ProfScope _ps(SLOT_REQUANT, st);
                requant_batch_kernel<<<g2, 256, 0, st>>>(*P, ids, xbuf, xstride, amnew, tma_on);
            }
            SCAO_CHECK_LAUNCH();
            if (tma_on) {
                ProfScope _ps(SLOT_REQUANT, st);
                requant_tile_kernel<<<dim3((int)ntri_tiles(mx), np), 256, 0, st>>>(*P, ids, xbuf, xstride, amnew);
            }
            SCAO_CHECK_LAUNCH();
        }
    }
    return SCAO_OK;
}

extern "C" int scao_plan_curvature_diag(const ScaoPlanDev* P,
                                        const int32_t* param_ids, int n_ids,
                                        double rho, void* stream) {
    if (!P || n_ids < 0) return SCAO_ERR_ARG;
    if (n_ids == 0) return SCAO_OK;
    dim3 grid(32, n_ids);
    { ProfScope _ps(SLOT_DIAG_EMA, (cudaStream_t)stream); diag_ema_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        *P, param_ids, (float)rho, (float)(1.0 - rho)); }
    SCAO_CHECK_LAUNCH();
    return SCAO_OK;
}
