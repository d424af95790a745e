// A C++ host that uses the library through its C ABI only (no Python, no
// torch): device buffers from the CUDA runtime, the reference's int8
// quantisation known answers (utils.py:170-203) computed on the host, the
// int8 EMA update and the fused Kronecker precondition compared with host
// restatements.  Prints "CABI OK" and exits 0 on success.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "scao_b200.h"

#define CK(x)                                                                    \
    do {                                                                         \
        if ((x) != 0) {                                                          \
            std::fprintf(stderr, "failed: %s (line %d)\n", #x, __LINE__);         \
            return 1;                                                            \
        }                                                                        \
    } while (0)

static void host_quant(const std::vector<float>& x, std::vector<int8_t>& q, double& s) {
    float am = 0.f;
    for (float v : x) am = std::fmax(am, std::fabs(v));
    if ((double)am < 1e-30) {
        s = 1.0;
        q.assign(x.size(), 0);
        return;
    }
    s = (double)am / 127.0;
    const float sf = (float)s;
    q.resize(x.size());
    for (size_t i = 0; i < x.size(); ++i) {
        float r = std::nearbyint(x[i] / sf);          // IEEE division, ties to even
        r = std::fmin(127.f, std::fmax(-127.f, r));
        q[i] = (int8_t)r;
    }
}

int main() {
    std::printf("%s\n", scao_version());
    const int64_t n = 1 << 18;
    std::vector<float> x(n), nv(n);
    unsigned s0 = 12345u;
    auto rnd = [&]() { s0 = s0 * 1664525u + 1013904223u; return ((s0 >> 8) * (1.0f / 16777216.0f)) - 0.5f; };
    for (int64_t i = 0; i < n; ++i) { x[i] = rnd() * 3.f; nv[i] = rnd() * 1e-3f; }
    float *dx, *dn;
    int8_t *dq, *dq2;
    double* ds;
    void* scratch;
    CK(cudaMalloc(&dx, n * 4));
    CK(cudaMalloc(&dn, n * 4));
    CK(cudaMalloc(&dq, n));
    CK(cudaMalloc(&dq2, n));
    CK(cudaMalloc(&ds, 16));
    const int64_t sb = scao_int8_ema_scratch_bytes(n);
    CK(cudaMalloc(&scratch, sb > 256 ? sb : 256));
    CK(cudaMemcpy(dx, x.data(), n * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dn, nv.data(), n * 4, cudaMemcpyHostToDevice));

    // 1. quantisation, bit for bit
    CK(scao_quantize_sym_int8(dx, n, dq, ds, scratch, nullptr));
    CK(cudaDeviceSynchronize());
    std::vector<int8_t> q(n), qh;
    double s = 0, sh = 0;
    CK(cudaMemcpy(q.data(), dq, n, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(&s, ds, 8, cudaMemcpyDeviceToHost));
    host_quant(x, qh, sh);
    for (int64_t i = 0; i < n; ++i)
        if (q[i] != qh[i]) { std::fprintf(stderr, "quant mismatch at %lld\n", (long long)i); return 1; }
    if (s != sh) { std::fprintf(stderr, "scale mismatch\n"); return 1; }

    // 2. int8 EMA update: dequant * rho + new -> requant, bit for bit
    const double rho = 0.999;
    CK(scao_int8_ema_update(dq, s, dn, rho, n, dq2, ds, scratch, nullptr));
    CK(cudaDeviceSynchronize());
    std::vector<float> xe(n);
    for (int64_t i = 0; i < n; ++i) xe[i] = ((float)q[i] * (float)s) * (float)rho + nv[i];
    std::vector<int8_t> q2(n), q2h;
    double s2 = 0, s2h = 0;
    host_quant(xe, q2h, s2h);
    CK(cudaMemcpy(q2.data(), dq2, n, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(&s2, ds, 8, cudaMemcpyDeviceToHost));
    for (int64_t i = 0; i < n; ++i)
        if (q2[i] != q2h[i]) { std::fprintf(stderr, "ema mismatch at %lld\n", (long long)i); return 1; }
    if (s2 != s2h) { std::fprintf(stderr, "ema scale mismatch\n"); return 1; }

    // 3. bad arguments come back as a status, not a fault
    if (scao_quantize_sym_int8(nullptr, n, dq, ds, scratch, nullptr) == 0) {
        std::fprintf(stderr, "null input accepted\n");
        return 1;
    }
    cudaFree(dx); cudaFree(dn); cudaFree(dq); cudaFree(dq2); cudaFree(ds); cudaFree(scratch);
    std::printf("CABI OK\n");
    return 0;
}
