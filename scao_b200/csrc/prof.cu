#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "prof.cuh"

namespace {

const char* kNames[SLOT_COUNT] = {
    "proj", "diag_pre", "leaf_coef", "param_pre", "apply_kron", "apply_flat", "param_post",
    "global_norm", "apply_p", "lookahead", "gram_ema", "requant", "diag_ema", "eig_prep",
    "eig_diag", "eig_gemm", "eig_jacobi", "eig_residual", "eig_cholinv", "eig_rank", "quant",
    "seam", "gram_tc", "transpose", "filter", "eig_iter"};

std::atomic<int64_t> g_launches{0};
std::atomic<int> g_enabled{0};
thread_local int g_suspended = 0;
std::mutex g_mu;
struct Pending { int slot; cudaEvent_t a, b; int dev; };
std::vector<Pending> g_pending;
// finished events for reuse, by device (an event records only on streams of
// the device it was created on)
std::vector<cudaEvent_t> g_pool[64];
cudaEvent_t g_open[SLOT_COUNT];
double g_ms[SLOT_COUNT];
int64_t g_cnt[SLOT_COUNT];

int cur_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) d = 0;
    return d;
}

cudaEvent_t get_event() {
    std::vector<cudaEvent_t>& pool = g_pool[cur_device()];
    if (!pool.empty()) { cudaEvent_t e = pool.back(); pool.pop_back(); return e; }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
}

}  // namespace

void scao_prof_suspend(int on) { g_suspended = on; }

void scao_prof_add_launches(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void scao_prof_begin(int slot, cudaStream_t st) {
    if (g_suspended) return;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (!g_enabled.load(std::memory_order_relaxed)) return;
    std::lock_guard<std::mutex> lk(g_mu);
    cudaEvent_t e = get_event();
    cudaEventRecord(e, st);
    g_open[slot] = e;
}

void scao_prof_end(int slot, cudaStream_t st) {
    if (g_suspended || !g_enabled.load(std::memory_order_relaxed)) return;
    std::lock_guard<std::mutex> lk(g_mu);
    cudaEvent_t e = get_event();
    cudaEventRecord(e, st);
    g_pending.push_back({slot, g_open[slot], e, cur_device()});
}

extern "C" int64_t scao_launch_count(void) { return g_launches.load(); }

extern "C" void scao_prof_enable(int on) { g_enabled.store(on ? 1 : 0); }

extern "C" int scao_prof_read(double* ms, int64_t* counts, int nslots) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& p : g_pending) {
        if (cudaEventSynchronize(p.b) != cudaSuccess) return SCAO_ERR_LAUNCH;
        float t = 0.f;
        cudaEventElapsedTime(&t, p.a, p.b);
        g_ms[p.slot] += t;
        g_cnt[p.slot] += 1;
        g_pool[p.dev].push_back(p.a);
        g_pool[p.dev].push_back(p.b);
    }
    g_pending.clear();
    for (int i = 0; i < nslots && i < SLOT_COUNT; ++i) {
        if (ms) ms[i] = g_ms[i];
        if (counts) counts[i] = g_cnt[i];
    }
    return SCAO_OK;
}

extern "C" void scao_prof_reset(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 0; i < SLOT_COUNT; ++i) { g_ms[i] = 0.0; g_cnt[i] = 0; }
}

extern "C" const char* scao_prof_name(int slot) {
    return (slot >= 0 && slot < SLOT_COUNT) ? kNames[slot] : "";
}

extern "C" int scao_prof_slots(void) { return SLOT_COUNT; }
