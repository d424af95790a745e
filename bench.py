"""Benchmark: SCAO optimizer step on the Llama-1B-shaped parameter set.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One "step" is one SCAO.step() over every parameter of the workload (bf16
params, fp32 state, int8 curvature EMA, max_precond_dim=1024, k_max=64,
precondition_freq=10) with synthetic seeded low-rank-plus-noise gradients.
The optimizer is first primed through the 20 Adam-warmup steps, then W
untimed and K timed Phase-2 steps run; K spans the natural curvature cadence
(every 10th step refreshes curvature + eigenfactors), so ``ms_per_step`` is the
amortised step time.  Inputs (2 GB of gradients, 16 GB of state) exceed L2.

N > 1 (torchrun): owner-compute sharding -- every parameter is owned by one
rank; gradients are reduce-scattered (average) into owner shards, each rank
runs the step on its own parameters, and the updated bf16 parameters are
all-gathered.  Time = max over ranks of CUDA-event time; the total work is
fixed, so scaling is "strong".

``--impl reference`` times the reference algorithm's CPU implementation (the
numpy restatement in oracle/, the reference package itself cannot travel) on
the host cores, on a bounded sample (one transformer layer) scaled to the full
parameter set by element count.
"""
from __future__ import annotations

import argparse
import re
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "SCAO optimizer step ms (Llama-1B shapes)"
UNIT = "ms"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def metric_for(workload):
    if workload.name.startswith("llama-1b"):
        return METRIC
    return f"SCAO optimizer step ms ({workload.name} shapes)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return PEAKS_FALLBACK, "fallback"


def algorithmic_bytes(workload, phase_of):
    """Bytes a step must move per parameter (bf16 p/g, fp32 state):
    Phase 2: read g,p,m,v,d,prev + write p,m,v,d,prev = 38 B/elem (44 fp32);
    Phase 1: read g,p,m,v + write p,m,v,prev = 26 B/elem (32 fp32)."""
    tot = 0
    for spec in workload.params:
        n = 1
        for d in spec.shape:
            n *= d
        b16 = workload.param_dtype != "float32"
        if phase_of(spec) == 2:
            tot += n * (38 if b16 else 44)
        else:
            tot += n * (26 if b16 else 32)
    return tot


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.out = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# reference (CPU) arm
# ---------------------------------------------------------------------------

def _layer_of(name):
    m = re.match(r"^[hl](\d+)\.", name)
    return int(m.group(1)) if m else None


def sample_split(workload, layers):
    """(the non-layer parameters, the first ``layers`` transformer layers,
    the workload's layer count) as two workloads with its settings."""
    import copy
    n_layers = 1 + max((_layer_of(p.name) for p in workload.params
                        if _layer_of(p.name) is not None), default=-1)
    w_e = copy.copy(workload)
    w_e.params = [p for p in workload.params if _layer_of(p.name) is None]
    w_l = copy.copy(workload)
    w_l.params = [p for p in workload.params
                  if _layer_of(p.name) is not None and _layer_of(p.name) < layers]
    return w_e, w_l, n_layers


def reference_arm(workload, steps, warmup, device="cpu", layers=1):
    """Time the reference package's own ``scao.SCAO.step()`` (the unmodified
    install under baseline/_ref; its CUDA extension is not built, so on CUDA
    tensors it runs its PyTorch fallback) on a bounded sample of the workload:
    the embedding + final norm (Adam-only group) and ``layers`` transformer
    layers, each sample its own optimizer with the workload's settings.  Both
    are primed through the 20 Adam-warmup steps + ``warmup`` steps untimed,
    then ``steps`` steps are timed (same global steps, hence the same
    curvature cadence, as the GPU arm); a step of the full set is
    t(non-layer part) + (layer count / layers) * t(layer sample), the first
    term absent when every parameter belongs to a layer."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref, "scao", "__init__.py")):
        return None
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import warnings
    warnings.filterwarnings("ignore", category=RuntimeWarning)
    import scao  # the reference package
    from scao_b200 import synthetic, workloads

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    if device == "cpu":
        torch.set_num_threads(threads)
    w_e, w_l, n_layers = sample_split(workload, layers)
    scale = n_layers / layers
    samples = []
    for w_s, weight in ((w_e, 1.0), (w_l, scale)):
        if not w_s.params:                  # e.g. no parameters outside the layers
            continue
        p0 = synthetic.init_params(w_s, device=device)
        params = [torch.nn.Parameter(p) for p in p0]
        opt = build_opt(w_s, params, scao.SCAO)
        gen = synthetic.LowRankGradients(w_s, device=device)
        sets = [gen.next() for _ in range(3)]
        samples.append((params, opt, sets, weight))
    pf = workload.scao_kwargs["precond_freq"]
    n_prime = workload.scao_kwargs["warmup_steps"] + warmup

    def one(k):
        t = 0.0
        for params, opt, sets, weight in samples:
            for p, g in zip(params, sets[k % 3]):
                p.grad = g
            if device != "cpu":
                torch.cuda.synchronize()
            t0 = time.perf_counter()
            opt.step()
            if device != "cpu":
                torch.cuda.synchronize()
            t += weight * (time.perf_counter() - t0) * 1e3
        return t

    for k in range(n_prime):
        one(k)
    per, curv = [], []
    for k in range(steps):
        per.append(one(n_prime + k))
        curv.append((n_prime + k + 1) % pf == 0)
    reg = [t for t, c in zip(per, curv) if not c]
    cur = [t for t, c in zip(per, curv) if c]
    sample = (f"reference scao.SCAO.step() on {device} tensors: the non-layer parameters "
              f"(embedding in its Adam-only group) and {layers} of {n_layers} transformer layers, each its own "
              f"optimizer, primed {n_prime} steps, {steps} timed; per step "
              f"t(embedding part) + {scale:g} x t(layer sample)")
    return {"ms_per_step": statistics.mean(per), "cores": threads if device == "cpu" else None,
            "sample": sample, "steps": steps, "warmup": warmup,
            "regular_step_ms": statistics.mean(reg) if reg else None,
            "curvature_step_ms": statistics.mean(cur) if cur else None}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def build_opt(workload, params, scao_cls, **extra):
    main = [p for p, s in zip(params, workload.params) if not s.adam_only]
    groups = [{"params": main}] if main else []
    adam = [p for p, s in zip(params, workload.params) if s.adam_only]
    if adam:
        # Adam-only (Phase-1-forever) group: warmup_steps beyond any run
        groups.append({"params": adam, "warmup_steps": 10 ** 9})
    return scao_cls(groups, **workload.scao_kwargs, **extra)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="fewer transformer layers (small cases)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--nondegenerate-steps", type=int, default=30,
                    help="after the timed region: steps with s0=1 gradients (factors off "
                         "127*I, iterative eigensolve on every curvature step), timed apart")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpu-fallback", action="store_true",
                    help="--impl reference: skip timing the reference's PyTorch path on the GPU")
    ap.add_argument("--grad-scale", type=float, default=None,
                    help="leading singular value s0 of the synthetic gradients (default 1e-2, "
                         "the benchmark configuration; 1.0 moves the int8 factors off 127*I so "
                         "every curvature step runs the iterative eigensolver)")
    ap.add_argument("--json-out", default=None)
    ap.add_argument("--profile-range", action="store_true",
                    help="cudaProfilerStart/Stop around the timed steps (ncu --profile-from-start off)")
    ap.add_argument("--sparsity", type=float, default=0.0,
                    help="gradient filter level (the reference default is 0.7; the headline "
                         "configuration runs the deterministic path, 0)")
    ap.add_argument("--dynamic-sparsity", action="store_true")
    ap.add_argument("--noise", type=float, default=0.0, help="noise_std_init")
    ap.add_argument("--buckets", type=int, default=4,
                    help="N>1: reduce-scatter / step / all-gather pipeline buckets")
    ap.add_argument("--sm-reserve", type=int, default=32,
                    help="N>1: SMs the persistent kernels leave to the collectives")
    ap.add_argument("--workload", default="llama-1b",
                    choices=["llama-1b", "qwen2.5-3b", "gpt2-small", "gpt2m-train"],
                    help="llama-1b: the headline optimizer step (configuration C4); "
                         "qwen2.5-3b: C5 (per-GPU peak HBM and the eigensolve step reported); "
                         "gpt2-small: C2 (fp32 parameters); gpt2m-train: the GPT-2-medium "
                         "data-parallel training step (C3)")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    if a.workload == "gpt2m-train":
        return gpt2_train_bench(a)

    from scao_b200 import workloads
    if a.workload == "qwen2.5-3b":
        workload = workloads.c5(n_layers=a.layers or 36)
    elif a.workload == "gpt2-small":
        workload = workloads.c2(n_layers=a.layers or 12)
    else:
        workload = workloads.c4(n_layers=a.layers or 16)
    if a.grad_scale is not None:
        workload.grad_scale = a.grad_scale
    workload.scao_kwargs.update(sparsity=a.sparsity, noise_std_init=a.noise,
                                dynamic_sparsity=a.dynamic_sparsity)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    kw = workload.scao_kwargs
    gbytes = sum(int(np.prod(p.shape)) for p in workload.params) * \
        (2 if workload.param_dtype != "float32" else 4)
    cfg = {"workload": workload.name, "params": workload.numel,
           "param_dtype": workload.param_dtype, "state_dtype": "float32",
           "int8_ema": kw["use_int8_ema"], "max_precond_dim": kw.get("max_precond_dim", 4096),
           "k_max": kw["k_max"], "precond_freq": kw["precond_freq"],
           "warmup_steps": kw["warmup_steps"], "blend_steps": kw["blend_steps"],
           "grad_rank": workload.grad_rank,
           "l2": f"inputs larger than L2 ({gbytes / 1e9:.2f} GB of gradients, "
                 f"{16 * workload.numel / 1e9:.1f} GB of fp32 state per step)",
           "sparsity": a.sparsity, "dynamic_sparsity": a.dynamic_sparsity,
           "noise_std_init": a.noise, "grad_scale": workload.grad_scale}

    if a.impl == "reference":
        if rank != 0:
            return
        r = reference_arm(workload, a.steps, a.warmup)
        if r is not None:
            kind, val, cores, sample = "reference", r["ms_per_step"], r["cores"], r["sample"]
            extra = {"regular_step_ms": r["regular_step_ms"],
                     "curvature_step_ms": r["curvature_step_ms"]}
        else:
            # reference package not installed: the oracle's numpy restatement
            amort, cores, sample, reg, curv = cpu_reference(workload, steps=2, warmup=1)
            kind, val = "port", amort
            sample += " (2 timed steps after 1 warm-up step; reference package not installed)"
            extra = {"regular_step_ms": reg, "curvature_step_ms": curv}
        line = {"impl": "reference", "metric": metric_for(workload), "value": round(val, 3),
                "unit": UNIT,
                "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": round(val, 3), "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": cfg,
                "cpu_baseline": {"value": round(val, 3), "unit": UNIT, "cores": cores,
                                 "kind": kind, "sample": sample,
                                 **{k: round(v, 1) for k, v in extra.items() if v is not None}},
                "e2e": {"value": round(val, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        if r is not None and torch.cuda.is_available() and not a.no_gpu_fallback:
            # the reference's own GPU path (PyTorch fallback + cuSOLVER eigh) on
            # one B200, same sample rule: 10 steps after the warmup, one of them
            # a curvature step
            torch.cuda.set_device(local)
            g = reference_arm(workload, 10, 0, device=f"cuda:{local}")
            line["reference_gpu_fallback"] = {
                "value": round(g["ms_per_step"], 3), "unit": UNIT, "sample": g["sample"],
                "regular_step_ms": round(g["regular_step_ms"], 3),
                "curvature_step_ms": round(g["curvature_step_ms"], 3)}
        print(json.dumps(line), flush=True)
        return

    from scao_b200 import SCAO, _lib, synthetic
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    L = _lib.lib()

    # ---------------- setup ----------------
    params0 = synthetic.init_params(workload, seed=0, device=dev)
    params = [torch.nn.Parameter(p) for p in params0]
    gen = synthetic.LowRankGradients(workload, seed=0, device=dev)
    n_sets = 3
    grad_sets = [gen.next() for _ in range(n_sets)]
    torch.cuda.synchronize()
    if world > 1:
        from scao_b200.distributed import ShardedSCAO
        opt = ShardedSCAO(params, workload, lambda ps: build_opt_list(workload, ps, SCAO),
                          buckets=a.buckets, sm_reserve=a.sm_reserve)
        # unsharded shadow of this rank's parameters (one optimizer per bucket,
        # as the owner runs them), replayed after the timed region on the
        # same gradients: every rank receives the same G_t, so the averaged
        # gradient is exactly G_t and the owned parameters must match it
        shadow = []
        lay = opt.layout
        for b in range(lay.nb):
            mine = [i for i in opt.my if lay.bucket[i] == b]
            if mine:
                ps = [torch.nn.Parameter(params[i].detach().clone()) for i in mine]
                shadow.append((mine, ps, build_opt_list(
                    workload, [(p, workload.params[i]) for p, i in zip(ps, mine)], SCAO)))
    else:
        opt = build_opt(workload, params, SCAO)

    def set_grads(k):
        if world > 1:
            opt.load_grads(grad_sets[k % n_sets])
        else:
            for p, g in zip(params, grad_sets[k % n_sets]):
                p.grad = g

    stream = torch.cuda.current_stream(dev)
    # prime through the Adam warmup (20 steps) + W warm-up steps
    n_prime = workload.scao_kwargs["warmup_steps"] + a.warmup
    for k in range(n_prime):
        set_grads(k)
        opt.step()
    torch.cuda.synchronize()

    # ---------------- timed region ----------------
    clocks = ClockSampler(local)
    L.scao_prof_reset()
    L.scao_prof_enable(1)
    launches0 = L.scao_launch_count()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.steps + 1)]
    curv_flags = []
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    if a.profile_range:
        torch.cuda.profiler.start()
    ev[0].record(stream)
    for k in range(a.steps):
        gstep = opt._global_step + 1 if world == 1 else opt.global_step + 1
        curv_flags.append(gstep % 10 == 0)
        set_grads(n_prime + k)
        opt.step()
        ev[k + 1].record(stream)
    torch.cuda.synchronize()
    if a.profile_range:
        torch.cuda.profiler.stop()
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop()
    peak_gb = torch.cuda.max_memory_allocated(dev) / 1e9   # through the timed region
    launches = L.scao_launch_count() - launches0
    L.scao_prof_enable(0)
    prof = _lib.prof_read()
    step_ms = [ev[k].elapsed_time(ev[k + 1]) for k in range(a.steps)]
    total_ms = ev[0].elapsed_time(ev[a.steps])
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = t.item()
    ms_per_step = total_ms / a.steps
    parity = None
    if world > 1:
        # the shadow runs the same n_prime + steps steps without sharding
        for k in range(n_prime + a.steps):
            for mine, ps, sopt in shadow:
                for i, p in zip(mine, ps):
                    p.grad = grad_sets[k % n_sets][i]
                sopt.step()
        torch.cuda.synchronize()
        d = 0.0
        for mine, ps, _ in shadow:
            for i, p in zip(mine, ps):
                d = max(d, (params[i].detach().float() - p.detach().float()).abs().max().item())
        t = torch.tensor([d], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        parity = {"parity_max_abs": t.item(), "steps_compared": n_prime + a.steps,
                  "note": "owned parameters after the run vs an unsharded optimizer per "
                          "bucket fed the same gradients (every rank's G_t is identical, so "
                          "the averaged gradient is G_t exactly); max over ranks"}
    reg = [t for t, c in zip(step_ms, curv_flags) if not c]
    cur = [t for t, c in zip(step_ms, curv_flags) if c]

    # ---------------- roofline of the apply (regular-step kernels) ----------
    pk, pname = peaks()
    hbm = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    apply_slots = ["proj", "diag_pre", "leaf_coef", "param_pre", "apply_kron", "apply_flat",
                   "param_post", "global_norm", "apply_p"]
    if a.sparsity > 0:
        apply_slots.append("filter")
    apply_ms = sum(prof.get(s, (0.0, 0))[0] for s in apply_slots) / a.steps
    owned = opt.owned_specs() if world > 1 else workload.params
    wl_local = type(workload)(workload.name, owned, workload.scao_kwargs, workload.grad_rank,
                              workload.grad_decay, workload.param_dtype)
    abytes = algorithmic_bytes(wl_local, lambda s: 1 if s.adam_only else 2)
    if a.sparsity > 0:
        # filter: magnitude EMA read + write and one read for the selection
        abytes += 12 * sum(int(np.prod(s.shape)) for s in wl_local.params)
    achieved = abytes / (apply_ms * 1e-3) / 1e9 if apply_ms > 0 else 0.0
    kern = {k: {"ms_total": round(v[0], 3), "launches": v[1]} for k, v in sorted(prof.items())}
    # dominant kernel: the Kronecker apply (slot "apply_kron": correction + Adan + write-back)
    kron_elems = sum(int(np.prod(s.shape)) for s in wl_local.params
                     if not s.adam_only and len(s.shape) == 2)
    b16 = wl_local.param_dtype != "float32"
    per_elem = (38 if b16 else 44) + (4 if a.sparsity > 0 else 0)
    k_ms, k_n = prof.get("apply_kron", (0.0, 0))
    k_avg = k_ms / max(k_n, 1)
    # with bucketed owner-compute (N > 1) one step launches the kernel once
    # per bucket: bytes and elements per launch are the step's share
    k_lps = max(k_n / max(a.steps, 1), 1.0)
    kron_elems = kron_elems / k_lps
    k_bytes = per_elem * kron_elems
    k_achieved = k_bytes / (k_avg * 1e-3) / 1e9 if k_avg > 0 else 0.0
    # DRAM bytes per launch from an ncu capture of the same kernel on the
    # 2-layer case (4.631 GB for 121,634,816 Kronecker elements), scaled by
    # the Kronecker elements of this workload: traffic equals the algorithmic
    # bytes there (no re-reads)
    k_traffic = (4.631e9 / 121634816 * kron_elems
                 if (b16 and a.sparsity == 0 and a.noise == 0) else None)
    # the curvature GEMMs (tensor bound): one triangle of L = GG^T and R = G^TG
    # per leaf, sum a*b*(a+b) FLOP, over the gram time of the timed curvature steps
    plans = [opt._plan] if world == 1 else [x._plan for x in opt.inner if x is not None]
    gflop = sum(float((p.ltab["a"].astype(np.float64) * p.ltab["b"] *
                       (p.ltab["a"] + p.ltab["b"].astype(np.float64))).sum())
                for p in plans if p is not None and p.n_leaves) / 1e9
    n_curv = sum(1 for c in curv_flags if c)
    g_ms = prof.get("gram_tc", (0.0, 0))[0] + prof.get("gram_ema", (0.0, 0))[0]
    gemm = None
    if n_curv and g_ms > 0:
        tf = gflop / (g_ms / n_curv * 1e-3) / 1e3
        peak_tf = float(pk.get("bf16_tflops", PEAKS_FALLBACK.get("bf16_tflops", 1590.0)))
        gemm = {"bound": "tensor", "achieved": round(tf, 1), "peak": peak_tf, "unit": "TFLOP/s",
                "frac": round(tf / peak_tf, 4), "kernel": "curvature EMA gram (gram_tma)",
                "gflop_per_curvature_step": round(gflop, 1),
                "ms_per_curvature_step": round(g_ms / n_curv, 3)}

    # ---------------- e2e: public API with host gradient buffers -------------
    e2e = None
    if world == 1 and a.e2e_steps > 0:
        # host gradients (pinned) -> device every step through opt.step(); the
        # next step's copy runs on a copy stream into the other of two
        # gradient buffers while this step computes (input prefetch)
        # one flat pinned host buffer and two flat device buffers (each
        # gradient a 16-byte aligned view), so a step is one large copy
        offs, tot = [], 0
        for g in grad_sets[0]:
            offs.append(tot)
            tot += (g.numel() + 7) // 8 * 8
        host_flat = torch.zeros(tot, dtype=grad_sets[0][0].dtype).pin_memory()
        for g, o in zip(grad_sets[0], offs):
            host_flat[o:o + g.numel()].copy_(g.reshape(-1))
        h2d = host_flat.numel() * host_flat.element_size()
        res = torch.empty(1, dtype=torch.float64).pin_memory()
        flats = [torch.empty(tot, dtype=host_flat.dtype, device=dev) for _ in range(2)]
        bufs = [[f[o:o + p.numel()].view_as(p) for p, o in zip(params, offs)] for f in flats]
        cstream = torch.cuda.Stream(dev)
        copied = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        cstream.wait_stream(stream)

        def upload(k):
            with torch.cuda.stream(cstream):
                if k >= 2:
                    cstream.wait_event(freed[k % 2])      # step k-2 is done with it
                flats[k % 2].copy_(host_flat, non_blocking=True)
                copied[k % 2].record(cstream)
        upload(0)
        for k in range(a.e2e_steps):
            if k + 1 < a.e2e_steps:
                upload(k + 1)
            stream.wait_event(copied[k % 2])
            for p, d_ in zip(params, bufs[k % 2]):
                p.grad = d_
            opt.step()
            freed[k % 2].record(stream)
            res.copy_(opt._plan.global_norm_ema, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e = {"value": round(e0.elapsed_time(e1) / a.e2e_steps, 3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 8,
               "note": "every step: all gradients copied H2D from pinned host memory (the next "
                       "step's copy overlaps this step's compute on a copy stream, double-"
                       "buffered), opt.step(), global-norm EMA read back"}

    if world > 1 and a.e2e_steps > 0:
        # each rank's full gradient list from pinned host memory into the
        # flat owner layout, then the sharded step; one scalar read back
        import torch.distributed as dist
        flat_idx = opt.stage_grads(grad_sets[0])
        host = opt.grad_sets[flat_idx].cpu().pin_memory()
        h2d = host.numel() * host.element_size()
        res = torch.empty(1, dtype=torch.float64).pin_memory()
        first = next(x for x in opt.inner if x is not None)
        torch.cuda.synchronize()
        dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(a.e2e_steps):
            opt.cur = opt.grad_sets[flat_idx]
            opt.cur.copy_(host, non_blocking=True)
            opt.step()
            res.copy_(first._plan.global_norm_ema, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / a.e2e_steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = {"value": round(t.item(), 3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 8,
               "note": "per rank: full gradient list copied H2D from pinned host memory into the "
                       "owner layout every step, then reduce-scatter / step / all-gather; "
                       "max over ranks"}

    split = None
    if world > 1:
        # communication and computation of the regular step measured apart
        # (same pipeline with the other half switched off); max over ranks
        import torch.distributed as dist

        def timed(n):
            opt.load_grads(grad_sets[0])
            torch.cuda.synchronize()
            dist.barrier()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(n):
                opt.step()
            t1.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([t0.elapsed_time(t1) / n], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return round(t.item(), 3)
        opt.skip_compute = True
        comm_ms = timed(3)
        opt.skip_compute = False
        opt.skip_comm = True
        compute_ms = timed(3)
        opt.skip_comm = False
        split = {"comm_only_ms": comm_ms, "compute_only_ms": compute_ms,
                 "note": "3 steps each after the timed region; compute-only steps include "
                         "curvature steps when the cadence lands on them"}

    eig_slots = ("eig_prep", "eig_diag", "eig_gemm", "eig_jacobi", "eig_residual",
                 "eig_cholinv", "eig_rank", "eig_iter")
    eig_ms = sum(prof.get(s_, (0.0, 0))[0] for s_ in eig_slots)
    diag_path = all(prof.get(s_, (0.0, 0))[1] == 0 for s_ in ("eig_gemm", "eig_jacobi"))

    nondeg = None
    if world == 1 and a.nondegenerate_steps > 0 and workload.grad_scale < 0.5:
        nondeg = nondegenerate_leg(a, opt, params, workload, dev, stream, L)

    if world > 1:
        t = torch.tensor([peak_gb], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        peak_gb = t.item()
    peak_gb = round(peak_gb, 2)
    if rank != 0:
        torch.distributed.destroy_process_group()
        return
    line = {
        "metric": metric_for(workload), "value": round(ms_per_step, 3), "unit": UNIT,
        "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16" if workload.param_dtype != "float32" else "f32",
        "data": "synthetic (seeded low-rank+noise gradients, N(0,0.02^2) params)",
        "config": dict(cfg, parallelism=f"owner-compute x{world}" if world > 1 else "single"),
        "regular_step_ms": round(statistics.mean(reg), 3) if reg else None,
        "curvature_step_ms": round(statistics.mean(cur), 3) if cur else None,
        "roofline": {"bound": "hbm", "achieved": round(k_achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(k_achieved / hbm, 4),
                     "traffic": round(k_traffic) if k_traffic else None,
                     "kernel": "apply (Kronecker correction + Adan + state write-back), slot apply_kron",
                     "algorithmic_bytes_per_launch": round(k_bytes),
                     "bytes_per_elem": per_elem, "elems_per_launch": round(kron_elems),
                     "launches_per_step": round(k_lps, 2),
                     "avg_launch_ms": round(k_avg, 3), "peak_source": pname,
                     "apply_sequence": {"kernels": "+".join(apply_slots),
                                        "algorithmic_bytes_per_step": abytes,
                                        "ms_per_step": round(apply_ms, 3),
                                        "achieved_gbs": round(achieved, 1),
                                        "frac": round(achieved / hbm, 4)}},
        "gemm_roofline": gemm,
        "eigensolve_ms_per_curvature_step": round(eig_ms / n_curv, 3) if n_curv else None,
        "eigensolve_diagonal_shortcut": bool(diag_path),
        **({"nondegenerate": nondeg} if nondeg else {}),
        "kernels": kern,
        "gpu_launches": int(launches),
        "peak_hbm_gb": peak_gb,
        **({"comm_compute_split": split} if split else {}),
        "clocks": clk,
        **({"sharded_parity": parity} if parity else {}),
    }
    if e2e:
        line["e2e"] = e2e
    if world == 1 and not a.no_cpu_baseline:
        # the reference package on the host cores: steps 21-30 (nine regular
        # steps and one curvature step) after the 20 Adam-warmup steps
        r = reference_arm(workload, 10, 0)
        if r is not None:
            line["cpu_baseline"] = {"value": round(r["ms_per_step"], 1), "unit": UNIT,
                                    "cores": r["cores"], "kind": "reference",
                                    "sample": r["sample"],
                                    "regular_step_ms": round(r["regular_step_ms"], 1),
                                    "curvature_step_ms": round(r["curvature_step_ms"], 1)}
        else:
            amort, cores, sample, creg, ccurv = cpu_reference(workload, steps=2, warmup=1)
            line["cpu_baseline"] = {"value": round(amort, 1), "unit": UNIT, "cores": cores,
                                    "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)
    if a.json_out:
        with open(a.json_out, "w") as f:
            json.dump(line, f, indent=1)
    if world > 1:
        torch.distributed.destroy_process_group()


def nondegenerate_leg(a, opt, params, workload, dev, stream, L):
    """Continue the optimizer with s0 = 1 gradients (the int8 factors leave
    127*I at the first curvature update, so every later curvature step runs
    the iterative eigensolver on all 1024 / 512 factors) and time
    ``--nondegenerate-steps`` steps with CUDA events; the eigensolve is timed
    per curvature step from the library's kernel events."""
    from scao_b200 import _lib, synthetic
    gen = synthetic.LowRankGradients(workload, seed=1, device=dev, s0=1.0)
    sets = [gen.next() for _ in range(3)]
    pf = workload.scao_kwargs["precond_freq"]
    # untimed up to and through one curvature step (leaves the 127*I regime)
    k = 0
    while True:
        for p, g in zip(params, sets[k % 3]):
            p.grad = g
        opt.step()
        k += 1
        if opt._global_step % pf == 0:
            break
    torch.cuda.synchronize()
    reg, curv, eig = [], [], []
    eig_slots = ("eig_prep", "eig_diag", "eig_gemm", "eig_jacobi", "eig_residual",
                 "eig_cholinv", "eig_rank", "eig_iter")
    last_split = {}
    for _ in range(a.nondegenerate_steps):
        for p, g in zip(params, sets[k % 3]):
            p.grad = g
        k += 1
        is_curv = (opt._global_step + 1) % pf == 0
        L.scao_prof_reset()
        L.scao_prof_enable(1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        opt.step()
        e1.record(stream)
        torch.cuda.synchronize()
        L.scao_prof_enable(0)
        t = e0.elapsed_time(e1)
        if is_curv:
            curv.append(t)
            pr = _lib.prof_read()
            eig.append(sum(pr.get(s_, (0.0, 0))[0] for s_ in eig_slots))
            last_split = {s_: round(pr[s_][0], 3) for s_ in eig_slots if s_ in pr}
            st = getattr(opt, "_last_eig_status", None)
            if st is not None:
                its = st.cpu().numpy()
                last_split["iterations_max"] = int(abs(its).max()) if its.size else 0
                last_split["iterations_mean"] = round(float(abs(its).mean()), 2) if its.size else 0
                last_split["capped"] = int((its < 0).sum())
        else:
            reg.append(t)
    r = statistics.mean(reg) if reg else None
    c = statistics.mean(curv) if curv else None
    return {"grad_scale": 1.0, "steps": a.nondegenerate_steps,
            "regular_step_ms": round(r, 3) if r else None,
            "curvature_step_ms": [round(x, 3) for x in curv],
            "eigensolve_ms": [round(x, 3) for x in eig],
            "eigensolve_last_split_ms": last_split,
            "amortised_ms": round(((pf - 1) * r + c) / pf, 3) if (r and c) else None,
            "note": "after the timed region: s0=1 gradients, first curvature step untimed; each "
                    "step timed alone (CUDA events, synchronised), eigensolve = eig_* kernels"}


def build_opt_list(workload, params_specs, scao_cls):
    """Optimizer over a rank's owned (param, spec) pairs."""
    ps = [p for p, s in params_specs if not s.adam_only]
    adam = [p for p, s in params_specs if s.adam_only]
    groups = []
    if ps:
        groups.append({"params": ps})
    if adam:
        groups.append({"params": adam, "warmup_steps": 10 ** 9})
    return scao_cls(groups, **workload.scao_kwargs)


def gpt2_train_bench(a):
    """GPT-2-medium training step (forward + backward under bf16 autocast +
    SCAO step; per rank 8 x 1024 tokens, fp32 weights and state) on N GPUs,
    data-parallel through the owner-compute ShardedSCAO; tokens/s over all
    ranks, CUDA events, max over ranks."""
    from scao_b200 import SCAO, gpt, workloads
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=dev)
    c = gpt.GPT2_MEDIUM
    model = gpt.GPT(c, seed=0).to(dev)
    params = list(model.parameters())
    kw = dict(lr=3e-4, betas=(0.9, 0.999), precond_freq=10, warmup_steps=20, blend_steps=50,
              min_precond_updates=1, k_max=64, max_precond_dim=1024, use_int8_ema=True,
              sparsity=0.0, noise_std_init=0.0, async_precond=False)
    sharded = None
    opt = None
    if world > 1:
        from scao_b200.distributed import ShardedSCAO
        specs = [workloads.ParamSpec(f"p{i}", tuple(p.shape)) for i, p in enumerate(params)]
        wl = workloads.Workload("gpt2-medium", specs, kw, 0, 0.0, "float32")
        sharded = ShardedSCAO(params, wl, lambda ps: SCAO([p for p, _ in ps], **kw),
                              buckets=a.buckets, sm_reserve=a.sm_reserve)
    else:
        opt = SCAO(params, **kw)
    batch = 8
    toks = [gpt.token_batch(c, batch, seed=1000 * rank + s, device=dev) for s in range(4)]
    stream = torch.cuda.current_stream(dev)
    for k in range(kw["warmup_steps"] + a.warmup):
        gpt.train_step(model, opt, toks[k % 4], sharded)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    losses = []
    for k in range(a.steps):
        losses.append(gpt.train_step(model, opt, toks[k % 4], sharded))
    ev[1].record(stream)
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / a.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    if rank != 0:
        return
    tokens = world * batch * c.seq_len
    print(json.dumps({
        "metric": "GPT-2-medium training step (forward+backward+SCAO) tokens/s",
        "value": round(tokens / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "dtype": "bf16 autocast, fp32 state",
        "data": "synthetic tokens, uniform over the vocabulary",
        "config": {"workload": "gpt2-medium-train", "layers": c.n_layer, "d_model": c.d_model,
                   "heads": c.n_head, "d_ff": c.d_ff, "vocab": c.vocab, "seq_len": c.seq_len,
                   "batch_per_gpu": batch, "params": sum(p.numel() for p in params),
                   "parallelism": f"data-parallel x{world}, owner-compute SCAO"},
        "loss_last": round(float(losses[-1].item()), 4),
    }), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
