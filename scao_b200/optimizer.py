"""SCAO optimizer facade (drop-in for ``scao.SCAO``, scao/optimizer.py:221-801).

The constructor keyword arguments, their defaults, the validation errors, the
per-group hyper-parameters, ``step(closure)``, callbacks, ``state_dict`` /
``load_state_dict`` schema and the diagnostics are those of the reference.
Behind ``step()`` the per-parameter Python loop is replaced by a fixed
sequence of batched sm_100a kernels (libscao_b200.so) covering every
parameter: the host only decides phases and per-parameter scalars, writes a
step table and launches.  There is no CPU path: parameters must be CUDA
tensors and the library must be built.
"""
from __future__ import annotations

import math
import os
from typing import Callable, Iterable

import numpy as np
import torch
from torch.optim import Optimizer

from . import _lib
from .plan import Plan
from .preconditioner import PrecondView



class _AdaptiveWarmupScheduler:
    """R1 (optimizer.py:104-150): leave the Adam warmup early once the mean
    gradient norm has changed by less than ``stability_threshold`` (relative)
    for ``patience`` consecutive steps.  Host logic on the per-step norms."""

    def __init__(self, warmup_steps=100, stability_threshold=0.05, patience=5, min_warmup=20):
        self.warmup_steps = warmup_steps
        self.stability_threshold = stability_threshold
        self.patience = patience
        self.min_warmup = min_warmup
        self._prev_norm = float("inf")
        self._stable_count = 0
        self._early_exit_step = None

    def update(self, step: int, avg_grad_norm: float) -> bool:
        if step < self.min_warmup:
            return True
        if self._prev_norm > 0:
            rel = abs(avg_grad_norm - self._prev_norm) / (self._prev_norm + 1e-8)
            self._stable_count = self._stable_count + 1 if rel < self.stability_threshold else 0
        self._prev_norm = avg_grad_norm
        if self._stable_count >= self.patience:
            self._early_exit_step = self._early_exit_step or step
            return False
        return step < self.warmup_steps

    @property
    def exited_early(self) -> bool:
        return self._early_exit_step is not None

    @property
    def actual_warmup_steps(self) -> int:
        return self._early_exit_step or self.warmup_steps


class _LazyPrecondTrigger:
    """R3 (optimizer.py:182-214): refresh the curvature when the gradient norm
    moved by more than ``delta_threshold`` (relative) or after ``max_skip``
    steps."""

    def __init__(self, delta_threshold=0.1, max_skip=50):
        self.delta_threshold = delta_threshold
        self.max_skip = max_skip
        self._prev_grad_norm = 0.0
        self._steps_since_update = 0

    def should_update(self, grad_norm: float) -> bool:
        self._steps_since_update += 1
        if self._steps_since_update >= self.max_skip:
            self._steps_since_update = 0
            self._prev_grad_norm = grad_norm
            return True
        if self._prev_grad_norm > 0:
            rel = abs(grad_norm - self._prev_grad_norm) / (self._prev_grad_norm + 1e-8)
            if rel > self.delta_threshold:
                self._steps_since_update = 0
                self._prev_grad_norm = grad_norm
                return True
        self._prev_grad_norm = grad_norm
        return False


class SCAO(Optimizer):
    """B200-native SCAO.  Same signature and defaults as the reference
    (optimizer.py:258-296)."""

    def __init__(
        self,
        params: Iterable,
        lr: float = 1e-3,
        betas: tuple = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 0.01,
        precond_freq: int = 20,
        epsilon_sparse: float = 0.05,
        k_min: int = 8,
        k_max: int = 128,
        rho: float = 0.999,
        tau: float | None = 1.0,
        warmup_steps: int = 100,
        blend_steps: int = 50,
        min_precond_updates: int = 10,
        max_precond_dim: int = 4096,
        use_newton_schulz: bool = False,
        use_int8_ema: bool = False,
        async_precond: bool = True,
        beta3: float = 0.99,
        sparsity: float = 0.7,
        noise_std_init: float = 0.01,
        noise_anneal: float = 0.998,
        lars_coeff: float = 1e-3,
        lookahead_k: int = 5,
        lookahead_alpha: float = 0.5,
        dynamic_sparsity: bool = False,
        adaptive_warmup: bool = False,
        warmup_stability_threshold: float = 0.05,
        warmup_patience: int = 5,
        lazy_precond: bool = False,
        lazy_delta_threshold: float = 0.1,
        lazy_max_skip: int = 50,
        use_gsnr_clip: bool = False,
        gsnr_threshold: float = 0.5,
        adaptive_rank: bool = False,
        eig_max_iters: int = 30,
        eig_tol: float = 5e-4,
    ) -> None:
        # optimizer.py:297-304
        if lr < 0:
            raise ValueError(f"Invalid lr: {lr}")
        if not (0.0 <= betas[0] < 1.0):
            raise ValueError(f"Invalid beta1: {betas[0]}")
        if not (0.0 <= betas[1] < 1.0):
            raise ValueError(f"Invalid beta2: {betas[1]}")
        if not (0.0 <= beta3 < 1.0):
            raise ValueError(f"Invalid beta3: {beta3}")
        defaults = dict(
            lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
            precond_freq=precond_freq, epsilon_sparse=epsilon_sparse,
            k_min=k_min, k_max=k_max, rho=rho, tau=tau,
            warmup_steps=warmup_steps, blend_steps=blend_steps,
            min_precond_updates=min_precond_updates,
            max_precond_dim=max_precond_dim, use_newton_schulz=use_newton_schulz,
            use_int8_ema=use_int8_ema, beta3=beta3, lars_coeff=lars_coeff,
        )
        super().__init__(params, defaults)
        self._callbacks: list = []
        self._global_step = 0
        self._noise_std = noise_std_init
        self._noise_anneal = noise_anneal
        self._lookahead_k = lookahead_k
        self._lookahead_alpha = lookahead_alpha
        self._lookahead_init = False
        self._sparsity = sparsity
        self._dynamic_sparsity = bool(dynamic_sparsity)
        # R1 / R3 / R4 / R5 (optimizer.py:332-345)
        self._adaptive_warmup = bool(adaptive_warmup)
        self._warmup_scheduler = _AdaptiveWarmupScheduler(
            warmup_steps=warmup_steps, stability_threshold=warmup_stability_threshold,
            patience=warmup_patience, min_warmup=max(20, warmup_steps // 5))
        self._lazy_precond = bool(lazy_precond)
        self._lazy_triggers: dict = {}
        self._lazy_delta_threshold = lazy_delta_threshold
        self._lazy_max_skip = lazy_max_skip
        self._use_gsnr_clip = bool(use_gsnr_clip)
        self._gsnr_threshold = gsnr_threshold
        self._adaptive_rank = bool(adaptive_rank)
        # R1 / R3 / R5 decide on the host from per-parameter gradient norms;
        # the host then keeps the global grad-norm EMA as well
        self._host_norms = self._adaptive_warmup or self._lazy_precond or self._adaptive_rank
        self._gema = 1.0
        self._sm_reserve = 0     # SMs the persistent kernels leave to concurrent collectives
        self._in_warmup_global = True
        self._eig_max_iters = int(eig_max_iters)
        self._eig_tol = float(eig_tol)
        self._plan: Plan | None = None
        # set by an owner-compute wrapper: the global grad-norm average over
        # all ranks' parameters for this step (callable(local norms) -> (avg, n))
        self._norm_average = None
        self._ema_scratch = None
        self._last_eig_status = None

    # ------------------------------------------------------------------
    # plan / state
    # ------------------------------------------------------------------
    def add_param_group(self, param_group: dict) -> None:
        """torch.optim.Optimizer.add_param_group.  Groups can be added until
        the first step; the device plan (arenas, tables, filter and
        lookahead state) is laid out for the parameter set of that step."""
        if getattr(self, "_plan", None) is not None:
            raise NotImplementedError(
                "scao_b200.SCAO: add_param_group after the first step is not supported; "
                "pass every parameter group to the constructor (or add them before stepping)")
        super().add_param_group(param_group)

    def _flat(self):
        ps, gs = [], []
        for g in self.param_groups:
            for p in g["params"]:
                ps.append(p)
                gs.append(g)
        return ps, gs

    def _build_plan(self):
        ps, gs = self._flat()
        if not ps:
            return
        dev = ps[0].device
        if dev.type != "cuda":
            raise RuntimeError("scao_b200.SCAO runs on CUDA tensors only (no CPU path)")
        if any(p.device != dev for p in ps):
            raise RuntimeError("all parameters must be on one CUDA device")
        int8 = {bool(g["use_int8_ema"]) for g in gs}
        if len(int8) != 1:
            raise NotImplementedError("mixed use_int8_ema across param groups")
        _lib.lib()
        with torch.cuda.device(dev):
            self._plan = Plan(ps, gs, dev, int8.pop())
            if self._sparsity > 0.0:
                self._plan.setup_filter(2 if self._dynamic_sparsity else 1, self._sparsity)
        f = self._plan.dev.filt
        f.gsnr_on = 1 if self._use_gsnr_clip else 0          # R4
        f.gsnr_thr = float(np.float32(self._gsnr_threshold))
        self._plan.dev.gnorm_host = 1 if self._host_norms else 0
        self._plan.dev.sm_reserve = int(self._sm_reserve)
        self._plan.gnorm_dev = torch.zeros(len(ps), dtype=torch.float32, device=dev)
        self._plan.gnorm_pin = torch.zeros(len(ps), dtype=torch.float32,
                                           pin_memory=torch.cuda.is_available())
        self._plan.k_pin = torch.zeros(max(self._plan.n_leaves, 1), dtype=torch.int32,
                                       pin_memory=torch.cuda.is_available())
        # noise stream key: the device generator's seed (consumes no draws)
        gen = torch.cuda.default_generators[dev.index if dev.index is not None
                                            else torch.cuda.current_device()]
        self._plan.dev.filt.noise_seed = (int(gen.initial_seed()) * 0x9E3779B97F4A7C15 + 1) \
            & 0xFFFFFFFFFFFFFFFF
        for i, (p, g) in enumerate(zip(ps, gs)):
            st = self.state[p]
            st["step"] = 0
            st["scao_step"] = 0
            st["exp_avg"] = self._plan.state_view(self._plan.exp_avg, i)
            st["exp_avg_sq"] = self._plan.state_view(self._plan.exp_avg_sq, i)
            st["exp_avg_diff"] = self._plan.state_view(self._plan.exp_avg_diff, i)
            st["prev_grad"] = self._plan.state_view(self._plan.prev_grad, i)
            st["preconditioner"] = PrecondView(self._plan, i, g)


    # ------------------------------------------------------------------
    # step
    # ------------------------------------------------------------------
    @torch.no_grad()
    def step(self, closure: Callable | None = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self._plan is None:
            self._build_plan()
            if self._plan is None:
                return loss
        # the library launches on the current device: make it the plan's
        with torch.cuda.device(self._plan.device):
            return self._device_step(loss)

    def _device_step(self, loss):
        plan = self._plan
        L = _lib.lib()
        if plan.step_event is not None:
            plan.step_event.synchronize()   # previous table upload has left the pinned buffer
        # a bounded device wait that ran out in an earlier step (read back
        # asynchronously; checked once its copy has landed, no synchronisation)
        if plan.err_event is not None and plan.err_event.query():
            plan.err_event = None
            if int(plan.err_pin[0]):
                raise RuntimeError("scao_b200: a device-side wait timed out in an earlier step "
                                   "(results of that step are not valid)")
        self._global_step += 1
        ps, gs = self._flat()
        tab = plan.step_np
        curv_leaves: dict = {}
        curv_diag: dict = {}
        eig_leaves, eig_bias = [], []
        keep = []
        grads = []
        for i, p in enumerate(ps):
            row = tab[i]
            row["p_ptr"] = p.data_ptr()
            grad = p.grad
            if grad is None:
                row["phase"] = 0
                grads.append(None)
                continue
            if grad.is_sparse:
                raise RuntimeError("SCAO does not support sparse gradients.")
            if grad.dtype != p.dtype or not grad.is_contiguous():
                grad = grad.to(p.dtype).contiguous()
                keep.append(grad)
            if not p.is_contiguous():
                raise RuntimeError("scao_b200 needs contiguous parameters")
            row["g_ptr"] = grad.data_ptr()
            row["phase"] = 1
            grads.append(grad)
        norms = kvec = None
        if self._host_norms:
            norms, kvec = self._grad_norms_and_ranks(plan)
            # the average takes p.grad.norm() in the gradient's dtype
            # (optimizer.py:440); R3 / R5 use the float32 norm (:531-532)
            avg_norms = _in_param_dtypes(norms, ps)
            live = [float(avg_norms[i]) for i in range(len(ps)) if grads[i] is not None]
            if self._norm_average is not None:
                # owner-compute across ranks: the all-parameter average
                avg, n_live = self._norm_average(live)
            else:
                avg, n_live = (sum(live) / len(live) if live else 0.0), len(live)
            if n_live:
                self._gema = 0.95 * self._gema + 0.05 * avg           # optimizer.py:445
            plan.global_norm_ema.fill_(self._gema)
        warm_max = max((g.get("warmup_steps", 100) for g in self.param_groups), default=100)
        if self._adaptive_warmup:                                       # R1, :470-474
            self._in_warmup_global = self._warmup_scheduler.update(self._global_step, avg)
        else:
            self._in_warmup_global = self._global_step <= warm_max
        k_changed = False
        for i, (p, g) in enumerate(zip(ps, gs)):
            row = tab[i]
            grad = grads[i]
            if grad is None:
                continue
            st = self.state[p]
            st["step"] += 1
            step = st["step"]
            pc = st["preconditioner"]
            lr = float(g["lr"])
            wd = float(g["weight_decay"])
            b1, b2 = g["betas"]
            b3 = g["beta3"]
            if self._adaptive_rank:                                     # R5, :383-401
                ratio = float(norms[i]) / (self._gema + 1e-8)
                cur = pc.k_host(kvec)
                new_k = None
                if ratio > 2.0:
                    new_k = min(g["k_max"], int(cur * 1.25))
                elif ratio < 0.5:
                    new_k = max(g["k_min"], int(cur * 0.8))
                if new_k is not None and new_k != cur:
                    k_changed |= pc.set_k_host(new_k, kvec)
            in_warmup = (self._in_warmup_global if self._adaptive_warmup
                         else step <= g["warmup_steps"]) or \
                (pc.precond_step < g["min_precond_updates"])
            if self._lazy_precond and not in_warmup:                    # R3, :594-599
                tr = self._lazy_triggers.get(i)
                if tr is None:
                    tr = self._lazy_triggers[i] = _LazyPrecondTrigger(
                        self._lazy_delta_threshold, self._lazy_max_skip)
                do_curv = tr.should_update(float(norms[i]))
            else:
                do_curv = step % g["precond_freq"] == 0
            if do_curv:
                pc.precond_step += 1
                rho = float(g["rho"])
                leaves = plan.param_leaves[i]
                if leaves:
                    curv_leaves.setdefault(rho, []).extend(leaves)
                    bf = 1.0 - rho ** pc.precond_step
                    eig_leaves.extend(leaves)
                    eig_bias.extend([bf] * len(leaves))
                if not leaves or plan.param_strips[i]:
                    # diagonal params, and the width-1 strips of Kronecker ones
                    curv_diag.setdefault(rho, []).append(i)
            row["lr"] = lr
            row["wd"] = wd
            row["wd_mult"] = np.float32(1.0 - lr * wd) if wd != 0.0 else np.float32(1.0)
            row["beta1"], row["beta2"], row["beta3"] = b1, b2, b3
            row["c1"], row["c2"], row["c3"] = 1.0 - b1, 1.0 - b2, 1.0 - b3
            row["eps"] = g["eps"]
            row["lars"] = g["lars_coeff"]
            row["diag_bias"] = pc.diag_bias
            bc1 = 1.0 - b1 ** step
            bc2 = 1.0 - b2 ** step
            if in_warmup:
                row["phase"] = 1
                row["alpha1"] = -(lr / bc1)
                row["sqrt_bc2"] = math.sqrt(bc2)
                row["rbc2"] = _recip32(row["sqrt_bc2"])   # RN(1/c) for the kernels' division
                continue
            row["phase"] = 2
            if not st.get("scao_phase_started", False):
                st["scao_phase_started"] = True
                st["phase2_start_step"] = step
                st["scao_step"] = 0
            st["scao_step"] += 1
            bs = g.get("blend_steps", 50)
            blend = min(1.0, st["scao_step"] / bs) if bs > 0 else 1.0
            row["blend"] = blend
            row["one_minus_blend"] = 1.0 - blend
            row["bc1"], row["bc2"], row["bc3"] = bc1, bc2, 1.0 - b3 ** step
            # correctly rounded float32 reciprocals for the kernels' division
            for k in ("bc1", "bc2", "bc3"):
                row["r" + k] = _recip32(row[k])
            tau = g["tau"]
            row["clip"] = 0 if tau is None else 1
            row["tau"] = 0.0 if tau is None else tau
        dev = plan.device
        stream = torch.cuda.current_stream(dev)
        sp = C_stream(stream)
        if k_changed:
            plan.upload_k(kvec)
        plan.t_step.copy_(plan.step_host, non_blocking=True)
        plan.step_event = torch.cuda.Event()
        plan.step_event.record(stream)
        dptr = plan.dev
        import ctypes
        pd = ctypes.byref(dptr)
        # TMA tensor maps of this step's gradients / parameters: one device
        # buffer per pointer set (a few kept, so alternating gradient buffers
        # do not re-encode); selected before any kernel that reads them
        if plan.has_bf16_kron and os.environ.get("SCAO_NO_TMA") != "1":
            plan.select_tensor_maps((tab["g_ptr"].tobytes(), tab["p_ptr"].tobytes(),
                                     tab["phase"].tobytes()), pd, sp)
        else:
            plan.dev.tmaps_ok = 0
        for rho, leaves in curv_leaves.items():
            ids_h = np.ascontiguousarray(leaves, dtype=np.int32)
            ids = plan.dev_ids(ids_h)
            ma, mb, _ = plan.max_dims(leaves)
            need = L.scao_ema_scratch_bytes(len(leaves), ma, mb)
            scratch = self._get_ema_scratch(need)
            _lib.check(L.scao_plan_curvature(pd, ids.data_ptr(), len(leaves), ma, mb, rho,
                                             scratch.data_ptr(), scratch.numel(),
                                             plan.ptab.ctypes.data, plan.step_host.data_ptr(),
                                             plan.ltab.ctypes.data, ids_h.ctypes.data, sp),
                       "scao_plan_curvature")
            keep.append(ids)
        for rho, pids in curv_diag.items():
            ids = plan.dev_ids(np.ascontiguousarray(pids, dtype=np.int32))
            _lib.check(L.scao_plan_curvature_diag(pd, ids.data_ptr(), len(pids), rho, sp),
                       "scao_plan_curvature_diag")
            keep.append(ids)
        if eig_leaves:
            eig_h = np.ascontiguousarray(eig_leaves, dtype=np.int32)
            ids = plan.dev_ids(eig_h)
            bias = plan.upload_bias(eig_h, eig_bias)
            ma, mb, smax = plan.max_dims(eig_leaves)
            status = plan.eig_status[: 2 * len(eig_leaves)]
            _lib.check(L.scao_plan_eigen(pd, ids.data_ptr(), len(eig_leaves), bias.data_ptr(),
                                         plan.t_eps_sparse.data_ptr(), self._eig_max_iters,
                                         self._eig_tol, status.data_ptr(), max(ma, mb), smax,
                                         sp), "scao_plan_eigen")
            self._last_eig_status = status
            keep.append(ids)
        plan.set_phases(np.array(tab["phase"], dtype=np.int32))
        if plan.n_leaves:
            # the cp.async projection runs only for Phase-2 leaves the TMA one cannot take
            ph = tab["phase"][plan.leaf_param]
            al = (tab["g_ptr"][plan.leaf_param] % 16) == 0
            plan.dev.proj_fallback = int(bool(np.any((ph == 2) & ~(plan.leaf_tma_shape & al))))
            alp = al & ((tab["p_ptr"][plan.leaf_param] % 16) == 0)
            plan.dev.apply_fallback = int(bool(np.any((ph == 2) & ~(plan.leaf_tma_apply & alp))))
        # lookahead (optimizer.py:356-365, after the parameter update): fused into
        # the Phase-2 parameter write; the lookahead kernel does the rest
        la_now = self._lookahead_k > 0 and self._global_step % self._lookahead_k == 0
        if la_now:
            plan.ensure_slow()
        plan.dev.la_fused = 1 if la_now else 0
        plan.dev.la_init = 0 if self._lookahead_init else 1
        plan.dev.la_alpha = float(self._lookahead_alpha)
        f = plan.dev.filt
        f.noise_on = 1 if self._noise_std > 1e-9 else 0     # optimizer.py:544
        f.noise_std = float(np.float32(self._noise_std))
        f.noise_step = self._global_step
        _lib.check(L.scao_plan_step(pd, sp), "scao_plan_step")
        if plan.err_event is None:
            plan.err_pin.copy_(plan.err, non_blocking=True)
            plan.err_event = torch.cuda.Event()
            plan.err_event.record(stream)
        self._noise_std *= self._noise_anneal
        if la_now:
            _lib.check(L.scao_plan_lookahead(pd, float(self._lookahead_alpha),
                                             0 if self._lookahead_init else 1, sp),
                       "scao_plan_lookahead")
            self._lookahead_init = True
        plan.dev.la_fused = 0
        self._keep = keep   # keep temporaries alive until the next step
        if self._callbacks:
            metrics = self.collect_metrics()
            for cb in self._callbacks:
                cb(metrics)
        return loss

    def _grad_norms_and_ranks(self, plan):
        """Per-parameter ||g|| of this step (device kernel over the step
        table's gradient pointers) and the current leaf ranks, read back
        together (one synchronisation)."""
        import ctypes
        L = _lib.lib()
        stream = torch.cuda.current_stream(plan.device)
        plan.t_step.copy_(plan.step_host, non_blocking=True)
        _lib.check(L.scao_plan_grad_norms(ctypes.byref(plan.dev), plan.gnorm_dev.data_ptr(),
                                          C_stream(stream)), "scao_plan_grad_norms")
        plan.gnorm_pin.copy_(plan.gnorm_dev, non_blocking=True)
        if plan.n_leaves:
            plan.k_pin.copy_(plan.k, non_blocking=True)
        stream.synchronize()
        return plan.gnorm_pin.numpy().copy(), plan.k_pin.numpy()[:plan.n_leaves].copy()

    def _get_ema_scratch(self, need):
        cap = 2 << 30
        need = min(int(need), cap)
        if self._ema_scratch is None or self._ema_scratch.numel() < need:
            self._ema_scratch = torch.empty(need, dtype=torch.uint8, device=self._plan.device)
        return self._ema_scratch

    # ------------------------------------------------------------------
    # callbacks / diagnostics (optimizer.py:716-801, logging.py:151-220)
    # ------------------------------------------------------------------
    def add_callback(self, callback) -> None:
        self._callbacks.append(callback)

    def remove_callback(self, callback) -> None:
        try:
            self._callbacks.remove(callback)
        except ValueError:
            pass

    def clear_callbacks(self) -> None:
        self._callbacks.clear()

    @property
    def _global_norm_ema(self) -> float:
        if self._plan is None:
            return self._gema
        if self._host_norms:
            return self._gema
        return float(self._plan.global_norm_ema.item())

    def collect_metrics(self) -> dict:
        """The callback metrics of optimizer.py:492-499: scao.logging's
        collect_metrics plus the noise level, the global grad-norm EMA and the
        warmup flag."""
        from .logging import collect_metrics
        m = collect_metrics(self)
        m["noise_std"] = self._noise_std
        m["global_norm_ema"] = self._global_norm_ema
        m["warmup_active"] = self._in_warmup_global
        return m

    def current_ranks(self) -> dict:
        return {idx: st["preconditioner"].k for idx, st in enumerate(self.state.values())
                if "preconditioner" in st}

    def precond_stats(self) -> dict:
        ks = list(self.current_ranks().values())
        if not ks:
            return {}
        return {"num_precond_layers": len(ks), "rank_min": min(ks), "rank_max": max(ks),
                "rank_mean": sum(ks) / len(ks), "global_norm_ema": self._global_norm_ema,
                "warmup_exited_early": self._warmup_scheduler.exited_early,
                "actual_warmup_steps": self._warmup_scheduler.actual_warmup_steps}

    def synchronize_precond(self) -> None:
        """Single-stream implementation: nothing is pending on a side stream."""
        return None

    def sync_preconditioner(self, process_group=None) -> None:
        """optimizer.py:686-710: broadcast the moments, step counters and
        preconditioner state of rank 0 to every rank (after a checkpoint was
        loaded on rank 0 only)."""
        import warnings

        import torch.distributed as dist
        if not dist.is_available() or not dist.is_initialized():
            warnings.warn("sync_preconditioner() called but distributed is not initialised.",
                          RuntimeWarning, stacklevel=2)
            return
        if self._plan is None:
            return
        ps, _ = self._flat()
        broadcast_plan_state(self._plan, [self.state[p] for p in ps], process_group)

    # ------------------------------------------------------------------
    # checkpoint (optimizer.py:732-776)
    # ------------------------------------------------------------------
    def state_dict(self) -> dict:
        ps, _ = self._flat()
        index = {id(p): i for i, p in enumerate(ps)}
        packed = {}
        precond = {}
        for p, st in self.state.items():
            i = index[id(p)]
            d = {}
            for k, v in st.items():
                if k == "preconditioner":
                    continue
                d[k] = v.clone() if torch.is_tensor(v) else v
            packed[i] = d
            if "preconditioner" in st:
                precond[i] = st["preconditioner"].state_dict()
        groups = []
        for g in self.param_groups:
            gg = {k: v for k, v in g.items() if k != "params"}
            gg["params"] = [index[id(p)] for p in g["params"]]
            groups.append(gg)
        return {
            "state": packed,
            "param_groups": groups,
            "_scao_precond": precond,
            "_scao_runtime": {
                "global_step": self._global_step,
                "noise_std": self._noise_std,
                "global_norm_ema": self._global_norm_ema,
                "warmup_prev_norm": self._warmup_scheduler._prev_norm,
                "warmup_stable_count": self._warmup_scheduler._stable_count,
                "warmup_early_exit_step": self._warmup_scheduler._early_exit_step,
            },
        }

    def load_state_dict(self, state_dict: dict) -> None:
        state_dict = dict(state_dict)
        extra = state_dict.pop("_scao_precond", {})
        runtime = state_dict.pop("_scao_runtime", {})
        for g, sg in zip(self.param_groups, state_dict["param_groups"]):
            for k, v in sg.items():
                if k != "params":
                    g[k] = v
        if self._plan is None:
            self._build_plan()
        ps, _ = self._flat()
        for i, p in enumerate(ps):
            if i not in state_dict["state"]:
                continue
            src = state_dict["state"][i]
            st = self.state[p]
            for k, v in src.items():
                if k == "preconditioner":
                    continue
                if torch.is_tensor(v) and k in st and torch.is_tensor(st[k]):
                    st[k].copy_(v)
                else:
                    st[k] = v
            if i in extra:
                st["preconditioner"].load_state_dict(extra[i])
        if runtime:
            self._global_step = int(runtime.get("global_step", self._global_step))
            self._noise_std = float(runtime.get("noise_std", self._noise_std))
            if "global_norm_ema" in runtime:
                self._gema = float(runtime["global_norm_ema"])
                self._plan.global_norm_ema.fill_(self._gema)
            ws = self._warmup_scheduler
            ws._prev_norm = float(runtime.get("warmup_prev_norm", ws._prev_norm))
            ws._stable_count = int(runtime.get("warmup_stable_count", ws._stable_count))
            ws._early_exit_step = runtime.get("warmup_early_exit_step", ws._early_exit_step)
        self._lookahead_init = False


def _recip32(c):
    """RN(1/c) in float32 (c rounded to float32 first, as the kernels see it)."""
    return float(np.float32(1.0) / np.float32(c))


def _in_param_dtypes(norms, params):
    """float32 values rounded (RNE) to each parameter's dtype."""
    out = np.asarray(norms, np.float32).copy()
    for dt in {p.dtype for p in params} - {torch.float32}:
        idx = [i for i, p in enumerate(params) if p.dtype == dt]
        out[idx] = torch.from_numpy(out[idx]).to(dt).float().numpy()
    return out


def C_stream(stream):
    return stream.cuda_stream


def broadcast_plan_state(plan, states, group=None):
    """Rank 0's optimizer state onto every rank, in place: the moment arenas
    (exp_avg, exp_avg_sq, exp_avg_diff -- prev_grad is not synchronised, as in
    the reference), each parameter's ``step`` and ``precond_step``, and the
    preconditioner arenas (factors and their absmax, eigenvectors and their
    bf16 operand tiles, eigenvalues, ranks, diagonal EMA)
    (optimizer.py:686-710, preconditioner.py:647-720)."""
    import torch.distributed as dist
    for t in (plan.exp_avg, plan.exp_avg_sq, plan.exp_avg_diff):
        dist.broadcast(t, src=0, group=group)
    counters = torch.tensor([[st.get("step", 0), st["preconditioner"].precond_step]
                             for st in states], dtype=torch.int64, device=plan.device)
    dist.broadcast(counters, src=0, group=group)
    for st, (step, pstep) in zip(states, counters.tolist()):
        st["step"] = int(step)
        st["preconditioner"].precond_step = int(pstep)
    for t in (plan.fac, plan.absmax, plan.u, plan.ev, plan.k, plan.diag_ema, plan.ua, plan.ut):
        dist.broadcast(t, src=0, group=group)
