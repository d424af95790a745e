"""``scao.SparsePreconditioner`` for a single tensor (scao/preconditioner.py:72-644).

The reference exports its per-parameter preconditioner for standalone use:
``update_curvature(grad)`` accumulates the Kronecker factors (or the diagonal
EMA) and refreshes the low-rank eigenfactors, ``precondition(grad)`` returns
the preconditioned gradient, ``natural_grad_norm(grad)`` the curvature-aware
norm.  Here one such object owns a one-parameter plan: its factors live in
the same device arenas, and curvature, eigen update and the Kronecker
correction run through the library's C ABI (``scao_plan_curvature``,
``scao_plan_curvature_diag``, ``scao_plan_eigen``,
``scao_fused_kronecker_precond``) -- the kernels the optimizer step uses.
The diagonal blocks' elementwise formula and the k x k projection of
``natural_grad_norm`` are small tensor expressions on the device.

CUDA tensors only: construction works anywhere (the checkpoint schema can be
inspected on the host), the compute methods raise on a CPU tensor.  The
kernels read gradients in the parameter's dtype: a float32 gradient passed for
a bf16 parameter is rounded to bf16 first (the reference takes it as float32).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .plan import Plan
from .preconditioner import LeafView, PrecondView, StripView

_EIG_MAX_ITERS = 30      # the optimizer's defaults (SCAO(eig_max_iters, eig_tol))
_EIG_TOL = 5e-4


class SparsePreconditioner(PrecondView):
    """Same constructor and methods as the reference class; ``use_newton_schulz``
    is accepted and, as in the reference, has no effect on the result."""

    def __init__(self, param, epsilon_sparse: float = 0.05, k_min: int = 8, k_max: int = 128,
                 rho: float = 0.999, max_precond_dim: int = 4096,
                 use_newton_schulz: bool = False, use_int8_ema: bool = False):
        p = param.detach()
        if not p.is_contiguous():
            p = p.contiguous()
        group = dict(epsilon_sparse=epsilon_sparse, k_min=k_min, k_max=k_max, rho=rho,
                     max_precond_dim=max_precond_dim)
        if p.device.type == "cuda":
            _lib.lib()
            with torch.cuda.device(p.device):      # the plan launches on its device
                plan = Plan([p], [group], p.device, bool(use_int8_ema))
        else:
            plan = Plan([p], [group], p.device, bool(use_int8_ema))
        super().__init__(plan, 0, group)
        self.epsilon_sparse = epsilon_sparse
        self.use_newton_schulz = use_newton_schulz
        self.param_dtype = p.dtype
        self.device = p.device
        self.k_min, self.k_max = (self._ktree[0], self._ktree[1]) if self._ktree else (1, 1)
        if self.use_block_diagonal:
            large = max(self.m, self.n)
            self._block_dim = 0 if self.m >= self.n else 1
            self._block_sizes = [max_precond_dim] * (large // max_precond_dim) + \
                ([large % max_precond_dim] if large % max_precond_dim else [])
        self._scratch = None
        self._keep = None

    # ------------------------------------------------------------------
    def _cuda(self, t):
        if self.device.type != "cuda" or t.device != self.device:
            raise RuntimeError("scao_b200.SparsePreconditioner computes on the CUDA device of "
                               "its parameter (no CPU path)")

    def _grad2d(self, grad):
        return grad.detach().reshape(self.m, self.n)

    @torch.no_grad()
    def update_curvature(self, grad):
        """preconditioner.py:297-361: factor EMAs (int8 or fp32) and the eigen
        update of every Kronecker block, the diagonal EMA of the others."""
        self._cuda(grad)
        with torch.cuda.device(self.device):
            self._update_curvature(grad)

    def _update_curvature(self, grad):
        plan = self.plan
        L = _lib.lib()
        # the kernels read the gradient in the parameter dtype
        g = grad.detach().to(self.param_dtype).contiguous()
        stream = torch.cuda.current_stream(self.device)
        sp = stream.cuda_stream
        if plan.step_event is not None:
            plan.step_event.synchronize()
        row = plan.step_np[0]
        row["g_ptr"] = g.data_ptr()
        row["p_ptr"] = g.data_ptr()
        row["phase"] = 1
        plan.t_step.copy_(plan.step_host, non_blocking=True)
        plan.step_event = torch.cuda.Event()
        plan.step_event.record(stream)
        self.precond_step += 1
        import ctypes
        pd = ctypes.byref(plan.dev)
        leaves = plan.param_leaves[0]
        if leaves:
            ids_h = np.ascontiguousarray(leaves, dtype=np.int32)
            ids = plan.dev_ids(ids_h)
            ma, mb, smax = plan.max_dims(leaves)
            need = int(L.scao_ema_scratch_bytes(len(leaves), ma, mb))
            if self._scratch is None or self._scratch.numel() < need:
                self._scratch = torch.empty(need, dtype=torch.uint8, device=self.device)
            _lib.check(L.scao_plan_curvature(pd, ids.data_ptr(), len(leaves), ma, mb, self.rho,
                                             self._scratch.data_ptr(), self._scratch.numel(),
                                             plan.ptab.ctypes.data, plan.step_host.data_ptr(),
                                             plan.ltab.ctypes.data, ids_h.ctypes.data, sp),
                       "scao_plan_curvature")
        if not leaves or plan.param_strips[0]:
            ids0 = plan.dev_ids(np.zeros(1, np.int32))
            _lib.check(L.scao_plan_curvature_diag(pd, ids0.data_ptr(), 1, self.rho, sp),
                       "scao_plan_curvature_diag")
        if leaves:
            bias = plan.upload_bias(ids_h, [1.0 - self.rho ** self.precond_step] * len(leaves))
            status = plan.eig_status[: 2 * len(leaves)]
            _lib.check(L.scao_plan_eigen(pd, ids.data_ptr(), len(leaves), bias.data_ptr(),
                                         plan.t_eps_sparse.data_ptr(), _EIG_MAX_ITERS, _EIG_TOL,
                                         status.data_ptr(), max(ma, mb), smax, sp),
                       "scao_plan_eigen")
        self._keep = g          # alive until the next call (stream-ordered reuse)

    def _leaf_factors(self, v):
        """(U_l, S_l, U_r, S_r) of a leaf, the reference's initial eye / ones
        before the first eigen update."""
        k = v.k
        if self.precond_step == 0:
            dev = self.device
            return (torch.eye(v.m, k, device=dev), torch.ones(k, device=dev),
                    torch.eye(v.n, k, device=dev), torch.ones(k, device=dev))
        return (v._u(0, k).contiguous(), v._s(0, k).clone(),
                v._u(1, k).contiguous(), v._s(1, k).clone())

    def _block(self, v):
        """Slices of the 2-D gradient covered by a leaf or strip view."""
        if isinstance(v, LeafView):
            Lr = self.plan.ltab[v.li]
            r0, c0 = int(Lr["row0"]), int(Lr["col0"])
            return slice(r0, r0 + v.m), slice(c0, c0 + v.n)
        r0, c0 = divmod(v.begin, self.n)
        return slice(r0, r0 + v.m), slice(c0, c0 + v.n)

    def _diag_out(self, g, d):
        """preconditioner.py:506-510."""
        return g / (d / self.diag_bias).pow(0.25).add_(1e-8)

    @torch.no_grad()
    def precondition(self, grad):
        """preconditioner.py:457-521: every block in float32, reassembled,
        returned in the gradient's dtype."""
        self._cuda(grad)
        with torch.cuda.device(self.device):
            return self._precondition(grad)

    def _precondition(self, grad):
        g2 = self._grad2d(grad).to(torch.float32)
        if not self._views:                                 # diagonal parameter
            return self._diag_out(g2, self.diag_ema.reshape(self.m, self.n)) \
                .reshape(grad.shape).to(grad.dtype)
        out = g2.clone()
        L = _lib.lib()
        sp = torch.cuda.current_stream(self.device).cuda_stream
        for v in self._views:
            rs, cs = self._block(v)
            if isinstance(v, StripView):
                out[rs, cs] = self._diag_out(g2[rs, cs], v.diag_ema)
                continue
            if self.precond_step == 0:
                continue          # U = eye, S = 1: the correction is exactly zero
            Ul, Sl, Ur, Sr = self._leaf_factors(v)
            k = Ul.shape[1]
            blk = g2[rs, cs].contiguous()
            res = torch.empty_like(blk)
            s4l = Sl.clamp(min=1e-8).pow(-0.25)
            s4r = Sr.clamp(min=1e-8).pow(-0.25)
            scratch = torch.empty(int(L.scao_fused_precond_scratch_bytes(v.m, v.n, k)),
                                  dtype=torch.uint8, device=self.device)
            _lib.check(L.scao_fused_kronecker_precond(Ul.data_ptr(), s4l.data_ptr(),
                                                      Ur.data_ptr(), s4r.data_ptr(),
                                                      blk.data_ptr(), res.data_ptr(), 0,
                                                      v.m, v.n, k, scratch.data_ptr(), sp),
                       "scao_fused_kronecker_precond")
            out[rs, cs] = res
        return out.reshape(grad.shape).to(grad.dtype)

    @torch.no_grad()
    def natural_grad_norm(self, grad, eps: float = 1e-8):
        """preconditioner.py:527-564: ||diag(S_l^-1/2) U_l^T G U_r diag(S_r^-1/2)||_F
        per Kronecker block, sqrt(sum g^2 / (sqrt(diag_ema) + eps)) per diagonal
        block, block-diagonal levels as sqrt of the sum of squares."""
        self._cuda(grad)
        g2 = self._grad2d(grad).to(torch.float32)
        if not self._views:
            d = self.diag_ema.reshape(self.m, self.n)
            return (g2.pow(2) / d.pow(0.5).add_(eps)).sum().sqrt()

        def node(x):
            if isinstance(x, list) or hasattr(x, "_blocks"):
                kids = x if isinstance(x, list) else x._blocks
                return torch.stack([node(c).pow(2) for c in kids]).sum().sqrt()
            rs, cs = self._block(x)
            gb = g2[rs, cs]
            if isinstance(x, StripView):
                return (gb.pow(2) / x.diag_ema.pow(0.5).add_(eps)).sum().sqrt()
            Ul, Sl, Ur, Sr = self._leaf_factors(x)
            P = (Ul.T @ gb) @ Ur
            return (Sl.clamp(min=eps).pow(-0.5).unsqueeze(1) * P *
                    Sr.clamp(min=eps).pow(-0.5).unsqueeze(0)).norm(p="fro")

        return node(self._blocks if self.use_block_diagonal else self._views[0])

    def memory_bytes(self) -> int:
        """preconditioner.py:602-619."""
        def one(v):
            if isinstance(v, StripView):
                return v.count * 4
            if hasattr(v, "_blocks"):
                return sum(one(c) for c in v._blocks)
            k = v.k
            fac = (v.m * v.m + 8 + v.n * v.n + 8) if self.use_int8_ema \
                else 4 * (v.m * v.m + v.n * v.n)
            return fac + 4 * (v.m * k + k + v.n * k + k)

        if not self._views:
            return self.m * self.n * 4
        return sum(one(c) for c in (self._blocks if self.use_block_diagonal else self._views))
