"""Seeded low-rank-plus-noise gradient generator for the benchmark workloads.

For every 2-D parameter of shape (m, n) the gradient at step t is

    G_t = U_t diag(s) V_t^T + 1e-4 * N(0, 1)

with s_i = 1e-2 * decay**i (i < rank), U_0 / V_0 sign-fixed QR factors of
Gaussian matrices, and a slow drift U_{t+1} = qr(U_t + 0.01 Z_t),
Z_t ~ N(0, 1/m) (same for V).  1-D parameters get 1e-4 * N(0, 1).  Every
draw is made in float64 from a torch.Generator seeded by (seed, param index,
step) and cast to the parameter dtype at the end.  Parameters are initialised
N(0, 0.02^2) from the seed.

The generator runs on CPU for parity tests (identical tensors are then fed to
the oracle and to the GPU path) and on the GPU for benchmarks.
"""
from __future__ import annotations

import torch

_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16,
           "float16": torch.float16}


def torch_dtype(name):
    return _DTYPES[name] if isinstance(name, str) else name


def _gen(device, *key):
    s = 0
    for k in key:
        s = (s * 1_000_003 + int(k) + 1) % (2 ** 62)
    g = torch.Generator(device=device)
    g.manual_seed(s)
    return g


def _signfix_qr(a):
    q, r = torch.linalg.qr(a)
    d = torch.sign(torch.diagonal(r))
    d[d == 0] = 1.0
    return q * d.unsqueeze(0)


def init_params(workload, seed=0, device="cpu"):
    """N(0, 0.02^2) parameter tensors for a workload, in its dtype."""
    out = []
    for i, spec in enumerate(workload.params):
        g = _gen(device, seed, 7, i)
        x = torch.randn(spec.shape, generator=g, device=device, dtype=torch.float64) * 0.02
        out.append(x.to(param_dtype(workload, i)))
    return out


def param_dtype(workload, i):
    """torch dtype of parameter i (its own, else the workload's)."""
    return torch_dtype(workload.params[i].dtype or workload.param_dtype)


class LowRankGradients:
    """Stateful generator: ``next()`` returns the list of gradients of step t."""

    def __init__(self, workload, seed=0, device="cpu", noise=1e-4, s0=None,
                 drift=0.01):
        if s0 is None:
            s0 = workload.grad_scale
        self.w = workload
        self.seed = seed
        self.device = torch.device(device)
        self.noise = noise
        self.drift = drift
        self.dtype = torch_dtype(workload.param_dtype)
        self.t = 0
        r = workload.grad_rank
        self.s = s0 * workload.grad_decay ** torch.arange(
            r, dtype=torch.float64, device=self.device)
        self.UV = []
        for i, spec in enumerate(workload.params):
            if len(spec.shape) < 2:
                self.UV.append(None)
                continue
            # parameters of 3+ dims get the low-rank gradient of their (d0, rest) view
            m, n = spec.shape[0], int(torch.Size(spec.shape[1:]).numel())
            rr = min(r, m, n)
            g = _gen(self.device, seed, 11, i)
            U = _signfix_qr(torch.randn(m, rr, generator=g, device=self.device,
                                        dtype=torch.float64))
            V = _signfix_qr(torch.randn(n, rr, generator=g, device=self.device,
                                        dtype=torch.float64))
            self.UV.append([U, V])

    def next(self):
        t = self.t
        grads = []
        for i, spec in enumerate(self.w.params):
            g = _gen(self.device, self.seed, 13, i, t)
            if self.UV[i] is None:
                x = torch.randn(spec.shape, generator=g, device=self.device,
                                dtype=torch.float64) * self.noise
                grads.append(x.to(param_dtype(self.w, i)))
                continue
            U, V = self.UV[i]
            rr = U.shape[1]
            x = (U * self.s[:rr].unsqueeze(0)) @ V.T
            x += torch.randn(x.shape, generator=g, device=self.device,
                             dtype=torch.float64) * self.noise
            if self.w.grad_scales is not None:
                x *= self.w.grad_scales[i]
            grads.append(x.reshape(spec.shape).to(param_dtype(self.w, i)))
            m, n = x.shape
            zu = torch.randn(U.shape, generator=g, device=self.device,
                             dtype=torch.float64) / m ** 0.5
            zv = torch.randn(V.shape, generator=g, device=self.device,
                             dtype=torch.float64) / n ** 0.5
            self.UV[i] = [_signfix_qr(U + self.drift * zu),
                          _signfix_qr(V + self.drift * zv)]
        self.t += 1
        return grads
