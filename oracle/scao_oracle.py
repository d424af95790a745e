"""CPU oracle for the SCAO optimizer step -- TEST INFRASTRUCTURE ONLY.

This module restates, in float32 numpy, the reference algorithm of
whispering3/scao for the optimizer-step hot path.  It exists to check the CUDA
implementation in ``scao_b200``: only the test-suite, ``__graft_entry__.smoke``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
it.  The product path never calls into this file.

Every function cites the reference file:line it follows (paths relative to the
reference project root).  Its outputs are pinned against golden vectors
produced by running the reference package itself
(``tests/golden/make_golden.py`` -> ``tests/golden/*.npz``).

Rounding points that the reference has and that matter for exact parity:
  * the int8 requant uses true IEEE division x / float32(scale) and
    round-half-even (``utils.py:187-188``), scale = float64(absmax) / 127;
  * bf16 / fp16 parameters round after every parameter-dtype op
    (``optimizer.py:549, 645``) and after ``precondition`` (``preconditioner.py:521``);
  * the LARS ``p.norm()`` is a parameter-dtype 0-dim tensor (``optimizer.py:373``).
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------
# parameter-dtype emulation
# ---------------------------------------------------------------------------

def round_bf16(x):
    """Round float32 values to the nearest bfloat16 (ties to even)."""
    x = np.ascontiguousarray(x, dtype=F32)
    b = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    lsb = (b >> 16) & 1
    b = (b + 0x7FFF + lsb) & 0xFFFF0000
    out = b.astype(np.uint32).view(F32).copy()
    out[nan] = np.nan
    return out


def round_to(x, dtype):
    """Cast float32 array ``x`` to the parameter dtype and back."""
    if dtype == "float32":
        return np.asarray(x, dtype=F32)
    if dtype == "bfloat16":
        return round_bf16(x)
    if dtype == "float16":
        return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)
    raise ValueError(dtype)


def fma(a, b, c):
    """float32 a*b + c with one rounding (torch CPU ``add_(x, alpha=)`` and
    ``addcmul_`` contract to a fused multiply-add)."""
    r = np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)
    return r.astype(F32)


def add_alpha(p, x, alpha, dtype):
    """``p.add_(x, alpha=alpha)`` in the parameter dtype: torch casts alpha to
    the tensor dtype first and evaluates with a fused multiply-add."""
    a = F32(round_to(np.array([alpha], F32), dtype)[0])
    return round_to(fma(a, x, p), dtype)


def norm_dt(x, dtype):
    """float(t.norm()) of a tensor of that dtype: torch accumulates in float32
    and returns the norm in the tensor's own dtype (rounded for bf16 / fp16)."""
    return float(round_to(np.array([norm_f32(x)], F32), dtype)[0])


def norm_f32(x):
    """Frobenius norm with float32 output (torch ``Tensor.norm``)."""
    x = np.asarray(x, dtype=F32)
    return F32(np.sqrt(np.sum(np.square(x, dtype=np.float64))))


# ---------------------------------------------------------------------------
# utils.py
# ---------------------------------------------------------------------------

def quantize_sym_int8(x):
    """utils.py:170-189.  Returns (int8 q, python-float scale)."""
    x = np.asarray(x, dtype=F32)
    abs_max = float(np.max(np.abs(x))) if x.size else 0.0
    if abs_max < 1e-30:
        return np.zeros(x.shape, np.int8), 1.0
    scale = abs_max / 127.0
    q = np.clip(np.rint(x / F32(scale)), -127, 127).astype(np.int8)
    return q, scale


def dequantize_sym_int8(q, scale):
    """utils.py:192-203."""
    return q.astype(F32) * F32(scale)


def adaptive_rank(eigenvalues, epsilon=0.05, k_min=4, k_max=128):
    """utils.py:121-151 (eigenvalues descending, float32)."""
    ev = np.asarray(eigenvalues, dtype=F32)
    total = float(np.sum(ev, dtype=F32))
    if total < 1e-12:
        return k_min
    threshold = (1.0 - epsilon) * total
    # torch's CPU cumsum accumulates in float64 and rounds each prefix
    cumsum = np.cumsum(ev.astype(np.float64)).astype(F32)
    idx = np.nonzero(cumsum >= F32(threshold))[0]
    k = int(idx[0]) + 1 if idx.size > 0 else len(ev)
    return int(min(k_max, max(k_min, k)))


def to_2d(g):
    """utils.py:208-219."""
    if g.ndim == 1:
        return g.reshape(1, -1)
    if g.ndim == 2:
        return g
    return g.reshape(g.shape[0], -1)


# ---------------------------------------------------------------------------
# preconditioner.py
# ---------------------------------------------------------------------------

class OraclePreconditioner:
    """preconditioner.py:72-644 (SparsePreconditioner), numpy float32."""

    def __init__(self, shape, epsilon_sparse=0.05, k_min=8, k_max=128,
                 rho=0.999, max_precond_dim=4096, use_int8_ema=False):
        # preconditioner.py:108-124
        shape = tuple(shape)
        ndim = len(shape)
        if ndim == 1:
            m, n = 1, shape[0]
        elif ndim == 2:
            m, n = shape
        else:
            m, n = shape[0], int(np.prod(shape[1:]))
        self.shape, self.m, self.n = shape, m, n
        self.epsilon_sparse = epsilon_sparse
        d_min = min(m, n)
        self.k_min = min(k_min, d_min)
        self.k_max = min(k_max, d_min // 2) if d_min > 2 * self.k_min else self.k_min
        self.rho = rho
        self.use_int8_ema = use_int8_ema
        # preconditioner.py:142-153
        self.use_block_diagonal = ndim >= 2 and m > 1 and n > 1 and max(m, n) > max_precond_dim
        self.use_kronecker = ndim >= 2 and m > 1 and n > 1 and max(m, n) <= max_precond_dim
        if self.use_block_diagonal:
            # preconditioner.py:163-194
            large, small = (m, n) if m >= n else (n, m)
            self.block_dim = 0 if m >= n else 1
            bs = max_precond_dim
            self.block_sizes = [bs] * (large // bs) + ([large % bs] if large % bs else [])
            self.blocks = []
            for b in self.block_sizes:
                fake = (b, small) if self.block_dim == 0 else (small, b)
                self.blocks.append(OraclePreconditioner(
                    fake, epsilon_sparse, k_min, k_max, rho, max_precond_dim,
                    use_int8_ema))
            self.k = self.blocks[0].k
        elif self.use_kronecker:
            # preconditioner.py:196-231
            k_init = min(k_min, min(m, n))
            self.k = k_init
            L0 = np.eye(m, dtype=F32) * F32(1e-4)
            R0 = np.eye(n, dtype=F32) * F32(1e-4)
            if use_int8_ema:
                self.L_q, self.L_scale = quantize_sym_int8(L0)
                self.R_q, self.R_scale = quantize_sym_int8(R0)
            else:
                self.L, self.R = L0, R0
            self.U_l = np.eye(m, k_init, dtype=F32)
            self.S_l = np.ones(k_init, F32)
            self.U_r = np.eye(n, k_init, dtype=F32)
            self.S_r = np.ones(k_init, F32)
        else:
            # preconditioner.py:232-236
            self.diag_ema = np.zeros(shape, F32)
            self.diag_bias = 1e-8
            self.k = 1
        self.precond_step = 0

    # -- iteration over leaf blocks (row/col slices of the 2-D gradient) ---
    def _slices(self):
        off = 0
        for bs, blk in zip(self.block_sizes, self.blocks):
            sl = (slice(off, off + bs), slice(None)) if self.block_dim == 0 else \
                 (slice(None), slice(off, off + bs))
            yield sl, blk
            off += bs

    def update_curvature(self, grad):
        """preconditioner.py:297-361."""
        self.precond_step += 1
        g = to_2d(np.asarray(grad, dtype=F32))
        if self.use_block_diagonal:
            for sl, blk in self._slices():
                blk.update_curvature(np.ascontiguousarray(g[sl]))
            self.k = sum(b.k for b in self.blocks) // max(len(self.blocks), 1)
            return
        if not self.use_kronecker:
            sq = g.reshape(self.diag_ema.shape)
            self.diag_ema = self.diag_ema * F32(self.rho) + (F32(1.0 - self.rho) * (sq * sq))
            self.diag_bias = max(1.0 - self.rho ** self.precond_step, 1e-8)
            return
        alpha = F32(1.0 - self.rho)
        rho = F32(self.rho)
        if self.use_int8_ema:
            L = dequantize_sym_int8(self.L_q, self.L_scale) * rho + alpha * (g @ g.T)
            self.L_q, self.L_scale = quantize_sym_int8(L)
            R = dequantize_sym_int8(self.R_q, self.R_scale) * rho + alpha * (g.T @ g)
            self.R_q, self.R_scale = quantize_sym_int8(R)
        else:
            self.L = self.L * rho + alpha * (g @ g.T)
            self.R = self.R * rho + alpha * (g.T @ g)
        self._update_eigenfactors(1.0 - self.rho ** self.precond_step)

    def factor_matrices(self, bias_factor):
        """L_reg, R_reg of preconditioner.py:383-406 (debias + Tikhonov)."""
        eps = 1e-8
        if self.use_int8_ema:
            L = dequantize_sym_int8(self.L_q, self.L_scale)
            R = dequantize_sym_int8(self.R_q, self.R_scale)
        else:
            L, R = self.L, self.R
        L = L / F32(max(bias_factor, eps))
        R = R / F32(max(bias_factor, eps))
        eps_l = max(eps, 1e-4 * float(np.trace(L, dtype=F32)) / self.m)
        eps_r = max(eps, 1e-4 * float(np.trace(R, dtype=F32)) / self.n)
        L = L.copy()
        R = R.copy()
        L[np.diag_indices(self.m)] += F32(eps_l)
        R[np.diag_indices(self.n)] += F32(eps_r)
        return L, R

    def _update_eigenfactors(self, bias_factor):
        """preconditioner.py:363-451."""
        L_reg, R_reg = self.factor_matrices(bias_factor)
        S_l, U_l = np.linalg.eigh(L_reg)
        S_r, U_r = np.linalg.eigh(R_reg)
        S_l = np.clip(S_l[::-1], 0.0, None).astype(F32)
        U_l = U_l[:, ::-1]
        S_r = np.clip(S_r[::-1], 0.0, None).astype(F32)
        U_r = U_r[:, ::-1]
        self.S_l_full, self.S_r_full = S_l, S_r
        k_l = adaptive_rank(S_l, self.epsilon_sparse, self.k_min, self.k_max)
        k_r = adaptive_rank(S_r, self.epsilon_sparse, self.k_min, self.k_max)
        k_new = min(k_l, k_r)
        k_new = max(k_new, self.k - 1)
        k_new = min(k_new, self.k + 4)
        k_new = int(min(self.k_max, max(self.k_min, k_new)))
        self.k = k_new
        self.U_l = np.ascontiguousarray(U_l[:, :k_new], dtype=F32)
        self.S_l = np.ascontiguousarray(S_l[:k_new])
        self.U_r = np.ascontiguousarray(U_r[:, :k_new], dtype=F32)
        self.S_r = np.ascontiguousarray(S_r[:k_new])

    def precondition(self, grad, dtype="float32"):
        """preconditioner.py:457-521 + cuda/__init__.py:95-99 (fp32 result
        before the final cast; the caller rounds to the parameter dtype)."""
        g = to_2d(np.asarray(grad, dtype=F32))
        if self.use_block_diagonal:
            out = np.zeros_like(g)
            for sl, blk in self._slices():
                out[sl] = blk.precondition(np.ascontiguousarray(g[sl]))
            return round_to(out.reshape(self.shape), dtype)
        if not self.use_kronecker:
            denom = np.power(self.diag_ema / F32(self.diag_bias), F32(0.25)).reshape(g.shape) + F32(1e-8)
            return round_to((g / denom).reshape(self.shape), dtype)
        s_l = np.power(np.maximum(self.S_l, F32(1e-8)), F32(-0.25))
        s_r = np.power(np.maximum(self.S_r, F32(1e-8)), F32(-0.25))
        P = (self.U_l.T @ g) @ self.U_r
        delta = (s_l[:, None] * s_r[None, :] - F32(1.0)) * P
        out = g + (self.U_l @ delta) @ self.U_r.T
        return round_to(out.reshape(self.shape), dtype)

    def natural_grad_norm(self, grad, eps=1e-8):
        """preconditioner.py:527-564 (float32 scalar)."""
        g = to_2d(np.asarray(grad, dtype=F32))
        if self.use_block_diagonal:
            sq = [F32(blk.natural_grad_norm(np.ascontiguousarray(g[sl]), eps)) ** 2
                  for sl, blk in self._slices()]
            return F32(np.sqrt(np.sum(np.array(sq, F32), dtype=F32)))
        if not self.use_kronecker:
            denom = np.sqrt(self.diag_ema).reshape(g.shape) + F32(eps)
            return F32(np.sqrt(np.sum(g * g / denom, dtype=F32)))
        s_l = np.power(np.maximum(self.S_l, F32(eps)), F32(-0.5))
        s_r = np.power(np.maximum(self.S_r, F32(eps)), F32(-0.5))
        P = (self.U_l.T @ g) @ self.U_r
        return norm_f32(s_l[:, None] * P * s_r[None, :])

    def set_k(self, new_k):
        """R5 rank assignment, preconditioner.py:249-291: clamp to
        [k_min, k_max]; a decrease truncates the eigenfactors, an increase is
        clamped to their current width (so it waits for the next eigen
        update); block-diagonal: every block, then the integer mean."""
        new_k = int(min(self.k_max, max(self.k_min, new_k)))
        if self.use_block_diagonal:
            for b in self.blocks:
                b.set_k(new_k)
            self.k = sum(b.k for b in self.blocks) // max(len(self.blocks), 1)
            return
        if self.use_kronecker:
            if new_k < self.k:
                self.U_l = np.ascontiguousarray(self.U_l[:, :new_k])
                self.S_l = np.ascontiguousarray(self.S_l[:new_k])
                self.U_r = np.ascontiguousarray(self.U_r[:, :new_k])
                self.S_r = np.ascontiguousarray(self.S_r[:new_k])
            elif new_k > self.k:
                cols = self.U_l.shape[1]
                new_k = min(new_k, cols) if new_k > cols else new_k
        self.k = new_k

    def leaves(self):
        """Leaf preconditioners in block order (self for non-split)."""
        if self.use_block_diagonal:
            out = []
            for b in self.blocks:
                out += b.leaves()
            return out
        return [self]


# ---------------------------------------------------------------------------
# optimizer.py
# ---------------------------------------------------------------------------

# ---------------------------------------------------------------------------
# gradient filter (optimizer.py:40-97)
# ---------------------------------------------------------------------------

QUANTILE_CAP = 1 << 24   # torch.quantile refuses larger inputs


def quantile_f32(x, q):
    """``torch.quantile(x, q)`` (linear interpolation) for a float32 vector,
    as ATen computes it: rank = float32(q) * (n - 1) in float32, the two
    neighbouring order statistics, and ``lerp`` with the weight
    rank - floor(rank) (fused multiply-add form, weight < 0.5 from below).
    Any NaN gives NaN.  Beyond torch's 2^24-element cap (where the reference
    raises) the rank is formed in float64 instead."""
    x = np.ascontiguousarray(x, dtype=F32).ravel()
    n = x.size
    if n == 0:
        return F32(np.nan)
    if np.isnan(x).any():
        return F32(np.nan)
    if n <= QUANTILE_CAP:
        rank = F32(F32(q) * F32(n - 1))
        lo = int(math.floor(rank))
        w = F32(rank - F32(lo))
    else:
        rank = float(F32(q)) * (n - 1)
        lo = int(math.floor(rank))
        w = F32(rank - lo)
    hi = min(lo + (1 if w > 0 else 0), n - 1)
    part = np.partition(x, (lo, hi)) if hi != lo else np.partition(x, lo)
    a, b = part[lo], part[hi]
    return lerp_f32(a, b, w)


def lerp_f32(a, b, w):
    """ATen ``lerp`` (Lerp.h) with its multiply-add contracted: exact
    products in float64, one rounding to float32."""
    a, b, w = F32(a), F32(b), F32(w)
    d = F32(b - a)
    if abs(w) < 0.5:
        return F32(float(w) * float(d) + float(a))
    return F32(float(b) - float(d) * float(F32(F32(1.0) - w)))


class OracleSparseFilter:
    """``_SparseGradFilter`` (optimizer.py:40-56) and, with ``dynamic``,
    ``_DynamicSparseFilter`` (:59-97)."""

    def __init__(self, sparsity=0.7, dynamic=False, ema=0.99, min_sparsity=0.3,
                 max_sparsity=0.9, norm_ema=0.95):
        self.base = sparsity
        self.sparsity = sparsity
        self.dynamic = dynamic
        self.ema = ema
        self.min_s, self.max_s, self.norm_coeff = min_sparsity, max_sparsity, norm_ema
        self.norm_ema = 1.0
        self.global_ref = 1.0
        self.mag = None

    def set_global_norm_ref(self, g):
        self.global_ref = max(g, 1e-8)

    def __call__(self, grad):
        if self.dynamic:
            layer = float(norm_f32(grad))        # grad = p.grad.float() (optimizer.py:531)
            self.norm_ema = self.norm_coeff * self.norm_ema + (1.0 - self.norm_coeff) * layer
            ratio = self.norm_ema / self.global_ref
            margin = 0.2 * (1.0 - min(ratio, 2.0) / 2.0)
            self.sparsity = float(max(self.min_s, min(self.max_s, self.base + margin)))
        mag = np.abs(grad).astype(F32)
        if self.mag is None:
            self.mag = mag.copy()
        else:
            self.mag = (self.mag * F32(self.ema)) + F32(1.0 - self.ema) * mag
        thr = quantile_f32(self.mag, self.sparsity)
        return grad * (self.mag >= thr).astype(F32)


# ---------------------------------------------------------------------------
# R1 adaptive warmup (optimizer.py:104-150), R3 lazy trigger (:182-214),
# R4 gSNR clip (:161-175)
# ---------------------------------------------------------------------------

class OracleWarmupScheduler:
    """``_AdaptiveWarmupScheduler`` (optimizer.py:104-150)."""

    def __init__(self, warmup_steps=100, stability_threshold=0.05, patience=5, min_warmup=20):
        self.warmup_steps, self.thr, self.patience = warmup_steps, stability_threshold, patience
        self.min_warmup = min_warmup
        self.prev = float("inf")
        self.stable = 0
        self.early = None

    def update(self, step, avg):
        if step < self.min_warmup:
            return True
        if self.prev > 0:
            rel = abs(avg - self.prev) / (self.prev + 1e-8)
            self.stable = self.stable + 1 if rel < self.thr else 0
        self.prev = avg
        if self.stable >= self.patience:
            self.early = self.early or step
            return False
        return step < self.warmup_steps


class OracleLazyTrigger:
    """``_LazyPrecondTrigger`` (optimizer.py:182-214)."""

    def __init__(self, delta_threshold=0.1, max_skip=50):
        self.thr, self.max_skip = delta_threshold, max_skip
        self.prev = 0.0
        self.since = 0

    def should_update(self, g):
        self.since += 1
        if self.since >= self.max_skip:
            self.since = 0
            self.prev = g
            return True
        if self.prev > 0:
            if abs(g - self.prev) / (self.prev + 1e-8) > self.thr:
                self.since = 0
                self.prev = g
                return True
        self.prev = g
        return False


def gsnr_clip(update, m, v, eps, thr):
    """optimizer.py:161-175: update * (|m| / (sqrt(v) + eps) >= thr)."""
    snr = np.abs(m) / (np.sqrt(v) + F32(eps))
    return update * (snr >= F32(thr)).astype(F32)


_DEFAULTS = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                 precond_freq=20, epsilon_sparse=0.05, k_min=8, k_max=128,
                 rho=0.999, tau=1.0, warmup_steps=100, blend_steps=50,
                 min_precond_updates=10, max_precond_dim=4096,
                 use_int8_ema=False, beta3=0.99, lars_coeff=1e-3)


class OracleSCAO:
    """optimizer.py:221-645 restricted to the deterministic path (no gradient
    noise; the sparse filter with its R2 dynamic form and the R1, R3, R4, R5
    extensions are included), numpy float32.

    ``params`` is a list of float32 arrays holding parameter-dtype values;
    ``groups`` is a list of dicts {"params": [indices], **overrides}.
    """

    def __init__(self, params, dtype="float32", groups=None, lookahead_k=5,
                 lookahead_alpha=0.5, threads=1, **kw):
        # one parameter dtype for all, or a list with one per parameter
        self.dtypes = list(dtype) if isinstance(dtype, (list, tuple)) else [dtype] * len(params)
        self.dtype = self.dtypes[0] if self.dtypes else dtype
        self.params = [round_to(np.array(p, dtype=F32), d) for p, d in zip(params, self.dtypes)]
        d = dict(_DEFAULTS)
        self.sparsity = float(kw.pop("sparsity", 0.0))
        self.dynamic_sparsity = bool(kw.pop("dynamic_sparsity", False))
        self.filters = {}
        # R1 / R3 / R4 / R5 (optimizer.py:325-345)
        self.adaptive_warmup = bool(kw.pop("adaptive_warmup", False))
        ws = kw.get("warmup_steps", _DEFAULTS["warmup_steps"])
        self.warmup_sched = OracleWarmupScheduler(
            ws, kw.pop("warmup_stability_threshold", 0.05), kw.pop("warmup_patience", 5),
            max(20, ws // 5))
        self.in_warmup_global = True
        self.lazy = bool(kw.pop("lazy_precond", False))
        self.lazy_thr = float(kw.pop("lazy_delta_threshold", 0.1))
        self.lazy_skip = int(kw.pop("lazy_max_skip", 50))
        self.triggers = {}
        self.gsnr = bool(kw.pop("use_gsnr_clip", False))
        self.gsnr_thr = float(kw.pop("gsnr_threshold", 0.5))
        self.adaptive_rank = bool(kw.pop("adaptive_rank", False))
        # gradient noise (optimizer.py:544-545) draws from torch's generator and
        # is not restated: the oracle is the noise-free path
        for k in ("noise_std_init", "async_precond", "noise_anneal"):
            kw.pop(k, None)
        d.update(kw)
        if groups is None:
            groups = [{"params": list(range(len(params)))}]
        self.groups = []
        for g in groups:
            gg = dict(d)
            gg.update(g)
            self.groups.append(gg)
        self.state = {}
        self.global_step = 0
        self.global_norm_ema = 1.0
        self.lookahead_k = lookahead_k
        self.lookahead_alpha = lookahead_alpha
        self.slow = {}
        self.threads = threads
        self._pool = None
        if threads > 1:
            from concurrent.futures import ThreadPoolExecutor
            self._pool = ThreadPoolExecutor(threads)

    def _init_state(self, i, group):
        """optimizer.py:407-433."""
        if i in self.state:
            return
        p = self.params[i]
        self.state[i] = dict(
            step=0, scao_step=0, started=False,
            m=np.zeros(p.shape, F32), v=np.zeros(p.shape, F32),
            d=np.zeros(p.shape, F32), prev=np.zeros(p.shape, F32),
            precond=OraclePreconditioner(
                p.shape, group["epsilon_sparse"], group["k_min"], group["k_max"],
                group["rho"], group["max_precond_dim"], group["use_int8_ema"]))

    def step(self, grads):
        """optimizer.py:452-503."""
        self.global_step += 1
        # optimizer.py:439-446: p.grad.norm() in the gradient's own dtype
        norms = [norm_dt(g, self.dtypes[i]) for i, g in enumerate(grads) if g is not None]
        avg = 0.0
        if norms:
            avg = sum(norms) / len(norms)
            self.global_norm_ema = 0.95 * self.global_norm_ema + 0.05 * avg
        if self.adaptive_warmup:                       # optimizer.py:470-479
            self.in_warmup_global = self.warmup_sched.update(self.global_step, avg)
        if self.dynamic_sparsity:
            for f in self.filters.values():
                f.set_global_norm_ref(self.global_norm_ema)
        for group in self.groups:
            self._step_group(group, grads)
        if self.lookahead_k > 0 and self.global_step % self.lookahead_k == 0:
            self._lookahead_sync()

    def _lookahead_sync(self):
        """optimizer.py:356-365."""
        a = F32(self.lookahead_alpha)
        for group in self.groups:
            for i in group["params"]:
                p = self.params[i]
                if i not in self.slow:
                    self.slow[i] = p.copy()
                s = self.slow[i]
                dt = self.dtypes[i]
                s = round_to(s + round_to(a * round_to(p - s, dt), dt), dt)
                self.slow[i] = s
                self.params[i] = s.copy()

    def _step_group(self, group, grads):
        """optimizer.py:509-645 (parameters are independent: optionally run
        on a thread pool; numpy releases the GIL inside its loops)."""
        for i in group["params"]:
            if grads[i] is not None:
                self._init_state(i, group)
        todo = [i for i in group["params"] if grads[i] is not None]
        if self._pool is not None:
            list(self._pool.map(lambda i: self._step_param(i, group, grads[i]), todo))
        else:
            for i in todo:
                self._step_param(i, group, grads[i])

    def _step_param(self, i, group, gr):
        dt = self.dtypes[i]
        lr = group["lr"]
        beta1, beta2 = group["betas"]
        beta3 = group["beta3"]
        eps = group["eps"]
        wd = group["weight_decay"]
        pf = group["precond_freq"]
        tau = group["tau"]
        lars = group["lars_coeff"]
        if True:
            st = self.state[i]
            st["step"] += 1
            step = st["step"]
            raw = np.asarray(gr, dtype=F32)       # p.grad (param dtype values)
            grad = raw
            grad_norm = float(norm_f32(raw))     # of p.grad.float(), optimizer.py:531-532
            if self.sparsity > 0.0:              # optimizer.py:536-542
                if i not in self.filters:
                    self.filters[i] = OracleSparseFilter(self.sparsity, self.dynamic_sparsity)
                grad = self.filters[i](grad)
            p = self.params[i]
            if wd != 0.0:
                p = round_to(p * F32(1.0 - lr * wd), dt)
            m, v, d, prev = st["m"], st["v"], st["d"], st["prev"]
            pc = st["precond"]
            if self.adaptive_rank:                      # R5, optimizer.py:383-401
                ratio = grad_norm / (self.global_norm_ema + 1e-8)
                if ratio > 2.0:
                    pc.set_k(min(group["k_max"], int(pc.k * 1.25)))
                elif ratio < 0.5:
                    pc.set_k(max(group["k_min"], int(pc.k * 0.8)))
            in_warmup = (self.in_warmup_global if self.adaptive_warmup
                         else step <= group["warmup_steps"]) or \
                (pc.precond_step < group["min_precond_updates"])
            if in_warmup:
                m = fma(grad, F32(1.0 - beta1), m * F32(beta1))
                v = fma(F32(1.0 - beta2) * grad, grad, v * F32(beta2))
                bc1 = 1.0 - beta1 ** step
                bc2 = 1.0 - beta2 ** step
                denom = np.sqrt(v) / F32(math.sqrt(bc2)) + F32(eps)
                if step % pf == 0:
                    pc.update_curvature(raw)
                p = add_alpha(p, round_to(m / denom, dt), -(lr / bc1), dt)
                st.update(m=m, v=v, prev=grad.copy())
                self.params[i] = p
                return
            if not st["started"]:
                st["started"] = True
                st["scao_step"] = 0
            st["scao_step"] += 1
            sstep = st["scao_step"]
            if self.lazy:                               # R3, optimizer.py:594-599
                if i not in self.triggers:
                    self.triggers[i] = OracleLazyTrigger(self.lazy_thr, self.lazy_skip)
                upd_now = self.triggers[i].should_update(grad_norm)
            else:
                upd_now = step % pf == 0
            if upd_now:
                pc.update_curvature(raw)
            gp = pc.precondition(raw, dt)
            if tau is not None:
                nat = pc.natural_grad_norm(raw, eps)
                if nat > tau:
                    gp = round_to(gp * (F32(tau) / max(nat, F32(eps))), dt)
            bs = group["blend_steps"]
            blend = min(1.0, sstep / bs) if bs > 0 else 1.0
            g_eff = F32(blend) * gp + F32(1.0 - blend) * grad
            delta = grad - prev
            prev = grad.copy()
            m = fma(g_eff, F32(1.0 - beta1), m * F32(beta1))
            d = fma(delta, F32(1.0 - beta3), d * F32(beta3))
            g_adan = g_eff + F32(1.0 - beta3) * delta
            v = fma(F32(1.0 - beta2) * g_adan, g_adan, v * F32(beta2))
            bc1 = 1.0 - beta1 ** step
            bc2 = 1.0 - beta2 ** step
            bc3 = 1.0 - beta3 ** step
            upd = (m / F32(bc1) + F32(1.0 - beta3) * (d / F32(bc3))) / \
                (np.sqrt(v / F32(bc2)) + F32(eps))
            if self.gsnr:                               # R4, optimizer.py:637-638
                upd = gsnr_clip(upd, m, v, eps, self.gsnr_thr)
            trust = self._lars(p, upd, lars, wd, dt) if lars > 0 else 1.0
            p = add_alpha(p, round_to(upd, dt), -(lr * trust), dt)
            st.update(m=m, v=v, d=d, prev=prev)
            self.params[i] = p

    def _lars(self, p, upd, lars, wd, dt):
        """optimizer.py:371-377 with parameter-dtype scalar roundings."""
        pn = F32(round_to(np.array([norm_f32(p)], F32), dt)[0])
        un = norm_f32(upd)
        if pn == 0 or un == 0:
            return 1.0
        num = F32(round_to(np.array([F32(lars) * pn], F32), dt)[0])
        wdp = F32(round_to(np.array([F32(wd) * pn], F32), dt)[0])
        den = F32(F32(un + wdp) + F32(1e-8))
        return float(F32(num / den))
