"""Helpers shared by the tests: load golden fixtures, replay a golden run."""
import os

import numpy as np

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

CASES = {
    # name: (dtype, max_precond_dim, steps, grad_scale, int8 EMA)
    "f32": ("float32", 4096, 40, 1e-2, True),
    "bf16": ("bfloat16", 4096, 40, 1e-2, True),
    "f32_blocks": ("float32", 48, 30, 1e-2, True),
    "f32_spec": ("float32", 4096, 30, 1.0, False),
    "int8_spec": ("float32", 48, 30, 1.0, True),
    "bf16_spec": ("bfloat16", 48, 30, 1.0, True),
    "f32_sparse": ("float32", 4096, 30, 1.0, True),
    "bf16_dyn": ("bfloat16", 48, 30, 1.0, True),
    "f32_r135": ("float32", 48, 30, 1.0, False),
    "bf16_gsnr": ("bfloat16", 4096, 30, 1.0, True),
    "f32_strips": ("float32", 48, 30, 1.0, True),
    "bf16_strips": ("bfloat16", 48, 30, 1.0, True),
    "mixed": ("float32", 48, 30, 1.0, True),
    "bf16_skip": ("bfloat16", 48, 30, 1.0, True),
}

# golden runs with a GPU check of their own (tests/test_gpu_goldens_extra.py);
# same fields as CASES
ORACLE_ONLY = {
    "bf16_r1235": ("bfloat16", 48, 30, 1.0, True),
    "f32_groups": ("float32", 48, 30, 1.0, True),
    "bf16_la": ("bfloat16", 4096, 30, 1.0, False),
    "f32_k128": ("float32", 4096, 24, 1.0, True),
    "f32_minpu": ("float32", 48, 30, 1.0, True),
    "f32_nd": ("float32", 48, 30, 1.0, True),
}

# optimizer keyword overrides of a case: the gradient filter of
# optimizer.py:40-97 (static and R2-dynamic), R1 adaptive warmup, R3 lazy
# curvature trigger, R5 adaptive rank, R4 gSNR clip
EXTRA = {
    "f32_sparse": dict(sparsity=0.7),
    "bf16_dyn": dict(sparsity=0.6, dynamic_sparsity=True),
    "f32_r135": dict(adaptive_warmup=True, warmup_patience=2, warmup_stability_threshold=0.5,
                     lazy_precond=True, lazy_delta_threshold=0.02, lazy_max_skip=4,
                     adaptive_rank=True, k_min=2, k_max=4,
                     _grad_scales=(1.0, 1.0, 0.05, 1.0, 1.0, 1.0)),
    "bf16_gsnr": dict(use_gsnr_clip=True, gsnr_threshold=0.3),
    # width-1 remainder blocks of the split (diagonal sub-preconditioners,
    # preconditioner.py:142-156, 232-236): a row strip, column strips, and
    # both inside a nested split
    "f32_strips": dict(_shapes=((49, 40), (40,), (40, 97), (97, 97))),
    "bf16_strips": dict(_shapes=((49, 40), (40,), (40, 97), (97, 97)), sparsity=0.5),
    # one optimizer over parameters of different dtypes
    "mixed": dict(_dtypes=("float32", "bfloat16", "float32", "float16", "float16",
                           "bfloat16")),
    # parameters without a gradient at some steps (skipped by the step,
    # still moved by lookahead, left out of the global-norm average)
    "bf16_skip": dict(_skip=((2, 3, 1), (0, 4, 2), (5, 7, 3))),
    # bf16 with R1 + R2 + R3 + R5: the global grad-norm average takes
    # float(p.grad.norm()) of the bf16 gradients, rounded to bf16
    "bf16_r1235": dict(adaptive_warmup=True, warmup_patience=2, warmup_stability_threshold=0.5,
                       lazy_precond=True, lazy_delta_threshold=0.02, lazy_max_skip=4,
                       adaptive_rank=True, k_min=2, k_max=4, sparsity=0.6,
                       dynamic_sparsity=True, _grad_scales=(1.0, 1.0, 0.05, 1.0, 1.0, 1.0)),
    # param groups with their own lr, weight decay, betas, rank bounds, clip
    # and warmup (the optimizer reads every group's values each step)
    "f32_groups": dict(_groups=(((0, 1, 2), dict(lr=2e-3, weight_decay=0.1, betas=(0.85, 0.99),
                                                   k_max=6)),
                                ((3, 4, 5), dict(lr=5e-4, weight_decay=0.0, tau=None, k_min=2,
                                                   warmup_steps=12, beta3=0.9)))),
    # lookahead every 2 steps with alpha 0.8, LARS off, fp32 factors
    "bf16_la": dict(lookahead_k=2, lookahead_alpha=0.8, lars_coeff=0.0),
    # the largest rank the kernels take (k_max 128: kpad 128)
    "f32_k128": dict(_shapes=((300, 272), (272,)), k_min=8, k_max=128, epsilon_sparse=0.01),
    # Phase 2 gated by min_precond_updates (3 curvature updates, the third one
    # made inside the warmup branch of the step that reaches it)
    "f32_minpu": dict(min_precond_updates=3, precond_freq=4, warmup_steps=4),
    # parameters of 3 and 4 dims (conv-like) flattened to (d0, rest) (utils.py:208-219)
    "f32_nd": dict(_shapes=((16, 4, 6), (24,), (8, 3, 3, 3), (6, 8, 10))),
}


def load(name):
    return dict(np.load(os.path.join(HERE, name + ".npz")))


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def principal_angle(U, V):
    """Largest principal angle (rad) between span(U) and span(V)."""
    U = np.linalg.qr(np.asarray(U, np.float64))[0]
    V = np.linalg.qr(np.asarray(V, np.float64))[0]
    s = np.linalg.svd(U.T @ V, compute_uv=False)
    return float(np.arccos(np.clip(s.min(), -1.0, 1.0)))


def separated_prefix(S, rel_gap=1e-2):
    """Largest j < len(S) such that the top-j eigen-subspace is separated from
    the rest of the listed spectrum by a relative gap >= rel_gap; 0 if none.
    Principal angles are only meaningful on such subspaces (near-equal
    eigenvalues make the individual vectors arbitrary)."""
    S = np.asarray(S, np.float64)
    if S.size == 0 or S[0] <= 0:
        return 0
    best = 0
    for j in range(1, len(S)):
        if (S[j - 1] - S[j]) >= rel_gap * S[0]:
            best = j
    return best


def subspace_angle(U, U_ref, S_ref, rel_gap=1e-2):
    j = separated_prefix(S_ref, rel_gap)
    if j == 0:
        return 0.0
    return principal_angle(np.asarray(U)[:, :j], np.asarray(U_ref)[:, :j])


def reference_root():
    """Directory holding the reference's ``scao`` package, for the CPU checks
    that import it: ``$SCAO_REFERENCE`` if set, else the offline install under
    ``baseline/_ref`` of this checkout; None when neither holds it."""
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for d in (os.environ.get("SCAO_REFERENCE"), os.path.join(repo, "baseline", "_ref")):
        if d and os.path.isfile(os.path.join(d, "scao", "__init__.py")):
            return d
    return None
