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
