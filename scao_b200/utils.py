"""Host-side utilities re-exported for API compatibility with ``scao``."""
from __future__ import annotations

import torch


def adaptive_rank(eigenvalues, epsilon: float = 0.05, k_min: int = 4, k_max: int = 128) -> int:
    """utils.py:121-151: smallest k whose top-k eigenvalues (descending) hold
    (1 - epsilon) of the spectral mass, clamped to [k_min, k_max].  The
    optimizer runs the same rule on the device (eig.cu adaptive_rank_dev)."""
    ev = torch.as_tensor(eigenvalues, dtype=torch.float32)
    total = ev.sum().item()
    if total < 1e-12:
        return k_min
    threshold = (1.0 - epsilon) * total
    cumsum = torch.cumsum(ev, dim=0)
    idx = (cumsum >= threshold).nonzero(as_tuple=True)[0]
    k = int(idx[0].item()) + 1 if idx.numel() > 0 else len(ev)
    return int(min(k_max, max(k_min, k)))


# ---------------------------------------------------------------------------
# Matrix inverse fourth roots (utils.py:17-114).  Exported for API
# compatibility; the optimizer step never calls them (its preconditioner
# keeps the low-rank factors and applies S^(-1/4) inside its kernels).
# ---------------------------------------------------------------------------

def newton_schulz_root_inv(A, steps: int = 10, eps: float = 1e-8):
    """utils.py:17-58: A^(-1/4) of a symmetric PSD matrix by two rounds of
    coupled Newton-Schulz iterations on A / ||A||_F (the first converges to
    the inverse square root, the second takes the square root of that),
    scaled back by ||A||_F^(1/4)."""
    assert A.ndim == 2 and A.shape[0] == A.shape[1], "A must be square"
    nrm = A.norm(p="fro").clamp(min=eps)
    eye = torch.eye(A.shape[0], dtype=A.dtype, device=A.device)

    def coupled(X):
        Y = eye.clone()
        for _ in range(steps):
            XY = X @ Y
            X, Y = (3.0 * X - XY @ X) * 0.5, (3.0 * eye - XY) @ Y * 0.5
        return X

    return coupled(coupled(A / nrm)) * nrm.pow(0.25)


def matrix_power_neg_quarter(A, use_newton_schulz: bool = False, ns_steps: int = 10,
                             eps: float = 1e-8):
    """utils.py:61-93: A^(-1/4) for symmetric PSD A, by eigendecomposition
    (eigenvalues floored at eps) or by Newton-Schulz."""
    if use_newton_schulz:
        return newton_schulz_root_inv(A, steps=ns_steps, eps=eps)
    w, V = torch.linalg.eigh(A)
    return (V * w.clamp(min=eps).pow(-0.25).unsqueeze(0)) @ V.T


def low_rank_matrix_power_neg_quarter(U, S, eps: float = 1e-8):
    """utils.py:96-114: the factors (U, S^(-1/4)) of A^(-1/4) ~ U diag(S^(-1/4)) U^T."""
    return U, S.clamp(min=eps).pow(-0.25)
