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
