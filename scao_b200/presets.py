"""Scale presets (scao/optimizer.py:958-1002; these v3 definitions shadow the
earlier ones at :808-951 in the reference module)."""
from __future__ import annotations

from .optimizer import SCAO


def _params(m):
    return m.parameters() if hasattr(m, "parameters") else m


def scao_sub1b(model_or_params, lr=1e-3, **kw):
    return SCAO(_params(model_or_params), lr=lr, k_max=64, use_int8_ema=False, **kw)


def scao_1b(model_or_params, lr=1e-3, **kw):
    return SCAO(_params(model_or_params), lr=lr, k_max=48, use_int8_ema=True,
                async_precond=True, **kw)


def scao_3b(model_or_params, lr=3e-4, **kw):
    return SCAO(_params(model_or_params), lr=lr, k_max=32, use_int8_ema=True,
                async_precond=True, warmup_steps=20, blend_steps=10, **kw)


def scao_7b(model_or_params, lr=1e-4, **kw):
    return SCAO(_params(model_or_params), lr=lr, k_max=24, use_int8_ema=True,
                async_precond=False, dynamic_sparsity=False, **kw)


def scao_40b(model_or_params, lr=1e-4, **kw):
    return SCAO(_params(model_or_params), lr=lr, k_max=16, use_int8_ema=True,
                async_precond=True, lazy_precond=True, use_gsnr_clip=True, **kw)


def scao_125b(model_or_params, lr=5e-5, **kw):
    return SCAO(_params(model_or_params), lr=lr, k_max=8, use_int8_ema=True,
                async_precond=True, lazy_precond=True, lazy_max_skip=100,
                use_gsnr_clip=True, adaptive_rank=True, **kw)
