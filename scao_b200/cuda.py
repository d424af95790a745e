"""Tensor-level kernel seam of the reference (scao/cuda/__init__.py:149-266):
``fused_kronecker_precond``, ``low_rank_precond_mm``, ``int8_ema_update``
with the reference's signatures and results, each one call into
``libscao_b200.so``.

The reference routes to its CUDA extension when it can and to a PyTorch
fallback otherwise; here there is no fallback: CPU tensors raise
RuntimeError, as does any error status of the library call.
"""
from __future__ import annotations

import torch

from . import _lib

_CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def _on_cuda(*ts):
    dev = ts[0].device
    if dev.type != "cuda" or any(t.device != dev for t in ts):
        raise RuntimeError("scao_b200.cuda: all tensors must be on one CUDA device "
                           "(no CPU path)")
    return dev


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def fused_kronecker_precond(U_l, s_l_inv4, U_r, s_r_inv4, G):
    """out = G + U_l ((s_l s_r^T - 1) o (U_l^T G U_r)) U_r^T, same shape and
    dtype as G (cuda/__init__.py:149-185, formula :78-99)."""
    dev = _on_cuda(G, U_l, s_l_inv4, U_r, s_r_inv4)
    if G.dtype not in _CODE:
        raise TypeError(f"unsupported gradient dtype {G.dtype}")
    m, n = G.shape
    k = U_l.shape[1]
    Ul, Ur = U_l.float().contiguous(), U_r.float().contiguous()
    sl, sr = s_l_inv4.float().contiguous(), s_r_inv4.float().contiguous()
    Gc = G.contiguous()
    out = torch.empty_like(Gc)
    L = _lib.lib()
    scratch = torch.empty(int(L.scao_fused_precond_scratch_bytes(m, n, k)), dtype=torch.uint8,
                          device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.scao_fused_kronecker_precond(Ul.data_ptr(), sl.data_ptr(), Ur.data_ptr(),
                                                  sr.data_ptr(), Gc.data_ptr(), out.data_ptr(),
                                                  _CODE[G.dtype], m, n, k, scratch.data_ptr(),
                                                  _stream(dev)), "scao_fused_kronecker_precond")
    return out


def low_rank_precond_mm(U, s, G, left: bool = True):
    """left: U diag(s) U^T G; otherwise G U diag(s) U^T (cuda/__init__.py:188-225),
    float32."""
    dev = _on_cuda(U, s, G)
    m, n = G.shape
    k = U.shape[1]
    Uc, sc, Gc = U.float().contiguous(), s.float().contiguous(), G.float().contiguous()
    out = torch.empty(m, n, dtype=torch.float32, device=dev)
    L = _lib.lib()
    scratch = torch.empty(int(L.scao_low_rank_precond_mm_scratch_bytes(m, n, k, int(left))),
                          dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.scao_low_rank_precond_mm(Uc.data_ptr(), sc.data_ptr(), Gc.data_ptr(),
                                              out.data_ptr(), m, n, k, int(left),
                                              scratch.data_ptr(), _stream(dev)),
                   "scao_low_rank_precond_mm")
    return out


def int8_ema_update(ema_q, ema_scale: float, new_val, rho: float):
    """(q_new, new_scale) of rho * dequantize(ema_q, ema_scale) + new_val,
    requantised (cuda/__init__.py:228-266; the library path's semantics,
    utils.py:170-203).  Reads the new scale back (one synchronisation, as
    the reference's ``.item()``)."""
    dev = _on_cuda(ema_q, new_val)
    q = ema_q.contiguous()
    nv = new_val.float().contiguous()
    n = q.numel()
    q_out = torch.empty_like(q)
    s_out = torch.empty(1, dtype=torch.float64, device=dev)
    L = _lib.lib()
    scratch = torch.empty(int(L.scao_int8_ema_scratch_bytes(n)), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.scao_int8_ema_update(q.data_ptr(), float(ema_scale), nv.data_ptr(), float(rho),
                                          n, q_out.data_ptr(), s_out.data_ptr(), scratch.data_ptr(),
                                          _stream(dev)), "scao_int8_ema_update")
    return q_out.view(ema_q.shape), float(s_out.item())
