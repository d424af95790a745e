"""The reference's tensor-level seam (scao/cuda/__init__.py:149-266) as
``scao_b200.cuda``: results against float64 torch restatements of its
formulas and against the oracle's int8 EMA update (bit-exact)."""
import numpy as np
import pytest
import torch

from oracle import scao_oracle as O
from scao_b200 import cuda as seam

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_fused_kronecker_precond(dt):
    gen = torch.Generator().manual_seed(3)
    m, n, k = 96, 80, 12
    Ul = torch.linalg.qr(torch.randn(m, k, generator=gen, dtype=torch.float64))[0]
    Ur = torch.linalg.qr(torch.randn(n, k, generator=gen, dtype=torch.float64))[0]
    sl, sr = torch.rand(k, generator=gen) + 0.5, torch.rand(k, generator=gen) + 0.5
    G = torch.randn(m, n, generator=gen).to(dt)
    Gd = G.double()
    ref = Gd + Ul @ ((sl.double()[:, None] * sr.double()[None, :] - 1) * (Ul.T @ Gd @ Ur)) @ Ur.T
    out = seam.fused_kronecker_precond(Ul.float().to(DEV), sl.to(DEV), Ur.float().to(DEV),
                                       sr.to(DEV), G.to(DEV))
    assert out.dtype == dt and out.shape == (m, n)
    if dt == torch.float32:
        assert (out.double().cpu() - ref).abs().max().item() < 1e-4
    else:
        assert torch.allclose(out.double().cpu(), ref.to(dt).double(), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("left", [True, False])
def test_low_rank_precond_mm(left):
    gen = torch.Generator().manual_seed(4)
    m, n, k = 64, 48, 8
    d = m if left else n
    U = torch.linalg.qr(torch.randn(d, k, generator=gen, dtype=torch.float64))[0].float()
    s = torch.rand(k, generator=gen)
    G = torch.randn(m, n, generator=gen)
    ref = (U * s) @ (U.T @ G) if left else (G @ (U * s)) @ U.T
    out = seam.low_rank_precond_mm(U.to(DEV), s.to(DEV), G.to(DEV), left)
    assert torch.allclose(out.cpu(), ref, atol=1e-5, rtol=1e-4)


def test_int8_ema_update_bit_exact():
    gen = torch.Generator().manual_seed(5)
    x0 = torch.randn(4096, generator=gen)
    q0, s0 = O.quantize_sym_int8(x0.numpy())
    new = (torch.randn(4096, generator=gen) * 1e-3).numpy().astype(np.float32)
    qr, sr = O.quantize_sym_int8(O.dequantize_sym_int8(q0, s0) * np.float32(0.99) + new)
    q, s = seam.int8_ema_update(torch.from_numpy(q0).to(DEV), s0, torch.from_numpy(new).to(DEV),
                                0.99)
    assert np.array_equal(q.cpu().numpy(), qr) and s == sr
