"""GPU tests of the sparse gradient filter and the gradient noise
(scao/optimizer.py:40-97, 536-545) through the optimizer facade.

The filter threshold must equal ``torch.quantile(mag_ema, sparsity)`` bit for
bit (the oracle's restatement beyond torch's 2^24-element cap); the
magnitude EMA must equal its float32 restatement; the full optimizer runs
with the filter on are compared with the reference's golden runs in
test_gpu_parity.py.  Noise cannot match torch's generator draw for draw: it
is checked for its distribution, its determinism and its independence
across parameters and steps.
"""
import numpy as np
import pytest
import torch

from oracle import scao_oracle as O
from scao_b200 import SCAO

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _opt(params, **kw):
    base = dict(lr=1e-3, warmup_steps=1000, noise_std_init=0.0, sparsity=0.7,
                async_precond=False, lookahead_k=0)
    base.update(kw)
    return SCAO(params, **base)


@pytest.mark.parametrize("shape", [(1,), (7,), (33,), (4096,), (257, 131), (1000, 1000)])
@pytest.mark.parametrize("q", [0.7, 0.05, 0.999])
def test_threshold_equals_torch_quantile(shape, q):
    gen = torch.Generator().manual_seed(hash((shape, q)) & 0xFFFF)
    p = torch.nn.Parameter(torch.zeros(shape, device=DEV))
    opt = _opt([p], sparsity=q)
    mag_ref = None
    for t in range(3):
        g = torch.randn(shape, generator=gen) * (1 + t)
        if t == 2:
            g = torch.round(g * 4) / 4          # many ties
        p.grad = g.to(DEV)
        opt.step()
        a = g.abs().numpy().astype(np.float32)
        mag_ref = a.copy() if mag_ref is None else \
            (mag_ref * np.float32(0.99)) + np.float32(1.0 - 0.99) * a
        plan = opt._plan
        mag = plan.state_view(plan.mag_ema, 0).cpu().numpy()
        assert np.array_equal(mag, mag_ref)
        thr = plan.filter_params()["thr"][0]
        ref = np.float32(torch.quantile(torch.from_numpy(mag_ref.ravel()), q).item())
        assert thr == ref, (t, thr, ref)


def test_threshold_beyond_torch_cap():
    """2^24 + 3 elements: torch.quantile refuses; the oracle's float64-rank
    restatement is the reference."""
    n = (1 << 24) + 3
    gen = torch.Generator().manual_seed(11)
    g = torch.rand(n, generator=gen)
    p = torch.nn.Parameter(torch.zeros(n, device=DEV))
    opt = _opt([p], sparsity=0.37)
    p.grad = g.to(DEV)
    opt.step()
    thr = opt._plan.filter_params()["thr"][0]
    assert thr == O.quantile_f32(g.numpy(), 0.37)


def test_nan_gradient_gives_nan_threshold():
    p = torch.nn.Parameter(torch.zeros(64, device=DEV))
    opt = _opt([p])
    g = torch.ones(64)
    g[5] = float("nan")
    p.grad = g.to(DEV)
    opt.step()
    assert np.isnan(opt._plan.filter_params()["thr"][0])


def test_filtered_moments_match_oracle_phase1():
    """Phase-1 Adam moments see the masked gradient; prev_grad holds it."""
    gen = torch.Generator().manual_seed(3)
    shapes = [(48, 40), (40,), (1000,)]
    p0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]
    params = [torch.nn.Parameter(x.clone().to(DEV)) for x in p0]
    kw = dict(lr=1e-3, warmup_steps=1000, noise_std_init=0.0, sparsity=0.6,
              async_precond=False, lookahead_k=0, weight_decay=0.0)
    opt = SCAO(params, **kw)
    orc = O.OracleSCAO([x.numpy() for x in p0], lookahead_k=0,
                       **{k: v for k, v in kw.items() if k != "lookahead_k"})
    for t in range(4):
        gs = [torch.randn(s, generator=gen) for s in shapes]
        for p, g in zip(params, gs):
            p.grad = g.to(DEV)
        opt.step()
        orc.step([g.numpy() for g in gs])
    for i, p in enumerate(params):
        st = opt.state[p]
        assert np.array_equal(st["prev_grad"].cpu().numpy(), orc.state[i]["prev"])
        assert np.allclose(st["exp_avg"].cpu().numpy(), orc.state[i]["m"], rtol=1e-6, atol=0)
        assert np.allclose(p.detach().cpu().numpy(), orc.params[i], rtol=1e-5, atol=1e-9)


def test_noise_distribution_and_determinism():
    n = 1 << 20

    def run(seed):
        torch.cuda.manual_seed(seed)
        ps = [torch.nn.Parameter(torch.zeros(n, device=DEV)) for _ in range(2)]
        opt = SCAO(ps, lr=1e-3, sparsity=0.0, noise_std_init=0.5, warmup_steps=100,
                   async_precond=False, lookahead_k=0)
        for p in ps:
            p.grad = torch.zeros(n, device=DEV)
        opt.step()
        z1 = [opt.state[p]["prev_grad"].clone() for p in ps]
        opt.step()
        z2 = [opt.state[p]["prev_grad"].clone() for p in ps]
        return z1, z2, opt._noise_std

    z1, z2, std_after = run(1234)
    for z in z1 + z2:
        m, s = z.mean().item(), z.std().item()
        assert abs(m) < 5 * 0.5 / n ** 0.5 * 2
        assert abs(s - 0.5 * (0.998 if z is z2[0] or z is z2[1] else 1.0)) < 0.5 * 5e-3
        # standard-normal tail mass beyond 3 sigma is 0.27 %
        frac = (z.abs() > 3 * s).float().mean().item()
        assert 0.002 < frac < 0.0035
    assert not torch.equal(z1[0], z1[1]) and not torch.equal(z1[0], z2[0])
    assert abs(torch.corrcoef(torch.stack([z1[0], z1[1]]))[0, 1].item()) < 0.01
    y1, y2, _ = run(1234)
    assert torch.equal(z1[0], y1[0]) and torch.equal(z2[1], y2[1])
    w1, _, _ = run(99)
    assert not torch.equal(z1[0], w1[0])
    assert std_after == pytest.approx(0.5 * 0.998 ** 2)


def test_reference_defaults_run():
    """SCAO(params) with the reference's defaults (sparsity 0.7, noise 0.01,
    lookahead 5, async) runs through Phase 1 into Phase 2 and stays finite."""
    gen = torch.Generator().manual_seed(0)
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(DEV))
              for s in [(64, 48), (48,), (96, 64)]]
    opt = SCAO(params, warmup_steps=4, min_precond_updates=1, precond_freq=2)
    for _ in range(12):
        for p in params:
            p.grad = (torch.randn(p.shape, generator=gen) * 1e-2).to(DEV)
        opt.step()
    torch.cuda.synchronize()
    opt._plan.check_error()
    for p in params:
        assert torch.isfinite(p).all()
    assert opt.state[params[0]]["scao_step"] > 0
