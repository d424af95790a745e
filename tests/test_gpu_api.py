"""GPU tests of the optimizer API, ported from the reference's test-suite
(scao/tests/test_optimizer.py): checkpoint round trips, block-diagonal
split, reduced-precision parameters, validation errors, callbacks."""
import copy
import io

import pytest
import torch
import torch.nn as nn

from scao_b200 import SCAO

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
KW = dict(sparsity=0.0, noise_std_init=0.0)


def _train(model, opt, x, steps):
    for _ in range(steps):
        opt.zero_grad()
        model(x).sum().backward()
        opt.step()


@pytest.mark.parametrize("mpd", [4096, 8])
def test_save_load_roundtrip(mpd):
    """test_optimizer.py:337-374 (plus a block-diagonal variant)."""
    torch.manual_seed(7)
    model = nn.Linear(32, 16).to(DEV)
    kw = dict(lr=1e-3, warmup_steps=5, precond_freq=2, lookahead_k=0, max_precond_dim=mpd,
              min_precond_updates=1, **KW)
    opt = SCAO(model.parameters(), **kw)
    x = torch.randn(4, 32, device=DEV)
    _train(model, opt, x, 10)
    buf = io.BytesIO()
    torch.save(opt.state_dict(), buf)
    buf.seek(0)
    state = torch.load(buf, weights_only=False)
    model2 = copy.deepcopy(model)
    opt2 = SCAO(model2.parameters(), **kw)
    opt2.load_state_dict(state)
    x2 = torch.randn(4, 32, device=DEV)
    for m_, o_ in ((model, opt), (model2, opt2)):
        o_.zero_grad()
        m_(x2).sum().backward()
        o_.step()
    for p1, p2 in zip(model.parameters(), model2.parameters()):
        assert torch.allclose(p1, p2, atol=1e-6)


def test_block_diagonal_activates_and_roundtrips():
    """test_optimizer.py:621-665 through the optimizer."""
    p = nn.Parameter(torch.randn(128, 16, device=DEV))
    opt = SCAO([p], lr=1e-3, max_precond_dim=64, k_min=4, warmup_steps=0,
               min_precond_updates=1, precond_freq=1, lookahead_k=0, **KW)
    for _ in range(3):
        p.grad = torch.randn_like(p)
        opt.step()
    sd = opt.state[p]["preconditioner"].state_dict()
    assert sd["use_block_diagonal"] and len(sd["blocks"]) == 2
    assert torch.isfinite(p).all()
    state = opt.state_dict()
    p2 = nn.Parameter(p.detach().clone())
    opt2 = SCAO([p2], lr=1e-3, max_precond_dim=64, k_min=4, warmup_steps=0,
                min_precond_updates=1, precond_freq=1, lookahead_k=0, **KW)
    opt2.load_state_dict(state)
    g = torch.randn_like(p)
    p.grad, p2.grad = g.clone(), g.clone()
    opt.step()
    opt2.step()
    assert torch.allclose(p, p2, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_reduced_precision_params(dtype):
    """test_optimizer.py:396-414: low-precision params, fp32 state."""
    model = nn.Sequential(nn.Linear(64, 64), nn.Linear(64, 8)).to(DEV).to(dtype)
    opt = SCAO(model.parameters(), lr=1e-3, warmup_steps=2, precond_freq=2,
               min_precond_updates=1, **KW)
    x = torch.randn(8, 64, device=DEV, dtype=dtype)
    _train(model, opt, x, 8)
    for p in model.parameters():
        assert p.dtype == dtype and torch.isfinite(p.float()).all()
        assert opt.state[p]["exp_avg"].dtype == torch.float32


def test_validation_errors():
    p = nn.Parameter(torch.zeros(4, device=DEV))
    with pytest.raises(ValueError):
        SCAO([p], lr=-1.0)
    with pytest.raises(ValueError):
        SCAO([p], betas=(1.0, 0.999))
    with pytest.raises(ValueError):
        SCAO([p], beta3=1.0)


def test_sparse_grad_raises():
    p = nn.Parameter(torch.zeros(8, 4, device=DEV))
    opt = SCAO([p], **KW)
    p.grad = torch.zeros(8, 4, device=DEV).to_sparse()
    with pytest.raises(RuntimeError):
        opt.step()


def test_callbacks_and_closure():
    model = nn.Linear(16, 8).to(DEV)
    opt = SCAO(model.parameters(), lr=1e-3, warmup_steps=0, min_precond_updates=0, **KW)
    seen = []
    opt.add_callback(seen.append)
    x = torch.randn(4, 16, device=DEV)

    def closure():
        opt.zero_grad()
        loss = model(x).sum()
        loss.backward()
        return loss

    loss = opt.step(closure)
    assert loss is not None and len(seen) == 1
    assert {"step", "scao/rank_mean", "noise_std", "global_norm_ema"} <= set(seen[0])
    opt.remove_callback(seen.append)


def test_weight_decay_shrinks_params():
    """test_optimizer.py:319-334."""
    p = nn.Parameter(torch.ones(16, 16, device=DEV))
    opt = SCAO([p], lr=0.1, weight_decay=0.5, warmup_steps=100, lookahead_k=0, **KW)
    for _ in range(3):
        p.grad = torch.zeros_like(p)
        opt.step()
    assert p.abs().max().item() < 1.0


def test_quadratic_converges():
    """test_optimizer.py:121-206: ill-conditioned quadratic, both phases."""
    torch.manual_seed(42)
    n = 32
    Q, _ = torch.linalg.qr(torch.randn(n, n))
    A = ((Q * torch.logspace(0, 2, n)) @ Q.T).to(DEV)
    b = torch.randn(n, device=DEV)
    X = nn.Parameter(torch.zeros(n, 4, device=DEV))
    B = torch.stack([b] * 4, 1)
    opt = SCAO([X], lr=0.05, warmup_steps=20, precond_freq=5, min_precond_updates=1,
               weight_decay=0.0, lars_coeff=0.0, lookahead_k=0, **KW)

    def loss():
        return (0.5 * (X * (A @ X)).sum() - (B * X).sum())
    l0 = loss().item()
    for _ in range(200):
        opt.zero_grad()
        loss().backward()
        opt.step()
    assert loss().item() < l0 - 1.0


def test_rank_setter_matches_oracle():
    """``preconditioner.k = v`` (preconditioner.py:249-291) on a nested
    block-diagonal parameter: clamping, truncation only, block mean."""
    from oracle import scao_oracle as O
    shape = (1100, 2500)
    p = torch.nn.Parameter(torch.zeros(shape, device=DEV))
    opt = SCAO([p], lr=1e-3, max_precond_dim=512, k_min=4, k_max=32, **KW)
    p.grad = torch.randn(shape, device=DEV) * 1e-2
    opt.step()
    pc = opt.state[p]["preconditioner"]
    ref = O.OraclePreconditioner(shape, k_min=4, k_max=32, max_precond_dim=512)
    assert pc.k == ref.k
    for v in (3, 40, 7, 2, 100):
        pc.k = v
        ref.set_k(v)
        assert pc.k == ref.k, v
        got = [lf["k"] for lf in pc.state_dict()["blocks"]]
        assert got == [b.k for b in ref.blocks], v


def test_large_model_presets_run():
    """The 40B / 125B presets (lazy trigger, gSNR clip, adaptive rank) step."""
    from scao_b200 import presets
    gen = torch.Generator().manual_seed(1)
    for make in (presets.scao_40b, presets.scao_125b):
        params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(DEV))
                  for s in [(96, 64), (64,), (128, 96)]]
        opt = make(params, warmup_steps=3, min_precond_updates=1)
        for _ in range(8):
            for q in params:
                q.grad = (torch.randn(q.shape, generator=gen) * 1e-2).to(DEV)
            opt.step()
        torch.cuda.synchronize()
        opt._plan.check_error()
        assert all(torch.isfinite(q).all() for q in params)
