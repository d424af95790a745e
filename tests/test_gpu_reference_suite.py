"""The reference test suite's behavioural checks of ``SCAO`` that the other GPU
tests do not already cover (scao/tests/test_optimizer.py:245-316, 396-527,
667-684): LR schedulers, AMP with GradScaler, fp32 preconditioner state for
reduced-precision parameters, rank bounds, clipping, a transformer block and
a block-diagonal layer -- on CUDA tensors, through the unchanged API."""
import pytest
import torch
import torch.nn as nn

from scao_b200 import SCAO

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _finite(model):
    return all(torch.isfinite(p).all() for p in model.parameters())


def _run(opt_factory, sched_factory, steps=20, plateau=False):
    torch.manual_seed(0)
    model = nn.Linear(16, 8).to(DEV)
    opt = opt_factory(model)
    sched = sched_factory(opt)
    x = torch.randn(4, 16, device=DEV)
    for _ in range(steps):
        opt.zero_grad()
        loss = model(x).sum()
        loss.backward()
        opt.step()
        sched.step(loss.item()) if plateau else sched.step()
    assert _finite(model)
    return opt.param_groups[0]["lr"]


def _scao(model, lr=1e-2):
    return SCAO(model.parameters(), lr=lr, warmup_steps=3, precond_freq=2)


def test_lr_schedulers():
    from torch.optim.lr_scheduler import (CosineAnnealingLR, LinearLR, OneCycleLR,
                                          ReduceLROnPlateau, SequentialLR, StepLR)
    assert _run(_scao, lambda o: CosineAnnealingLR(o, T_max=20, eta_min=1e-5)) <= 1e-2
    assert _run(_scao, lambda o: StepLR(o, step_size=5, gamma=0.5)) < 1e-2
    assert _run(_scao, lambda o: SequentialLR(
        o, [LinearLR(o, start_factor=0.1, total_iters=5),
            LinearLR(o, start_factor=1.0, end_factor=0.1, total_iters=15)], milestones=[5])) < 1e-2
    _run(lambda m: _scao(m, 1e-3), lambda o: OneCycleLR(o, max_lr=1e-2, total_steps=20))
    _run(_scao, lambda o: ReduceLROnPlateau(o, factor=0.5, patience=3, min_lr=1e-5), steps=15,
         plateau=True)


def test_zero_lr_leaves_parameters_unchanged():
    """The step reads each group's current lr (what the schedulers rely on)."""
    torch.manual_seed(1)
    model = nn.Linear(16, 8).to(DEV)
    opt = SCAO(model.parameters(), lr=1e-2, warmup_steps=2, precond_freq=2, lookahead_k=0,
               sparsity=0.0, noise_std_init=0.0)
    x = torch.randn(4, 16, device=DEV)
    for t in range(6):
        if t == 4:
            for g in opt.param_groups:
                g["lr"] = 0.0
            before = [p.detach().clone() for p in model.parameters()]
        opt.zero_grad()
        model(x).sum().backward()
        opt.step()
    assert all(torch.equal(a, p) for a, p in zip(before, model.parameters()))


def test_amp_autocast_gradscaler():
    torch.manual_seed(2)
    model = nn.Linear(32, 16).to(DEV)
    opt = SCAO(model.parameters(), lr=1e-3, warmup_steps=5, precond_freq=2)
    scaler = torch.amp.GradScaler("cuda")
    x = torch.randn(4, 32, device=DEV) * 0.1
    w0 = model.weight.detach().clone()
    for _ in range(10):      # steps whose scaled fp16 gradients overflow are skipped
        opt.zero_grad()
        with torch.autocast("cuda", dtype=torch.float16):
            loss = model(x).sum()
        scaler.scale(loss).backward()
        scaler.step(opt)
        scaler.update()
    assert _finite(model) and not torch.equal(w0, model.weight)


def test_preconditioner_state_always_float32():
    torch.manual_seed(3)
    model = nn.Linear(16, 8).to(DEV, torch.bfloat16)
    opt = SCAO(model.parameters(), lr=1e-3, warmup_steps=0, precond_freq=1)
    opt.zero_grad()
    model(torch.randn(4, 16, device=DEV, dtype=torch.bfloat16)).sum().backward()
    opt.step()
    for st in opt.state.values():
        assert st["exp_avg"].dtype == torch.float32
        prec = st["preconditioner"]
        if prec.use_kronecker:
            assert prec.L_ema.dtype == torch.float32
            assert prec.U_l.dtype == torch.float32 and prec.S_l.dtype == torch.float32


def test_rank_bounds_and_stats():
    torch.manual_seed(4)
    model = nn.Linear(64, 64, bias=False).to(DEV)
    opt = SCAO(model.parameters(), lr=1e-3, warmup_steps=0, precond_freq=1, k_min=4, k_max=32)
    x = torch.randn(16, 64, device=DEV)
    for _ in range(5):
        opt.zero_grad()
        model(x).sum().backward()
        opt.step()
    ranks = opt.current_ranks()
    assert ranks and all(4 <= k <= 32 for k in ranks.values())
    stats = opt.precond_stats()
    assert "rank_mean" in stats and stats["num_precond_layers"] >= 1


def test_clipping_extremes():
    torch.manual_seed(5)
    for tau in (1e-6, None):
        model = nn.Linear(16, 8, bias=False).to(DEV)
        opt = SCAO(model.parameters(), lr=1e-3, warmup_steps=0, precond_freq=1, tau=tau)
        for p in model.parameters():
            p.grad = torch.ones_like(p) * 1e6 if tau else torch.randn_like(p)
        opt.step()
        assert _finite(model)


def test_transformer_block_and_large_layer():
    torch.manual_seed(6)
    layer = nn.TransformerEncoderLayer(d_model=64, nhead=4, dim_feedforward=128,
                                       batch_first=True).to(DEV)
    big = nn.Linear(256, 64).to(DEV)        # 64 x 256 weight: block-diagonal at 128
    params = list(layer.parameters()) + list(big.parameters())
    opt = SCAO(params, lr=1e-3, warmup_steps=5, precond_freq=2, max_precond_dim=128)
    x = torch.randn(2, 10, 64, device=DEV)
    for _ in range(10):
        opt.zero_grad()
        (layer(x).pow(2).mean() + big(torch.randn(4, 256, device=DEV)).pow(2).mean()).backward()
        opt.step()
    assert _finite(layer) and _finite(big)
    assert opt.state[big.weight]["preconditioner"].use_block_diagonal
