"""The training-step caller (scao_b200/gpt.py): a small GPT-2-shaped model
trains with SCAO (loss goes down), and on real gradients of that model the
CUDA optimizer follows the oracle (relative L2 <= 1e-3 on the updates)."""
import numpy as np
import pytest
import torch

from oracle import scao_oracle as O
from scao_b200 import SCAO, gpt

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
SMALL = gpt.GPTConfig(n_layer=2, d_model=128, n_head=4, d_ff=512, vocab=512, seq_len=64)
KW = dict(lr=3e-3, warmup_steps=5, precond_freq=5, min_precond_updates=1, blend_steps=5,
          k_min=4, k_max=16, max_precond_dim=256, sparsity=0.0, noise_std_init=0.0,
          async_precond=False)


def test_small_gpt_trains():
    torch.manual_seed(0)
    model = gpt.GPT(SMALL).to(DEV)
    opt = SCAO(model.parameters(), **KW)
    tokens = gpt.token_batch(SMALL, 8, seed=1, device=DEV)
    losses = [gpt.train_step(model, opt, tokens).item() for _ in range(40)]
    torch.cuda.synchronize()
    opt._plan.check_error()
    assert np.isfinite(losses).all()
    assert np.mean(losses[-5:]) < np.mean(losses[:5]) - 0.5, losses


def test_real_gradients_match_oracle():
    """Gradients of the model at its initial weights (fixed sequence of
    batches) drive both the CUDA optimizer and the oracle."""
    model = gpt.GPT(SMALL).to(DEV)
    params = [p for p in model.parameters()]
    p0 = [p.detach().float().cpu().numpy() for p in params]
    grads = []
    for s in range(15):
        model.zero_grad(set_to_none=True)
        gpt.loss_fn(model, gpt.token_batch(SMALL, 4, seed=100 + s, device=DEV)).backward()
        grads.append([p.grad.detach().clone() for p in params])
    opt = SCAO(params, **KW)
    orc = O.OracleSCAO(p0, **{k: v for k, v in KW.items()})
    for gl in grads:
        for p, g in zip(params, gl):
            p.grad = g
        opt.step()
        orc.step([g.float().cpu().numpy() for g in gl])
    torch.cuda.synchronize()
    for i, p in enumerate(params):
        d_got = p.detach().float().cpu().numpy() - p0[i]
        d_ref = orc.params[i] - p0[i]
        den = np.linalg.norm(d_ref)
        assert np.linalg.norm(d_got - d_ref) <= 1e-3 * den + 1e-9, (i, tuple(p.shape))
