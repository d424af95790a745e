"""GPU parity checks beyond the core golden set:

* the golden runs of ``ORACLE_ONLY`` (the oracle matches the reference on them
  on CPU): param groups, lookahead without LARS, k_max 128, the
  min_precond_updates gate, 3-D / 4-D parameters, bf16 with R1+R2+R3+R5;
* parity at the reference's default max_precond_dim (leaves of 2048-4096);
* a checkpoint written by the reference package, loaded and continued here.
"""
import os

import numpy as np
import pytest
import torch

from golden_util import EXTRA, HERE, ORACLE_ONLY, load, rel_err
from oracle import scao_oracle as O
from scao_b200 import SCAO, synthetic, workloads
from scao_b200.workloads import ParamSpec, Workload

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

DEV = "cuda:0"
TOL = 1e-3


def _run_gpu(name):
    dt, mpd, steps, gs, i8 = ORACLE_ONLY[name]
    w = workloads.tiny(dtype=dt, max_precond_dim=mpd, steps=steps, grad_scale=gs, int8=i8,
                       extra=EXTRA.get(name))
    p0 = synthetic.init_params(w)
    params = [torch.nn.Parameter(p.clone().to(DEV)) for p in p0]
    opt = SCAO(workloads.param_groups(w, params), **w.scao_kwargs)
    gen = synthetic.LowRankGradients(w)
    ks = []
    for t in range(steps):
        for i, (p, g) in enumerate(zip(params, gen.next())):
            p.grad = g.to(DEV) if workloads.has_grad(w, i, t) else None
        opt.step()
        ks.append([opt.state[p]["preconditioner"].k for p in params])
    torch.cuda.synchronize()
    opt._plan.check_error()
    return p0, params, opt, np.array(ks)


@pytest.mark.parametrize("name", list(ORACLE_ONLY))
def test_oracle_only_goldens_on_gpu(name):
    G = load("run_" + name)
    p0, params, opt, ks = _run_gpu(name)
    assert np.array_equal(ks, G["ks"])
    for i, p in enumerate(params):
        st = opt.state[p]
        a0 = p0[i].float().numpy()
        assert rel_err(p.detach().float().cpu().numpy() - a0, G[f"p{i}"] - a0) < TOL, i
        assert rel_err(st["exp_avg"].cpu().numpy(), G[f"exp_avg{i}"]) < TOL, i


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_large_leaves_match_oracle(dtype):
    """Leaves of 4096 x 1024 and a 2048 x 3000 layer split at the default
    max_precond_dim (4096): ranks every step and the final state against the
    oracle."""
    w = Workload("large", [ParamSpec("a", (4096, 1024)), ParamSpec("b", (2048, 3000)),
                           ParamSpec("c", (1024,))],
                 dict(lr=1e-3, precond_freq=5, warmup_steps=8, blend_steps=10,
                      min_precond_updates=1, k_min=4, k_max=32, use_int8_ema=True,
                      sparsity=0.0, noise_std_init=0.0, async_precond=False),
                 grad_rank=16, grad_decay=0.8, param_dtype=dtype, steps=20, grad_scale=1.0)
    p0 = synthetic.init_params(w)
    params = [torch.nn.Parameter(p.clone().to(DEV)) for p in p0]
    opt = SCAO(params, **w.scao_kwargs)
    orc = O.OracleSCAO([p.float().numpy() for p in p0], dtype=dtype, threads=8,
                       **w.scao_kwargs)
    gen = synthetic.LowRankGradients(w)
    for _ in range(w.steps):
        gs = gen.next()
        for p, g in zip(params, gs):
            p.grad = g.to(DEV)
        opt.step()
        orc.step([g.float().numpy() for g in gs])
        assert [opt.state[p]["preconditioner"].k for p in params] == \
            [orc.state[i]["precond"].k for i in range(len(params))]
    torch.cuda.synchronize()
    for i, p in enumerate(params):
        a0 = p0[i].float().numpy()
        assert rel_err(p.detach().float().cpu().numpy() - a0, orc.params[i] - a0) < TOL
        assert rel_err(opt.state[p]["exp_avg"].cpu().numpy(), orc.state[i]["m"]) < TOL


def test_reference_checkpoint_loads_and_continues():
    """tests/golden/ckpt_tiny_f32.pt (the reference's state_dict after 12
    steps) loads into SCAO, which continues 10 steps on the same gradients and
    ends where the reference did."""
    d = torch.load(os.path.join(HERE, "ckpt_tiny_f32.pt"))
    after = np.load(os.path.join(HERE, "ckpt_tiny_f32_after.npz"))
    nb, na = int(after["steps_before"]), int(after["steps_after"])
    w = workloads.tiny(dtype="float32", max_precond_dim=48, steps=nb + na, grad_scale=1.0,
                       int8=True)
    params = [torch.nn.Parameter(p.clone().to(DEV)) for p in d["params"]]
    opt = SCAO(params, **w.scao_kwargs)
    opt.load_state_dict(d["state_dict"])
    gen = synthetic.LowRankGradients(w, seed=0)
    for _ in range(nb):
        gen.next()
    for _ in range(na):
        for p, g in zip(params, gen.next()):
            p.grad = g.to(DEV)
        opt.step()
    torch.cuda.synchronize()
    for i, p in enumerate(params):
        assert opt.state[p]["preconditioner"].k == int(after[f"k{i}"])
        p0 = d["params"][i].numpy()
        assert rel_err(p.detach().cpu().numpy() - p0, after[f"p{i}"] - p0) < TOL
        assert rel_err(opt.state[p]["exp_avg"].cpu().numpy(), after[f"exp_avg{i}"]) < TOL
