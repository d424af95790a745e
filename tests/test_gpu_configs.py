"""BASELINE config 0 at full size (4-layer d=256 GPT set, int8 EMA, 100 steps):
the CUDA optimizer against the oracle on the same seeded gradients -- ranks
equal at every step, parameter updates and moments within 1e-3 relative L2."""
import numpy as np
import pytest
import torch

from oracle import scao_oracle as O
from scao_b200 import SCAO, synthetic, workloads

pytestmark = pytest.mark.gpu


def _rel(a, b):
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))


def test_config0_full_run_matches_oracle():
    w = workloads.c1()
    p0 = synthetic.init_params(w)
    params = [torch.nn.Parameter(p.clone().cuda()) for p in p0]
    opt = SCAO(params, **w.scao_kwargs)
    orc = O.OracleSCAO([p.float().numpy() for p in p0], dtype="float32", **w.scao_kwargs)
    gen = synthetic.LowRankGradients(w)
    for _ in range(w.steps):
        gs = gen.next()
        for p, g in zip(params, gs):
            p.grad = g.cuda()
        opt.step()
        orc.step([g.float().numpy() for g in gs])
        ks = [opt.state[p]["preconditioner"].k for p in params]
        assert ks == [orc.state[i]["precond"].k for i in range(len(params))]
    torch.cuda.synchronize()
    opt._plan.check_error()
    for i, p in enumerate(params):
        st = opt.state[p]
        a0 = p0[i].float().numpy()
        assert _rel(p.detach().cpu().numpy() - a0, orc.params[i] - a0) < 1e-3, i
        assert _rel(st["exp_avg"].cpu().numpy(), orc.state[i]["m"]) < 1e-3, i
        assert _rel(st["exp_avg_sq"].cpu().numpy(), orc.state[i]["v"]) < 1e-3, i
