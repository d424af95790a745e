"""Host utilities exported for API compatibility (scao/utils.py:17-151),
checked against the reference's own functions when its checkout is present
and against their defining properties otherwise."""
import os
import sys

import pytest
import torch

import scao_b200
from scao_b200 import utils

from golden_util import reference_root  # noqa: E402

REF = reference_root()


def _spd(m, seed):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(m, m, generator=g, dtype=torch.float64)
    return (X @ X.T / m + 0.1 * torch.eye(m, dtype=torch.float64)).float()


@pytest.mark.parametrize("m", [1, 5, 64])
def test_neg_quarter_eigh_property(m):
    A = _spd(m, m)
    X = utils.matrix_power_neg_quarter(A).double()
    # X^4 A = I
    P = X @ X @ X @ X @ A.double()
    assert torch.allclose(P, torch.eye(m, dtype=torch.float64), atol=1e-3)


def test_low_rank_factors():
    U = torch.eye(6, 3)
    S = torch.tensor([16.0, 1.0, 0.0])
    U2, s = utils.low_rank_matrix_power_neg_quarter(U, S)
    assert U2 is U
    assert torch.allclose(s, torch.tensor([0.5, 1.0, 1e-8 ** -0.25]))


def test_exports():
    for name in ("adaptive_rank", "matrix_power_neg_quarter", "newton_schulz_root_inv",
                 "low_rank_matrix_power_neg_quarter"):
        assert callable(getattr(scao_b200, name))


@pytest.mark.skipif(REF is None, reason="reference checkout not present")
@pytest.mark.parametrize("ns", [False, True])
@pytest.mark.parametrize("m", [4, 32])
def test_neg_quarter_matches_reference(m, ns):
    sys.path.insert(0, REF)
    from scao import utils as ru
    A = _spd(m, 100 + m)
    ref = ru.matrix_power_neg_quarter(A, use_newton_schulz=ns)
    got = utils.matrix_power_neg_quarter(A, use_newton_schulz=ns)
    if ns:
        # same iteration, same operation order: identical in float32
        assert torch.equal(got, ref)
    else:
        assert torch.allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_seam_refuses_cpu():
    """scao_b200.cuda has no CPU fallback (the reference's routes to PyTorch)."""
    from scao_b200 import cuda as seam
    z = torch.zeros(4, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        seam.fused_kronecker_precond(torch.zeros(4, 2), torch.ones(2), torch.zeros(4, 2),
                                     torch.ones(2), z)
    with pytest.raises(RuntimeError, match="CUDA"):
        seam.low_rank_precond_mm(torch.zeros(4, 2), torch.ones(2), z)
    with pytest.raises(RuntimeError, match="CUDA"):
        seam.int8_ema_update(torch.zeros(4, dtype=torch.int8), 1.0, torch.zeros(4), 0.9)


def test_average_norms_in_param_dtype():
    """The global grad-norm average takes p.grad.norm() in the gradient's dtype
    (optimizer.py:440): float32 norms rounded like torch's own casts."""
    import numpy as np
    from scao_b200.optimizer import _in_param_dtypes
    ps = [torch.zeros(1, dtype=d) for d in (torch.bfloat16, torch.float32, torch.float16)]
    x = np.array([32.2302131652832, 1.2345678, 1.2345678], np.float32)
    got = _in_param_dtypes(x, ps)
    g = torch.randn(1000, generator=torch.Generator().manual_seed(0))
    assert got[0] == float(torch.tensor(x[0]).bfloat16()) == 32.25
    assert got[1] == x[1] and got[2] == float(np.float16(x[2]))
    # what the reference's float(p.grad.norm()) returns for a bf16 gradient
    assert float(g.bfloat16().norm()) == float(_in_param_dtypes(
        np.array([g.bfloat16().float().norm().item()], np.float32), ps[:1])[0])


@pytest.mark.skipif(REF is None, reason="reference checkout not present")
def test_host_policies_match_reference_classes():
    """R1 warmup scheduler and R3 lazy trigger (optimizer.py:104-214): the
    host classes against the reference's own on random norm sequences
    (drifting, flat, jumping), decision for decision."""
    import numpy as np
    sys.path.insert(0, REF)
    from scao import optimizer as ro
    from scao_b200 import optimizer as so
    rng = np.random.default_rng(7)
    for trial in range(40):
        kind = trial % 4
        n = 200
        if kind == 0:
            x = np.abs(1 + 0.01 * np.cumsum(rng.standard_normal(n)))
        elif kind == 1:
            x = np.full(n, 0.5) + 1e-4 * rng.standard_normal(n)
        elif kind == 2:
            x = np.abs(rng.standard_normal(n)) + 0.1
        else:
            x = np.where(rng.random(n) < 0.1, 5.0, 1.0) * (1 + 0.02 * rng.standard_normal(n))
        kw = dict(warmup_steps=int(rng.integers(20, 150)),
                  stability_threshold=float(rng.choice([0.01, 0.05, 0.2])),
                  patience=int(rng.integers(1, 8)), min_warmup=int(rng.integers(5, 30)))
        a, b = ro._AdaptiveWarmupScheduler(**kw), so._AdaptiveWarmupScheduler(**kw)
        for t, v in enumerate(x, 1):
            assert a.update(t, float(v)) == b.update(t, float(v)), (trial, t)
        assert (a.exited_early, a.actual_warmup_steps) == (b.exited_early, b.actual_warmup_steps)
        tk = dict(delta_threshold=float(rng.choice([0.02, 0.1, 0.5])),
                  max_skip=int(rng.integers(1, 30)))
        c, d = ro._LazyPrecondTrigger(**tk), so._LazyPrecondTrigger(**tk)
        assert [c.should_update(float(v)) for v in x] == [d.should_update(float(v)) for v in x]


@pytest.mark.skipif(REF is None, reason="reference checkout not present")
@pytest.mark.parametrize("name", ["scao_sub1b", "scao_1b", "scao_3b", "scao_7b", "scao_40b",
                                  "scao_125b"])
def test_presets_configure_like_reference(name):
    """optimizer.py:958-1002 (the module's final definitions): same group
    hyperparameters and the same extensions switched on."""
    sys.path.insert(0, REF)
    import scao
    import scao_b200
    ref = getattr(scao, name)([torch.nn.Parameter(torch.zeros(4, 4))])
    ours = getattr(scao_b200, name)([torch.nn.Parameter(torch.zeros(4, 4))])
    rg = {k: v for k, v in ref.param_groups[0].items() if k != "params"}
    og = {k: v for k, v in ours.param_groups[0].items() if k != "params"}
    assert rg == {k: og[k] for k in rg}
    for attr in ("_sparsity", "_dynamic_sparsity", "_adaptive_warmup", "_lazy_precond",
                 "_use_gsnr_clip", "_adaptive_rank", "_noise_std", "_lookahead_k",
                 "_lookahead_alpha"):
        assert getattr(ref, attr) == getattr(ours, attr), attr


@pytest.mark.skipif(REF is None, reason="reference checkout not present")
def test_constructor_defaults_and_errors_match_reference():
    """optimizer.py:258-304: same defaults in every param group, same
    attributes of the extensions, same ValueError cases."""
    sys.path.insert(0, REF)
    import scao
    import scao_b200
    mk = lambda: [torch.nn.Parameter(torch.zeros(3, 3))]
    ref, ours = scao.SCAO(mk()), scao_b200.SCAO(mk())
    assert ref.defaults == {k: ours.defaults[k] for k in ref.defaults}
    for attr in ("_sparsity", "_dynamic_sparsity", "_adaptive_warmup", "_lazy_precond",
                 "_use_gsnr_clip", "_adaptive_rank", "_noise_std", "_noise_anneal",
                 "_lookahead_k", "_lookahead_alpha", "_global_step"):
        assert getattr(ref, attr) == getattr(ours, attr), attr
    for bad in (dict(lr=-1.0), dict(betas=(1.0, 0.9)), dict(betas=(0.9, -0.1)),
                dict(beta3=1.5)):
        with pytest.raises(ValueError):
            scao.SCAO(mk(), **bad)
        with pytest.raises(ValueError):
            scao_b200.SCAO(mk(), **bad)


@pytest.mark.skipif(REF is None, reason="reference checkout not present")
def test_state_dict_top_level_schema_matches_reference():
    """optimizer.py:732-756: same top-level keys, runtime keys and group keys."""
    sys.path.insert(0, REF)
    import scao
    import scao_b200
    mk = lambda: [torch.nn.Parameter(torch.zeros(3, 3))]
    r, o = scao.SCAO(mk()).state_dict(), scao_b200.SCAO(mk()).state_dict()
    assert sorted(r) == sorted(o)
    assert sorted(r["_scao_runtime"]) == sorted(o["_scao_runtime"])
    assert r["param_groups"][0].keys() == o["param_groups"][0].keys()


def test_add_param_group_before_first_step_only():
    """Groups added before the first step join the plan with the defaults
    filled in; after it (plan laid out) the call raises instead of failing
    later inside the step."""
    import scao_b200
    o = scao_b200.SCAO([torch.nn.Parameter(torch.zeros(3, 3))])
    o.add_param_group({"params": [torch.nn.Parameter(torch.zeros(4))], "lr": 1e-2})
    assert len(o.param_groups) == 2 and o.param_groups[1]["lr"] == 1e-2
    assert o.param_groups[1]["k_max"] == o.defaults["k_max"]
    o._plan = object()          # stands for the plan the first step builds
    with pytest.raises(NotImplementedError):
        o.add_param_group({"params": [torch.nn.Parameter(torch.zeros(2))]})
