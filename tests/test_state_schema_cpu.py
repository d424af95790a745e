"""Checkpoint schema of the preconditioner state (preconditioner.py:570-600)
matches the reference's, including the nesting of block-diagonal splits.
Runs on CPU: the plan's arenas can live on the host for this check."""
import os
import sys

import pytest
import torch

from scao_b200.plan import Plan
from scao_b200.preconditioner import PrecondView

from golden_util import reference_root  # noqa: E402

REF = reference_root()

SHAPES = [((96, 128), 48), ((100, 30), 48), ((50, 7), 48), ((16,), 48), ((33, 200), 64),
          # width-1 remainders: diagonal sub-preconditioners inside the split
          ((49, 40), 48), ((40, 97), 48), ((97, 97), 48)]


def _ours(shape, mpd, int8):
    p = torch.zeros(shape)
    g = dict(max_precond_dim=mpd, k_min=4, k_max=8, epsilon_sparse=0.05, rho=0.999)
    plan = Plan([p], [g], torch.device("cpu"), int8)
    return PrecondView(plan, 0, g).state_dict()


def _structure(d):
    out = {}
    for k, v in d.items():
        if k == "blocks":
            out[k] = [_structure(b) for b in v]
        elif torch.is_tensor(v):
            out[k] = (tuple(v.shape), v.dtype)
        else:
            out[k] = v
    return out


@pytest.mark.skipif(REF is None, reason="reference checkout not present")
@pytest.mark.parametrize("int8", [True, False])
@pytest.mark.parametrize("shape,mpd", SHAPES)
def test_schema_matches_reference(shape, mpd, int8):
    sys.path.insert(0, REF)
    from scao.preconditioner import SparsePreconditioner
    ref = SparsePreconditioner(torch.zeros(shape), k_min=4, k_max=8, max_precond_dim=mpd,
                               use_int8_ema=int8).state_dict()
    assert _structure(_ours(shape, mpd, int8)) == _structure(ref)


def test_nested_schema_without_reference():
    d = _ours((96, 128), 48, True)
    assert d["use_block_diagonal"] and len(d["blocks"]) == 3
    assert all(b["use_block_diagonal"] and len(b["blocks"]) == 2 for b in d["blocks"])
    leaf = d["blocks"][0]["blocks"][0]
    assert leaf["use_kronecker"] and leaf["L_ema_q"].dtype == torch.int8


@pytest.mark.parametrize("shape,mpd", [((49, 40), 48), ((40, 97), 48), ((97, 97), 48),
                                       ((3, 2049), 1024)])
def test_strips_and_leaves_tile_the_parameter(shape, mpd):
    """Kronecker leaves and diagonal strips cover every element once; strip
    diag_ema views address exactly their elements."""
    import numpy as np
    p = torch.zeros(shape)
    g = dict(max_precond_dim=mpd, k_min=4, k_max=8, epsilon_sparse=0.05, rho=0.999)
    plan = Plan([p], [g], torch.device("cpu"), True)
    m, n = shape
    cover = np.zeros(m * n, np.int32)
    for L in plan.ltab:
        r0, c0, a, b = (int(L[k]) for k in ("row0", "col0", "a", "b"))
        for r in range(r0, r0 + a):
            cover[r * n + c0: r * n + c0 + b] += 1
    for S in plan.stab:
        cover[int(S["begin"]) + np.arange(int(S["count"])) * int(S["stride"])] += 1
    assert (cover == 1).all()
    pv = PrecondView(plan, 0, g)
    strips = [v for v in pv._views if not v.use_kronecker]
    assert len(strips) == plan.n_strips > 0
    for v in strips:
        v.diag_ema.fill_(1.0)
    assert int(plan.diag_ema.sum().item()) == sum(int(S["count"]) for S in plan.stab)
    assert pv.k_host(plan.k.numpy()) >= 1


def test_reference_checkpoint_schema_matches_ours():
    """The committed reference checkpoint (make_golden.py --ckpt) has, per
    parameter, the same nested preconditioner schema as ours -- keys, block
    nesting, factor shapes and dtypes -- so load_state_dict can take it."""
    from golden_util import HERE
    from scao_b200 import workloads
    d = torch.load(os.path.join(HERE, "ckpt_tiny_f32.pt"))
    w = workloads.tiny(dtype="float32", max_precond_dim=48, grad_scale=1.0, int8=True)
    g = dict(dict(epsilon_sparse=0.05, rho=0.999), **w.scao_kwargs)
    plan = Plan([torch.zeros(s.shape) for s in w.params], [g] * len(w.params),
                torch.device("cpu"), True)

    def shape_only(x):
        if isinstance(x, dict):
            return {k: shape_only(v) for k, v in x.items()
                    if k not in ("k", "precond_step", "U_l", "S_l", "U_r", "S_r")}
        if isinstance(x, list):
            return [shape_only(v) for v in x]
        if torch.is_tensor(x):
            return (tuple(x.shape), x.dtype)
        return type(x).__name__ if isinstance(x, float) else x

    for i in range(len(w.params)):
        ours = PrecondView(plan, i, g).state_dict()
        assert shape_only(d["state_dict"]["_scao_precond"][i]) == shape_only(ours), i


def test_plan_tables_cover_random_shapes():
    """The plan's tables for random parameter sets (remainders of width 1,
    nested splits, 1-D and 3-D parameters): leaves and strips tile every
    matrix exactly once, tiles tile every leaf, panels cover its rows, flat
    chunks cover every parameter, arena offsets are 8-element aligned."""
    import numpy as np
    from scao_b200 import plan as P
    rng = np.random.default_rng(3)
    for trial in range(40):
        mpd = int(rng.choice([16, 48, 64, 128]))
        shapes = []
        for _ in range(int(rng.integers(1, 5))):
            kind = rng.integers(0, 4)
            if kind == 0:
                shapes.append((int(rng.integers(1, 300)),))
            elif kind == 1:
                shapes.append((int(mpd * rng.integers(1, 4) + rng.choice([0, 1, 7])),
                               int(rng.integers(2, 3 * mpd))))
            elif kind == 2:
                shapes.append((int(rng.integers(2, 3 * mpd)),
                               int(mpd * rng.integers(1, 4) + rng.choice([0, 1, 5]))))
            else:
                shapes.append((int(rng.integers(2, 20)), int(rng.integers(1, 6)),
                               int(rng.integers(2, 9))))
        g = dict(max_precond_dim=mpd, k_min=4, k_max=16, epsilon_sparse=0.05, rho=0.999)
        params = [torch.zeros(s) for s in shapes]
        try:
            plan = Plan(params, [g] * len(params), torch.device("cpu"), True)
        except NotImplementedError:
            continue            # a split leaving no Kronecker block at all
        for i, p in enumerate(params):
            r = plan.ptab[i]
            assert int(r["offset"]) % 8 == 0
            n = p.numel()
            cov = np.zeros(n, np.int32)
            for c in plan.ctab[int(r["chunk_begin"]):int(r["chunk_end"])]:
                cov[int(c["begin"]):int(c["end"])] += 1
            assert (cov == 1).all(), (shapes[i], mpd)
            if int(r["mode"]) != 1:
                continue
            m, ncol = P.to_2d_shape(tuple(p.shape))
            cov = np.zeros(m * ncol, np.int32)
            for li in plan.param_leaves[i]:
                L = plan.ltab[li]
                r0, c0, a, b = (int(L[k]) for k in ("row0", "col0", "a", "b"))
                assert a > 1 and b > 1
                for rr in range(r0, r0 + a):
                    cov[rr * ncol + c0: rr * ncol + c0 + b] += 1
                tcov = np.zeros((a, b), np.int32)
                for t in plan.ttab[int(L["tile_begin"]):int(L["tile_end"])]:
                    tr, tc = int(t["row0"]), int(t["col0"])
                    tcov[tr:tr + P.TILE, tc:tc + P.TILE] += 1
                assert (tcov == 1).all()
                rows = sum(int(pn["nrows"]) for pn in plan.pantab[int(L["panel_begin"]):int(L["panel_end"])])
                assert rows == a
            for si in plan.param_strips[i]:
                S = plan.stab[si]
                cov[int(S["begin"]) + np.arange(int(S["count"])) * int(S["stride"])] += 1
            assert (cov == 1).all(), (shapes[i], mpd)
