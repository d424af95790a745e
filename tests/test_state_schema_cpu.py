"""Checkpoint schema of the preconditioner state (preconditioner.py:570-600)
matches the reference's, including the nesting of block-diagonal splits.
Runs on CPU: the plan's arenas can live on the host for this check."""
import os
import sys

import pytest
import torch

from scao_b200.plan import Plan
from scao_b200.preconditioner import PrecondView

REF = "/root/reference"

SHAPES = [((96, 128), 48), ((100, 30), 48), ((50, 7), 48), ((16,), 48), ((33, 200), 64)]


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


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference checkout not present")
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
