"""``SparsePreconditioner`` (scao/preconditioner.py:72-644) on the host: mode
selection, block structure, rank bounds, checkpoint schema and memory
accounting against the reference class; compute methods refuse CPU tensors
(the product has no CPU path)."""
import os
import sys

import pytest
import torch

from scao_b200 import SparsePreconditioner

from golden_util import reference_root  # noqa: E402

REF = reference_root()
SHAPES = [((64, 48), 4096), ((128, 16), 64), ((49, 40), 48), ((97, 97), 48), ((40,), 48),
          ((8, 4, 5), 4096)]


def test_block_diagonal_activates():
    """The reference's own check (tests/test_optimizer.py:621-636)."""
    prec = SparsePreconditioner(torch.randn(128, 16), max_precond_dim=64)
    assert prec.use_block_diagonal and not prec.use_kronecker
    assert len(prec._blocks) == 2 and prec._block_dim == 0
    assert all(b.use_kronecker for b in prec._blocks)


def test_diag_and_kron_modes():
    assert not SparsePreconditioner(torch.zeros(7)).use_kronecker
    p = SparsePreconditioner(torch.zeros(32, 24), k_min=4, k_max=8)
    assert p.use_kronecker and p.k == 4 and (p.k_min, p.k_max) == (4, 8)
    assert p.U_l.shape == (32, 4) and torch.equal(p.S_l, torch.ones(4))


def test_compute_refuses_cpu():
    p = SparsePreconditioner(torch.zeros(16, 8))
    for f in (p.update_curvature, p.precondition, p.natural_grad_norm):
        with pytest.raises(RuntimeError, match="CUDA"):
            f(torch.zeros(16, 8))


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
def test_matches_reference_class(shape, mpd, int8):
    sys.path.insert(0, REF)
    from scao.preconditioner import SparsePreconditioner as Ref
    kw = dict(k_min=4, k_max=8, max_precond_dim=mpd, use_int8_ema=int8)
    ref = Ref(torch.zeros(shape), **kw)
    ours = SparsePreconditioner(torch.zeros(shape), **kw)
    for a in ("use_kronecker", "use_block_diagonal", "k", "k_min", "k_max", "m", "n"):
        assert getattr(ours, a) == getattr(ref, a), a
    if ref.use_block_diagonal:
        assert ours._block_sizes == ref._block_sizes and ours._block_dim == ref._block_dim
        assert [b.use_kronecker for b in ours._blocks] == [b.use_kronecker for b in ref._blocks]
    assert _structure(ours.state_dict()) == _structure(ref.state_dict())
    assert ours.memory_bytes() == ref.memory_bytes()
