"""Per-parameter preconditioner view over the plan's device arenas.

``state["preconditioner"]`` of the reference is a ``SparsePreconditioner``
object (scao/preconditioner.py:72-644).  Here the factors of all parameters
live in flat device arenas owned by the plan; this class exposes one
parameter's slice of them with the reference's attribute names and its exact
``state_dict`` schema (preconditioner.py:570-600, 621-644).
"""
from __future__ import annotations

import numpy as np
import torch

from .plan import k_bounds, to_2d_shape


def _scale_from_absmax(am):
    """utils.py:184-187: Python-float scale from the float32 absmax."""
    am = float(np.float32(am))
    return 1.0 if am < 1e-30 else am / 127.0


def _absmax_from_scale(scale, q_nonzero):
    """Inverse of _scale_from_absmax (exact: picks the float32 absmax whose
    float64(absmax)/127 reproduces ``scale``)."""
    if not q_nonzero or scale == 1.0 and not q_nonzero:
        return np.float32(0.0)
    a = np.float32(scale * 127.0)
    for cand in (a, np.nextafter(a, np.float32(np.inf)), np.nextafter(a, np.float32(0))):
        if float(cand) / 127.0 == scale:
            return cand
    return a


class LeafView:
    """One Kronecker leaf (a block of the reference's block-diagonal split)."""

    def __init__(self, plan, li, owner):
        self.plan, self.li, self.owner = plan, li, owner
        L = plan.ltab[li]
        self.m, self.n = int(L["a"]), int(L["b"])
        self.k_min, self.k_max = int(L["kmin"]), int(L["kmax"])
        self.use_kronecker = True
        self.use_block_diagonal = False
        self.use_int8_ema = plan.int8_ema

    @property
    def precond_step(self):
        return self.owner.precond_step

    @property
    def k(self):
        return int(self.plan.k[self.li].item())

    def __getattr__(self, name):
        # the reference's tensor attributes (U_l, S_l, L_ema_q, ...), as copies
        if name in PrecondView._KRON_ATTRS:
            st = self.state_dict()
            if name in st:
                return st[name]
        raise AttributeError(name)

    def _fac(self, side):
        L = self.plan.ltab[self.li]
        n = self.m if side == 0 else self.n
        o = int(L["lq_off"] if side == 0 else L["rq_off"])
        return self.plan.fac[o:o + n * n].view(n, n)

    def _u(self, side, k):
        L = self.plan.ltab[self.li]
        n = self.m if side == 0 else self.n
        s = int(L["sl"] if side == 0 else L["sr"])
        o = int(L["ul_off"] if side == 0 else L["ur_off"])
        return self.plan.u[o:o + n * s].view(n, s)[:, :k]

    def _s(self, side, k):
        L = self.plan.ltab[self.li]
        o = int(L["evl_off"] if side == 0 else L["evr_off"])
        return self.plan.ev[o:o + k]

    @property
    def L_ema_scale(self):
        return _scale_from_absmax(self.plan.absmax[2 * self.li].item())

    @property
    def R_ema_scale(self):
        return _scale_from_absmax(self.plan.absmax[2 * self.li + 1].item())

    def state_dict(self):
        k = self.k
        d = {"precond_step": self.precond_step, "k": k, "use_kronecker": True,
             "use_block_diagonal": False}
        if self.use_int8_ema:
            d.update({"L_ema_q": self._fac(0).clone(), "L_ema_scale": self.L_ema_scale,
                      "R_ema_q": self._fac(1).clone(), "R_ema_scale": self.R_ema_scale})
        else:
            d.update({"L_ema": self._fac(0).clone(), "R_ema": self._fac(1).clone()})
        if self.precond_step == 0:
            # before the first eigen update the reference holds eye(m, k), ones(k)
            dev = self.plan.device
            d.update({"U_l": torch.eye(self.m, k, device=dev), "S_l": torch.ones(k, device=dev),
                      "U_r": torch.eye(self.n, k, device=dev), "S_r": torch.ones(k, device=dev)})
        else:
            d.update({"U_l": self._u(0, k).contiguous(), "S_l": self._s(0, k).clone(),
                      "U_r": self._u(1, k).contiguous(), "S_r": self._s(1, k).clone()})
        return d

    def load_state_dict(self, st):
        k = int(st["k"])
        self.plan.k[self.li] = k
        if self.use_int8_ema:
            for side, qk, sk in ((0, "L_ema_q", "L_ema_scale"), (1, "R_ema_q", "R_ema_scale")):
                q = st[qk].to(device=self.plan.device, dtype=torch.int8)
                self._fac(side).copy_(q)
                am = _absmax_from_scale(float(st[sk]), bool(q.ne(0).any().item()))
                self.plan.absmax[2 * self.li + side] = float(am)
        else:
            self._fac(0).copy_(st["L_ema"])
            self._fac(1).copy_(st["R_ema"])
        for side, uk, sk in ((0, "U_l", "S_l"), (1, "U_r", "S_r")):
            S = st[sk].to(device=self.plan.device, dtype=torch.float32)
            self._u_full(side).copy_(self._complete_basis(st[uk], side))
            self._s(side, S.shape[0]).copy_(S)

    def _u_full(self, side):
        L = self.plan.ltab[self.li]
        n = self.m if side == 0 else self.n
        s = int(L["sl"] if side == 0 else L["sr"])
        o = int(L["ul_off"] if side == 0 else L["ur_off"])
        return self.plan.u[o:o + n * s].view(n, s)

    def _complete_basis(self, U, side):
        """The stored top-k eigenvectors as the first k columns of an
        orthonormal n x s basis (the eigensolver's warm start must be
        orthonormal: the direct solve (s = n) and the first Rayleigh-Ritz step
        read it as such).  Householder QR of [U, I] in float64 on the host: the
        first k columns of Q are +-U, the rest are orthogonal to it."""
        n = self.m if side == 0 else self.n
        s = int(self.plan.ltab[self.li]["sl" if side == 0 else "sr"])
        U = U.detach().to("cpu", torch.float64)
        k = U.shape[1]
        if k >= s:
            return U[:, :s].to(torch.float32)
        Q, R = torch.linalg.qr(torch.cat([U, torch.eye(n, dtype=torch.float64)], 1),
                               mode="reduced")
        Q = Q[:, :s].clone()
        sg = torch.sign(torch.diagonal(R)[:k])
        sg[sg == 0] = 1.0
        Q[:, :k] *= sg
        Q[:, :k] = U                   # bit-exact stored columns
        return Q.to(torch.float32)


class StripView:
    """A width-1 block of the split (1 x b or a x 1): the reference's diagonal
    sub-preconditioner (preconditioner.py:232-236), whose ``diag_ema`` is a
    strided slice of the plan's diagonal arena."""

    def __init__(self, plan, si, owner):
        self.plan, self.si, self.owner = plan, si, owner
        S = plan.stab[si]
        self.count, self.stride = int(S["count"]), int(S["stride"])
        self.begin = int(S["begin"])
        self.pi = int(S["param"])
        self.m, self.n = (1, self.count) if self.stride == 1 else (self.count, 1)
        self.k_min = self.k_max = 1
        self.use_kronecker = False
        self.use_block_diagonal = False
        self.use_int8_ema = plan.int8_ema

    @property
    def precond_step(self):
        return self.owner.precond_step

    @property
    def k(self):
        return 1

    @property
    def diag_ema(self):
        o = int(self.plan.ptab[self.pi]["offset"]) + self.begin
        return self.plan.diag_ema.as_strided((self.m, self.n),
                                             (self.stride, 1) if self.stride != 1 else (self.count, 1),
                                             o)

    def state_dict(self):
        return {"precond_step": self.precond_step, "k": 1, "use_kronecker": False,
                "use_block_diagonal": False, "diag_ema": self.diag_ema.clone()}

    def load_state_dict(self, st):
        self.diag_ema.copy_(st["diag_ema"].reshape(self.m, self.n))


class _BlockNode:
    """An inner node of a nested block-diagonal split (a block whose own
    larger dimension still exceeds max_precond_dim, preconditioner.py:163-194)."""

    use_kronecker = False
    use_block_diagonal = True

    def __init__(self, owner, kids):
        self.owner = owner
        self._blocks = [_BlockNode(owner, x) if isinstance(x, list) else x for x in kids]

    @property
    def precond_step(self):
        return self.owner.precond_step

    @property
    def k(self):
        ks = [b.k for b in self._blocks]
        if self.owner.precond_step == 0 and not self.owner._k_mean:
            return ks[0]
        return sum(ks) // max(len(ks), 1)


class PrecondView:
    """``state["preconditioner"]`` of one parameter."""

    def __init__(self, plan, pi, group):
        self.plan, self.pi = plan, pi
        p = plan.params[pi]
        self.original_shape = tuple(p.shape)
        self.m, self.n = to_2d_shape(self.original_shape)
        self.precond_step = 0
        self.rho = group["rho"]
        self.use_int8_ema = plan.int8_ema
        leaves = plan.param_leaves[pi]
        self.use_kronecker = len(leaves) == 1 and int(plan.ptab[pi]["mode"]) == 1 and \
            plan.ltab[leaves[0]]["a"] == self.m and plan.ltab[leaves[0]]["b"] == self.n
        self.use_block_diagonal = int(plan.ptab[pi]["mode"]) == 1 and not self.use_kronecker
        self._leaves = [LeafView(plan, li, self) for li in leaves]
        # every block of the split in order: Kronecker leaves and diagonal strips
        self._views = [LeafView(plan, x, self) if kind == "L" else StripView(plan, x, self)
                       for kind, x in plan.param_blocks[pi]]
        # the reference's ``_blocks`` hierarchy: children of the top split
        # (leaf / strip views, or nodes of a nested split)
        self._blocks = [_BlockNode(self, x) if isinstance(x, list) else x
                        for x in self._nest(plan.param_trees[pi], iter(self._views))] \
            if self.use_block_diagonal else []
        # rank bounds of every node of the block tree (preconditioner.py:122-124)
        self._ktree = self._bounds_tree(self.m, self.n, group["max_precond_dim"],
                                        group["k_min"], group["k_max"],
                                        iter(plan.param_blocks[pi])) if leaves else None
        self._k_mean = False     # an R5 assignment made every level a block mean
        self._k_plain = None     # R5-assigned k of a leaf-free (diagonal) parameter

    # the reference's tensor attributes of a single Kronecker block (copies)
    _KRON_ATTRS = ("U_l", "S_l", "U_r", "S_r", "L_ema_q", "L_ema_scale", "R_ema_q",
                   "R_ema_scale", "L_ema", "R_ema")

    def __getattr__(self, name):
        d = self.__dict__
        if d.get("use_kronecker") and name in PrecondView._KRON_ATTRS:
            st = d["_views"][0].state_dict()
            if name in st:
                return st[name]
        raise AttributeError(name)

    @staticmethod
    def _nest(t, views):
        """Views of tree t: a leaf / strip view, or the list of its children."""
        if t == 1 or t == 0:
            return next(views)
        return [PrecondView._nest(c, views) for c in t]

    @staticmethod
    def _bounds_tree(m, n, mpd, kmin, kmax, blocks):
        """(k_min, k_max, child): child = a leaf index, None for a diagonal
        strip (rank 1), or the list of sub-trees."""
        lo, hi = k_bounds(m, n, kmin, kmax)
        if m <= 1 or n <= 1:
            next(blocks)
            return (1, 1, None)
        if max(m, n) <= mpd:
            return (lo, hi, next(blocks)[1])
        large, small = (m, n) if m >= n else (n, m)
        sizes = [mpd] * (large // mpd) + ([large % mpd] if large % mpd else [])
        kids = [PrecondView._bounds_tree(*((bs, small) if m >= n else (small, bs)), mpd, kmin,
                                         kmax, blocks) for bs in sizes]
        return (lo, hi, kids)

    def _walk_k(self, node, kvec):
        lo, hi, c = node
        if c is None:
            return 1
        if not isinstance(c, list):
            return int(kvec[c])
        sub = [self._walk_k(x, kvec) for x in c]
        if self.precond_step == 0 and not self._k_mean:   # initialised as the first block's k (:194)
            return sub[0]
        return sum(sub) // max(len(sub), 1)              # mean of the blocks (:329)

    def k_host(self, kvec):
        """``k`` from a host copy of the per-leaf ranks."""
        if self._ktree is None:
            return 1 if self._k_plain is None else self._k_plain
        return self._walk_k(self._ktree, kvec)

    def set_k_host(self, new_k, kvec):
        """R5 rank assignment (preconditioner.py:249-291) on a host copy of
        the per-leaf ranks: clamp to each node's [k_min, k_max]; a leaf only
        ever shrinks (growth waits for the next eigen update, because the
        eigenfactors hold exactly k columns); block-diagonal nodes propagate
        and become the mean of their blocks.  Returns True if kvec changed."""
        if self._ktree is None:
            lo, hi = k_bounds(self.m, self.n, 1, 1) if self.m > 1 else (1, 1)
            self._k_plain = int(min(hi, max(lo, new_k)))
            return False
        changed = False

        def setk(node, k):
            nonlocal changed
            lo, hi, c = node
            k = int(min(hi, max(lo, k)))
            if isinstance(c, list):
                for x in c:
                    setk(x, k)
                return
            if c is None:
                return
            if k < int(kvec[c]):
                kvec[c] = k
                changed = True

        setk(self._ktree, new_k)
        if isinstance(self._ktree[2], list):
            self._k_mean = True
        return changed

    @property
    def diag_bias(self):
        return max(1.0 - self.rho ** self.precond_step, 1e-8) if self.precond_step else 1e-8

    @property
    def k(self):
        if not self._leaves:
            return 1 if self._k_plain is None else self._k_plain
        return self._walk_k(self._ktree, self.plan.k.cpu().numpy())

    @k.setter
    def k(self, new_k):
        """preconditioner.py:249-291 (external rank assignment, R5)."""
        kvec = self.plan.k.cpu().numpy().copy()
        if self.set_k_host(int(new_k), kvec):
            self.plan.k.copy_(torch.from_numpy(kvec).to(self.plan.device))

    @property
    def diag_ema(self):
        return self.plan.state_view(self.plan.diag_ema, self.pi)

    def _tree_state(self, t, leaves):
        if t == 1 or t == 0:
            return next(leaves).state_dict()
        blocks = [self._tree_state(c, leaves) for c in t]
        k = blocks[0]["k"] if self.precond_step == 0 and not self._k_mean else \
            sum(b["k"] for b in blocks) // max(len(blocks), 1)
        return {"precond_step": self.precond_step, "k": k, "use_kronecker": False,
                "use_block_diagonal": True, "blocks": blocks}

    def _tree_load(self, t, st, leaves):
        if t == 1 or t == 0:
            next(leaves).load_state_dict(st)
            return
        for c, bs in zip(t, st["blocks"]):
            self._tree_load(c, bs, leaves)

    def state_dict(self):
        """Same schema as preconditioner.py:570-600, nested like the
        reference's ``_blocks`` hierarchy."""
        if self.use_block_diagonal or self.use_kronecker:
            return self._tree_state(self.plan.param_trees[self.pi], iter(self._views))
        return {"precond_step": self.precond_step, "k": 1, "use_kronecker": False,
                "use_block_diagonal": False, "diag_ema": self.diag_ema.clone()}

    def load_state_dict(self, st):
        self.precond_step = int(st["precond_step"])
        if self.use_block_diagonal or self.use_kronecker:
            self._tree_load(self.plan.param_trees[self.pi], st, iter(self._views))
            # the apply reads the eigenvectors through their bf16 operand tiles
            self.plan.prep_leaves(self.plan.param_leaves[self.pi])
        else:
            self.diag_ema.copy_(st["diag_ema"])
