"""Owner-compute sharding of the SCAO step across the GPUs of one node.

The reference's distributed helpers (scao/distributed.py:60-160) keep the full
optimizer state on every rank and all-reduce-average preconditioner factors
after curvature steps.  Here every parameter -- with its moments, its int8
curvature factors and its eigenfactors -- is owned by exactly one rank:

    1. reduce-scatter (average) of the gradients into owner-contiguous shards
       (the data-parallel gradient reduction, done once, by owner);
    2. each rank runs the batched SCAO step on the parameters it owns;
    3. all-gather of the updated parameters.

Because the step is independent per parameter (the LARS trust ratio and the
curvature clip are per-parameter reductions), the result is identical to the
single-GPU step on the averaged gradient.  The global grad-norm
EMA (optimizer.py:439-446), which steers the optional R1 adaptive warmup, R2
dynamic sparsity and R5 adaptive rank, is an average over all parameters:
when one of them is on, the owners exchange their per-parameter norms each
step (one small all-reduce) before any bucket steps.  ``sync_preconditioners`` and
``wrap_scao_for_fsdp`` keep the reference's API for replicated optimizers.
"""
from __future__ import annotations

import heapq

import torch
import torch.distributed as dist

ALIGN = 64   # elements: every parameter slot starts on a 128-byte boundary


def partition(costs, world):
    """Greedy LPT: assign items (largest cost first) to the least-loaded rank.
    Deterministic (ties broken by rank, then item index)."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    owner = [0] * len(costs)
    for i in order:
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + costs[i], r))
    return owner


def _round_up(x, k):
    return (x + k - 1) // k * k


class FlatLayout:
    """Bucket-major owner layout of a flat buffer.  Each rank's parameters (in
    model order) are cut into ``buckets`` contiguous groups of similar size;
    bucket b occupies [base_b, base_b + world * seg_b) with rank r's part at
    base_b + r * seg_b, so one reduce-scatter / all-gather per bucket works on
    a contiguous range and the buckets can be pipelined."""

    def __init__(self, numels, owner, world, buckets=1):
        self.world = world
        self.owner = owner
        self.numels = numels
        n = len(numels)
        self.bucket = [0] * n
        self.offsets = [0] * n
        size = [_round_up(x, ALIGN) for x in numels]
        # each rank's items, largest first (ties by index)
        queue = [sorted((i for i in range(n) if owner[i] == r), key=lambda i: (-size[i], i))
                 for r in range(world)]
        fill = {}

        def pick(q, cap):
            """Largest-first fit of q's items into cap (the largest always)."""
            took, f = [], 0
            for i in q:
                if not took or f + size[i] <= cap:
                    took.append(i)
                    f += size[i]
            return took, f

        # Buckets are filled for all ranks together so that each bucket's
        # segment (the max over ranks) carries little padding: a bucket's
        # segment is set by the rank that needs most for a target share of
        # its remaining load (its largest item at least), then every rank
        # packs up to it; the last bucket takes what is left.  A few target
        # shares per bucket are tried and the layout with the smallest sum of
        # segments is kept.  Within a bucket items keep model order.
        def plan(queue, b):
            if b == buckets - 1:
                return (max(sum(size[i] for i in q) for q in queue), [list(q) for q in queue]),
            base = max(sum(size[i] for i in q) for q in queue) / (buckets - b)
            if base == 0:
                return ((0, [[] for _ in queue]),) * (buckets - b)
            best = None
            for s in (0.8, 0.9, 1.0, 1.12, 1.25):
                seg = max(pick(q, base * s)[1] if q else 0 for q in queue)
                took = [pick(q, seg)[0] if q else [] for q in queue]
                rest = [[i for i in q if i not in ts] for q, ts in zip(queue, map(set, took))]
                tail = plan(rest, b + 1)
                tot = max(sum(size[i] for i in t) for t in took) + sum(x[0] for x in tail)
                # the first bucket's reduce-scatter and the last one's
                # all-gather are the pipeline's exposed ends: large end
                # segments are charged a little extra
                tot += 0.1 * tail[-1][0]
                if b == 0:
                    tot += 0.1 * max(sum(size[i] for i in t) for t in took)
                if best is None or tot < best[0]:
                    best = (tot, ((max(sum(size[i] for i in t) for t in took), took),) + tail)
            return best[1]

        for b, (_, took) in enumerate(plan(queue, 0)):
            for r in range(world):
                f = 0
                for i in sorted(took[r]):
                    self.bucket[i], self.offsets[i] = b, f
                    f += size[i]
                fill[(r, b)] = f
        self.nb = buckets
        self.seg = [max([fill.get((r, b), 0) for r in range(world)] + [ALIGN])
                    for b in range(buckets)]
        self.base = [0] * buckets
        self.gbase = [0] * buckets      # bucket start inside a rank's own shard
        for b in range(1, buckets):
            self.base[b] = self.base[b - 1] + world * self.seg[b - 1]
            self.gbase[b] = self.gbase[b - 1] + self.seg[b - 1]
        self.total = self.base[-1] + world * self.seg[-1]
        self.shard = sum(self.seg)

    def global_offset(self, i):
        b = self.bucket[i]
        return self.base[b] + self.owner[i] * self.seg[b] + self.offsets[i]

    def shard_offset(self, i):
        return self.gbase[self.bucket[i]] + self.offsets[i]


class ShardedSCAO:
    """Owner-compute wrapper.  ``make_inner(list of (param, spec))`` builds the
    per-rank optimizer over the owned parameters of one bucket (a
    ``scao_b200.SCAO`` on GPUs; tests inject CPU stand-ins).  Parameters are
    re-pointed into one flat buffer so the all-gather writes them in place.
    On NCCL the buckets are pipelined: all reduce-scatters are queued on a
    communication stream, bucket b's step runs as soon as its gradients have
    arrived, and its all-gather is queued right after its step."""

    def __init__(self, params, workload, make_inner, group=None, costs=None, buckets=4,
                 comm_priority=True, sm_reserve=32):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.params = list(params)
        self.specs = list(workload.params)
        numels = [p.numel() for p in self.params]
        self.owner = partition(costs or numels, self.world)
        self.layout = lay = FlatLayout(numels, self.owner, self.world, buckets)
        p0 = self.params[0]
        self.dtype, self.device = p0.dtype, p0.device
        self.flat_p = torch.zeros(lay.total, dtype=self.dtype, device=self.device)
        for i, p in enumerate(self.params):
            o = lay.global_offset(i)
            view = self.flat_p[o:o + p.numel()].view_as(p)
            view.copy_(p.data)
            p.data = view
        self.my = [i for i in range(len(self.params)) if self.owner[i] == self.rank]
        self.my_g = torch.zeros(lay.shard, dtype=self.dtype, device=self.device)
        for i in self.my:
            o = lay.shard_offset(i)
            self.params[i].grad = self.my_g[o:o + numels[i]].view_as(self.params[i])
        self.inner = []
        for b in range(lay.nb):
            mine = [i for i in self.my if lay.bucket[i] == b]
            self.inner.append(make_inner([(self.params[i], self.specs[i]) for i in mine])
                              if mine else None)
        # the step's persistent kernels leave SMs to the concurrent NCCL kernels
        for opt in self.inner:
            if opt is not None and hasattr(opt, "_sm_reserve"):
                opt._sm_reserve = sm_reserve if dist.get_backend(group) == "nccl" else 0
        self.global_step = 0
        self.grad_sets = []
        self.cur = None
        self.nccl = dist.get_backend(group) == "nccl"
        # a high-priority communication stream: the collectives' blocks are
        # scheduled ahead of queued compute blocks, so the pipeline keeps moving
        self.comm = (torch.cuda.Stream(self.device, priority=-1 if comm_priority else 0)
                     if self.nccl else None)
        self.skip_comm = False       # measurement only: compute without collectives
        self.skip_compute = False    # measurement only: collectives without compute
        # R1 / R2-dynamic / R5 steer by the global grad-norm EMA, an average
        # over ALL parameters: the owners exchange their norms each step
        # (one small all-reduce) and every inner optimizer takes that average
        self.norm_sync = any(o is not None and (getattr(o, "_host_norms", False) or
                                                getattr(o, "_dynamic_sparsity", False))
                             for o in self.inner)
        if self.norm_sync:
            for o in self.inner:
                if o is not None:
                    o._host_norms = True      # the host keeps the EMA (from the average)

    @property
    def param_groups(self):
        """The param groups of this rank's inner optimizers (the same dicts):
        learning-rate changes made here reach the step, e.g.
        ``for g in sharded.param_groups: g["lr"] = lr``."""
        return [g for o in self.inner if o is not None for g in getattr(o, "param_groups", [])]

    def owned_specs(self):
        return [self.specs[i] for i in self.my]

    # bucket views ------------------------------------------------------------
    def _views(self, flat, b):
        lay = self.layout
        full = flat[lay.base[b]:lay.base[b] + self.world * lay.seg[b]]
        mine_p = self.flat_p[lay.base[b] + self.rank * lay.seg[b]:
                             lay.base[b] + (self.rank + 1) * lay.seg[b]]
        mine_g = self.my_g[lay.gbase[b]:lay.gbase[b] + lay.seg[b]]
        return full, mine_p, mine_g

    # gradients ------------------------------------------------------------
    def stage_grads(self, full_grads):
        """Lay a full (per-rank) gradient list out as one flat buffer in the
        bucket-major owner layout; returns its index."""
        flat = torch.zeros(self.layout.total, dtype=self.dtype, device=self.device)
        for i, g in enumerate(full_grads):
            o = self.layout.global_offset(i)
            flat[o:o + g.numel()].copy_(g.reshape(-1))
        self.grad_sets.append(flat)
        return len(self.grad_sets) - 1

    def load_grads(self, full_grads):
        key = id(full_grads)
        if not hasattr(self, "_staged"):
            self._staged = {}
        if key not in self._staged:
            self._staged[key] = self.stage_grads(full_grads)
        self.cur = self.grad_sets[self._staged[key]]

    def flat_grad_from_params(self):
        """Training-loop entry: gather every parameter's local .grad (as left
        by backward) into the flat buffer, then point the owned parameters'
        .grad back at their shard of the reduced gradient.  With
        ``attach_grad_hooks`` the hooks have done this already (no-op)."""
        if getattr(self, "_pending", None) is not None:
            return
        if getattr(self, "_train_flat", None) is None:
            self._train_flat = torch.zeros(self.layout.total, dtype=self.dtype, device=self.device)
        flat = self._train_flat
        for i, p in enumerate(self.params):
            o = self.layout.global_offset(i)
            if p.grad is None:
                flat[o:o + p.numel()].zero_()
            else:
                flat[o:o + p.numel()].copy_(p.grad.reshape(-1))
        for i in self.my:
            o = self.layout.shard_offset(i)
            self.params[i].grad = self.my_g[o:o + self.params[i].numel()].view_as(self.params[i])
        self.cur = flat

    # reduce-scatter overlapped with backward -------------------------------
    def attach_grad_hooks(self):
        """For training loops with one backward per step: every parameter's
        gradient is copied into the flat buffer as soon as autograd has
        accumulated it (a post-accumulate-grad hook, which then drops the
        local .grad), and a bucket's reduce-scatter is queued -- NCCL: on the
        communication stream -- when its last gradient has arrived, so the
        gradient reduction overlaps the rest of backward.  ``step()`` reduces
        the buckets still pending (parameters that got no gradient count as
        zero).  With gradient accumulation over several backward passes use
        ``flat_grad_from_params`` instead."""
        lay = self.layout
        if getattr(self, "_train_flat", None) is None:
            self._train_flat = torch.zeros(lay.total, dtype=self.dtype, device=self.device)
        self._bucket_size = [sum(1 for i in range(len(self.params)) if lay.bucket[i] == b)
                             for b in range(lay.nb)]
        self._pending = None
        from functools import partial
        self._hooks = [p.register_post_accumulate_grad_hook(partial(self._grad_ready, i))
                       for i, p in enumerate(self.params)]

    def _grad_ready(self, i, p):
        if self._pending is None:            # first gradient of this backward
            self._pending = list(self._bucket_size)
            self._got = [False] * len(self.params)
            self._ev_rs = [None] * self.layout.nb
        o = self.layout.global_offset(i)
        self._train_flat[o:o + p.numel()].copy_(p.grad.reshape(-1))
        self._got[i] = True
        p.grad = None
        b = self.layout.bucket[i]
        self._pending[b] -= 1
        if self._pending[b] == 0:
            self._reduce_bucket(b)

    def _reduce_bucket(self, b):
        full_g, _, mine_g = self._views(self._train_flat, b)
        if self.nccl:
            D = torch.cuda.current_stream(self.device)
            ready = torch.cuda.Event()
            ready.record(D)
            with torch.cuda.stream(self.comm):
                self.comm.wait_event(ready)
                if not self.skip_comm:
                    dist.reduce_scatter_tensor(mine_g, full_g, op=dist.ReduceOp.AVG,
                                               group=self.group)
                done = torch.cuda.Event()
                done.record(self.comm)
            self._ev_rs[b] = done
        else:
            tmp = full_g.clone()
            dist.all_reduce(tmp, group=self.group)
            seg = self.layout.seg[b]
            mine_g.copy_(tmp[self.rank * seg:(self.rank + 1) * seg] / self.world)
            self._ev_rs[b] = True
        self._pending[b] = -1

    def _finish_hooked_reduction(self):
        """Reduce the buckets whose gradients did not all arrive, then point
        the owned parameters' .grad at their reduced shard."""
        lay = self.layout
        for b in range(lay.nb):
            if self._pending[b] != -1:
                for i in range(len(self.params)):
                    if lay.bucket[i] == b and not self._got[i]:
                        o = lay.global_offset(i)
                        self._train_flat[o:o + self.params[i].numel()].zero_()
                self._reduce_bucket(b)
        for i in self.my:
            o = lay.shard_offset(i)
            self.params[i].grad = self.my_g[o:o + self.params[i].numel()].view_as(self.params[i])
        self.cur = self._train_flat

    # global grad-norm average ---------------------------------------------
    def _share_norm_average(self):
        """optimizer.py:439-446 over all parameters: each owner contributes
        float(p.grad.norm()) of its averaged gradients (in the gradient's
        dtype), one all-reduce makes the full list known everywhere, and the
        average is summed in parameter order; every inner optimizer uses it
        this step."""
        from .optimizer import _in_param_dtypes
        n = len(self.params)
        vec = torch.zeros(n, dtype=torch.float64, device=self.device)
        if self.my:
            mine = [self.params[i] for i in self.my]
            f32 = torch.stack([torch.linalg.vector_norm(p.grad.float()) for p in mine])
            rounded = _in_param_dtypes(f32.cpu().numpy(), mine)
            vec[self.my] = torch.from_numpy(rounded.astype("float64")).to(self.device)
        dist.all_reduce(vec, group=self.group)
        norms = vec.cpu().tolist()
        avg = sum(norms) / n if n else 0.0
        for o in self.inner:
            if o is not None:
                o._norm_average = (lambda a, c: (lambda _live: (a, c)))(avg, n)
        return avg

    # step -------------------------------------------------------------------
    def step(self):
        self.global_step += 1
        hooked = getattr(self, "_pending", None) is not None
        if hooked:
            self._finish_hooked_reduction()
        if self.cur is None:
            raise RuntimeError("no gradients staged (load_grads / flat_grad_from_params)")
        try:
            self._step(hooked)
        finally:
            if hooked:
                self._pending = None

    def _step(self, hooked):
        nb = self.layout.nb
        if not self.nccl:
            for b in range(nb):
                if hooked:
                    break                       # reduced during backward
                full_g, mine_p, mine_g = self._views(self.cur, b)
                tmp = full_g.clone()
                dist.all_reduce(tmp, group=self.group)
                seg = self.layout.seg[b]
                mine_g.copy_(tmp[self.rank * seg:(self.rank + 1) * seg] / self.world)
            if self.norm_sync:
                self._share_norm_average()
            for b in range(nb):
                if self.inner[b] is not None:
                    self.inner[b].step()
                full_p, mine_p, _ = self._views(self.flat_p, b)
                parts = list(full_p.chunk(self.world))
                dist.all_gather(parts, mine_p.clone(), group=self.group)
                full_p.copy_(torch.cat(parts))
            return
        D = torch.cuda.current_stream(self.device)
        C = self.comm
        C.wait_stream(D)
        if hooked:
            ev_rs = self._ev_rs                 # queued during backward
        else:
            ev_rs = [torch.cuda.Event() for _ in range(nb)]
            with torch.cuda.stream(C):
                for b in range(nb):
                    full_g, _, mine_g = self._views(self.cur, b)
                    if not self.skip_comm:
                        dist.reduce_scatter_tensor(mine_g, full_g, op=dist.ReduceOp.AVG,
                                                   group=self.group)
                    ev_rs[b].record(C)
        if self.norm_sync:
            # the average needs every bucket's gradients: no step starts before
            for b in range(nb):
                D.wait_event(ev_rs[b])
            self._share_norm_average()
        for b in range(nb):
            D.wait_event(ev_rs[b])
            if self.inner[b] is not None and not self.skip_compute:
                self.inner[b].step()
            ev = torch.cuda.Event()
            ev.record(D)
            full_p, mine_p, _ = self._views(self.flat_p, b)
            with torch.cuda.stream(C):
                C.wait_event(ev)
                if not self.skip_comm:
                    dist.all_gather_into_tensor(full_p, mine_p, group=self.group)
        D.wait_stream(C)

    @property
    def _global_step(self):
        return self.global_step

    # checkpoint -------------------------------------------------------------
    def state_dict(self):
        """This rank's shard of the optimizer state: the state of the
        parameters it owns (one inner optimizer per bucket, in the
        reference's schema), with the layout it belongs to.  Each rank saves
        its own; the parameters themselves are the model's (views into the
        flat parameter buffer)."""
        return {"world_size": self.world, "rank": self.rank, "owner": list(self.owner),
                "buckets": self.layout.nb, "global_step": self.global_step,
                "inner": [o.state_dict() if o is not None else None for o in self.inner]}

    def load_state_dict(self, state):
        """Load this rank's shard saved by ``state_dict`` under the same
        world size, ownership and bucket layout."""
        if (state["world_size"], state["rank"], list(state["owner"]), state["buckets"]) != \
                (self.world, self.rank, list(self.owner), self.layout.nb):
            raise ValueError("sharded optimizer checkpoint of a different layout "
                             "(world size, rank, ownership or buckets)")
        self.global_step = int(state["global_step"])
        for o, s in zip(self.inner, state["inner"]):
            if o is not None:
                o.load_state_dict(s)


# ---------------------------------------------------------------------------
# reference-API helpers for replicated optimizers (scao/distributed.py)
# ---------------------------------------------------------------------------

def sync_preconditioners(optimizer, process_group=None):
    """scao/distributed.py:60-128: all-reduce-average the preconditioner state
    of a replicated optimizer.  Here the state lives in flat arenas, so the
    average is one all-reduce per arena; int8 factors are dequantised,
    averaged and requantised on the device (same as the reference's
    dequant -> all_reduce -> quant)."""
    if not dist.is_available() or not dist.is_initialized():
        return
    world = dist.get_world_size(process_group)
    if world == 1:
        return
    plan = getattr(optimizer, "_plan", None)
    if plan is None:
        return
    for t in (plan.u, plan.ev, plan.diag_ema):
        dist.all_reduce(t, group=process_group)
        t.div_(world)
    if plan.int8_ema:
        with torch.cuda.device(plan.device):      # library launches on the plan's device
            _requant_average(plan, process_group, world)
    else:
        dist.all_reduce(plan.fac, group=process_group)
        plan.fac.div_(world)


def wrap_scao_for_fsdp(optimizer):
    """scao/distributed.py:131-160: run sync_preconditioners after every
    curvature step."""
    original = optimizer.step

    def patched(closure=None):
        out = original(closure)
        step = next((s.get("step", 0) for s in optimizer.state.values() if "step" in s), 0)
        if step % optimizer.defaults["precond_freq"] == 0:
            sync_preconditioners(optimizer)
        return out

    optimizer.step = patched
    return optimizer


def _requant_average(plan, group, world):
    """int8 factors: dequantise (utils.py:192-203), all-reduce, average,
    requantise (utils.py:170-189) -- each step through the library's C ABI."""
    import numpy as np
    from . import _lib
    L = _lib.lib()
    stream = torch.cuda.current_stream(plan.device).cuda_stream
    scratch = torch.empty(256, dtype=torch.uint8, device=plan.device)
    sc = torch.zeros(1, dtype=torch.float64, device=plan.device)
    lt = plan.ltab
    for li in range(plan.n_leaves):
        for side in (0, 1):
            n = int(lt["a"][li] if side == 0 else lt["b"][li])
            o = int(lt["lq_off"][li] if side == 0 else lt["rq_off"][li])
            q = plan.fac[o:o + n * n]
            am = float(np.float32(plan.absmax[2 * li + side].item()))
            scale = 1.0 if am < 1e-30 else am / 127.0
            x = torch.empty(n * n, dtype=torch.float32, device=plan.device)
            _lib.check(L.scao_dequantize_sym_int8(q.data_ptr(), scale, n * n, x.data_ptr(),
                                                  stream), "dequantize")
            dist.all_reduce(x, group=group)
            x.div_(world)
            _lib.check(L.scao_quantize_sym_int8(x.data_ptr(), n * n, q.data_ptr(), sc.data_ptr(),
                                                scratch.data_ptr(), stream), "quantize")
            s_new = sc.item()
            plan.absmax[2 * li + side] = float(np.float32(s_new * 127.0)) if s_new != 1.0 or \
                bool(q.ne(0).any().item()) else 0.0
