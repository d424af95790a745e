"""Owner-compute sharding host logic on CPU: 2 gloo ranks (127.0.0.1)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from scao_b200 import workloads
from scao_b200.distributed import FlatLayout, ShardedSCAO, partition


def test_partition_balanced_and_deterministic():
    costs = [100, 7, 50, 50, 3, 99, 1, 60]
    a = partition(costs, 3)
    assert a == partition(costs, 3)
    loads = [sum(c for c, o in zip(costs, a) if o == r) for r in range(3)]
    assert max(loads) - min(loads) <= max(costs)
    assert set(a) == {0, 1, 2}


def test_flat_layout_disjoint_aligned():
    numels = [10, 300, 64, 1, 1000, 77, 5000, 3]
    owner = partition(numels, 2)
    for nb in (1, 3):
        lay = FlatLayout(numels, owner, 2, nb)
        spans = sorted((lay.global_offset(i), lay.global_offset(i) + n)
                       for i, n in enumerate(numels))
        for (a0, a1), (b0, _) in zip(spans, spans[1:]):
            assert a1 <= b0
        assert spans[-1][1] <= lay.total
        assert all(lay.offsets[i] % 64 == 0 for i in range(len(numels)))
        assert all(lay.offsets[i] + numels[i] <= lay.seg[lay.bucket[i]]
                   for i in range(len(numels)))
        # a rank's bucket segments tile its own shard
        assert lay.shard == sum(lay.seg)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_flat_layout_padding_llama_shapes(world):
    """The bucket-major layout of the Llama-1B parameter set carries little
    padding (each collective moves world x segment elements), every bucket
    holds parameters of every rank that owns any, and items stay disjoint."""
    numels = [int(torch.Size(s.shape).numel()) for s in workloads.c4().params]
    owner = partition(numels, world)
    lay = FlatLayout(numels, owner, world, 4)
    assert lay.total <= 1.06 * sum(numels)
    spans = sorted((lay.global_offset(i), lay.global_offset(i) + n) for i, n in enumerate(numels))
    assert all(a1 <= b0 for (_, a1), (b0, _) in zip(spans, spans[1:]))
    assert all(lay.offsets[i] + numels[i] <= lay.seg[lay.bucket[i]] for i in range(len(numels)))


class _SGD:
    """Stand-in for the per-rank optimizer: p -= 0.1 * grad (grads are views
    into the reduce-scattered shard)."""

    def __init__(self, pairs):
        self.ps = [p for p, _ in pairs]

    def step(self):
        for p in self.ps:
            p.data.add_(p.grad, alpha=-0.1)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = workloads.tiny()
        torch.manual_seed(0)
        params = [torch.randn(s.shape) for s in w.params]
        ref = [p.clone() for p in params]
        # per-rank gradients differ; the owner update must use their average
        grads = [torch.full(s.shape, float(rank + 1)) * (i + 1) for i, s in enumerate(w.params)]
        avg = [torch.full(s.shape, (1 + world) / 2.0) * (i + 1) for i, s in enumerate(w.params)]
        opt = ShardedSCAO(params, w, _SGD, buckets=2)
        opt.load_grads(grads)
        opt.step()
        errs = [float((p - (r - 0.1 * g)).abs().max()) for p, r, g in zip(params, ref, avg)]
        ok = max(errs) < 1e-5
        if not ok:
            print(rank, errs, opt.my, flush=True)
        q.put((rank, ok, sorted(opt.my)))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_sharded_step_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res)
    owned = sorted(i for _, _, m in res for i in m)
    assert owned == list(range(len(workloads.tiny().params)))


def _sync_worker(rank, world, port, q):
    """Plans on the host (arenas only, no kernels): rank 0's state after
    broadcast_plan_state on every rank."""
    from scao_b200.optimizer import broadcast_plan_state
    from scao_b200.plan import Plan
    from scao_b200.preconditioner import PrecondView
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = dict(max_precond_dim=48, k_min=4, k_max=8, epsilon_sparse=0.05, rho=0.999)
        params = [torch.zeros(49, 40), torch.zeros(40), torch.zeros(64, 48)]
        plan = Plan(params, [g] * 3, torch.device("cpu"), True)
        states = [{"step": 10 * (rank + 1) + i, "preconditioner": PrecondView(plan, i, g)}
                  for i in range(3)]
        for i, st in enumerate(states):
            st["preconditioner"].precond_step = rank + i
        gen = torch.Generator().manual_seed(rank)
        arenas = ("exp_avg", "exp_avg_sq", "exp_avg_diff", "prev_grad", "fac", "absmax", "u",
                  "ev", "k", "diag_ema", "ua", "ut")
        for name in arenas:
            t = getattr(plan, name)
            t.copy_((torch.rand(t.shape, generator=gen) * 100).to(t.dtype))
        # numpy copies travel through the queue by value
        before = {n: getattr(plan, n).numpy().copy() for n in arenas}
        broadcast_plan_state(plan, states)
        got = {n: getattr(plan, n).numpy().copy() for n in arenas}
        q.put((rank, [st["step"] for st in states],
               [st["preconditioner"].precond_step for st in states], before, got))
    finally:
        dist.destroy_process_group()


def test_sync_preconditioner_broadcasts_rank0_state():
    """optimizer.py:686-710: moments, counters and preconditioner state from
    rank 0; prev_grad stays per rank (the reference does not broadcast it)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sync_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=120) for _ in procs), key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    (_, s0, p0, b0, g0), (_, s1, p1, b1, g1) = res
    assert s0 == s1 == [10, 11, 12] and p0 == p1 == [0, 1, 2]
    for name in g0:
        eq = np.array_equal
        if name == "prev_grad":
            assert eq(g1[name], b1[name]) and not eq(g1[name], b0[name])
        else:
            assert eq(g1[name], b0[name]) and eq(g0[name], b0[name]), name


def test_replicated_helpers_single_process():
    """scao/tests/test_optimizer.py:686-720 on the host: without an initialised
    process group the helpers are silent no-ops; the FSDP wrapper returns the
    optimizer with its step patched."""
    from scao_b200 import SCAO
    from scao_b200.distributed import sync_preconditioners, wrap_scao_for_fsdp
    assert not dist.is_initialized()
    opt = SCAO([torch.nn.Parameter(torch.zeros(64, 256))], lr=1e-3, max_precond_dim=64)
    sync_preconditioners(opt)
    with pytest.warns(RuntimeWarning):
        opt.sync_preconditioner()
    wrapped = wrap_scao_for_fsdp(opt)
    assert wrapped is opt and callable(wrapped.step)


class _NormProbe(_SGD):
    """Inner stand-in with a host-norm extension switched on: records the
    global grad-norm average the wrapper hands it each step."""
    _host_norms = True

    def __init__(self, pairs):
        super().__init__(pairs)
        self._norm_average = None
        self.seen = []

    def step(self):
        self.seen.append(self._norm_average(None))
        super().step()


def _norm_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = workloads.tiny()
        torch.manual_seed(0)
        params = [torch.randn(s.shape) for s in w.params]
        gen = torch.Generator().manual_seed(5)
        base = [torch.randn(s.shape, generator=gen) for s in w.params]
        opt = ShardedSCAO(params, w, _NormProbe, buckets=2)
        assert opt.norm_sync
        res = []
        for t in range(2):
            grads = [b * (rank + 1) * (t + 1) for b in base]
            opt.load_grads(grads)
            opt.step()
            avg_g = [b * (1 + world) / 2.0 * (t + 1) for b in base]
            want = sum(float(torch.linalg.vector_norm(g.float())) for g in avg_g) / len(avg_g)
            got = [o.seen[-1] for o in opt.inner if o is not None]
            res.append((want, got))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_sharded_global_norm_average_over_all_parameters():
    """With R1 / R2-dynamic / R5 on, every inner optimizer of every rank gets
    the average of all parameters' norms (optimizer.py:439-446), not of the
    ones it owns."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_norm_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, steps in res:
        for want, got in steps:
            assert got and all(abs(a - want) <= 1e-6 * want and n == 6 for a, n in got)


def _hook_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch.nn as nn
        from scao_b200.workloads import ParamSpec, Workload

        def model_and_inputs():
            torch.manual_seed(0)
            m = nn.Sequential(nn.Linear(16, 32), nn.ReLU(), nn.Linear(32, 8))
            xs = [torch.randn(4, 16, generator=torch.Generator().manual_seed(10 + r))
                  for r in range(world)]
            return m, xs

        # expected: SGD on the gradient averaged over the ranks' batches
        m_ref, xs = model_and_inputs()
        grads = []
        for x in xs:
            m_ref.zero_grad()
            m_ref(x).pow(2).mean().backward()
            grads.append([p.grad.clone() for p in m_ref.parameters()])
        want = [p.detach() - 0.1 * sum(g[i] for g in grads) / world
                for i, p in enumerate(m_ref.parameters())]

        m, xs = model_and_inputs()
        params = list(m.parameters())
        wl = Workload("mlp", [ParamSpec(f"p{i}", tuple(p.shape)) for i, p in enumerate(params)],
                      {}, 1, 1.0)
        opt = ShardedSCAO(params, wl, _SGD, buckets=2)
        opt.attach_grad_hooks()
        m.zero_grad(set_to_none=True)
        m(xs[rank]).pow(2).mean().backward()
        # every bucket holding parameters was reduced before step() (a bucket
        # the layout leaves empty is reduced in step(), on every rank alike)
        reduced_in_backward = all(x == -1 for x, n in zip(opt._pending, opt._bucket_size) if n) \
            and any(opt._bucket_size)
        opt.step()
        err = max(float((p.detach() - w).abs().max()) for p, w in zip(params, want))
        q.put((rank, reduced_in_backward, err, opt._pending is None))
    finally:
        dist.destroy_process_group()


def test_reduce_scatter_overlapped_with_backward():
    """attach_grad_hooks: every bucket is reduced during backward (as its
    last gradient arrives) and the step equals SGD on the rank-averaged
    gradient."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_hook_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, in_bwd, err, reset in res:
        assert in_bwd and reset and err < 1e-6, (in_bwd, err)


class _Momentum:
    """Stateful inner stand-in: heavy-ball SGD with a checkpointable buffer."""

    def __init__(self, pairs):
        self.ps = [p for p, _ in pairs]
        self.buf = [torch.zeros_like(p) for p in self.ps]

    def step(self):
        for p, b in zip(self.ps, self.buf):
            b.mul_(0.9).add_(p.grad)
            p.data.add_(b, alpha=-0.1)

    def state_dict(self):
        return {"buf": [b.clone() for b in self.buf]}

    def load_state_dict(self, st):
        for b, s in zip(self.buf, st["buf"]):
            b.copy_(s)


def _ckpt_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = workloads.tiny()

        def fresh():
            torch.manual_seed(0)
            params = [torch.randn(s.shape) for s in w.params]
            return params, ShardedSCAO(params, w, _Momentum, buckets=2)

        grads = [[torch.full(s.shape, float(t + rank + 1)) for s in w.params] for t in range(3)]
        pa, a = fresh()
        for t in range(3):
            a.load_grads(grads[t])
            a.step()
        pb, b = fresh()
        for t in range(2):
            b.load_grads(grads[t])
            b.step()
        sd = b.state_dict()
        saved_p = [p.detach().clone() for p in pb]
        pc, c = fresh()
        for p, s in zip(pc, saved_p):
            p.data.copy_(s)
        c.load_state_dict(sd)
        c.load_grads(grads[2])
        c.step()
        err = max(float((x - y).abs().max()) for x, y in zip(pa, pc))
        assert c.param_groups == []           # stand-ins carry no param groups
        bad = False
        try:
            sd2 = dict(sd, buckets=3)
            c.load_state_dict(sd2)
        except ValueError:
            bad = True
        q.put((rank, err, bad, c.global_step))
    finally:
        dist.destroy_process_group()


def test_sharded_checkpoint_resume():
    """Each rank saves its shard; a fresh wrapper that loads it (and the
    parameters) continues exactly like the uninterrupted run; a checkpoint of
    another layout is refused."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ckpt_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, err, bad, gs in res:
        assert err == 0.0 and bad and gs == 3
