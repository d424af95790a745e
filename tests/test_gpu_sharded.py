"""Owner-compute sharding (ShardedSCAO, NCCL) against the unsharded optimizer
on 2 GPUs: every rank receives the same gradients, so the reduce-scatter
average equals them exactly and each rank's owned parameters must equal an
unsharded optimizer's (one per bucket, as the owner runs them) bit for bit.
Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, steps, out):
    import torch.distributed as dist
    from scao_b200 import SCAO, synthetic, workloads
    from scao_b200.distributed import ShardedSCAO
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        w = workloads.c4(n_layers=1)
        w.grad_scale = 1.0                      # non-degenerate: the eigensolver runs
        params = [torch.nn.Parameter(p) for p in synthetic.init_params(w, device=dev)]
        opt = ShardedSCAO(params, w, lambda ps: bench.build_opt_list(w, ps, SCAO), buckets=2)
        lay = opt.layout
        shadow = []
        for b in range(lay.nb):
            mine = [i for i in opt.my if lay.bucket[i] == b]
            if mine:
                ps = [torch.nn.Parameter(params[i].detach().clone()) for i in mine]
                shadow.append((mine, ps, bench.build_opt_list(
                    w, [(p, w.params[i]) for p, i in zip(ps, mine)], SCAO)))
        gen = synthetic.LowRankGradients(w, device=dev)
        sets = [gen.next() for _ in range(3)]
        for k in range(steps):
            opt.load_grads(sets[k % 3])
            opt.step()
        for k in range(steps):
            for mine, ps, sopt in shadow:
                for i, p in zip(mine, ps):
                    p.grad = sets[k % 3][i]
                sopt.step()
        torch.cuda.synchronize()
        d = 0.0
        for mine, ps, _ in shadow:
            for i, p in zip(mine, ps):
                d = max(d, (params[i].detach().float() - p.detach().float()).abs().max().item())
        # every rank also holds the other ranks' parameters (all-gather)
        t = torch.tensor([d], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ref = [p.detach().clone() for p in params]
        chk = [torch.zeros_like(p) for p in ref]
        for c, p in zip(chk, ref):
            c.copy_(p)
            dist.broadcast(c, src=0)
        same = all(torch.equal(c, p) for c, p in zip(chk, ref))
        out[rank] = (t.item(), bool(same))
    finally:
        dist.destroy_process_group()


def test_sharded_step_equals_unsharded_two_gpus():
    world, steps = 2, 25                         # 20 Adam-warmup steps, then Phase 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_rank, args=(world, _free_port(), steps, out), nprocs=world, join=True)
    for r in range(world):
        diff, same = out[r]
        assert diff == 0.0, (r, diff)
        assert same, r
