"""Profiling case for the eigensolver kernels (run under ncu, see profiles/):

    python tests/prof/eig_case.py LAYERS STEPS

The Llama-1B layer shapes with LAYERS transformer layers, bf16 parameters,
int8 curvature EMA, fed s0 = 1 gradients from the first step, so the curvature
update at step 10 is non-degenerate and runs the iterative eigensolver from its
cold start.  Not a test (pytest does not collect it)."""
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from scao_b200 import SCAO, synthetic, workloads  # noqa: E402


def main():
    w = workloads.c4(n_layers=int(sys.argv[1]))
    dev = torch.device("cuda", 0)
    params = [torch.nn.Parameter(p) for p in synthetic.init_params(w, device=dev)]
    opt = bench.build_opt(w, params, SCAO)
    gen = synthetic.LowRankGradients(w, device=dev, s0=1.0)
    sets = [gen.next() for _ in range(3)]
    for k in range(int(sys.argv[2])):
        for p, g in zip(params, sets[k % 3]):
            p.grad = g
        opt.step()
    torch.cuda.synchronize()
    print("ok: mean eigen iterations", opt._last_eig_status.abs().float().mean().item())


if __name__ == "__main__":
    main()
