"""Generate the golden fixtures in this folder by running the REFERENCE package.

Usage (needs the reference source tree, which only exists where fixtures are
made; the fixtures themselves are committed and travel):

    python tests/golden/make_golden.py --ref <path to whispering3/scao checkout>

It imports ``scao`` from the reference checkout, runs the deterministic SCAO
path (sparsity=0, noise_std_init=0, async_precond=False) on the ``tiny``
workload of ``scao_b200.workloads`` with gradients from
``scao_b200.synthetic``, and stores inputs checksums and outputs as .npz:

  * quant.npz      -- ``utils.quantize_sym_int8`` on edge-case tensors
  * rank.npz       -- ``utils.adaptive_rank`` on spectra incl. near-ties
  * run_<case>.npz -- final params / moments / per-leaf preconditioner state
                       and per-step ranks of a full optimizer run
"""
from __future__ import annotations

import argparse
import copy
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

from scao_b200 import workloads, synthetic  # noqa: E402

CASES = {
    # name: (dtype, max_precond_dim, steps, grad_scale, int8 EMA)
    "f32": ("float32", 4096, 40, 1e-2, True),
    "bf16": ("bfloat16", 4096, 40, 1e-2, True),
    "f32_blocks": ("float32", 48, 30, 1e-2, True),
    "f32_spec": ("float32", 4096, 30, 1.0, False),
    "int8_spec": ("float32", 48, 30, 1.0, True),
    "bf16_spec": ("bfloat16", 48, 30, 1.0, True),
    "f32_sparse": ("float32", 4096, 30, 1.0, True),
    "bf16_dyn": ("bfloat16", 48, 30, 1.0, True),
    "f32_r135": ("float32", 48, 30, 1.0, False),
    "bf16_gsnr": ("bfloat16", 4096, 30, 1.0, True),
    "f32_strips": ("float32", 48, 30, 1.0, True),
    "bf16_strips": ("bfloat16", 48, 30, 1.0, True),
    "mixed": ("float32", 48, 30, 1.0, True),
    "bf16_skip": ("bfloat16", 48, 30, 1.0, True),
}

# golden runs the oracle is pinned against whose GPU parity run is still to be
# recorded (same fields as CASES)
ORACLE_ONLY = {
    "bf16_r1235": ("bfloat16", 48, 30, 1.0, True),
    "f32_groups": ("float32", 48, 30, 1.0, True),
    "bf16_la": ("bfloat16", 4096, 30, 1.0, False),
    "f32_k128": ("float32", 4096, 24, 1.0, True),
    "f32_minpu": ("float32", 48, 30, 1.0, True),
    "f32_nd": ("float32", 48, 30, 1.0, True),
}

# optimizer keyword overrides of a case: the gradient filter of
# optimizer.py:40-97 (static and R2-dynamic), R1 adaptive warmup, R3 lazy
# curvature trigger, R5 adaptive rank, R4 gSNR clip
EXTRA = {
    "f32_sparse": dict(sparsity=0.7),
    "bf16_dyn": dict(sparsity=0.6, dynamic_sparsity=True),
    "f32_r135": dict(adaptive_warmup=True, warmup_patience=2, warmup_stability_threshold=0.5,
                     lazy_precond=True, lazy_delta_threshold=0.02, lazy_max_skip=4,
                     adaptive_rank=True, k_min=2, k_max=4,
                     _grad_scales=(1.0, 1.0, 0.05, 1.0, 1.0, 1.0)),
    "bf16_gsnr": dict(use_gsnr_clip=True, gsnr_threshold=0.3),
    # width-1 remainder blocks of the split (diagonal sub-preconditioners,
    # preconditioner.py:142-156, 232-236): a row strip, column strips, and
    # both inside a nested split
    "f32_strips": dict(_shapes=((49, 40), (40,), (40, 97), (97, 97))),
    "bf16_strips": dict(_shapes=((49, 40), (40,), (40, 97), (97, 97)), sparsity=0.5),
    # one optimizer over parameters of different dtypes
    "mixed": dict(_dtypes=("float32", "bfloat16", "float32", "float16", "float16",
                           "bfloat16")),
    # parameters without a gradient at some steps (skipped by the step,
    # still moved by lookahead, left out of the global-norm average)
    "bf16_skip": dict(_skip=((2, 3, 1), (0, 4, 2), (5, 7, 3))),
    # bf16 with R1 + R2 + R3 + R5: the global grad-norm average takes
    # float(p.grad.norm()) of the bf16 gradients, rounded to bf16
    "bf16_r1235": dict(adaptive_warmup=True, warmup_patience=2, warmup_stability_threshold=0.5,
                       lazy_precond=True, lazy_delta_threshold=0.02, lazy_max_skip=4,
                       adaptive_rank=True, k_min=2, k_max=4, sparsity=0.6,
                       dynamic_sparsity=True, _grad_scales=(1.0, 1.0, 0.05, 1.0, 1.0, 1.0)),
    # param groups with their own lr, weight decay, betas, rank bounds, clip
    # and warmup (the optimizer reads every group's values each step)
    "f32_groups": dict(_groups=(((0, 1, 2), dict(lr=2e-3, weight_decay=0.1, betas=(0.85, 0.99),
                                                   k_max=6)),
                                ((3, 4, 5), dict(lr=5e-4, weight_decay=0.0, tau=None, k_min=2,
                                                   warmup_steps=12, beta3=0.9)))),
    # lookahead every 2 steps with alpha 0.8, LARS off, fp32 factors
    "bf16_la": dict(lookahead_k=2, lookahead_alpha=0.8, lars_coeff=0.0),
    # the largest rank the kernels take (k_max 128: kpad 128)
    "f32_k128": dict(_shapes=((300, 272), (272,)), k_min=8, k_max=128, epsilon_sparse=0.01),
    # Phase 2 gated by min_precond_updates (3 curvature updates, the third one
    # made inside the warmup branch of the step that reaches it)
    "f32_minpu": dict(min_precond_updates=3, precond_freq=4, warmup_steps=4),
    # parameters of 3 and 4 dims (conv-like) flattened to (d0, rest) (utils.py:208-219)
    "f32_nd": dict(_shapes=((16, 4, 6), (24,), (8, 3, 3, 3), (6, 8, 10))),
}


def grad_digest(grads):
    h = hashlib.sha1()
    for g in grads:
        h.update(g.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def run_case(scao_mod, name, dtype, mpd, steps, gs, int8):
    w = workloads.tiny(dtype=dtype, max_precond_dim=mpd, steps=steps,
                       grad_scale=gs, int8=int8, extra=EXTRA.get(name))
    params0 = synthetic.init_params(w, seed=0)
    params = [torch.nn.Parameter(p.clone()) for p in params0]
    opt = scao_mod.SCAO(workloads.param_groups(w, params), **w.scao_kwargs)
    gen = synthetic.LowRankGradients(w, seed=0)
    digests, ks = [], []
    for t in range(steps):
        grads = gen.next()
        digests.append(grad_digest(grads))
        for i, (p, g) in enumerate(zip(params, grads)):
            p.grad = g.clone() if workloads.has_grad(w, i, t) else None
        opt.step()
        ks.append([opt.state[p]["preconditioner"].k for p in params])
    out = {"steps": np.array(steps), "digests": np.array(digests),
           "ks": np.array(ks, np.int32)}
    for i, p in enumerate(params):
        st = opt.state[p]
        out[f"p{i}"] = p.detach().float().numpy()
        for key in ("exp_avg", "exp_avg_sq", "exp_avg_diff", "prev_grad"):
            out[f"{key}{i}"] = st[key].numpy()
        pc = st["preconditioner"]

        def flat(node):
            # every leaf of the (possibly nested) block tree, in order
            return [x for b in node._blocks for x in flat(b)] if node.use_block_diagonal \
                else [node]
        leaves = flat(pc)
        for j, lf in enumerate(leaves):
            pre = f"leaf{i}_{j}_"
            out[pre + "precond_step"] = np.array(lf.precond_step)
            out[pre + "k"] = np.array(lf.k)
            if lf.use_kronecker and lf.use_int8_ema:
                out[pre + "Lq"] = lf.L_ema_q.numpy()
                out[pre + "Ls"] = np.array(lf.L_ema_scale, np.float64)
                out[pre + "Rq"] = lf.R_ema_q.numpy()
                out[pre + "Rs"] = np.array(lf.R_ema_scale, np.float64)
            elif lf.use_kronecker:
                out[pre + "L"] = lf.L_ema.numpy()
                out[pre + "R"] = lf.R_ema.numpy()
            if lf.use_kronecker:
                for key in ("U_l", "S_l", "U_r", "S_r"):
                    out[pre + key] = getattr(lf, key).numpy()
            else:
                out[pre + "diag_ema"] = lf.diag_ema.numpy()
    np.savez_compressed(os.path.join(HERE, f"run_{name}.npz"), **out)
    print("wrote", name)


def quant_cases(utils):
    g = torch.Generator().manual_seed(1234)
    xs = {
        "randn": torch.randn(64, 64, generator=g),
        "tiny_scale": torch.randn(32, 32, generator=g) * 1e-6,
        "zeros": torch.zeros(16, 16),
        "below_floor": torch.full((8, 8), 1e-31),
        "eye": torch.eye(48) * 1e-4,
        "ema_like": torch.eye(40) * 0.999e-4 + torch.randn(40, 40, generator=g) * 3e-7,
        # values placed exactly on half-code boundaries of scale 1/127
        "ties": (torch.arange(-254, 255, dtype=torch.float32) / 254.0).reshape(1, -1),
        "huge": torch.randn(17, 33, generator=g) * 1e30,
    }
    out = {}
    for k, x in xs.items():
        q, s = utils.quantize_sym_int8(x.clone())
        out[k + "_x"] = x.numpy()
        out[k + "_q"] = q.numpy()
        out[k + "_s"] = np.array(s, np.float64)
        out[k + "_deq"] = utils.dequantize_sym_int8(q, s).numpy()
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **out)
    print("wrote quant")


def rank_cases(utils):
    g = torch.Generator().manual_seed(99)
    specs = []
    for i in range(24):
        n = [16, 64, 200, 1024][i % 4]
        ev = torch.rand(n, generator=g).pow(6 + i % 5).sort(descending=True).values
        specs.append((ev, 0.05, 4, 64))
    specs.append((torch.zeros(32), 0.05, 4, 16))
    specs.append((torch.full((50,), 0.5), 0.05, 3, 20))
    specs.append((torch.tensor([1.0, 0.0, 0.0, 0.0]), 0.05, 1, 4))
    out = {}
    for i, (ev, e, kmin, kmax) in enumerate(specs):
        out[f"ev{i}"] = ev.numpy()
        out[f"args{i}"] = np.array([e, kmin, kmax], np.float64)
        out[f"k{i}"] = np.array(utils.adaptive_rank(ev, e, kmin, kmax))
    out["n"] = np.array(len(specs))
    np.savez_compressed(os.path.join(HERE, "rank.npz"), **out)
    print("wrote rank")


def ckpt_case(scao_mod, steps_before=12, steps_after=10):
    """A checkpoint of the reference after ``steps_before`` steps of the tiny
    fp32 int8 workload (Phase 2 reached), saved as its state_dict without the
    pickled preconditioner objects (everything the schema needs is in
    ``_scao_precond``), and the reference's state ``steps_after`` steps later:
    the GPU test loads the checkpoint into scao_b200.SCAO and continues."""
    w = workloads.tiny(dtype="float32", max_precond_dim=48, steps=steps_before + steps_after,
                       grad_scale=1.0, int8=True)
    params = [torch.nn.Parameter(p.clone()) for p in synthetic.init_params(w, seed=0)]
    opt = scao_mod.SCAO(params, **w.scao_kwargs)
    gen = synthetic.LowRankGradients(w, seed=0)
    for t in range(steps_before):
        for p, g in zip(params, gen.next()):
            p.grad = g.clone()
        opt.step()
    sd = opt.state_dict()
    sd["state"] = {i: {k: v for k, v in st.items() if k != "preconditioner"}
                   for i, st in sd["state"].items()}
    torch.save({"state_dict": sd, "params": [p.detach().clone() for p in params]},
               os.path.join(HERE, "ckpt_tiny_f32.pt"))
    # the reference itself resumes from its own (full) checkpoint: a fresh
    # optimizer loads it, so state the checkpoint does not hold (the
    # lookahead slow weights) starts afresh, as it does for any resumed run
    full = copy.deepcopy(opt.state_dict())
    params = [torch.nn.Parameter(p.detach().clone()) for p in params]
    opt = scao_mod.SCAO(params, **w.scao_kwargs)
    opt.load_state_dict(full)
    for t in range(steps_after):
        for p, g in zip(params, gen.next()):
            p.grad = g.clone()
        opt.step()
    out = {"steps_before": np.array(steps_before), "steps_after": np.array(steps_after)}
    for i, p in enumerate(params):
        out[f"p{i}"] = p.detach().numpy()
        out[f"exp_avg{i}"] = opt.state[p]["exp_avg"].numpy()
        out[f"k{i}"] = np.array(opt.state[p]["preconditioner"].k)
    np.savez_compressed(os.path.join(HERE, "ckpt_tiny_f32_after.npz"), **out)
    print("wrote ckpt")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference checkout root")
    ap.add_argument("--only", nargs="*", help="regenerate only these run cases")
    ap.add_argument("--ckpt", action="store_true", help="regenerate only the checkpoint case")
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    import scao  # noqa: E402  (the reference package)
    from scao import utils  # noqa: E402
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    if a.ckpt:
        ckpt_case(scao)
        return
    if not a.only:
        quant_cases(utils)
        rank_cases(utils)
        ckpt_case(scao)
    for name, args in {**CASES, **ORACLE_ONLY}.items():
        if not a.only or name in a.only:
            run_case(scao, name, *args)


if __name__ == "__main__":
    main()
