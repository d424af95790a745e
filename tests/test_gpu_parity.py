"""GPU parity: the CUDA path against the oracle and the reference's golden runs.

Bars (from the north star): int8 quantisation bit-exact on identical fp32
inputs; ranks equal; eigen-subspaces within 1e-3 rad principal angle;
parameter updates and moments within relative L2 1e-3.
"""

import numpy as np
import pytest
import torch

from golden_util import CASES, EXTRA, load, rel_err, subspace_angle
from oracle import scao_oracle as O
from scao_b200 import SCAO, _lib, synthetic, workloads

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = 1e-3


def _stream():
    return torch.cuda.current_stream().cuda_stream


# ---------------------------------------------------------------------------
# single-matrix C-ABI entry points
# ---------------------------------------------------------------------------

def test_quantize_bit_exact_golden():
    L = _lib.lib()
    g = load("quant")
    names = sorted({k[:-2] for k in g if k.endswith("_x")})
    for n in names:
        x = torch.from_numpy(g[n + "_x"]).to(DEV).contiguous()
        q = torch.empty(x.shape, dtype=torch.int8, device=DEV)
        sc = torch.zeros(1, dtype=torch.float64, device=DEV)
        scratch = torch.empty(256, dtype=torch.uint8, device=DEV)
        _lib.check(L.scao_quantize_sym_int8(x.data_ptr(), x.numel(), q.data_ptr(),
                                            sc.data_ptr(), scratch.data_ptr(), _stream()), n)
        torch.cuda.synchronize()
        assert np.array_equal(q.cpu().numpy(), g[n + "_q"]), n
        assert sc.item() == float(g[n + "_s"]), n
        out = torch.empty(x.shape, dtype=torch.float32, device=DEV)
        _lib.check(L.scao_dequantize_sym_int8(q.data_ptr(), float(g[n + "_s"]), q.numel(),
                                              out.data_ptr(), _stream()), n)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), g[n + "_deq"]), n


@pytest.mark.parametrize("n", [1, 1000, 1 << 20])
def test_int8_ema_update_bit_exact(n):
    """dequant -> rho*x + new -> requant vs the oracle on identical fp32 input."""
    L = _lib.lib()
    gen = torch.Generator().manual_seed(n)
    x0 = torch.randn(n, generator=gen)
    q0, s0 = O.quantize_sym_int8(x0.numpy())
    new = (torch.randn(n, generator=gen) * 1e-3).numpy().astype(np.float32)
    rho = 0.999
    ref = O.dequantize_sym_int8(q0, s0) * np.float32(rho) + new
    qr, sr = O.quantize_sym_int8(ref)
    qd = torch.from_numpy(q0).to(DEV)
    nd = torch.from_numpy(new).to(DEV)
    qo = torch.empty_like(qd)
    so = torch.zeros(1, dtype=torch.float64, device=DEV)
    scratch = torch.empty(L.scao_int8_ema_scratch_bytes(n), dtype=torch.uint8, device=DEV)
    _lib.check(L.scao_int8_ema_update(qd.data_ptr(), s0, nd.data_ptr(), rho, n, qo.data_ptr(),
                                      so.data_ptr(), scratch.data_ptr(), _stream()), "ema")
    torch.cuda.synchronize()
    assert np.array_equal(qo.cpu().numpy(), qr)
    assert so.item() == sr


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("m,n,k", [(64, 48, 8), (300, 200, 16), (1024, 1024, 64), (5, 7, 3)])
def test_fused_kronecker_precond(m, n, k, dt):
    """Formula of scao/cuda/__init__.py:78-99 against a float64 torch reference
    (the reference's KAT, scripts/kaggle_kernel_scao.py:64-82, uses max-abs 1e-4)."""
    L = _lib.lib()
    gen = torch.Generator().manual_seed(m * 7 + n)
    Ul = torch.linalg.qr(torch.randn(m, k, generator=gen, dtype=torch.float64))[0].float()
    Ur = torch.linalg.qr(torch.randn(n, k, generator=gen, dtype=torch.float64))[0].float()
    sl = torch.rand(k, generator=gen) + 0.5
    sr = torch.rand(k, generator=gen) + 0.5
    G = torch.randn(m, n, generator=gen).to(dt)
    Gd = G.double()
    P = Ul.double().T @ Gd @ Ur.double()
    ref = Gd + Ul.double() @ ((sl.double()[:, None] * sr.double()[None, :] - 1) * P) @ Ur.double().T
    d = {k_: v.to(DEV).contiguous() for k_, v in dict(Ul=Ul, Ur=Ur, sl=sl, sr=sr, G=G).items()}
    out = torch.empty_like(d["G"])
    code = {torch.float32: 0, torch.bfloat16: 1}[dt]
    scratch = torch.empty(L.scao_fused_precond_scratch_bytes(m, n, k), dtype=torch.uint8, device=DEV)
    _lib.check(L.scao_fused_kronecker_precond(d["Ul"].data_ptr(), d["sl"].data_ptr(),
                                              d["Ur"].data_ptr(), d["sr"].data_ptr(),
                                              d["G"].data_ptr(), out.data_ptr(), code, m, n, k,
                                              scratch.data_ptr(), _stream()), "fused")
    torch.cuda.synchronize()
    got = out.double().cpu()
    if dt == torch.float32:
        assert (got - ref).abs().max().item() < 1e-4
    else:
        # one bf16 rounding of the result
        assert torch.allclose(got, ref.to(dt).double(), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("left", [1, 0])
def test_low_rank_precond_mm(left):
    L = _lib.lib()
    gen = torch.Generator().manual_seed(5 + left)
    m, n, k = 96, 80, 12
    d = m if left else n
    U = torch.linalg.qr(torch.randn(d, k, generator=gen, dtype=torch.float64))[0].float()
    s = torch.rand(k, generator=gen)
    G = torch.randn(m, n, generator=gen)
    ref = (U * s) @ (U.T @ G) if left else (G @ (U * s)) @ U.T
    dU, ds, dG = (x.contiguous().to(DEV) for x in (U, s, G))
    out = torch.empty(m, n, device=DEV)
    scratch = torch.empty(L.scao_low_rank_precond_mm_scratch_bytes(m, n, k, left),
                          dtype=torch.uint8, device=DEV)
    _lib.check(L.scao_low_rank_precond_mm(dU.data_ptr(), ds.data_ptr(), dG.data_ptr(),
                                          out.data_ptr(), m, n, k, left, scratch.data_ptr(),
                                          _stream()), "lrmm")
    torch.cuda.synchronize()
    assert torch.allclose(out.cpu(), ref, atol=1e-5, rtol=1e-4)


# ---------------------------------------------------------------------------
# full optimizer runs
# ---------------------------------------------------------------------------

def run_gpu(name, steps=None):
    dt, mpd, nsteps, gs, i8 = CASES[name]
    steps = steps or nsteps
    w = workloads.tiny(dtype=dt, max_precond_dim=mpd, steps=steps, grad_scale=gs, int8=i8,
                       extra=EXTRA.get(name))
    p0 = synthetic.init_params(w)
    params = [torch.nn.Parameter(p.clone().to(DEV)) for p in p0]
    opt = SCAO(workloads.param_groups(w, params), **w.scao_kwargs)
    gen = synthetic.LowRankGradients(w)
    ks = []
    for t in range(steps):
        for i, (p, g) in enumerate(zip(params, gen.next())):
            p.grad = g.to(DEV) if workloads.has_grad(w, i, t) else None
        opt.step()
        ks.append([opt.state[p]["preconditioner"].k for p in params])
    torch.cuda.synchronize()
    opt._plan.check_error()
    return p0, params, opt, np.array(ks)


@pytest.mark.parametrize("name", list(CASES))
def test_optimizer_matches_reference_run(name):
    G = load("run_" + name)
    p0, params, opt, ks = run_gpu(name)
    assert np.array_equal(ks, G["ks"]), (ks[-1], G["ks"][-1])
    for i, p in enumerate(params):
        st = opt.state[p]
        p0i = p0[i].float().numpy()
        got = p.detach().float().cpu().numpy()
        assert rel_err(got - p0i, G[f"p{i}"] - p0i) < TOL, i
        assert rel_err(st["exp_avg"].cpu().numpy(), G[f"exp_avg{i}"]) < TOL, i
        assert rel_err(st["exp_avg_sq"].cpu().numpy(), G[f"exp_avg_sq{i}"]) < TOL, i
        assert rel_err(st["exp_avg_diff"].cpu().numpy(), G[f"exp_avg_diff{i}"]) < TOL, i
        pc = st["preconditioner"]
        sd = pc.state_dict()

        def flat(d):
            return [x for b in d["blocks"] for x in flat(b)] if d["use_block_diagonal"] else [d]
        leaves = flat(sd)
        for j, lf in enumerate(leaves):
            pre = f"leaf{i}_{j}_"
            assert lf["k"] == int(G[pre + "k"])
            assert lf["precond_step"] == int(G[pre + "precond_step"])
            if "diag_ema" in lf:
                assert rel_err(lf["diag_ema"].cpu().numpy(), G[pre + "diag_ema"]) < 1e-5
                continue
            if "L_ema_q" in lf:
                lq, rq = lf["L_ema_q"].cpu().numpy(), lf["R_ema_q"].cpu().numpy()
                # identical codes except rare +-1 flips from GEMM summation order
                assert np.abs(lq.astype(int) - G[pre + "Lq"]).max() <= 1
                assert np.abs(rq.astype(int) - G[pre + "Rq"]).max() <= 1
                assert np.mean(lq != G[pre + "Lq"]) < 1e-3
            else:
                assert rel_err(lf["L_ema"].cpu().numpy(), G[pre + "L"]) < 1e-5
            assert subspace_angle(lf["U_l"].cpu().numpy(), G[pre + "U_l"], G[pre + "S_l"]) < 1e-3
            assert subspace_angle(lf["U_r"].cpu().numpy(), G[pre + "U_r"], G[pre + "S_r"]) < 1e-3
            # eigenvalues: 1e-4 on fp32 factors; an int8 factor carries its
            # rare +-1 code flips (one code = absmax / 127) into them
            stol = 1e-3 if "L_ema_q" in lf else 1e-4
            assert rel_err(lf["S_l"].cpu().numpy(), G[pre + "S_l"]) < stol
            assert rel_err(lf["S_r"].cpu().numpy(), G[pre + "S_r"]) < stol


def test_bf16_degenerate_run_is_bit_exact():
    """In the degenerate int8 regime every step is deterministic elementwise
    work: the bf16 parameters must equal the reference run bit for bit except
    for rare one-ulp flips from reduction order in the LARS norms."""
    G = load("run_bf16")
    p0, params, opt, _ = run_gpu("bf16")
    for i, p in enumerate(params):
        got = p.detach().float().cpu().numpy()
        assert np.mean(got != G[f"p{i}"]) < 1e-2, i
