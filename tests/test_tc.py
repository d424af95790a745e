"""tcgen05 toolkit known-answer test (bf16 x bf16 -> fp32 in TMEM)."""
import pytest
import torch

from scao_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mn", [0, 1])
@pytest.mark.parametrize("N,K", [(16, 16), (64, 64), (128, 64), (256, 128), (96, 32)])
def test_tc_selftest(N, K, mn):
    L = _lib.lib()
    g = torch.Generator().manual_seed(N * 1000 + K)
    A = torch.randn(128, K, generator=g).bfloat16()
    B = torch.randn(N, K, generator=g).bfloat16()
    ref = A.double() @ B.double().T
    dA, dB = A.cuda().contiguous(), B.cuda().contiguous()
    C = torch.zeros(128, N, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(L.scao_tc_selftest(dA.data_ptr(), dB.data_ptr(), C.data_ptr(), N, K,
                                  err.data_ptr(), mn, torch.cuda.current_stream().cuda_stream), "tc")
    torch.cuda.synchronize()
    assert err.item() == 0
    assert (C.double().cpu() - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())


def test_division_by_constant_is_ieee():
    """x / c in the Adan update runs as x*r plus one FMA correction; it must
    give the IEEE quotient for the value ranges the moments take."""
    L = _lib.lib()
    g = torch.Generator().manual_seed(7)
    n = 1 << 22
    x = (torch.randn(n, generator=g) * torch.exp(torch.randn(n, generator=g) * 8)).cuda()
    # bias corrections 1 - beta**t for beta in (0.9, 0.999, 0.99), t in 1..1024
    t = torch.arange(1, 1025, dtype=torch.float64)
    c = torch.cat([1 - 0.9 ** t[:342], 1 - 0.999 ** t[:341], 1 - 0.99 ** t[:341]]).float().cuda()
    m = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(L.scao_divc_check(x.data_ptr(), c.data_ptr(), n, m.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream), "divc")
    torch.cuda.synchronize()
    assert m.item() == 0


def test_bounded_wait_gives_up_and_context_survives():
    """A wait nobody satisfies runs out, reports through the status flag, and
    the context keeps working (a tensor-core self-check right after)."""
    L = _lib.lib()
    err = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    _lib.check(L.scao_wait_timeout_check(err.data_ptr(), 1 << 16,
                                         torch.cuda.current_stream().cuda_stream), "wait")
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    x = torch.ones(1024, device="cuda")
    assert float((x * 2).sum().item()) == 2048.0


def test_device_error_flag_raises_on_a_later_step():
    """A timed-out wait inside a step (simulated by setting the plan's error
    flag) is reported by an exception on a following step."""
    from scao_b200 import SCAO
    p = torch.nn.Parameter(torch.zeros(64, 32, device="cuda"))
    opt = SCAO([p], sparsity=0.0, noise_std_init=0.0)
    p.grad = torch.ones_like(p)
    opt.step()
    torch.cuda.synchronize()
    opt._plan.err.fill_(1)
    with pytest.raises(RuntimeError, match="timed out"):
        for _ in range(4):
            p.grad = torch.ones_like(p)
            opt.step()
            torch.cuda.synchronize()
