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
