"""The allocation-free int8 EMA update against the regular entry point.

Callers embedded in a host that owns all device memory (a serving process or
plugin with its own pool) cannot hand this library a scratch buffer; the
``_noalloc`` entry point stages through a fixed device array inside the
library instead.  Its results must equal the regular entry point's bit for
bit (the int8 requant is exact), on consecutive calls that reuse the array.
This file is collected last so a stop-at-first-failure run has already run
everything else.
"""
import pytest
import torch

from scao_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _regular(L, q, s, new, rho, st):
    n = q.numel()
    qo = torch.empty_like(q)
    so = torch.zeros(1, dtype=torch.float64, device=DEV)
    scratch = torch.empty(L.scao_int8_ema_scratch_bytes(n), dtype=torch.uint8, device=DEV)
    _lib.check(L.scao_int8_ema_update(q.data_ptr(), s, new.data_ptr(), rho, n, qo.data_ptr(),
                                      so.data_ptr(), scratch.data_ptr(), st), "regular")
    return qo, so


def _noalloc(L, q, s, new, rho, st):
    qo = torch.empty_like(q)
    so = torch.zeros(1, dtype=torch.float64, device=DEV)
    _lib.check(L.scao_int8_ema_update_noalloc(q.data_ptr(), s, new.data_ptr(), rho, q.numel(),
                                              qo.data_ptr(), so.data_ptr(), st), "noalloc")
    return qo, so


def test_noalloc_matches_regular_two_calls():
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    gen = torch.Generator().manual_seed(11)
    # second call is smaller and has a smaller max: a stale max slot from the
    # first call would show up as a wrong scale
    for n, mag in ((1 << 20, 1.0), (300_000, 1e-3)):
        q = torch.randint(-127, 128, (n,), generator=gen, dtype=torch.int8).to(DEV)
        new = (torch.randn(n, generator=gen) * mag).to(DEV)
        s = mag / 127.0
        qa, sa = _regular(L, q, s, new, 0.999, st)
        qb, sb = _noalloc(L, q, s, new, 0.999, st)
        torch.cuda.synchronize()
        assert torch.equal(qa, qb)
        assert sa.item() == sb.item()


def test_noalloc_rejects_oversize():
    L = _lib.lib()
    mx = L.scao_int8_ema_update_noalloc_max_n()
    assert mx == 1 << 20
    q = torch.zeros(8, dtype=torch.int8, device=DEV)
    new = torch.zeros(8, device=DEV)
    out = torch.empty_like(q)
    so = torch.zeros(1, dtype=torch.float64, device=DEV)
    rc = L.scao_int8_ema_update_noalloc(q.data_ptr(), 1.0, new.data_ptr(), 0.9, mx + 1,
                                        out.data_ptr(), so.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 1   # SCAO_ERR_ARG, nothing launched


def test_noalloc_in_place():
    """q_out may alias q (the header allows it): same codes and scale as the
    regular entry point writing to a separate buffer."""
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    gen = torch.Generator().manual_seed(12)
    n = 200_003
    q = torch.randint(-127, 128, (n,), generator=gen, dtype=torch.int8).to(DEV)
    new = (torch.randn(n, generator=gen) * 0.1).to(DEV)
    qa, sa = _regular(L, q, 0.1 / 127.0, new, 0.99, st)
    qq = q.clone()
    so = torch.zeros(1, dtype=torch.float64, device=DEV)
    _lib.check(L.scao_int8_ema_update_noalloc(qq.data_ptr(), 0.1 / 127.0, new.data_ptr(), 0.99,
                                              n, qq.data_ptr(), so.data_ptr(), st), "in place")
    torch.cuda.synchronize()
    assert torch.equal(qa, qq)
    assert sa.item() == so.item()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_noalloc_second_device():
    """The staging array's address is looked up per device: a call on cuda:1
    (with cuda:1 current) matches the regular entry point there."""
    L = _lib.lib()
    dev = "cuda:1"
    gen = torch.Generator().manual_seed(13)
    n = 65_536
    with torch.cuda.device(1):
        st = torch.cuda.current_stream().cuda_stream
        q = torch.randint(-127, 128, (n,), generator=gen, dtype=torch.int8).to(dev)
        new = torch.randn(n, generator=gen).to(dev)
        qo = torch.empty_like(q)
        so = torch.zeros(1, dtype=torch.float64, device=dev)
        scratch = torch.empty(L.scao_int8_ema_scratch_bytes(n), dtype=torch.uint8, device=dev)
        _lib.check(L.scao_int8_ema_update(q.data_ptr(), 1.0 / 127.0, new.data_ptr(), 0.9, n,
                                          qo.data_ptr(), so.data_ptr(), scratch.data_ptr(), st),
                   "regular")
        qb = torch.empty_like(q)
        sb = torch.zeros(1, dtype=torch.float64, device=dev)
        _lib.check(L.scao_int8_ema_update_noalloc(q.data_ptr(), 1.0 / 127.0, new.data_ptr(), 0.9,
                                                  n, qb.data_ptr(), sb.data_ptr(), st), "noalloc")
        torch.cuda.synchronize()
    assert torch.equal(qo, qb)
    assert so.item() == sb.item()
