"""The clock probe (rouge_b200_set_clock_probe): while it is set, each CTA
of a GEMM launch writes its %clock64 and %globaltimer at start and end;
switched off, launches write nothing. No reference counterpart (a
measurement aid of this library)."""
import pytest

pytestmark = pytest.mark.gpu


def _gemm(rb, torch, cuda, M, N, K):
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=cuda)
    b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=cuda)
    c = torch.empty((M, N), dtype=torch.int32, device=cuda)
    return lambda: rb.gemm_i8(a, b, rb.B_NK, c, rb.OUT_I32)


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 512), (512, 512, 512)])
def test_probe_stamps_every_cta(rb, cuda, M, N, K):
    import torch
    f = _gemm(rb, torch, cuda, M, N, K)
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    with rb.clock_probe(2 * sms, cuda) as p:
        f()
        torch.cuda.synchronize()
        mhz = p.sm_mhz()
        w = p.stamps.view(-1, 4).cpu()
    rb.sync_status()
    ctas = int((w[:, 1] > 0).sum())
    assert ctas >= 1 and len(mhz) == ctas            # every started CTA also ended
    assert ((mhz > 200.0) & (mhz < 2600.0)).all(), mhz
    assert (w[ctas:] == 0).all()                      # no stamps past the grid


def test_probe_off_writes_nothing(rb, cuda):
    import torch
    f = _gemm(rb, torch, cuda, 1024, 1024, 256)
    p = rb.clock_probe(64, cuda)
    with p:
        pass
    f()
    torch.cuda.synchronize()
    rb.sync_status()
    assert int(p.stamps.abs().sum()) == 0


def test_probe_arguments(rb, cuda):
    L = rb.lib()
    assert L.rouge_b200_set_clock_probe(None, -1) == rb.EINVAL
    assert L.rouge_b200_set_clock_probe(None, 0) == rb.OK
