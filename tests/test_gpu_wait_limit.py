"""Failure detection of the device-side waits, without a GPU fault.

Every wait of the kernels (TMA stage barriers, MMA commits, TMEM drains) is
bounded by %globaltimer and leaves through an abort flag shared by the
block. rouge_b200_check_wait_limit launches one CTA whose mbarrier nothing
ever arrives at: the wait must run out after the requested limit, the other
warps must leave on the abort flag rather than on their own 5 s limit, the
error word must read ROUGE_B200_ETIMEOUT once (and be cleared by the read),
and the context must still run an int8 GEMM bit-exact afterwards."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_wait_runs_out_and_context_survives(rb, orc, cuda):
    import torch
    L = rb.lib()
    assert L.rouge_b200_sync_status(None) == rb.OK
    for limit_ms in (20, 250):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        st = rb.check_wait_limit(limit_ms * 1_000_000)
        dt = time.perf_counter() - t0
        assert st == rb.ETIMEOUT, L.rouge_b200_status_string(st)
        assert limit_ms / 1000 <= dt < limit_ms / 1000 + 2.0, dt   # ended on the limit, not at 5 s
        assert L.rouge_b200_sync_status(None) == rb.OK                # the read cleared the word

    rng = np.random.default_rng(11)
    M, N, K = 256, 384, 512
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (N, K), dtype=np.int8)
    acc = torch.empty((M, N), dtype=torch.int32, device=cuda)
    rb.gemm_i8(torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda), rb.B_NK, acc, rb.OUT_I32)
    rb.sync_status()
    want, _ = orc.gemm_i8(A, B, True)
    assert (acc.cpu().numpy() == want).all()


def test_wait_limit_arguments(rb, cuda):
    L = rb.lib()
    for bad in (0, 999_999, 2_000_000_001):
        assert L.rouge_b200_check_wait_limit(bad, None) == rb.EINVAL
    assert L.rouge_b200_sync_status(None) == rb.OK
