"""rouge_gemm_i8_noalloc — the int8 GEMM for callers that cannot let the
library allocate device memory (for example a process that reserves the
GPU's memory for its own allocator at start-up, or a loop that must not
allocate once it runs). It stages everything in a fixed 64 MiB device array
instead of an allocated workspace. Checked through the C ABI against the
existing entry point rouge_gemm_i8 and against the oracle on two calls in a
row (the second call reuses the array the first one left behind, with a
different shape), with the same tolerance as the other int8 GEMM tests:
bit-exact f32 outputs. A call after the first ones of its shape class must
leave the device's free memory unchanged: that is what such a caller needs.

This file is collected last, so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed):
    rng = np.random.default_rng(seed)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (K, N), dtype=np.int8)     # [K][N], as rouge_gemm_i8 takes it
    sa = rng.uniform(1e-3, 2e-2, M).astype(np.float32)
    sb = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    return A, B, sa, sb


def _noalloc(rb, A, B, sa, a_rows, sb, b_cols):
    M, K = A.shape
    N = B.shape[1]
    out = np.full((M, N), np.nan, np.float32)
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    st = rb.lib().rouge_gemm_i8_noalloc(M, N, K, p(A), p(B), p(sa), a_rows, p(sb), b_cols, p(out))
    return st, out


CASES = (((300, 200, 100), (1, 1), 1),       # K, N padded inside the array
         ((1024, 768, 512), (0, 1), 2))      # a larger one, single row scale


def test_noalloc_matches_rouge_gemm_i8_on_two_calls(rb, orc, cuda):
    for (M, N, K), (a_rows, b_cols), seed in CASES:
        A, B, sa, sb = _operands(M, N, K, seed)
        if not a_rows:
            sa = sa[:1].copy()
        st, got = _noalloc(rb, A, B, sa, a_rows, sb, b_cols)
        assert st == rb.OK, rb.lib().rouge_b200_status_string(st)
        want = rb.host_gemm_i8(A, B, sa, a_rows, sb, b_cols)
        assert (got.view(np.uint32) == want.view(np.uint32)).all()
        # the oracle's ((float)acc * sa) * sb (quant_int8.cpp:189-211), B[K][N]
        _, oc = orc.gemm_i8(A, B, False, sa, a_rows, sb, b_cols)
        assert (got.view(np.uint32) == oc.view(np.uint32)).all()


def test_noalloc_warm_call_allocates_nothing(rb, cuda):
    import torch
    for (M, N, K), (a_rows, b_cols), seed in CASES:
        A, B, sa, sb = _operands(M, N, K, seed + 10)
        st, first = _noalloc(rb, A, B, sa, 1, sb, 1)    # the set-up call of this shape class
        assert st == rb.OK
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        st, again = _noalloc(rb, A, B, sa, 1, sb, 1)
        assert st == rb.OK
        assert torch.cuda.mem_get_info()[0] == free0     # the driver reserved nothing more
        assert (again.view(np.uint32) == first.view(np.uint32)).all()


def test_noalloc_refuses_problems_beyond_its_array(rb, cuda):
    M = N = K = 4096        # 16 + 16 MiB operands + 64 MiB output: more than 64 MiB
    A = np.zeros((M, K), np.int8)
    B = np.zeros((K, N), np.int8)
    s = np.ones(M, np.float32)
    st, out = _noalloc(rb, A, B, s, 1, s, 1)
    assert st == rb.ETOOBIG
    assert np.isnan(out).all()          # nothing written
