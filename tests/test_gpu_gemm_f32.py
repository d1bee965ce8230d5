"""rouge_gemm_f32 and the tuner entries (numerics.h:54-55, 311-324;
gemm.cpp:291-383, autotune.cpp:32-127) on the GPU, through the C ABI with
host arrays, checked the way the reference's own test checks its CPU GEMM
(tests/test_gemm.cpp:25-63): its eight sizes, every candidate
configuration, the default configuration, the tuner's result and profile,
against a naive f64 product with max|C - ref| / max(||ref||_inf, 1) <= 1e-5.
The reference library itself (oracle/_ref) is held to the same bound on the
same inputs, which pins the metric."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# tests/test_gemm.cpp:25-29
SIZES = [(1, 1, 1), (3, 5, 7), (17, 33, 65), (128, 128, 128), (200, 100, 50), (64, 64, 128),
         (129, 131, 127), (256, 192, 128)]
TOL = 1e-5  # tests/test_gemm.cpp:32


def rel_error(got, ref):
    """tests/test_gemm.cpp:37-45: max|got - ref| / max(||ref||_inf, 1)."""
    return float(np.max(np.abs(got.astype(np.float64) - ref)) / max(np.max(np.abs(ref)), 1.0))


def inputs(M, N, K):
    rng = np.random.default_rng(M * 7919 + N * 104729 + K)
    A = rng.uniform(-1.0, 1.0, (M, K)).astype(np.float32)
    B = rng.uniform(-1.0, 1.0, (K, N)).astype(np.float32)
    return A, B, A.astype(np.float64) @ B.astype(np.float64)


@pytest.mark.parametrize("M,N,K", SIZES)
def test_every_candidate_and_default(cuda, rb, M, N, K):
    A, B, want = inputs(M, N, K)
    results = []
    for cfg in rb.gemm_candidates() + [None]:
        C_ = np.full((M, N), -7.0, np.float32)       # C is overwritten, not accumulated
        rb.host_gemm_f32(A, B, cfg, out=C_)
        err = rel_error(C_, want)
        assert np.isfinite(err) and err <= TOL, (cfg and cfg.astuple(), err)
        results.append(C_)
    # every tile shape accumulates each element over K in the same order
    for r in results[1:]:
        assert (r.view(np.uint32) == results[0].view(np.uint32)).all()


@pytest.mark.parametrize("M,N,K", SIZES)
def test_tuner_result_and_profile(cuda, rb, M, N, K):
    A, B, want = inputs(M, N, K)
    C_ = np.full((M, N), -7.0, np.float32)
    prof = rb.gemm_tuned(A, B, C_)
    rb.lib().rouge_b200_clear_error()
    assert rel_error(C_, want) <= TOL
    assert prof.gflops > 0.0 and prof.iters == 4 * rb.lib().rouge_gemm_candidate_count()
    assert prof.cfg.astuple() in [c.astuple() for c in rb.gemm_candidates()]
    C2 = np.zeros_like(C_)
    assert rb.gemm_flops_per_sec(A, B, C2, prof.cfg) > 0.0
    assert (C2.view(np.uint32) == C_.view(np.uint32)).all()


def test_reference_meets_the_same_bound(ref):
    # the metric is the reference's: its own CPU GEMM passes it on these inputs
    for M, N, K in SIZES:
        A, B, want = inputs(M, N, K)
        assert rel_error(ref.gemm_f32(A, B), want) <= TOL


@pytest.mark.parametrize("M,N,K", [(1000, 1200, 640), (2048, 1536, 1024), (4096, 4096, 4096)])
def test_larger_shapes_against_reference(cuda, rb, ref, M, N, K):
    # past the reference test's sizes: the same metric against f64 on
    # sampled rows, and the reference library's own result on those rows
    rng = np.random.default_rng(M + N + K)
    A = rng.uniform(-1.0, 1.0, (M, K)).astype(np.float32)
    B = rng.uniform(-1.0, 1.0, (K, N)).astype(np.float32)
    got = rb.host_gemm_f32(A, B)
    rows = np.unique(np.r_[0, 1, M // 2, M - 1, rng.integers(0, M, 12)])
    want = A[rows].astype(np.float64) @ B.astype(np.float64)
    assert rel_error(got[rows], want) <= TOL
    theirs = ref.gemm_f32(A[rows], B)
    assert rel_error(theirs, want) <= TOL
