"""librouge_b200_cublas.so: the cuBLAS GEMM API subset (the reference's
cublas_shim.cpp entry names, statuses and column-major semantics) on the
tcgen05 kernels. Device pointers, the handle's stream.

Checked against an f64 product of the same operands: f32 (3xTF32 split
operands) relative L2 <= 1e-5; f16 / bf16 / e4m3 inputs <= 1e-4 (f32
accumulation); int8 exact. beta == 0 must not read C (C is NaN there)."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "rouge-v_b200", "lib", "librouge_b200_cublas.so")
OP = {"N": 0, "T": 1, "C": 2}
CUDA_R_32F, CUDA_R_16F, CUDA_R_16BF, CUDA_R_8I, CUDA_R_32I, CUDA_R_8F_E4M3 = 0, 2, 14, 3, 10, 28
COMPUTE_32F, COMPUTE_32I = 68, 72


@pytest.fixture(scope="module")
def blas(cuda):
    L = C.CDLL(SHIM)
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    yield L, h
    assert L.cublasDestroy_v2(h) == 0


def colmajor(rows, cols, ld, dtype, fill=None, gen=None):
    """Device storage of a column-major rows x cols matrix with leading
    dimension ld: a [cols][ld] row-major tensor; returns (storage, view)."""
    t = torch.empty((cols, ld), dtype=dtype, device="cuda")
    if fill is not None:
        t.fill_(fill)
    else:
        t.copy_(gen((cols, ld)))
    return t, t[:, :rows].T   # view[i, j] = element (i, j)


def op(x, o):
    return x if o == "N" else x.T


def rel_l2(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _f32(shape):
    return torch.randn(shape, device="cuda")


@pytest.mark.parametrize("ta", ["N", "T", "C"])
@pytest.mark.parametrize("tb", ["N", "T"])
@pytest.mark.parametrize("m,n,k", [(67, 45, 33), (256, 128, 512), (130, 257, 96)])
def test_sgemm(blas, ta, tb, m, n, k):
    L, h = blas
    torch.manual_seed(m + n + k)
    ar, ac = (m, k) if ta == "N" else (k, m)
    br, bc = (k, n) if tb == "N" else (n, k)
    A, Av = colmajor(ar, ac, ar + 3, torch.float32, gen=_f32)
    B, Bv = colmajor(br, bc, br + 5, torch.float32, gen=_f32)
    Cs, Cv = colmajor(m, n, m + 1, torch.float32, gen=_f32)
    c0 = Cv.double().clone()
    alpha, beta = C.c_float(1.5), C.c_float(-0.5)
    st = L.cublasSgemm_v2(h, OP[ta], OP[tb], m, n, k, C.byref(alpha), C.c_void_p(A.data_ptr()),
                          ar + 3, C.c_void_p(B.data_ptr()), br + 5, C.byref(beta),
                          C.c_void_p(Cs.data_ptr()), m + 1)
    assert st == 0
    torch.cuda.synchronize()
    want = 1.5 * (op(Av.double(), ta) @ op(Bv.double(), tb)) - 0.5 * c0
    assert rel_l2(Cv, want) < 1e-5


def test_sgemm_beta_zero_ignores_c_and_k_zero(blas):
    L, h = blas
    m, n, k = 96, 80, 64
    A, Av = colmajor(m, k, m, torch.float32, gen=_f32)
    B, Bv = colmajor(k, n, k, torch.float32, gen=_f32)
    Cs, Cv = colmajor(m, n, m, torch.float32, fill=float("nan"))
    one, zero = C.c_float(1.0), C.c_float(0.0)
    assert L.cublasSgemm_v2(h, 0, 0, m, n, k, C.byref(one), C.c_void_p(A.data_ptr()), m,
                            C.c_void_p(B.data_ptr()), k, C.byref(zero), C.c_void_p(Cs.data_ptr()),
                            m) == 0
    torch.cuda.synchronize()
    assert torch.isfinite(Cv).all()
    assert rel_l2(Cv, Av.double() @ Bv.double()) < 1e-5
    # k == 0: C = beta * C
    two = C.c_float(2.0)
    before = Cv.clone()
    assert L.cublasSgemm_v2(h, 0, 0, m, n, 0, C.byref(one), C.c_void_p(A.data_ptr()), m,
                            C.c_void_p(B.data_ptr()), 1, C.byref(two), C.c_void_p(Cs.data_ptr()),
                            m) == 0
    torch.cuda.synchronize()
    assert torch.equal(Cv, 2.0 * before)


def test_sgemm_device_pointer_mode_and_batched(blas):
    L, h = blas
    m, n, k, nb = 64, 48, 40, 3
    A = torch.randn((nb, k, m), device="cuda")   # batch of column-major m x k, lda = m
    B = torch.randn((nb, n, k), device="cuda")   # column-major k x n, ldb = k
    Cs = torch.randn((nb, n, m), device="cuda")
    c0 = Cs.double().clone()
    ab = torch.tensor([0.75, 0.25], device="cuda")
    assert L.cublasSetPointerMode_v2(h, 1) == 0
    try:
        st = L.cublasSgemmStridedBatched(h, 0, 0, m, n, k, C.c_void_p(ab.data_ptr()),
                                         C.c_void_p(A.data_ptr()), m, C.c_longlong(k * m),
                                         C.c_void_p(B.data_ptr()), k, C.c_longlong(n * k),
                                         C.c_void_p(ab.data_ptr() + 4), C.c_void_p(Cs.data_ptr()),
                                         m, C.c_longlong(n * m), nb)
    finally:
        assert L.cublasSetPointerMode_v2(h, 0) == 0
    assert st == 0
    torch.cuda.synchronize()
    for b in range(nb):
        want = 0.75 * (A[b].double().T @ B[b].double().T) + 0.25 * c0[b].T
        assert rel_l2(Cs[b].T, want) < 1e-5


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("ta,tb", [("N", "N"), ("T", "N"), ("N", "T")])
def test_gemm_ex_half(blas, dt, ta, tb):
    L, h = blas
    m, n, k = 200, 136, 264
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    ctype = CUDA_R_16F if dt == "f16" else CUDA_R_16BF
    ar, ac = (m, k) if ta == "N" else (k, m)
    br, bc = (k, n) if tb == "N" else (n, k)
    gen = lambda s: torch.rand(s, device="cuda").to(tdt) - 0.5  # noqa: E731
    A, Av = colmajor(ar, ac, ar, tdt, gen=gen)
    B, Bv = colmajor(br, bc, br, tdt, gen=gen)
    Cs, Cv = colmajor(m, n, m, torch.float32, fill=float("nan"))
    one, zero = C.c_float(1.0), C.c_float(0.0)
    st = L.cublasGemmEx(h, OP[ta], OP[tb], m, n, k, C.byref(one), C.c_void_p(A.data_ptr()), ctype, ar,
                        C.c_void_p(B.data_ptr()), ctype, br, C.byref(zero), C.c_void_p(Cs.data_ptr()),
                        CUDA_R_32F, m, COMPUTE_32F, -1)
    assert st == 0
    torch.cuda.synchronize()
    want = op(Av.double(), ta) @ op(Bv.double(), tb)
    assert rel_l2(Cv, want) < 1e-4


def test_gemm_ex_int8_exact(blas):
    L, h = blas
    m, n, k = 160, 96, 128
    gen = lambda s: torch.randint(-127, 128, s, device="cuda", dtype=torch.int8)  # noqa: E731
    A, Av = colmajor(k, m, k, torch.int8, gen=gen)     # op(A) = A^T: stored k x m
    B, Bv = colmajor(k, n, k, torch.int8, gen=gen)
    Cs, Cv = colmajor(m, n, m, torch.int32, fill=-7)
    one, zero = C.c_int32(1), C.c_int32(0)
    st = L.cublasGemmEx(h, 1, 0, m, n, k, C.byref(one), C.c_void_p(A.data_ptr()), CUDA_R_8I, k,
                        C.c_void_p(B.data_ptr()), CUDA_R_8I, k, C.byref(zero), C.c_void_p(Cs.data_ptr()),
                        CUDA_R_32I, m, COMPUTE_32I, -1)
    assert st == 0
    torch.cuda.synchronize()
    want = (Av.double().T @ Bv.double()).round().to(torch.int32)
    assert torch.equal(Cv, want)


def test_invalid_arguments(blas):
    L, h = blas
    one = C.c_float(1.0)
    x = torch.zeros(64, device="cuda")
    p = C.c_void_p(x.data_ptr())
    assert L.cublasSgemm_v2(h, 5, 0, 4, 4, 4, C.byref(one), p, 4, p, 4, C.byref(one), p, 4) == 7
    assert L.cublasSgemm_v2(h, 0, 0, 4, 4, 4, C.byref(one), p, 2, p, 4, C.byref(one), p, 4) == 7
    assert L.cublasGemmEx(h, 0, 0, 4, 4, 4, C.byref(one), p, CUDA_R_16F, 4, p, CUDA_R_16BF, 4,
                          C.byref(one), p, CUDA_R_32F, 4, COMPUTE_32F, -1) == 15
    assert L.cublasGetStatusString(7) is not None
