"""The drop-in host-pointer entries (same names and semantics as the
reference numerics.h) against the golden outputs of the reference library,
on the reference's own test shapes (odd sizes included: the entries pad
operands internally)."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def test_quantize_i8_channel_golden(rb, cuda, golden):
    q, s = rb.host_quantize_i8_channel(golden["q8_x"])
    assert (q == golden["q8_codes"]).all()
    assert (s.view(np.uint32) == golden["q8_scales"].view(np.uint32)).all()


def test_quantize_i8_tensor_golden(rb, cuda, golden):
    q, s = rb.host_quantize_i8_tensor(golden["q8_x"][:20])
    assert (q == golden["q8t_codes"].ravel()).all()
    assert np.float32(s) == golden["q8t_scale"]


def test_quantize_i8_group_golden(rb, cuda, golden):
    q, s, z = rb.host_quantize_i8_group(golden["qg_x"], 4)
    assert (q == golden["qg_codes"]).all()
    assert (s.view(np.uint32) == golden["qg_scales"].view(np.uint32)).all()
    assert (z == golden["qg_zeros"]).all()
    back = rb.host_dequantize_i8_group(q, 4, s, z)
    assert (back.view(np.uint32) == golden["qg_back"].view(np.uint32)).all()
    # cols % groups != 0 is refused (quant_int8.cpp:98)
    with pytest.raises(rb.RougeB200Error):
        rb.host_quantize_i8_group(golden["qg_x"][:, :63], 4)


def test_quantize_i8_odd_columns(rb, orc, cuda):
    rng = np.random.default_rng(4)
    for shape in ((5, 3), (9, 41), (2, 1)):
        x = rng.standard_normal(shape).astype(np.float32)
        q, s = rb.host_quantize_i8_channel(x)
        oq, os_ = orc.quantize_i8_rows(x)
        assert (q == oq).all() and (s == os_).all()


def test_dequantize_round_trip(rb, orc, cuda, golden):
    # tests/test_ai.cpp:100-123: per-row error <= half a step
    x = golden["q8_x"][:3]
    q, s = rb.host_quantize_i8_channel(x)
    back = rb.host_dequantize_i8_channel(q, s)
    assert (back.view(np.uint32) == orc.dequantize_i8_rows(q, s).view(np.uint32)).all()
    step = np.abs(x).max(axis=1, keepdims=True).astype(np.float64) / 127.0
    assert (np.abs(x - back) <= step * 0.5 + 1e-6).all()
    qt, st = rb.host_quantize_i8_tensor(x)
    bt = rb.host_dequantize_i8_tensor(qt, st)
    assert (bt == qt.astype(np.float32) * np.float32(st)).all()


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_gemm_i8_golden(rb, cuda, golden, tag):
    A, B = golden[f"g8{tag}_A"], golden[f"g8{tag}_B"]
    C = rb.host_gemm_i8(A, B, golden[f"g8{tag}_sa"], 1, golden[f"g8{tag}_sb"], 1)
    assert (C.view(np.uint32) == golden[f"g8{tag}_C"].view(np.uint32)).all()


def test_gemm_i8_exact_small(rb, cuda):
    # tests/test_ai.cpp:163-184: llround(C / (sa*sb)) == integer product
    rng = np.random.default_rng(0xA1)
    A = rng.integers(-127, 128, (7, 11)).astype(np.int8)
    B = rng.integers(-127, 128, (11, 5)).astype(np.int8)
    sa, sb = np.float32(0.013), np.float32(0.021)
    C = rb.host_gemm_i8(A, B, [sa], 0, [sb], 0)
    want = A.astype(np.int64) @ B.astype(np.int64)
    assert (np.rint(C.astype(np.float64) / (float(sa) * float(sb))).astype(np.int64) == want).all()


def test_gemm_f16_bf16_golden(rb, cuda, golden):
    # tests/test_gemm_f16.cpp:61-94: 1e-2 of scale vs the f32 GEMM
    for a, b, c, fn in (("gh_A16", "gh_B16", "gh_C16", rb.host_gemm_f16),
                        ("gh_Ab", "gh_Bb", "gh_Cb", rb.host_gemm_bf16)):
        got = fn(golden[a], golden[b])
        want = golden[c]
        assert np.abs(got - want).max() / max(np.abs(want).max(), 1.0) < 1e-5
        assert rel_l2(got, want) < 1e-2


def test_gemm_e4m3_golden_exact(rb, cuda, golden):
    got = rb.host_gemm_e4m3(golden["ge_A"], golden["ge_B"])
    assert (got == golden["ge_C"]).all()


def test_null_and_empty_are_noops(rb, cuda):
    out = np.full((4, 4), 3.0, np.float32)
    rb.lib().rouge_gemm_f16(0, 4, 4, None, None, out.ctypes.data, None)
    assert (out == 3.0).all()


# Operands of 8 MB and more move in row bands on three streams (copy in,
# kernels, copy out overlapping). These shapes give several bands with a
# ragged last one; rows on both sides of every band edge are checked.

def _band_rows(M, step):
    edges = [r for b in range(step, M, step) for r in (b - 1, b)]
    return np.unique(np.array([0, 1, M - 1] + edges, np.int32))


@pytest.mark.parametrize("rows,cols", [(3000, 1000), (2500, 1003)])
def test_quantize_i8_channel_banded(rb, orc, cuda, rows, cols):
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[rng.random((rows, cols)) < 0.01] *= 20.0
    q, s = rb.host_quantize_i8_channel(x)
    oq, os_ = orc.quantize_i8_rows(x)
    assert (q == oq).all()
    assert (s.view(np.uint32) == os_.view(np.uint32)).all()


# Ragged last bands, per-row and single scales on either side; the last
# of the first four is below the banding threshold. The last two have a B
# of 8 MB and more, which comes in four column blocks that the first band
# is computed and copied out by (a ragged last block in the last case).
@pytest.mark.parametrize("M,N,K,a_rows,b_cols", [(1000, 2048, 1024, 1, 1), (1100, 2000, 1000, 0, 1),
                                                 (1300, 1700, 528, 1, 0), (700, 600, 256, 1, 1),
                                                 (1024, 4096, 2048, 1, 1), (600, 4100, 2064, 0, 1)])
def test_gemm_i8_banded(rb, orc, cuda, M, N, K, a_rows, b_cols):
    rng = np.random.default_rng(M + N + K)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (K, N), dtype=np.int8)   # [K][N], as rouge_gemm_i8 takes it
    sa = rng.uniform(1e-3, 2e-2, M if a_rows else 1).astype(np.float32)
    sb = rng.uniform(1e-3, 2e-2, N if b_cols else 1).astype(np.float32)
    C = rb.host_gemm_i8(A, B, sa, a_rows, sb, b_cols)
    rows = _band_rows(M, 256)
    _, oc = orc.gemm_i8(A, B, False, sa, a_rows, sb, b_cols, rows=rows)
    assert (C[rows].view(np.uint32) == oc.view(np.uint32)).all()


def test_gemm_f16_banded(rb, orc, cuda):
    M, N, K = 2000, 1024, 520
    rng = np.random.default_rng(7)
    a = orc.f16_encode(rng.uniform(-1, 1, (M, K)).astype(np.float32))
    b = orc.f16_encode(rng.uniform(-1, 1, (K, N)).astype(np.float32))   # [K][N]
    C = rb.host_gemm_f16(a, b)
    rows = _band_rows(M, 256)
    want = orc.gemm_f32(orc.f16_decode(a), orc.f16_decode(b), False, rows=rows)
    err = rel_l2(C[rows], want)
    assert err < 1e-2 and err < 1e-4, err
