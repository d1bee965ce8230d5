"""Pins the CPU oracle (oracle/rouge_oracle.c) to the reference.

Two sources of truth, neither of which needs the reference at test time:
  * the known-answer vectors written in the reference's own tests
    (tests/test_gemm_fp8.cpp:38-70,73-99; tests/test_gemm_f16.cpp:36-58;
    tests/test_ai.cpp:89-96,163-184);
  * tests/golden/golden.npz, produced by running the reference library itself
    (tests/golden/make_golden.py).
Integer and code outputs must match bit for bit.
"""
import numpy as np

from conftest import rel_l2


def f32(x):
    return np.float32(x)


def test_e4m3_point_vectors(orc):
    # tests/test_gemm_fp8.cpp:38-51
    enc = orc.lib.or_e4m3_encode
    assert enc(1.0) == 0x38
    assert enc(-1.0) == 0xB8
    assert enc(448.0) == 0x7E
    assert enc(1000.0) == 0x7E
    assert enc(-1000.0) == 0xFE
    assert enc(float("inf")) == 0x7E
    assert enc(float("nan")) == 0x7F
    assert enc(-0.0) == 0x80
    assert np.float32(orc.lib.or_e4m3_decode(0x80)).view(np.uint32) == 0x80000000
    assert orc.lib.or_e4m3_decode(0x38) == 1.0
    assert orc.lib.or_e4m3_decode(0xB8) == -1.0


def test_e4m3_all_codes_round_trip(orc):
    # tests/test_gemm_fp8.cpp:55-70: every finite code is a fixed point
    codes = np.arange(256, dtype=np.uint8)
    vals = orc.e4m3_decode(codes)
    finite = np.isfinite(vals)
    assert (orc.e4m3_encode(vals[finite]) == codes[finite]).all()
    assert (orc.e4m3_encode(vals[~finite]) & 0x7F == 0x7F).all()


def test_e4m3_sign_dropped_below_half_subnormal(orc):
    # fp8.cpp:86: |x| < 2^-10 encodes as +0 whatever its sign
    assert orc.lib.or_e4m3_encode(-(2.0 ** -11)) == 0x00
    assert orc.lib.or_e4m3_encode(-(2.0 ** -10)) == 0x80  # exact tie rounds to even (-0)


def test_f16_bf16_point_vectors(orc):
    # tests/test_gemm_f16.cpp:36-58
    L = orc.lib
    assert L.or_f16_decode(0x3C00) == 1.0
    assert L.or_f16_decode(0xBC00) == -1.0
    assert L.or_f16_decode(0x3800) == 0.5
    assert np.float32(L.or_f16_decode(0x8000)).view(np.uint32) == 0x80000000
    assert np.isinf(L.or_f16_decode(0x7C00))
    assert np.isnan(L.or_f16_decode(0x7E00))
    assert L.or_f16_encode(1.0) == 0x3C00
    assert L.or_f16_encode(-0.0) == 0x8000
    assert L.or_f16_encode(100000.0) & 0x7FFF == 0x7C00
    assert L.or_f16_encode(float("nan")) & 0x7FFF == 0x7E00
    assert L.or_bf16_decode(0x3F80) == 1.0
    assert L.or_bf16_decode(0xBF80) == -1.0
    assert L.or_bf16_encode(1.0) == 0x3F80
    for i in range(1, 33):
        assert L.or_f16_decode(L.or_f16_encode(float(i))) == i
        assert L.or_bf16_decode(L.or_bf16_encode(float(i))) == i


def test_formats_match_golden(orc, golden):
    x = golden["fmt_x"]
    assert (orc.e4m3_encode(x) == golden["e4m3_codes"]).all()
    assert (orc.f16_encode(x) == golden["f16_codes"]).all()
    assert (orc.bf16_encode(x) == golden["bf16_codes"]).all()
    assert (orc.e4m3_decode(np.arange(256, dtype=np.uint8)).view(np.uint32)
            == golden["e4m3_decode_bits"]).all()
    assert (orc.f16_decode(golden["f16_decode_in"]).view(np.uint32) == golden["f16_decode_bits"]).all()


def test_int8_saturation(orc):
    # tests/test_ai.cpp:89-96
    q, _ = orc.quantize_i8_tensor(np.array([1000.0], np.float32))
    assert q[0] == 127
    q, _ = orc.quantize_i8_tensor(np.array([-1000.0], np.float32))
    assert q[0] == -127


def test_int8_rows_match_golden(orc, golden):
    q, s = orc.quantize_i8_rows(golden["q8_x"])
    assert (q == golden["q8_codes"]).all()
    assert (s.view(np.uint32) == golden["q8_scales"].view(np.uint32)).all()
    qt, st = orc.quantize_i8_tensor(golden["q8_x"][:20])
    assert (qt == golden["q8t_codes"]).all()
    assert np.float32(st) == golden["q8t_scale"]


def test_int8_group_matches_golden(orc, golden):
    q, s, z = orc.quantize_i8_group(golden["qg_x"], 4)
    assert (q == golden["qg_codes"]).all()
    assert (s.view(np.uint32) == golden["qg_scales"].view(np.uint32)).all()
    assert (z == golden["qg_zeros"]).all()
    back = orc.dequantize_i8_group(q, 4, s, z)
    assert (back.view(np.uint32) == golden["qg_back"].view(np.uint32)).all()


def test_int8_group_one_step_bound(orc):
    # tests/test_ai.cpp:130-160: error within one step of the stored scale
    rng = np.random.default_rng(0xA1)
    x = rng.uniform(-2, 2, (4, 64)).astype(np.float32)
    q, s, z = orc.quantize_i8_group(x, 8)
    back = orc.dequantize_i8_group(q, 8, s, z)
    step = np.repeat(s.reshape(4, 8), 8, axis=1).astype(np.float64)
    assert (np.abs(x - back) <= step * (1.0 + 1e-5) + 1e-6).all()


def test_int8_rows_half_step_bound(orc):
    # tests/test_ai.cpp:100-123
    rng = np.random.default_rng(0xA1)
    x = rng.uniform(-2, 2, (8, 64)).astype(np.float32)
    x[0, 0], x[0, 1] = 100.0, 0.001
    q, s = orc.quantize_i8_rows(x)
    back = orc.dequantize_i8_rows(q, s)
    step = np.abs(x).max(axis=1, keepdims=True).astype(np.float64) / 127.0
    assert (np.abs(x.astype(np.float64) - back) <= step * 0.5 + 1e-6).all()


def test_gemm_i8_exact_vs_long_long(orc):
    # tests/test_ai.cpp:163-184 (M=7, N=5, K=11)
    rng = np.random.default_rng(0xA1)
    A = rng.integers(-127, 128, (7, 11)).astype(np.int8)
    B = rng.integers(-127, 128, (11, 5)).astype(np.int8)
    acc, _ = orc.gemm_i8(A, B, b_nk=False)
    assert (acc == A.astype(np.int64) @ B.astype(np.int64)).all()
    accT, _ = orc.gemm_i8(A, np.ascontiguousarray(B.T), b_nk=True)
    assert (accT == acc).all()


def test_gemm_i8_matches_golden(orc, golden):
    for tag in "abc":
        A, B = golden[f"g8{tag}_A"], golden[f"g8{tag}_B"]
        acc, c = orc.gemm_i8(A, B, False, golden[f"g8{tag}_sa"], 1, golden[f"g8{tag}_sb"], 1)
        assert (acc == golden[f"g8{tag}_acc"]).all()
        assert (c.view(np.uint32) == golden[f"g8{tag}_C"].view(np.uint32)).all()


def test_float_gemms_match_golden(orc, golden):
    for a, b, c, dec in (("gh_A16", "gh_B16", "gh_C16", orc.f16_decode),
                         ("gh_Ab", "gh_Bb", "gh_Cb", orc.bf16_decode),
                         ("ge_A", "ge_B", "ge_C", orc.e4m3_decode)):
        got = orc.gemm_f32(dec(golden[a]), dec(golden[b]), b_nk=False)
        assert rel_l2(got, golden[c]) < 1e-6
    # integer e4m3 data: the product is exact (tests/test_gemm_fp8.cpp:73-99)
    got = orc.gemm_f32(orc.e4m3_decode(golden["ge_A"]), orc.e4m3_decode(golden["ge_B"]), False)
    assert (got == golden["ge_C"]).all()


def test_conv_matches_golden(orc, golden):
    x = np.ascontiguousarray(golden["cv_x"].transpose(0, 2, 3, 1))      # NCHW -> NHWC
    w = np.ascontiguousarray(golden["cv_w"].transpose(0, 2, 3, 1))      # OIHW -> OHWI
    y = orc.conv2d_nhwc(x, w, golden["cv_b"], 1, 1)
    N, C, H, W = golden["cv_y"].shape
    want = golden["cv_y"].transpose(0, 2, 3, 1).reshape(-1, C)
    assert rel_l2(y, want) < 1e-6
