"""Cross-checks the oracle restatement against the reference library itself
(oracle/_ref/librouge_ref.so, compiled from the reference sources) on many
seeded inputs. Skipped where the reference library was not built."""
import numpy as np
import pytest

from conftest import rel_l2


@pytest.mark.parametrize("fmt", ["e4m3", "f16", "bf16"])
def test_encoders_over_float_space(orc, ref, fmt):
    # Every 251st float bit pattern (17M values, all exponents and signs),
    # plus a dense window around the small-magnitude boundaries.
    bits = np.arange(0, 2 ** 32, 251, dtype=np.uint64).astype(np.uint32)
    dense = np.arange(0x38000000 - 2 ** 22, 0x38000000 + 2 ** 22, dtype=np.uint32)  # ~2^-15
    e4 = np.arange(0x3A000000, 0x3B800000, 3, dtype=np.uint32)                      # ~2^-11..2^-8
    x = np.concatenate([bits, dense, dense | 0x80000000, e4, e4 | 0x80000000]).view(np.float32)
    mine = getattr(orc, f"{fmt}_encode")(x)
    theirs = ref.encode_n(fmt, x)
    bad = np.nonzero(mine != theirs)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x bits {x[bad[:4]].view(np.uint32)}"


@pytest.mark.parametrize("shape", [(1, 1), (3, 7), (64, 33), (256, 4096)])
def test_quantize_rows_vs_reference(orc, ref, shape):
    rng = np.random.default_rng(shape[0] * 1000 + shape[1])
    x = rng.standard_normal(shape).astype(np.float32)
    x[rng.random(shape) < 0.01] *= 20.0
    q1, s1 = orc.quantize_i8_rows(x)
    q2, s2 = ref.quantize_i8_channel(x)
    assert (q1 == q2).all()
    assert (s1.view(np.uint32) == s2.view(np.uint32)).all()
    q3, s3 = ref.quantize_i8_channel(x, threads=4)  # row-sliced driver is bit-identical
    assert (q3 == q2).all() and (s3 == s2).all()


@pytest.mark.parametrize("shape,groups", [((1, 4), 1), ((33, 96), 8), ((5, 7), 7), ((128, 4096), 32)])
def test_quantize_group_vs_reference(orc, ref, shape, groups):
    rng = np.random.default_rng(shape[1] + groups)
    x = (rng.standard_normal(shape) * 3).astype(np.float32)
    x[0, 0] = abs(x[0, 0]) + 5.0
    mine = orc.quantize_i8_group(x, groups)
    theirs = ref.quantize_i8_group(x, groups)
    for a, b in zip(mine, theirs):
        assert (a.view(np.uint8) == b.view(np.uint8)).all()
    assert (orc.dequantize_i8_group(*mine[:1], groups, mine[1], mine[2]).view(np.uint32)
            == ref.dequantize_i8_group(theirs[0], groups, theirs[1], theirs[2]).view(np.uint32)).all()


def test_gemm_i8_vs_reference(orc, ref):
    rng = np.random.default_rng(3)
    M, N, K = 97, 80, 300
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (K, N), dtype=np.int8)
    sa = rng.uniform(1e-3, 1e-2, M).astype(np.float32)
    sb = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    acc, c = orc.gemm_i8(A, B, False, sa, 1, sb, 1)
    assert (acc == ref.gemm_i8_acc(A, B)).all()
    assert (c.view(np.uint32) == ref.gemm_i8(A, B, sa, 1, sb, 1).view(np.uint32)).all()
    assert (ref.gemm_i8(A, B, sa, 1, sb, 1, threads=3) == ref.gemm_i8(A, B, sa, 1, sb, 1)).all()
    # per-tensor scales (a_rows = b_cols = 0)
    _, c0 = orc.gemm_i8(A, B, False, sa[:1], 0, sb[:1], 0)
    assert (c0.view(np.uint32) == ref.gemm_i8(A, B, sa[:1], 0, sb[:1], 0).view(np.uint32)).all()


def test_e4m3_tensor_scaling_vs_reference(orc, ref):
    rng = np.random.default_rng(11)
    x = rng.standard_normal(1 << 16).astype(np.float32)
    codes, s, amax = orc.quantize_e4m3_tensor(x)
    assert amax == np.abs(x).max()
    assert np.float32(s) == np.float32(amax) / np.float32(448.0)
    assert (codes == ref.encode_n("e4m3", x / np.float32(s))).all()


def test_float_gemm_vs_reference(orc, ref):
    rng = np.random.default_rng(5)
    A = rng.uniform(-1, 1, (40, 72)).astype(np.float32)
    B = rng.uniform(-1, 1, (72, 56)).astype(np.float32)
    assert rel_l2(orc.gemm_f32(A, B, False), ref.gemm_f32(A, B)) < 1e-6
    assert rel_l2(orc.gemm_f32(A, np.ascontiguousarray(B.T), True), ref.gemm_f32(A, B)) < 1e-6


def test_conv_vs_reference(orc, ref):
    rng = np.random.default_rng(9)
    x = rng.uniform(-1, 1, (2, 16, 12, 10)).astype(np.float32)
    w = (rng.standard_normal((24, 16, 3, 3)) * 0.1).astype(np.float32)
    b = rng.standard_normal(24).astype(np.float32)
    for stride, pad in ((1, 1), (2, 0), (1, 0)):
        want = ref.conv2d_f32(x, w, b, stride, pad)
        got = orc.conv2d_nhwc(x.transpose(0, 2, 3, 1), w.transpose(0, 2, 3, 1), b, stride, pad)
        assert rel_l2(got, want.transpose(0, 2, 3, 1).reshape(-1, 24)) < 1e-6


def test_reference_arm_inputs_match_the_library_generator(rb, ref):
    # bench.py's reference arm builds its inputs with the checker library's
    # copy of the generator (so its process never maps librouge_b200.so);
    # both arms must see the same bits.
    a = ref.synth_normal(1, (300, 129), 0.0, 1.0)
    na = ref.synth_outliers(1, a, 0.01, 20.0)
    b = rb.synth_normal(1, (300, 129), 0.0, 1.0)
    nb = rb.synth_outliers(1, b, 0.01, 20.0)
    assert na == nb and (a.view(np.uint32) == b.view(np.uint32)).all()
    a = ref.synth_normal(9, (6, 8192), 0.0, 0.02, offset=4 * 8192)
    b = rb.synth_normal_at(9, 4 * 8192, (6, 8192), 0.0, 0.02)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
    a = ref.synth_uniform(0, (77, 33), -1.0, 1.0)
    b = rb.synth_uniform(0, (77, 33), -1.0, 1.0)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
