"""The oracle's restatement of narrow.cpp (e4m3 / e5m2 / e3m2 / e2m3 / e2m1,
E8M0, MXFP8 / MXFP4 / NVFP4 blocks) pinned two ways: the known answers of
the reference's own test (test_narrow.cpp:29-82, 86-180) and the reference
library compiled from its sources (oracle/_ref), on every code, on ~4 M
f32 bit patterns per format, and on random and special-value blocks."""
import numpy as np
import pytest

FMTS = ["e5m2", "e3m2", "e2m3", "e2m1"]
WIDTH = {"e4m3": 8, "e5m2": 8, "e3m2": 6, "e2m3": 6, "e2m1": 4}


def _same_f32(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return bool((na == nb).all() and (a[~na].view(np.uint32) == b[~nb].view(np.uint32)).all())


def test_known_answers(orc):
    # test_narrow.cpp:30-51: e5m2 round trip of every code, the special points
    codes = np.arange(256, dtype=np.uint8)
    v = orc.narrow_decode(codes, "e5m2")
    back = orc.narrow_encode(v, "e5m2")
    nan, inf = np.isnan(v), np.isinf(v)
    assert ((back[nan] & 0x7F) == 0x7F).all()
    assert ((back[inf] & 0x7F) == 0x7B).all()
    assert (back[~nan & ~inf] == codes[~nan & ~inf]).all()
    assert orc.narrow_decode([0x7B], "e5m2")[0] == 57344.0
    assert np.isinf(orc.narrow_decode([0x7C, 0xFC], "e5m2")).all()
    assert np.isnan(orc.narrow_decode([0x7F], "e5m2")[0])
    assert orc.narrow_encode([57344.0, 1e30], "e5m2").tolist() == [0x7B, 0x7B]
    assert orc.narrow_encode([-0.0], "e5m2")[0] & 0x80
    # :54-66: e2m1 round trip, values, NaN -> +MAX
    c16 = np.arange(16, dtype=np.uint8)
    assert (orc.narrow_encode(orc.narrow_decode(c16, "e2m1"), "e2m1") == c16).all()
    assert orc.narrow_decode([0x07, 0x0F, 0x00, 0x02, 0x04], "e2m1").tolist() == [6, -6, 0, 1, 2]
    assert orc.narrow_encode([np.nan], "e2m1")[0] == 0x07
    # :69-82: e3m2 / e2m3 points and signed saturation
    assert orc.narrow_decode([0x1F, 0x3F, 0x04], "e3m2").tolist() == [28, -28, 0.25]
    assert orc.narrow_decode([0x1F, 0x3F, 0x08], "e2m3").tolist() == [7.5, -7.5, 1.0]
    for fmt, mx in (("e3m2", 0x1F), ("e2m3", 0x1F), ("e2m1", 0x07)):
        sign = 1 << (WIDTH[fmt] - 1)
        assert orc.narrow_encode([100.0, -100.0], fmt).tolist() == [mx, mx | sign]


@pytest.mark.parametrize("fmt", FMTS)
def test_decode_every_code_matches_reference(orc, ref, fmt):
    codes = np.arange(1 << WIDTH[fmt], dtype=np.uint8)
    assert _same_f32(orc.narrow_decode(codes, fmt), ref.narrow_decode(codes, fmt))


def _patterns():
    u = np.arange(0, 1 << 32, 1021, dtype=np.uint64).astype(np.uint32)
    special = np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00000, 0x00000001,
                        0x807FFFFF, 0x3E800000, 0xBE800000, 0x3F400000, 0x43E00000, 0x43E80000,
                        0x44000000, 0x47600000, 0x47700000], np.uint32)
    return np.concatenate([u, special]).view(np.float32)


@pytest.mark.parametrize("fmt", FMTS)
def test_encode_bit_patterns_match_reference(orc, ref, fmt):
    x = _patterns()
    assert (orc.narrow_encode(x, fmt) == ref.narrow_encode(x, fmt)).all()


def _blocks(rng, n):
    x = rng.uniform(-10, 10, n).astype(np.float32)
    x[0], x[1] = 37.5, -37.5                              # test_narrow.cpp:94-95
    x[32:64] = 0.0                                         # an all-zero block
    x[64:96] *= np.float32(1e-30)                          # tiny block (f32 subnormal products)
    x[96:128] *= np.float32(3e30)                          # huge block (scale 2^p, p large)
    x[130], x[131], x[133] = np.inf, -np.inf, np.nan       # non-finite elements
    x[160:192] = rng.choice([448.0, -464.0, 480.0, 224.0, 6.0, -3.25], 32).astype(np.float32)
    return x


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m1"])
def test_mx_quantize_matches_reference(orc, ref, fmt):
    rng = np.random.default_rng(0x4D58)
    for n in (32, 96, 1000, 4096 + 7):
        x = _blocks(rng, max(n, 200))[:n] if n >= 200 else rng.uniform(-10, 10, n).astype(np.float32)
        q, s = orc.mx_quantize(x, fmt)
        rq, rs = ref.mx_quantize(x, fmt)
        assert (q == rq).all() and (s == rs).all()
        assert _same_f32(orc.mx_dequantize(q, s, fmt), ref.mx_dequantize(rq, rs, fmt))


@pytest.mark.parametrize("gs", [1.0, 0.5, 3.0, 1e-20, 0.0, -2.0, float("nan")])
def test_nvfp4_quantize_matches_reference(orc, ref, gs):
    rng = np.random.default_rng(16)
    x = _blocks(rng, 1024)
    q, s = orc.nvfp4_quantize(x, gs)
    rq, rs = ref.nvfp4_quantize(x, gs)
    assert (q == rq).all() and (s == rs).all()


def test_e8m0_scale_is_twice_the_chosen_power(orc):
    # f32_to_e8m0 (narrow.cpp:155-163) codes 2^p as p + 128 (frexp's exponent)
    for p in range(0, 20):
        assert orc.lib.or_e8m0_encode(float(2.0 ** p)) == p + 128
    assert orc.lib.or_e8m0_decode(128) == 2.0
    assert np.isnan(orc.lib.or_e8m0_decode(255))
