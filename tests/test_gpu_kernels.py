"""GPU parity of the sm_100a kernels, called through the C ABI with device
pointers, against the CPU oracle on the same seeded inputs.

Integer, code and scale outputs must be bit-exact. Floating-point GEMM
outputs must be within the north-star tolerance (relative L2 <= 1e-2) and,
as a kernel-health bound, within 1e-4 of the double-accumulated oracle
(e4m3/f16 products are exact in f32, so only summation order differs)."""
import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL_CONTRACT = 1e-2
TOL_KERNEL = 1e-4


def dev_tensor(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


# ---------------------------------------------------------------- int8 quant

# Row counts of 296 and more take the warp-per-row kernel (one per register
# size: rows up to 1024, 2048 and 4096 elements), fewer rows and longer
# rows the CTA-per-row kernels. The warp-per-row cases cover 1 to 24 rows
# per SM (148 SMs), so that every count of rows left after whole rounds of
# an SM's 12 warps occurs.
@pytest.mark.parametrize("shape", [(1, 4), (3, 8), (48, 40), (257, 1028), (64, 8192), (16, 12288),
                                   (1024, 1024), (700, 2044), (1200, 4096), (4096, 4096),
                                   (640, 4100), (800, 12), (1924, 12), (1924, 4096), (2072, 1028),
                                   (592, 1020), (3552, 256)])
def test_quantize_i8_rows(rb, orc, cuda, shape):
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    x = rng.standard_normal(shape).astype(np.float32)
    x[rng.random(shape) < 0.01] *= 20.0
    xd = dev_tensor(x, cuda)
    q = torch.empty(shape, dtype=torch.int8, device=cuda)
    s = torch.empty(shape[0], dtype=torch.float32, device=cuda)
    rb.quantize_i8_rows(xd, s, q)
    rb.sync_status()
    oq, os_ = orc.quantize_i8_rows(x)
    assert (q.cpu().numpy() == oq).all()
    assert (s.cpu().numpy().view(np.uint32) == os_.view(np.uint32)).all()


def test_quantize_i8_rows_golden(rb, cuda, golden):
    x = golden["q8_x"]
    q = torch.empty(x.shape, dtype=torch.int8, device=cuda)
    s = torch.empty(x.shape[0], dtype=torch.float32, device=cuda)
    rb.quantize_i8_rows(dev_tensor(x, cuda), s, q)
    rb.sync_status()
    assert (q.cpu().numpy() == golden["q8_codes"]).all()
    assert (s.cpu().numpy().view(np.uint32) == golden["q8_scales"].view(np.uint32)).all()


@pytest.mark.parametrize("reps", [1, 200, 250])
def test_quantize_i8_rows_special_values(rb, orc, cuda, reps):
    x = np.zeros((8, 16), np.float32)
    x[1] = np.inf                        # scale inf, codes from NaN products
    x[2, :4] = [np.inf, -np.inf, 1.0, -1.0]
    x[3] = 1e-44                         # subnormal row: scale underflows to 0
    x[4, :3] = [np.nan, 2.0, -3.0]
    x[5] = -0.0
    x[6] = np.linspace(-1e-36, 1e-36, 16)  # subnormal scale, finite reciprocal
    x[7] = np.linspace(-3e-37, 3e-37, 16)  # subnormal scale, reciprocal beyond f32
    x = np.tile(x, (reps, 1))
    q = torch.empty(x.shape, dtype=torch.int8, device=cuda)
    s = torch.empty(x.shape[0], dtype=torch.float32, device=cuda)
    rb.quantize_i8_rows(dev_tensor(x, cuda), s, q)
    rb.sync_status()
    oq, os_ = orc.quantize_i8_rows(x)
    assert (q.cpu().numpy() == oq).all()
    assert (s.cpu().numpy().view(np.uint32) == os_.view(np.uint32)).all()


@pytest.mark.parametrize("reps", [1, 30, 60])
def test_quantize_i8_rows_near_ties(rb, orc, cuda, reps):
    # Values a few ulps around k + 1/2 under several scales: the products the
    # single-precision fast path must hand to the exact double path.
    rows = []
    base = np.arange(-126, 127, dtype=np.float32) + np.float32(0.5)
    for amax in (127.0, 100.0, 3.0, 1e-3, 12345.678):
        s = np.float32(np.float64(amax) / 127.0)
        for d in range(-3, 4):
            v = (base.astype(np.float64) * float(s)).astype(np.float32)
            v = (v.view(np.int32) + d).view(np.float32)
            row = np.concatenate([[np.float32(amax)], v, np.zeros(256 - 1 - v.size, np.float32)])
            rows.append(row[:256])
    x = np.tile(np.stack(rows).astype(np.float32), (reps, 1))
    q = torch.empty(x.shape, dtype=torch.int8, device=cuda)
    s = torch.empty(x.shape[0], dtype=torch.float32, device=cuda)
    rb.quantize_i8_rows(dev_tensor(x, cuda), s, q)
    rb.sync_status()
    oq, os_ = orc.quantize_i8_rows(x)
    assert (s.cpu().numpy() == os_).all()
    assert (q.cpu().numpy() == oq).all()


@pytest.mark.parametrize("shape,groups", [((1, 4), 1), ((33, 96), 8), ((5, 7), 7), ((512, 4096), 32)])
def test_quantize_i8_group(rb, orc, cuda, shape, groups):
    rng = np.random.default_rng(shape[0] + groups)
    x = (rng.standard_normal(shape) * 3).astype(np.float32)
    x[0] = np.abs(x[0])
    rows, cols = shape
    q = torch.empty(shape, dtype=torch.uint8, device=cuda)
    s = torch.empty(rows * groups, dtype=torch.float32, device=cuda)
    z = torch.empty(rows * groups, dtype=torch.uint8, device=cuda)
    rb.quantize_i8_group(dev_tensor(x, cuda), groups, s, z, q)
    back = torch.empty(shape, dtype=torch.float32, device=cuda)
    rb.dequantize_i8_group(q, groups, s, z, back)
    rb.sync_status()
    oq, os_, oz = orc.quantize_i8_group(x, groups)
    assert (q.cpu().numpy() == oq).all()
    assert (s.cpu().numpy().view(np.uint32) == os_.view(np.uint32)).all()
    assert (z.cpu().numpy() == oz).all()
    ob = orc.dequantize_i8_group(oq, groups, os_, oz)
    assert (back.cpu().numpy().view(np.uint32) == ob.view(np.uint32)).all()


def test_quantize_i8_group_golden(rb, cuda, golden):
    x = golden["qg_x"]
    q = torch.empty(x.shape, dtype=torch.uint8, device=cuda)
    s = torch.empty(x.shape[0] * 4, dtype=torch.float32, device=cuda)
    z = torch.empty(x.shape[0] * 4, dtype=torch.uint8, device=cuda)
    rb.quantize_i8_group(dev_tensor(x, cuda), 4, s, z, q)
    rb.sync_status()
    assert (q.cpu().numpy() == golden["qg_codes"]).all()
    assert (s.cpu().numpy().view(np.uint32) == golden["qg_scales"].view(np.uint32)).all()
    assert (z.cpu().numpy() == golden["qg_zeros"]).all()


def test_dequantize_i8_rows(rb, orc, cuda):
    rng = np.random.default_rng(1)
    q = rng.integers(-127, 128, (33, 64), dtype=np.int8)
    s = rng.uniform(1e-3, 1.0, 33).astype(np.float32)
    out = torch.empty((33, 64), dtype=torch.float32, device=cuda)
    rb.dequantize_i8_rows(dev_tensor(q, cuda), dev_tensor(s, cuda), out)
    rb.sync_status()
    assert (out.cpu().numpy().view(np.uint32) == orc.dequantize_i8_rows(q, s).view(np.uint32)).all()


# ---------------------------------------------------------------- formats

def float_space():
    bits = np.arange(0, 2 ** 32, 61, dtype=np.uint64).astype(np.uint32)
    dense = np.arange(0x3A000000, 0x3C000000, dtype=np.uint32)  # |x| in [2^-11, 2^-7)
    return np.concatenate([bits, dense, dense | 0x80000000]).view(np.float32)


def test_e4m3_encode_float_space(rb, orc, cuda):
    # amax = 448 gives s = 1, so the kernel encodes x / 1 = x itself.
    x = float_space()
    x = x[: x.size // 16 * 16]
    amax = torch.tensor([448.0], dtype=torch.float32, device=cuda)
    s = torch.zeros(1, dtype=torch.float32, device=cuda)
    out = torch.empty(x.size, dtype=torch.uint8, device=cuda)
    rb.quantize_e4m3_scaled(dev_tensor(x, cuda), amax, s, out)
    rb.sync_status()
    assert s.item() == 1.0
    got = out.cpu().numpy()
    want = orc.e4m3_encode(x)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, x[bad[:8]].view(np.uint32)


@pytest.mark.parametrize("fmt", ["f16", "bf16"])
def test_half_encode_float_space(rb, orc, cuda, fmt):
    x = float_space()
    out = torch.empty(x.size, dtype=torch.int16, device=cuda)
    fn = rb.convert_f32_to_f16 if fmt == "f16" else rb.convert_f32_to_bf16
    fn(dev_tensor(x, cuda), out)
    rb.sync_status()
    got = out.cpu().numpy().view(np.uint16)
    want = getattr(orc, f"{fmt}_encode")(x)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, x[bad[:8]].view(np.uint32)


def test_e4m3_decode_all_codes(rb, orc, cuda):
    c = np.tile(np.arange(256, dtype=np.uint8), 5)
    out = torch.empty(c.size, dtype=torch.float32, device=cuda)
    rb.convert_e4m3_to_f32(dev_tensor(c, cuda), out)
    rb.sync_status()
    assert (out.cpu().numpy().view(np.uint32) == orc.e4m3_decode(c).view(np.uint32)).all()


@pytest.mark.parametrize("n", [1, 17, 1 << 20, (1 << 24) + 13])
def test_e4m3_per_tensor(rb, orc, cuda, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    if n > 20:
        x[5] = np.nan                    # ignored by the max
        x[7] = -1e-7                     # far below 2^-10 after scaling: +0
    xd = dev_tensor(x, cuda)
    am = torch.empty(2, dtype=torch.float32, device=cuda)
    out = torch.empty(n, dtype=torch.uint8, device=cuda)
    if n % 4 == 0:
        rb.quantize_e4m3_tensor(xd, am[0:1], am[1:2], out)
    else:  # unaligned sizes go through the scalar tail
        rb.quantize_e4m3_tensor(xd, am[0:1], am[1:2], out)
    rb.sync_status()
    oc, os_, oamax = orc.quantize_e4m3_tensor(x)
    assert am[0].item() == np.float32(oamax)
    assert np.float32(am[1].item()) == np.float32(os_)
    assert (out.cpu().numpy() == oc).all()


@pytest.mark.parametrize("amax", [3.7, 1000.0, 0.0123, 6.02e-5])
def test_e4m3_per_tensor_near_code_boundaries(rb, orc, cuda, amax):
    # Values a few ulps around (s * m) for every e4m3 midpoint and code value
    # m, under scales that are not powers of two: the quotients the
    # division-free encoder must hand to the exact path.
    s = np.float32(np.float32(amax) / np.float32(448.0))
    codes = orc.e4m3_decode(np.arange(256, dtype=np.uint8))
    vals = np.unique(np.abs(codes[np.isfinite(codes)]).astype(np.float64))
    mids = (vals[:-1] + vals[1:]) / 2
    base = np.concatenate([vals, mids, [2.0 ** -10, 2.0 ** -9, 464.0]])
    x = (base * float(s)).astype(np.float32)
    x = np.concatenate([(x.view(np.int32) + d).view(np.float32) for d in range(-4, 5)])
    x = np.concatenate([x, -x])
    x = x[np.abs(x) < np.float32(amax)]
    x = np.concatenate([[np.float32(amax)], x]).astype(np.float32)
    x = np.resize(x, (x.size + 15) // 16 * 16)
    xd = dev_tensor(x, cuda)
    am = torch.empty(2, dtype=torch.float32, device=cuda)
    out = torch.empty(x.size, dtype=torch.uint8, device=cuda)
    rb.quantize_e4m3_tensor(xd, am[0:1], am[1:2], out)
    rb.sync_status()
    oc, os_, _ = orc.quantize_e4m3_tensor(x)
    assert np.float32(am[1].item()) == np.float32(os_)
    got = out.cpu().numpy()
    bad = np.nonzero(got != oc)[0]
    assert bad.size == 0, (x[bad[:8]], got[bad[:8]], oc[bad[:8]])


def test_e4m3_per_tensor_special_values(rb, orc, cuda):
    # x86-64 results the reference produces: a NaN operand keeps its sign,
    # inf/inf is the negative default NaN, x/inf is +-0.
    nan_neg = np.array([0xFFC00001], np.uint32).view(np.float32)[0]
    cases = [
        np.array([np.inf, -np.inf, 1.0, 0.0, -2.0, nan_neg, np.nan, -0.0] * 2, np.float32),
        np.array([1e-44, -1e-44, 0.0, 3e-45] * 4, np.float32),    # amax/448 underflows to 0
        np.array([0.0] * 16, np.float32),                          # amax 0 -> s = 1
    ]
    for x in cases:
        am = torch.empty(2, dtype=torch.float32, device=cuda)
        out = torch.empty(x.size, dtype=torch.uint8, device=cuda)
        rb.quantize_e4m3_tensor(dev_tensor(x, cuda), am[0:1], am[1:2], out)
        rb.sync_status()
        oc, os_, _ = orc.quantize_e4m3_tensor(x)
        assert np.float32(am[1].item()).view(np.uint32) == np.float32(os_).view(np.uint32)
        assert (out.cpu().numpy() == oc).all(), (x, out.cpu().numpy(), oc)


def test_absmax_all_zero(rb, cuda):
    x = torch.zeros(1000, dtype=torch.float32, device=cuda)
    am = torch.full((1,), 5.0, dtype=torch.float32, device=cuda)
    rb.absmax(x, am)
    rb.sync_status()
    assert am.item() == 0.0


# ---------------------------------------------------------------- GEMMs

# Tile widths the shapes take (148 SMs): 32 for the small ones, 64 for
# (1024, 1024, 1024), (256, 4096, 512) and (600, 1000, 128) (ragged N), 128
# and CTA pairs for the rest.
GEMM_SHAPES = [(128, 256, 128), (7, 5, 16), (300, 200, 96), (130, 96, 64), (1024, 1024, 1024),
               (256, 4096, 512), (4096, 128, 256), (600, 1000, 128), (1000, 1200, 640)]


def gemm_operands(rng, M, N, K):
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (N, K), dtype=np.int8)   # [N][K]
    sa = rng.uniform(1e-3, 2e-2, M).astype(np.float32)
    sb = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    return A, B, sa, sb


@pytest.mark.parametrize("shape", GEMM_SHAPES)
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_gemm_i8_int32_exact(rb, orc, cuda, shape, layout):
    M, N, K = shape
    if layout == "kn" and N % 16:
        pytest.skip("B[K][N] needs N % 16 == 0 (16-byte rows)")
    if K % 16:
        pytest.skip("K % 16 == 0 required")
    rng = np.random.default_rng(M * 31 + N * 7 + K)
    A, B, sa, sb = gemm_operands(rng, M, N, K)
    Bdev = B if layout == "nk" else np.ascontiguousarray(B.T)
    lay = rb.B_NK if layout == "nk" else rb.B_KN
    acc = torch.empty((M, N), dtype=torch.int32, device=cuda)
    rb.gemm_i8(dev_tensor(A, cuda), dev_tensor(Bdev, cuda), lay, acc, rb.OUT_I32)
    c = torch.empty((M, N), dtype=torch.float32, device=cuda)
    rb.gemm_i8(dev_tensor(A, cuda), dev_tensor(Bdev, cuda), lay, c, rb.OUT_F32,
               dev_tensor(sa, cuda), 1, dev_tensor(sb, cuda), 1)
    rb.sync_status()
    oacc, oc = orc.gemm_i8(A, B, True, sa, 1, sb, 1)
    got = acc.cpu().numpy()
    assert (got == oacc).all(), np.argwhere(got != oacc)[:5]
    assert (c.cpu().numpy().view(np.uint32) == oc.view(np.uint32)).all()


def test_gemm_i8_bf16_and_scalar_scales(rb, orc, cuda):
    rng = np.random.default_rng(77)
    M, N, K = 384, 512, 256
    A, B, sa, sb = gemm_operands(rng, M, N, K)
    cb = torch.empty((M, N), dtype=torch.int16, device=cuda)
    rb.gemm_i8(dev_tensor(A, cuda), dev_tensor(B, cuda), rb.B_NK, cb, rb.OUT_BF16,
               dev_tensor(sa, cuda), 1, dev_tensor(sb, cuda), 1)
    c0 = torch.empty((M, N), dtype=torch.float32, device=cuda)
    rb.gemm_i8(dev_tensor(A, cuda), dev_tensor(B, cuda), rb.B_NK, c0, rb.OUT_F32,
               dev_tensor(sa[:1], cuda), 0, dev_tensor(sb[:1], cuda), 0)
    rb.sync_status()
    _, oc = orc.gemm_i8(A, B, True, sa, 1, sb, 1)
    assert (cb.cpu().numpy().view(np.uint16) == orc.bf16_encode(oc)).all()
    _, oc0 = orc.gemm_i8(A, B, True, sa[:1], 0, sb[:1], 0)
    assert (c0.cpu().numpy().view(np.uint32) == oc0.view(np.uint32)).all()


def test_gemm_i8_strided_output(rb, orc, cuda):
    rng = np.random.default_rng(5)
    M, N, K = 200, 96, 128
    A, B, sa, sb = gemm_operands(rng, M, N, K)
    big = torch.full((M, 160), -7, dtype=torch.int32, device=cuda)
    rb.gemm_i8(dev_tensor(A, cuda), dev_tensor(B, cuda), rb.B_NK, big[:, 16:16 + N], rb.OUT_I32)
    rb.sync_status()
    oacc, _ = orc.gemm_i8(A, B, True)
    g = big.cpu().numpy()
    assert (g[:, 16:16 + N] == oacc).all()
    assert (g[:, :16] == -7).all() and (g[:, 16 + N:] == -7).all()


@pytest.mark.parametrize("shape", [(128, 256, 128), (33, 48, 64), (512, 512, 512), (1000, 1200, 640)])
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_gemm_e4m3(rb, orc, cuda, shape, layout):
    M, N, K = shape
    rng = np.random.default_rng(M + N + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((N, K)).astype(np.float32)
    qa, sa, _ = orc.quantize_e4m3_tensor(a)
    qb, sb, _ = orc.quantize_e4m3_tensor(b)
    Bdev = qb if layout == "nk" else np.ascontiguousarray(qb.T)
    lay = rb.B_NK if layout == "nk" else rb.B_KN
    sad = torch.tensor([sa], dtype=torch.float32, device=cuda)
    sbd = torch.tensor([sb], dtype=torch.float32, device=cuda)
    c = torch.empty((M, N), dtype=torch.float32, device=cuda)
    rb.gemm_e4m3(dev_tensor(qa, cuda), dev_tensor(Bdev, cuda), lay, c, rb.OUT_F32)
    cb = torch.empty((M, N), dtype=torch.int16, device=cuda)
    rb.gemm_e4m3(dev_tensor(qa, cuda), dev_tensor(Bdev, cuda), lay, cb, rb.OUT_BF16, sad, sbd)
    rb.sync_status()
    want = orc.gemm_f32(orc.e4m3_decode(qa), orc.e4m3_decode(qb), True)
    err = rel_l2(c.cpu().numpy(), want)
    assert err < TOL_CONTRACT and err < TOL_KERNEL, err
    wantb = want * np.float32(np.float32(sa) * np.float32(sb))
    errb = rel_l2(orc.bf16_decode(cb.cpu().numpy().view(np.uint16)), wantb)
    assert errb < TOL_CONTRACT, errb


def test_gemm_e4m3_integer_data_exact(rb, orc, cuda, golden):
    # tests/test_gemm_fp8.cpp:73-99: integers 1..8, the f32 result is exact
    qa, qb_kn, want = golden["ge_A"], golden["ge_B"], golden["ge_C"]
    c = torch.empty(want.shape, dtype=torch.float32, device=cuda)
    rb.gemm_e4m3(dev_tensor(qa, cuda), dev_tensor(qb_kn, cuda), rb.B_KN, c, rb.OUT_F32)
    rb.sync_status()
    assert (c.cpu().numpy() == want).all()


@pytest.mark.parametrize("shape", [(128, 256, 64), (40, 56, 72), (512, 512, 512), (777, 640, 320),
                                   (600, 1000, 128)])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_gemm_f16(rb, orc, cuda, shape, bf16, layout):
    M, N, K = shape
    if layout == "kn" and N % 8:
        pytest.skip("B[K][N] needs N % 8 == 0")
    rng = np.random.default_rng(M * 3 + N + K)
    enc = orc.bf16_encode if bf16 else orc.f16_encode
    dec = orc.bf16_decode if bf16 else orc.f16_decode
    a = enc(rng.uniform(-1, 1, (M, K)).astype(np.float32))
    b = enc(rng.uniform(-1, 1, (N, K)).astype(np.float32))
    Bdev = b if layout == "nk" else np.ascontiguousarray(b.T)
    lay = rb.B_NK if layout == "nk" else rb.B_KN
    c = torch.empty((M, N), dtype=torch.float32, device=cuda)
    rb.gemm_f16(dev_tensor(a.view(np.int16), cuda), dev_tensor(Bdev.view(np.int16), cuda), lay, c,
                rb.OUT_F32, is_bf16=bf16)
    rb.sync_status()
    want = orc.gemm_f32(dec(a), dec(b), True)
    err = rel_l2(c.cpu().numpy(), want)
    assert err < TOL_CONTRACT and err < TOL_KERNEL, err


def test_unsupported_layouts_are_refused(rb, cuda):
    A = torch.zeros((64, 24), dtype=torch.int8, device=cuda)   # K = 24: rows not 16-byte
    B = torch.zeros((64, 24), dtype=torch.int8, device=cuda)
    C = torch.zeros((64, 64), dtype=torch.int32, device=cuda)
    with pytest.raises(rb.RougeB200Error) as e:
        rb.gemm_i8(A, B, rb.B_NK, C, rb.OUT_I32)
    assert e.value.status == rb.EUNSUPPORTED
