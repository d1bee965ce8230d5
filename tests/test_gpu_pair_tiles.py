"""CTA-pair tiles (tcgen05.mma.cta_group::2, 256 x 256 tiles over a 2-CTA
cluster) against the oracle, with the tile mode forced so that the pair
kernel runs on small shapes too. Each case runs in both modes (SINGLE and
PAIR); int8 results must be bit-exact in both (int32 accumulation is exact,
quant_int8.cpp:189-211), floating-point GEMMs and convolutions within the
relative-L2 bound 1e-2 (and 1e-4 as a kernel-health bound).

Shapes cover the pair kernel's edges: M below 128 (the second CTA's A rows
are all out of range), M and N not multiples of the tile, N <= 128 (the
second CTA's half of B is out of range), several tiles per cluster and
both B layouts."""
import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu

MODES = ["single", "pair"]


def _mode(rb, name):
    return rb.tile_mode(rb.TILES_PAIR if name == "pair" else rb.TILES_SINGLE)


def _dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


# Few tiles: the launcher also cuts the last round's tiles N-wise into two
# units (K-major B), so these cover split units too, (256, 96, 128) one
# whose second part lies wholly beyond N.
I8_SHAPES = [(100, 256, 128), (256, 256, 256), (300, 200, 96), (520, 384, 640),
             (1024, 1024, 1024), (4096, 512, 256), (256, 4096, 128), (256, 96, 128)]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", I8_SHAPES)
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_pair_gemm_i8_exact(rb, orc, cuda, mode, shape, layout):
    M, N, K = shape
    if layout == "kn" and N % 16:
        pytest.skip("B[K][N] needs N % 16 == 0")
    rng = np.random.default_rng(M * 5 + N * 3 + K)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sa = rng.uniform(1e-3, 2e-2, M).astype(np.float32)
    sb = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    Bd = B if layout == "nk" else B.T
    lay = rb.B_NK if layout == "nk" else rb.B_KN
    acc = torch.empty((M, N), dtype=torch.int32, device=cuda)
    c = torch.empty((M, N), dtype=torch.float32, device=cuda)
    cb = torch.empty((M, N), dtype=torch.int16, device=cuda)
    with _mode(rb, mode):
        rb.gemm_i8(_dev(A, cuda), _dev(Bd, cuda), lay, acc, rb.OUT_I32)
        rb.gemm_i8(_dev(A, cuda), _dev(Bd, cuda), lay, c, rb.OUT_F32,
                   _dev(sa, cuda), 1, _dev(sb, cuda), 1)
        rb.gemm_i8(_dev(A, cuda), _dev(Bd, cuda), lay, cb, rb.OUT_BF16,
                   _dev(sa, cuda), 1, _dev(sb, cuda), 1)
        rb.sync_status()
    oacc, oc = orc.gemm_i8(A, B, True, sa, 1, sb, 1)
    got = acc.cpu().numpy()
    assert (got == oacc).all(), np.argwhere(got != oacc)[:5]
    assert (c.cpu().numpy().view(np.uint32) == oc.view(np.uint32)).all()
    assert (cb.cpu().numpy().view(np.uint16) == orc.bf16_encode(oc)).all()


@pytest.mark.parametrize("mode", MODES)
def test_pair_gemm_i8_strided_output(rb, orc, cuda, mode):
    rng = np.random.default_rng(11)
    M, N, K = 272, 96, 128
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (N, K), dtype=np.int8)
    big = torch.full((M, 160), -7, dtype=torch.int32, device=cuda)
    with _mode(rb, mode):
        rb.gemm_i8(_dev(A, cuda), _dev(B, cuda), rb.B_NK, big[:, 16:16 + N], rb.OUT_I32)
        rb.sync_status()
    oacc, _ = orc.gemm_i8(A, B, True)
    g = big.cpu().numpy()
    assert (g[:, 16:16 + N] == oacc).all()
    assert (g[:, :16] == -7).all() and (g[:, 16 + N:] == -7).all()


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [(100, 128, 128), (600, 528, 384), (1024, 1024, 2048)])
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_pair_gemm_e4m3(rb, orc, cuda, mode, shape, layout):
    M, N, K = shape
    rng = np.random.default_rng(M + 2 * N + K)
    qa, _, _ = orc.quantize_e4m3_tensor(rng.standard_normal((M, K)).astype(np.float32))
    qb, _, _ = orc.quantize_e4m3_tensor(rng.standard_normal((N, K)).astype(np.float32))
    Bd = qb if layout == "nk" else qb.T
    lay = rb.B_NK if layout == "nk" else rb.B_KN
    c = torch.empty((M, N), dtype=torch.float32, device=cuda)
    with _mode(rb, mode):
        rb.gemm_e4m3(_dev(qa, cuda), _dev(Bd, cuda), lay, c, rb.OUT_F32)
        rb.sync_status()
    want = orc.gemm_f32(orc.e4m3_decode(qa), orc.e4m3_decode(qb), True)
    err = rel_l2(c.cpu().numpy(), want)
    assert err < 1e-2 and err < 1e-4, err


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [(90, 64, 64), (640, 384, 512)])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_pair_gemm_f16(rb, orc, cuda, mode, shape, bf16, layout):
    M, N, K = shape
    rng = np.random.default_rng(M * 7 + N + K)
    enc = orc.bf16_encode if bf16 else orc.f16_encode
    dec = orc.bf16_decode if bf16 else orc.f16_decode
    a = enc(rng.uniform(-1, 1, (M, K)).astype(np.float32))
    b = enc(rng.uniform(-1, 1, (N, K)).astype(np.float32))
    Bd = b if layout == "nk" else b.T
    lay = rb.B_NK if layout == "nk" else rb.B_KN
    c = torch.empty((M, N), dtype=torch.float32, device=cuda)
    with _mode(rb, mode):
        rb.gemm_f16(_dev(a.view(np.int16), cuda), _dev(Bd.view(np.int16), cuda), lay, c,
                    rb.OUT_F32, is_bf16=bf16)
        rb.sync_status()
    want = orc.gemm_f32(dec(a), dec(b), True)
    err = rel_l2(c.cpu().numpy(), want)
    assert err < 1e-2 and err < 1e-4, err


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [
    # N, H, W, Cin, Cout, KH, KW, stride, pad
    (4, 16, 16, 64, 64, 3, 3, 1, 1),       # Cout below the second CTA's B half
    (4, 9, 11, 192, 256, 3, 3, 1, 0),      # odd spatial sizes, pixel count not a tile multiple
    (4, 20, 20, 64, 320, 3, 3, 2, 1),      # stride 2, Cout over one tile
])
def test_pair_conv(rb, orc, cuda, mode, shape):
    N, H, W, Cin, Cout, KH, KW, stride, pad = shape
    rng = np.random.default_rng(Cout + H)
    x = orc.f16_encode(rng.uniform(-1, 1, (N, H, W, Cin)).astype(np.float32))
    w = orc.f16_encode((rng.standard_normal((Cout, KH, KW, Cin)) *
                        np.sqrt(2.0 / (KH * KW * Cin))).astype(np.float32))
    b = rng.standard_normal(Cout).astype(np.float32)
    OH = (H + 2 * pad - KH) // stride + 1
    OW = (W + 2 * pad - KW) // stride + 1
    y = torch.full((N, OH, OW, Cout), float("nan"), dtype=torch.float32, device=cuda)
    with _mode(rb, mode):
        rb.conv2d_nhwc_f16(_dev(x.view(np.int16), cuda), _dev(w.view(np.int16), cuda),
                           _dev(b, cuda), y, stride, pad)
        rb.sync_status()
    got = y.cpu().numpy().reshape(-1, Cout)
    want = orc.conv2d_nhwc(orc.f16_decode(x), orc.f16_decode(w), b, stride, pad)
    assert np.isfinite(got).all()
    err = rel_l2(got, want)
    assert err < 1e-2 and err < 1e-4, err


def test_pair_and_single_agree_on_large_i8(rb, cuda):
    # 4096 x 4096 x 4096 (the W8A8 headline shape) through both kernels:
    # identical int32 accumulators.
    M = N = K = 4096
    g = torch.Generator(device=cuda).manual_seed(3)
    A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=cuda, generator=g)
    B = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=cuda, generator=g)
    out = {}
    for mode in MODES:
        acc = torch.empty((M, N), dtype=torch.int32, device=cuda)
        with _mode(rb, mode):
            rb.gemm_i8(A, B, rb.B_NK, acc, rb.OUT_I32)
            rb.sync_status()
        out[mode] = acc
    assert torch.equal(out["single"], out["pair"])
    # spot-check two row blocks against an f64 product (every partial sum is
    # an integer below 2^53, so it is exact)
    for r0 in (0, 4032):
        ref = (A[r0:r0 + 64].double() @ B.double().T).to(torch.int32)
        assert torch.equal(out["pair"][r0:r0 + 64], ref)
