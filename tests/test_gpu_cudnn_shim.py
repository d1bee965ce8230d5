"""librouge_b200_cudnn.so on the GPU against the reference's cuDNN shim
(cudnn_shim.cpp, compiled from its sources into oracle/_ref) run on the same
inputs, call for call through the same API:

* convolution forward FLOAT + NCHW (the reference's only case, test_shims.cpp:
  277-325 included): relative error <= 1e-5 of the largest output
  (3xTF32 tensor-core sums against the reference's f32 CPU sums);
* HALF / BFLOAT16 in NHWC and NCHW (the reference refuses them): against the
  oracle's double-precision convolution of the decoded operands, within one
  unit in the last place of the output type;
* AddTensor and BatchNorm inference bit-exact, activation and softmax
  within a few f32 ulps (the GPU's exp / tanh), host and device operands.
"""
import os

import numpy as np
import pytest

import dnn_api as D

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ours(cuda):
    d = D.Dnn(D.B200_DNN)
    assert d.create() == D.SUCCESS
    yield d
    d.close()


@pytest.fixture(scope="module")
def theirs():
    if not os.path.exists(D.REF_SHIMS):
        pytest.skip("reference shims library not built")
    d = D.Dnn(D.REF_SHIMS)
    assert d.create() == D.SUCCESS
    yield d
    d.close()


def _dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _host(t):
    return t.cpu().numpy()


def _descs(lib, dtype, xfmt, wfmt, yfmt, N, Cin, H, W, Cout, KH, KW, pad, stride):
    xd = lib.tensor(xfmt, dtype, N, Cin, H, W)[0]
    wd = lib.filter(dtype, wfmt, Cout, Cin, KH, KW)[0]
    cd, st = lib.conv(pad, stride)
    assert st == D.SUCCESS
    st, (n, c, oh, ow) = lib.output_dim(cd, xd, wd)
    assert st == D.SUCCESS
    yd = lib.tensor(yfmt, dtype, n, c, oh, ow)[0]
    return xd, wd, cd, yd, (oh, ow)


FLOAT_CASES = [  # N, Cin, H, W, Cout, KH, KW, pad, stride
    (1, 2, 8, 8, 3, 3, 3, 1, 1),        # test_shims.cpp:286-325
    (2, 5, 13, 11, 7, 3, 3, 1, 2),
    (2, 16, 20, 20, 32, 1, 1, 0, 1),
    (1, 3, 32, 32, 8, 7, 7, 3, 2),
    (3, 8, 9, 9, 4, 5, 5, 2, 1),
    (2, 64, 28, 28, 64, 3, 3, 1, 1),
]


@pytest.mark.parametrize("case", FLOAT_CASES)
@pytest.mark.parametrize("algo", [D.ALGO_IMPLICIT_GEMM, D.ALGO_WINOGRAD])
def test_conv_float_nchw_matches_reference(ours, theirs, cuda, case, algo):
    N, Cin, H, W, Cout, KH, KW, pad, stride = case
    rng = np.random.default_rng(sum(case) + algo)
    x = rng.uniform(-1, 1, (N, Cin, H, W)).astype(np.float32)
    w = rng.uniform(-1, 1, (Cout, Cin, KH, KW)).astype(np.float32)
    al, be = 2.0, 0.5
    outs = {}
    for name, lib in (("ref", theirs), ("ours", ours)):
        xd, wd, cd, yd, (oh, ow) = _descs(lib, D.FLOAT, D.NCHW, D.NCHW, D.NCHW, N, Cin, H, W, Cout,
                                          KH, KW, pad, stride)
        y = np.full((N, Cout, oh, ow), 0.25, np.float32)
        assert lib.conv_forward(al, xd, x, wd, w, cd, algo, yd, y, be) == D.SUCCESS
        outs[name] = y
        if lib is ours:  # device operands give the same bits as host operands
            yt = _dev(np.full((N, Cout, oh, ow), 0.25, np.float32), cuda)
            assert lib.conv_forward(al, xd, _dev(x, cuda), wd, _dev(w, cuda), cd, algo, yd, yt,
                                    be) == D.SUCCESS
            assert (_host(yt).view(np.uint32) == y.view(np.uint32)).all()
    want, got = outs["ref"], outs["ours"]
    md = float(np.abs(got.astype(np.float64) - want).max())
    # the reference's Winograd path carries its own f32 error (its test: 1e-4)
    tol = 1e-4 if algo == D.ALGO_WINOGRAD and (KH, KW, stride, pad) == (3, 3, 1, 1) else 1e-5
    assert md / max(1.0, float(np.abs(want).max())) <= tol, md


def _decode(a, dtype):
    if dtype == D.HALF:
        return a.view(np.float16).astype(np.float64)
    return (a.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _encode(v, dtype):
    v = np.asarray(v, np.float32)
    if dtype == D.HALF:
        return v.astype(np.float16).view(np.uint16)
    b = v.view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def _to(a, fmt):
    """NCHW-ordered array -> the memory order of fmt (NHWC: channels last)."""
    return np.ascontiguousarray(a if fmt == D.NCHW else a.transpose(0, 2, 3, 1))


def _from(a, fmt):
    return a if fmt == D.NCHW else a.transpose(0, 3, 1, 2)


HALF_CASES = [  # N, Cin, H, W, Cout, KH, KW, pad, stride, dtype, x/w/y formats, no workspace
    (4, 64, 28, 28, 128, 3, 3, 1, 1, D.HALF, (D.NHWC, D.NHWC, D.NHWC), True),
    (4, 64, 28, 28, 128, 3, 3, 1, 1, D.BFLOAT16, (D.NHWC, D.NHWC, D.NHWC), True),
    (2, 128, 16, 16, 256, 3, 3, 1, 2, D.HALF, (D.NHWC, D.NHWC, D.NHWC), True),
    (2, 3, 32, 32, 5, 7, 7, 3, 2, D.HALF, (D.NHWC, D.NHWC, D.NHWC), False),
    (2, 24, 17, 15, 16, 3, 3, 1, 1, D.HALF, (D.NCHW, D.NCHW, D.NCHW), False),
    (1, 128, 14, 14, 64, 1, 1, 0, 1, D.HALF, (D.NHWC, D.NCHW, D.NHWC), False),
    (8, 64, 16, 16, 64, 3, 3, 1, 2, D.BFLOAT16, (D.NHWC, D.NHWC, D.NCHW), False),
    (3, 64, 20, 20, 72, 5, 5, 2, 1, D.HALF, (D.NHWC, D.NHWC, D.NHWC), True),
]


@pytest.mark.parametrize("case", HALF_CASES)
def test_conv_16bit_against_oracle(ours, orc, cuda, case):
    N, Cin, H, W, Cout, KH, KW, pad, stride, dtype, (xf, wf, yf), direct = case
    rng = np.random.default_rng(N * Cin + Cout)
    xs = _encode(rng.uniform(-1, 1, (N, Cin, H, W)), dtype)
    ws = _encode(rng.uniform(-1, 1, (Cout, Cin, KH, KW)) * 0.1, dtype)
    xd, wd, cd, yd, (oh, ow) = _descs(ours, dtype, xf, wf, yf, N, Cin, H, W, Cout, KH, KW, pad,
                                      stride)
    st, ws_bytes = ours.workspace(xd, wd, cd, yd)
    assert st == D.SUCCESS and (ws_bytes == 0) == direct, ws_bytes
    y0 = _encode(rng.uniform(-1, 1, (N, Cout, oh, ow)), dtype)
    al, be = 1.5, 0.5
    yt = _dev(_to(y0, yf), cuda)
    assert ours.conv_forward(al, xd, _dev(_to(xs, xf), cuda), wd, _dev(_to(ws, wf), cuda), cd,
                             D.ALGO_IMPLICIT_GEMM, yd, yt, be) == D.SUCCESS
    got = _decode(_from(_host(yt), yf), dtype)
    # oracle: double sums of the decoded operands, NHWC
    xn = _decode(xs, dtype).astype(np.float32).transpose(0, 2, 3, 1)
    wn = _decode(ws, dtype).astype(np.float32).transpose(0, 2, 3, 1)
    conv = orc.conv2d_nhwc(xn, wn, None, stride, pad).reshape(N, oh, ow, Cout).transpose(0, 3, 1, 2)
    want = al * conv.astype(np.float64) + be * _decode(y0, dtype)
    ulp = 2.0 ** (-10 if dtype == D.HALF else -7)
    err = np.abs(got - want)
    assert (err <= ulp * np.abs(want) + 1e-4 * np.abs(want).max()).all(), float(err.max())


def test_conv_16bit_beta_zero_never_reads_y(ours, cuda):
    import torch
    N, Cin, H, W, Cout = 2, 64, 32, 32, 64
    xd, wd, cd, yd, (oh, ow) = _descs(ours, D.HALF, D.NHWC, D.NHWC, D.NHWC, N, Cin, H, W, Cout,
                                      3, 3, 1, 1)
    x = torch.randn(N, H, W, Cin, device=cuda).half()
    w = torch.randn(Cout, 3, 3, Cin, device=cuda).half() * 0.05
    y = torch.full((N, oh, ow, Cout), float("nan"), device=cuda).half()
    assert ours.conv_forward(1.0, xd, x, wd, w, cd, D.ALGO_IMPLICIT_GEMM, yd, y, 0.0) == D.SUCCESS
    want = torch.nn.functional.conv2d(x.double().cpu().permute(0, 3, 1, 2),
                                      w.double().cpu().permute(0, 3, 1, 2), padding=1)
    want = want.permute(0, 2, 3, 1)
    assert not torch.isnan(y).any()
    assert float((y.double().cpu() - want).norm() / want.norm()) < 1e-3


def test_conv_float_nhwc_layouts(ours, theirs, cuda):
    """FLOAT in NHWC (direct f32 epilogue when K % 4 == 0) and mixed layouts
    equal the reference's NCHW result."""
    N, Cin, H, W, Cout, K, pad, stride = 2, 24, 18, 18, 16, 3, 1, 1
    rng = np.random.default_rng(7)
    x = rng.uniform(-1, 1, (N, Cin, H, W)).astype(np.float32)
    w = rng.uniform(-1, 1, (Cout, Cin, K, K)).astype(np.float32)
    y0 = rng.uniform(-1, 1, (N, Cout, H, W)).astype(np.float32)
    xd, wd, cd, yd, _ = _descs(theirs, D.FLOAT, D.NCHW, D.NCHW, D.NCHW, N, Cin, H, W, Cout, K, K,
                               pad, stride)
    want = y0.copy()
    assert theirs.conv_forward(0.75, xd, x, wd, w, cd, 0, yd, want, -1.25) == D.SUCCESS
    for xf, wf, yf in ((D.NHWC, D.NHWC, D.NHWC), (D.NCHW, D.NHWC, D.NHWC), (D.NHWC, D.NCHW, D.NCHW)):
        xd, wd, cd, yd, _ = _descs(ours, D.FLOAT, xf, wf, yf, N, Cin, H, W, Cout, K, K, pad, stride)
        yt = _dev(_to(y0, yf), cuda)
        assert ours.conv_forward(0.75, xd, _dev(_to(x, xf), cuda), wd, _dev(_to(w, wf), cuda), cd, 0,
                                 yd, yt, -1.25) == D.SUCCESS
        got = _from(_host(yt), yf)
        assert float(np.abs(got - want).max()) <= 1e-5 * max(1.0, float(np.abs(want).max()))


def test_conv_refusals(ours, theirs):
    for lib in (ours, theirs):
        xd, wd, cd, yd, _ = _descs(lib, D.FLOAT, D.NCHW, D.NCHW, D.NCHW, 1, 2, 8, 8, 3, 3, 3, 1, 1)
        x = np.zeros((1, 2, 8, 8), np.float32)
        w = np.zeros((3, 2, 3, 3), np.float32)
        y = np.zeros((1, 3, 8, 8), np.float32)
        # mixed element types: NOT_SUPPORTED (test_shims.cpp:327-335)
        hd = lib.tensor(D.NCHW, D.HALF, 1, 2, 8, 8)[0]
        assert lib.conv_forward(2.0, hd, x, wd, w, cd, 0, yd, y, 0.5) == D.NOT_SUPPORTED
        # y of the wrong size, channel mismatch: BAD_PARAM
        bad = lib.tensor(D.NCHW, D.FLOAT, 1, 3, 7, 8)[0]
        assert lib.conv_forward(2.0, xd, x, wd, w, cd, 0, bad, y, 0.5) == D.BAD_PARAM
        bad = lib.tensor(D.NCHW, D.FLOAT, 1, 4, 8, 8)[0]
        assert lib.conv_forward(2.0, bad, x, wd, w, cd, 0, yd, y, 0.5) == D.BAD_PARAM
        # an algorithm outside the list, INT8 / DOUBLE tensors: NOT_SUPPORTED
        assert lib.conv_forward(2.0, xd, x, wd, w, cd, 1, yd, y, 0.5) == D.NOT_SUPPORTED
        for t in (D.INT8, D.DOUBLE):
            td = lib.tensor(D.NCHW, t, 1, 2, 8, 8)[0]
            tw = lib.filter(t, D.NCHW, 3, 2, 3, 3)[0]
            ty = lib.tensor(D.NCHW, t, 1, 3, 8, 8)[0]
            assert lib.conv_forward(2.0, td, x, tw, w, cd, 0, ty, y, 0.5) == D.NOT_SUPPORTED
        # dilation 2: NOT_SUPPORTED at the descriptor (test_shims.cpp:337-339)
        assert lib.conv(1, 1, dil=2)[1] == D.NOT_SUPPORTED


# ------------------------------------------------------------ element-wise

SHAPES = [(2, 3, 4, 5), (4, 32, 17, 9), (1, 7, 64, 64)]


def _pair(lib, fmt, dtype, shape):
    return lib.tensor(fmt, dtype, *shape)[0], lib.tensor(fmt, dtype, *shape)[0]


@pytest.mark.parametrize("shape", SHAPES)
def test_add_tensor_bit_exact(ours, theirs, cuda, shape):
    rng = np.random.default_rng(shape[1])
    A = rng.uniform(-1, 1, shape).astype(np.float32)
    B = rng.uniform(-1, 1, shape).astype(np.float32)
    want = B.copy()
    ad, bd = _pair(theirs, D.NCHW, D.FLOAT, shape)
    assert theirs.add(2.0, ad, A, -1.0, bd, want) == D.SUCCESS
    ad, bd = _pair(ours, D.NCHW, D.FLOAT, shape)
    got = B.copy()
    assert ours.add(2.0, ad, A, -1.0, bd, got) == D.SUCCESS           # host operands
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    gt = _dev(B, cuda)
    assert ours.add(2.0, ad, _dev(A, cuda), -1.0, bd, gt) == D.SUCCESS  # device operands
    assert (_host(gt).view(np.uint32) == want.view(np.uint32)).all()
    # mismatched dims: NOT_SUPPORTED in both (test_shims.cpp:364-370)
    bad = shape[:3] + (shape[3] - 1,)
    for lib in (ours, theirs):
        ad, _ = _pair(lib, D.NCHW, D.FLOAT, shape)
        bd = lib.tensor(D.NCHW, D.FLOAT, *bad)[0]
        assert lib.add(2.0, ad, A, -1.0, bd, B) == D.NOT_SUPPORTED


@pytest.mark.parametrize("fmt", [D.NCHW, D.NHWC])
@pytest.mark.parametrize("dtype", [D.FLOAT, D.HALF, D.BFLOAT16])
def test_add_bias_broadcast(ours, cuda, fmt, dtype):
    N, Cc, H, W = 3, 48, 10, 12
    rng = np.random.default_rng(fmt * 10 + dtype)
    bias = rng.uniform(-1, 1, (1, Cc, 1, 1)).astype(np.float32)
    B = rng.uniform(-1, 1, (N, Cc, H, W)).astype(np.float32)
    if dtype != D.FLOAT:
        bias = _decode(_encode(bias, dtype), dtype).astype(np.float32)
        B = _decode(_encode(B, dtype), dtype).astype(np.float32)
    want = np.float32(1.5) * bias + np.float32(0.5) * B
    ad = ours.tensor(fmt, dtype, 1, Cc, 1, 1)[0]
    bd = ours.tensor(fmt, dtype, N, Cc, H, W)[0]
    enc = (lambda a: a) if dtype == D.FLOAT else (lambda a: _encode(a, dtype))
    bt = _dev(_to(enc(B), fmt), cuda)
    assert ours.add(1.5, ad, _dev(enc(bias), cuda), 0.5, bd, bt) == D.SUCCESS
    got = _from(_host(bt), fmt)
    if dtype == D.FLOAT:
        assert (got == want).all()
    else:
        assert (got == _encode(want, dtype)).all()


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("mode,coef", [(D.RELU, 0.0), (D.CLIPPED_RELU, 6.0), (D.CLIPPED_RELU, 0.0),
                                       (D.SIGMOID, 0.0), (D.TANH, 0.0)])
def test_activation_matches_reference(ours, theirs, cuda, shape, mode, coef):
    rng = np.random.default_rng(shape[2] + mode)
    x = (rng.uniform(-1, 1, shape) * 8).astype(np.float32)
    y0 = rng.uniform(-1, 1, shape).astype(np.float32)
    want = y0.copy()
    xd, yd = _pair(theirs, D.NCHW, D.FLOAT, shape)
    assert theirs.activation(mode, coef, 1.5, xd, x, 0.5, yd, want) == D.SUCCESS
    xd, yd = _pair(ours, D.NCHW, D.FLOAT, shape)
    yt = _dev(y0, cuda)
    assert ours.activation(mode, coef, 1.5, xd, _dev(x, cuda), 0.5, yd, yt) == D.SUCCESS
    got = _host(yt)
    if mode in (D.RELU, D.CLIPPED_RELU):
        assert (got.view(np.uint32) == want.view(np.uint32)).all()
    else:
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=2e-7)


def test_activation_in_place_and_16bit(ours, cuda):
    import torch
    x = torch.randn(4, 16, 8, 8, device=cuda)
    ref = torch.sigmoid(x.clone())
    xd, _ = _pair(ours, D.NCHW, D.FLOAT, (4, 16, 8, 8))
    assert ours.activation(D.SIGMOID, 0.0, 1.0, xd, x, 0.0, xd, x) == D.SUCCESS   # y == x
    assert float((x - ref).abs().max()) < 1e-6
    h = torch.randn(4, 8, 8, 16, device=cuda).half()
    hd, _ = _pair(ours, D.NHWC, D.HALF, (4, 16, 8, 8))
    out = torch.empty_like(h)
    assert ours.activation(D.RELU, 0.0, 1.0, hd, h, 0.0, hd, out) == D.SUCCESS
    assert torch.equal(out, torch.relu(h))


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("algo", [D.SOFTMAX_ACCURATE, D.SOFTMAX_LOG])
@pytest.mark.parametrize("mode", [D.MODE_INSTANCE, D.MODE_CHANNEL])
def test_softmax_matches_reference(ours, theirs, cuda, shape, algo, mode):
    rng = np.random.default_rng(shape[1] + algo * 3 + mode)
    x = (rng.uniform(-1, 1, shape) * 6).astype(np.float32)
    y0 = rng.uniform(-1, 1, shape).astype(np.float32)
    want = y0.copy()
    xd, yd = _pair(theirs, D.NCHW, D.FLOAT, shape)
    assert theirs.softmax(algo, mode, 1.25, xd, x, 0.5, yd, want) == D.SUCCESS
    for fmt in (D.NCHW, D.NHWC):
        xd, yd = _pair(ours, fmt, D.FLOAT, shape)
        yt = _dev(_to(y0, fmt), cuda)
        assert ours.softmax(algo, mode, 1.25, xd, _dev(_to(x, fmt), cuda), 0.5, yd, yt) == D.SUCCESS
        got = _from(_host(yt), fmt)
        if mode == D.MODE_INSTANCE and fmt == D.NHWC:
            continue  # an NHWC instance is the same values in another order: not comparable
        np.testing.assert_allclose(got, want, rtol=3e-7, atol=1e-7)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("fmt", [D.NCHW, D.NHWC])
def test_batchnorm_bit_exact(ours, theirs, cuda, shape, fmt):
    N, Cc, H, W = shape
    rng = np.random.default_rng(Cc + fmt)
    x = rng.uniform(-2, 2, shape).astype(np.float32)
    y0 = rng.uniform(-1, 1, shape).astype(np.float32)
    scale = rng.uniform(0.5, 2, Cc).astype(np.float32)
    bias = rng.uniform(-1, 1, Cc).astype(np.float32)
    mean = rng.uniform(-1, 1, Cc).astype(np.float32)
    var = rng.uniform(0.1, 4, Cc).astype(np.float32)
    want = y0.copy()
    xd, yd = _pair(theirs, D.NCHW, D.FLOAT, shape)
    bnd = theirs.tensor(D.NCHW, D.FLOAT, 1, Cc, 1, 1)[0]
    assert theirs.batchnorm(D.BN_SPATIAL, 1.25, 0.5, xd, x, yd, want, bnd, scale, bias, mean, var,
                            1e-5) == D.SUCCESS
    xd, yd = _pair(ours, fmt, D.FLOAT, shape)
    bnd = ours.tensor(D.NCHW, D.FLOAT, 1, Cc, 1, 1)[0]
    yt = _dev(_to(y0, fmt), cuda)
    assert ours.batchnorm(D.BN_SPATIAL, 1.25, 0.5, xd, _dev(_to(x, fmt), cuda), yd, yt, bnd,
                          _dev(scale, cuda), _dev(bias, cuda), _dev(mean, cuda), _dev(var, cuda),
                          1e-5) == D.SUCCESS
    got = np.ascontiguousarray(_from(_host(yt), fmt))
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    # host operands, and the reference's refusal of a negative epsilon
    got = y0.copy()
    xd, yd = _pair(ours, D.NCHW, D.FLOAT, shape)
    assert ours.batchnorm(D.BN_SPATIAL, 1.25, 0.5, xd, x, yd, got, bnd, scale, bias, mean, var,
                          1e-5) == D.SUCCESS
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    for lib in (ours, theirs):
        xd, yd = _pair(lib, D.NCHW, D.FLOAT, shape)
        bnd = lib.tensor(D.NCHW, D.FLOAT, 1, Cc, 1, 1)[0]
        assert lib.batchnorm(D.BN_SPATIAL, 1.0, 0.0, xd, x, yd, got, bnd, scale, bias, mean, var,
                             -1.0) == D.BAD_PARAM
