"""rouge_conv2d_f32 / rouge_conv_implicit_f32 drop-ins (NCHW f32, conv.cpp:26-66,
conv_implicit.cpp:24-79) on tf32 tensor cores with split operands, against
the oracle's double-accumulated direct convolution and, where the reference
library was built, against the reference's own rouge_conv2d_f32.

Tolerance: relative L2 <= 1e-2 (the north-star bound for float paths) and,
as a kernel-health bound, <= 1e-5: the three tf32 products hi*hi + hi*lo +
lo*hi carry about 2^-21 of relative error per product, the same order as the
reference's own f32 accumulation."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

SHAPES = [
    # N, Cin, H, W, Cout, KH, KW, stride, pad, bias
    (1, 3, 32, 32, 16, 3, 3, 1, 1, True),     # tiny input (padded to 128 KB), Cin 3
    (2, 64, 28, 28, 64, 3, 3, 1, 1, True),
    (2, 16, 17, 19, 30, 5, 5, 2, 2, True),    # stride 2, odd sizes, Cout not a multiple of 4
    (1, 8, 10, 10, 6, 1, 1, 1, 0, True),      # 1x1
    (4, 32, 16, 16, 32, 3, 3, 1, 0, False),   # no padding, no bias
    (2, 40, 9, 7, 300, 3, 3, 1, 1, True),     # Cout over one 256-wide tile
]


def _case(shape, seed):
    N, Cin, H, W, Cout, KH, KW, stride, pad, has_bias = shape
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (N, Cin, H, W)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, KH, KW)) * np.sqrt(2.0 / (Cin * KH * KW))).astype(np.float32)
    b = rng.standard_normal(Cout).astype(np.float32) if has_bias else None
    return x, w, b, stride, pad


def _oracle(orc, x, w, b, stride, pad):
    N = x.shape[0]
    Cout = w.shape[0]
    y = orc.conv2d_nhwc(x.transpose(0, 2, 3, 1), w.transpose(0, 2, 3, 1), b, stride, pad)
    OH = (x.shape[2] + 2 * pad - w.shape[2]) // stride + 1
    OW = (x.shape[3] + 2 * pad - w.shape[3]) // stride + 1
    return y.reshape(N, OH, OW, Cout).transpose(0, 3, 1, 2)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("implicit", [False, True])
def test_conv2d_f32_vs_oracle(rb, orc, cuda, shape, implicit):
    x, w, b, stride, pad = _case(shape, sum(shape[:9]))
    y = rb.host_conv2d_f32(x, w, b, stride, pad, implicit=implicit)
    want = _oracle(orc, x, w, b, stride, pad)
    assert np.isfinite(y).all()
    err = rel_l2(y, want)
    assert err < 1e-2 and err < 1e-5, err


@pytest.mark.parametrize("shape", SHAPES[:3])
def test_conv2d_f32_vs_reference(rb, ref, cuda, shape):
    x, w, b, stride, pad = _case(shape, 7 + shape[1])
    y = rb.host_conv2d_f32(x, w, b, stride, pad)
    want = ref.conv2d_f32(x, w, b, stride, pad)
    err = rel_l2(y, want)
    assert err < 1e-2 and err < 1e-5, err


def test_conv2d_f32_refusals(rb, cuda):
    L = rb.lib()
    x = np.ones((1, 3, 8, 8), np.float32)
    w = np.ones((4, 3, 3, 3), np.float32)
    y = np.full((1, 4, 6, 6), 7.0, np.float32)
    p = lambda a: a.ctypes.data_as(rb.C.c_void_p)  # noqa: E731
    # NULL or invalid sizes: no-op (conv.cpp:30-36)
    L.rouge_conv2d_f32(1, 3, 8, 8, 4, 3, 3, 1, 0, None, p(w), None, p(y), None)
    L.rouge_conv2d_f32(1, 3, 8, 8, 4, 3, 3, 0, 0, p(x), p(w), None, p(y), None)
    L.rouge_conv2d_f32(1, 3, 2, 2, 4, 3, 3, 1, 0, p(x), p(w), None, p(y), None)   # OH <= 0
    assert (y == 7.0).all()
    # stride beyond the im2col tensor map's limit: no-op, EUNSUPPORTED
    L.rouge_b200_clear_error()
    L.rouge_conv2d_f32(1, 3, 8, 8, 4, 3, 3, 9, 0, p(x), p(w), None, p(y), None)
    assert (y == 7.0).all()
    assert L.rouge_b200_last_error() == rb.EUNSUPPORTED
    L.rouge_b200_clear_error()
