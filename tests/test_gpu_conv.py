"""Implicit-GEMM convolution (NHWC f16/bf16, f32 accumulation, fused bias) on
tcgen05 against the oracle's direct convolution (double accumulation) —
the same arithmetic as the reference's im2col + f32 GEMM conv
(conv.cpp:26-66) on the decoded inputs. Tolerance: relative L2 <= 1e-2 (the
north-star bound) and, as a kernel-health bound, <= 1e-4 (f16 products are
exact in f32; only the summation order differs)."""
import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def run_conv(rb, orc, cuda, N, H, W, Cin, Cout, KH, KW, stride, pad, bias=True, bf16=False,
             seed=0, pixels=None):
    rng = np.random.default_rng(seed)
    enc = orc.bf16_encode if bf16 else orc.f16_encode
    dec = orc.bf16_decode if bf16 else orc.f16_decode
    x = enc(rng.uniform(-1, 1, (N, H, W, Cin)).astype(np.float32))
    w = enc((rng.standard_normal((Cout, KH, KW, Cin)) * np.sqrt(2.0 / (KH * KW * Cin))).astype(np.float32))
    b = rng.standard_normal(Cout).astype(np.float32) if bias else None
    OH = (H + 2 * pad - KH) // stride + 1
    OW = (W + 2 * pad - KW) // stride + 1
    y = torch.full((N, OH, OW, Cout), float("nan"), dtype=torch.float32, device=cuda)
    bd = torch.from_numpy(b).to(cuda) if bias else None
    rb.conv2d_nhwc_f16(torch.from_numpy(x.view(np.int16)).to(cuda),
                       torch.from_numpy(w.view(np.int16)).to(cuda), bd, y, stride, pad, is_bf16=bf16)
    rb.sync_status()
    got = y.cpu().numpy().reshape(-1, Cout)
    xf, wf = dec(x), dec(w)
    if pixels is None:
        want = orc.conv2d_nhwc(xf, wf, b, stride, pad)
        return got, want
    wants, gots = [], []
    for p0, p1 in pixels:
        wants.append(orc.conv2d_nhwc(xf, wf, b, stride, pad, p0, p1))
        gots.append(got[p0:p1])
    return np.concatenate(gots), np.concatenate(wants)


@pytest.mark.parametrize("shape", [
    # N, H, W, Cin, Cout, KH, KW, stride, pad
    (4, 16, 16, 64, 64, 3, 3, 1, 1),
    (4, 14, 14, 128, 96, 3, 3, 1, 1),      # Cout not a tile multiple
    (4, 20, 20, 64, 128, 3, 3, 2, 1),      # stride 2
    (2, 28, 28, 128, 64, 1, 1, 1, 0),      # 1x1
    (4, 16, 16, 64, 64, 5, 5, 1, 2),       # 5x5, pad 2
    (4, 9, 11, 192, 256, 3, 3, 1, 0),      # no padding, odd spatial sizes
])
def test_conv_vs_oracle(rb, orc, cuda, shape):
    got, want = run_conv(rb, orc, cuda, *shape)
    assert np.isfinite(got).all()
    err = rel_l2(got, want)
    assert err < 1e-2 and err < 1e-4, err


def test_conv_bf16_no_bias(rb, orc, cuda):
    got, want = run_conv(rb, orc, cuda, 8, 12, 12, 64, 64, 3, 3, 1, 1, bias=False, bf16=True, seed=3)
    err = rel_l2(got, want)
    assert err < 1e-2 and err < 1e-4, err


def test_conv_config4_sampled(rb, orc, cuda):
    # BASELINE config 4 at full size: N=32, 56x56, 256 -> 256, 3x3, s1 p1.
    # Output pixels checked: the first and last image's borders and corners
    # (where padding is exercised), tile boundaries and rows crossing images.
    OHW = 56 * 56
    pix = [(0, 200), (OHW - 60, OHW + 60), (5 * OHW + 1000, 5 * OHW + 1130),
           (31 * OHW - 56, 31 * OHW), (32 * OHW - 130, 32 * OHW)]
    got, want = run_conv(rb, orc, cuda, 32, 56, 56, 256, 256, 3, 3, 1, 1, seed=5, pixels=pix)
    err = rel_l2(got, want)
    assert err < 1e-2 and err < 1e-4, err


def test_conv_rejects_unsupported(rb, cuda):
    x = torch.zeros((4, 16, 16, 48), dtype=torch.int16, device=cuda)   # Cin % 64 != 0
    w = torch.zeros((64, 3, 3, 48), dtype=torch.int16, device=cuda)
    y = torch.zeros((4, 16, 16, 64), dtype=torch.float32, device=cuda)
    with pytest.raises(rb.RougeB200Error) as e:
        rb.conv2d_nhwc_f16(x, w, None, y, 1, 1)
    assert e.value.status == rb.EUNSUPPORTED
