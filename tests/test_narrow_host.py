"""Host-side narrow-format codecs of librouge_b200.so (rouge_quantize_e5m2,
..., rouge_dequantize_e2m1: the drop-ins of numerics.h:257-264) against the
reference library on every code and ~4 M f32 bit patterns, without a GPU."""
import numpy as np
import pytest

FMTS = ["e5m2", "e3m2", "e2m3", "e2m1"]
WIDTH = {"e5m2": 8, "e3m2": 6, "e2m3": 6, "e2m1": 4}


@pytest.mark.parametrize("fmt", FMTS)
def test_scalar_codecs_match_reference(rb, ref, fmt):
    L = rb.lib()
    enc = getattr(L, f"rouge_quantize_{fmt}")
    dec = getattr(L, f"rouge_dequantize_{fmt}")
    codes = np.arange(1 << WIDTH[fmt], dtype=np.uint8)
    got = np.array([dec(int(c)) for c in codes], np.float32)
    want = ref.narrow_decode(codes, fmt)
    nan = np.isnan(want)
    assert (np.isnan(got) == nan).all() and (got[~nan].view(np.uint32) == want[~nan].view(np.uint32)).all()
    u = np.arange(0, 1 << 32, 65537 * 13, dtype=np.uint64).astype(np.uint32)
    special = np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0x3E800000,
                        0xBE800000, 0x47700000, 0x43E80000, 0x00000001], np.uint32)
    x = np.concatenate([u, special]).view(np.float32)
    got = np.array([enc(float(v)) for v in x.tolist()], np.uint8)
    assert (got == ref.narrow_encode(x, fmt)).all()
