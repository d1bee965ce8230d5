"""MX / NVFP4 block quantizers on the GPU (narrow.cpp:200-331), bit-exact
against the oracle (codes, scales, decoded values with their NaN bits) and,
through the host drop-in entries, against the reference library itself.
Cases: full and partial last blocks, unaligned operands (the scalar path),
special values (NaN, +-Inf, zeros, f32 subnormals, values at the format
edges), global scales of NVFP4 including the refused ones, 64 M elements."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FMT = {"e4m3": 0, "e5m2": 1, "e2m1": 4}


def _data(rng, n):
    x = (rng.standard_normal(n) * rng.choice([1e-3, 1.0, 50.0, 3e4], n)).astype(np.float32)
    k = min(n, 4096)
    spec = np.array([np.nan, -np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, -1e-42, 448.0, -464.0,
                     480.0, 57344.0, 61440.0, 6.0, -0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0,
                     1e38, -3e38], np.float32)
    idx = rng.choice(k, size=min(k, 512), replace=False)
    x[idx] = rng.choice(spec, idx.size)
    if n >= 96:
        x[32:64] = 0.0                              # all-zero block
        x[64:96] = np.float32(1e-39)                # block of subnormals
    return x


def _same_bits(a, b):
    return bool((np.asarray(a).view(np.uint32) == np.asarray(b).view(np.uint32)).all())


def _eq(got, want, x=None):
    """Array equality with the first mismatches in the failure message."""
    bad = np.nonzero(got != want)[0]
    if bad.size:
        rows = [(int(i), None if x is None else float(x[i]) if i < x.size else None,
                 int(got[i]), int(want[i])) for i in bad[:8]]
        raise AssertionError(f"{bad.size} mismatches (index, x, got, want): {rows}")


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m1"])
@pytest.mark.parametrize("n,offset", [(32, 0), (4096, 0), (1000, 0), (4099, 0), (777, 1),
                                      (1 << 20, 0), (1 << 20, 3)])
def test_mx_quantize_bit_exact(rb, orc, cuda, fmt, n, offset):
    import torch
    rng = np.random.default_rng(n + offset + FMT[fmt])
    x = _data(rng, n)
    buf = torch.zeros(n + 8, dtype=torch.float32, device=cuda)
    buf[offset:offset + n] = torch.from_numpy(x).to(cuda)
    xd = buf[offset:offset + n]
    qb = torch.full((n + 8,), 0xAA, dtype=torch.uint8, device=cuda)
    q = qb[offset:offset + n]
    s = torch.full(((n + 31) // 32,), 0xAA, dtype=torch.uint8, device=cuda)
    rb.mx_quantize(xd, FMT[fmt], q, s)
    wq, ws = orc.mx_quantize(x, fmt)
    _eq(q.cpu().numpy(), wq, x)
    _eq(s.cpu().numpy(), ws)
    assert (qb[:offset].cpu().numpy() == 0xAA).all() and (qb[offset + n:].cpu().numpy() == 0xAA).all()
    out = torch.empty(n, dtype=torch.float32, device=cuda)
    rb.mx_dequantize(q, s, FMT[fmt], out)
    assert _same_bits(out.cpu().numpy(), orc.mx_dequantize(wq, ws, fmt))


@pytest.mark.parametrize("gs", [1.0, 0.37, 12.0, 0.0, -1.0])
@pytest.mark.parametrize("n", [16, 1000, 1 << 20])
def test_nvfp4_quantize_bit_exact(rb, orc, cuda, gs, n):
    import torch
    rng = np.random.default_rng(n)
    x = _data(rng, n)
    q = torch.empty(n, dtype=torch.uint8, device=cuda)
    s = torch.empty((n + 15) // 16, dtype=torch.uint8, device=cuda)
    rb.nvfp4_quantize(torch.from_numpy(x).to(cuda), gs, q, s)
    wq, ws = orc.nvfp4_quantize(x, gs)
    _eq(q.cpu().numpy(), wq, x)
    _eq(s.cpu().numpy(), ws)


def test_full_size_block_quantizers(rb, orc, cuda):
    """64 M elements (256 MB of f32, larger than L2), whole arrays compared."""
    import torch
    n = 64 << 20
    xt = torch.randn(n, device=cuda) * 3
    x = xt.cpu().numpy()
    q = torch.empty(n, dtype=torch.uint8, device=cuda)
    s = torch.empty(n // 32, dtype=torch.uint8, device=cuda)
    for fmt in ("e4m3", "e2m1"):
        rb.mx_quantize(xt, FMT[fmt], q, s)
        wq, ws = orc.mx_quantize(x, fmt)
        assert (q.cpu().numpy() == wq).all() and (s.cpu().numpy() == ws).all()


def test_host_drop_ins_match_reference(rb, ref, cuda):
    L = rb.lib()
    rng = np.random.default_rng(0x4D58)
    P = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    for n in (31, 32, 96, 4097, 100000):
        x = _data(rng, n)
        for eb, fmt in ((1, "e4m3"), (2, "e5m2")):
            q = np.empty(n, np.uint8)
            s = np.empty((n + 31) // 32, np.uint8)
            assert L.rouge_mx_quantize_f32(P(x), n, eb, P(q), P(s)) == s.size
            rq, rs = ref.mx_quantize(x, fmt)
            assert (q == rq).all() and (s == rs).all()
            back = np.empty(n, np.float32)
            L.rouge_mx_dequantize_f32(P(q), P(s), n, eb, P(back))
            assert _same_bits(back, ref.mx_dequantize(rq, rs, fmt))
        q = np.empty(n, np.uint8)
        s = np.empty((n + 31) // 32, np.uint8)
        assert L.rouge_mx_quantize_f32_e2m1(P(x), n, P(q), P(s)) == s.size
        rq, rs = ref.mx_quantize(x, "e2m1")
        assert (q == rq).all() and (s == rs).all()
        back = np.empty(n, np.float32)
        L.rouge_mx_dequantize_f32_e2m1(P(q), P(s), n, P(back))
        assert _same_bits(back, ref.mx_dequantize(rq, rs, "e2m1"))
        for gs in (1.0, 0.5, -3.0):
            q = np.empty(n, np.uint8)
            s = np.empty((n + 15) // 16, np.uint8)
            assert L.rouge_nvfp4_quantize_f32(P(x), n, gs, P(q), P(s)) == s.size
            rq, rs = ref.nvfp4_quantize(x, gs)
            assert (q == rq).all() and (s == rs).all()
    # invalid arguments: 0 and nothing written (narrow.cpp:202-204)
    x = np.ones(64, np.float32)
    q = np.full(64, 7, np.uint8)
    s = np.full(2, 7, np.uint8)
    assert L.rouge_mx_quantize_f32(P(x), 64, 3, P(q), P(s)) == 0
    assert L.rouge_mx_quantize_f32(P(x), 0, 1, P(q), P(s)) == 0
    assert L.rouge_nvfp4_quantize_f32(None, 64, 1.0, P(q), P(s)) == 0
    assert (q == 7).all() and (s == 7).all()


@pytest.mark.parametrize("gs", [1.0, 0.37, -2.0])
def test_nvfp4_packed_equals_codes_packed(rb, orc, cuda, gs):
    import torch
    n = 1 << 20
    x = _data(np.random.default_rng(5), n)
    xd = torch.from_numpy(x).to(cuda)
    p = torch.empty(n // 2, dtype=torch.uint8, device=cuda)
    s = torch.empty(n // 16, dtype=torch.uint8, device=cuda)
    rb.nvfp4_quantize_packed(xd, gs, p, s)
    wq, ws = orc.nvfp4_quantize(x, gs)
    _eq(s.cpu().numpy(), ws)
    _eq(p.cpu().numpy(), (wq[0::2] | (wq[1::2] << 4)).astype(np.uint8))
