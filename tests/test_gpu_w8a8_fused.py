"""The W8A8 linear step in one launch (rouge_b200_w8a8_linear): per-row int8
quantization of the activations fused into the CTA-pair int8 GEMM. Its
codes, scales and output must equal, bit for bit, those of the two calls it
replaces (rouge_b200_quantize_i8_rows, then rouge_b200_gemm_i8 with per-row
and per-column scales), which the other tests pin to the oracle; sampled
rows are also checked against the oracle directly. Cases: the BASELINE
config-2 shape, ragged M and N, short K, special values (NaN, +-Inf, zero
and subnormal rows), each output type, shapes whose last round of tiles is
cut N-wise (more tiles than the 74 CTA pairs, not a multiple of them),
repeated calls on one workspace (left zeroed every time), one workspace
used for several M, and the two-launch path for K > 4096."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _x(rng, M, K, special=True):
    x = (rng.standard_normal((M, K)) * rng.choice([1e-3, 1.0, 40.0], (M, 1))).astype(np.float32)
    if special and M >= 8:
        x[1, :] = 0.0                                          # all-zero row: scale 1
        x[2, :] = np.float32(1e-41)                            # subnormal row
        x[3, 5], x[3, 9], x[3, 11] = np.nan, np.inf, -np.inf   # non-finite elements
        x[4, :] = np.float32(3e38) * np.sign(x[4, :])           # huge row
        x[5, ::7] = 127.5 * x[5, 0] / 127.0                    # values near rounding ties
    return x


def _two_calls(rb, torch, xd, wq, sw, out_type, cuda):
    M, K = xd.shape
    N = wq.shape[0]
    aq = torch.empty((M, K), dtype=torch.int8, device=cuda)
    sa = torch.empty(M, dtype=torch.float32, device=cuda)
    rb.quantize_i8_rows(xd, sa, aq)
    dt = {rb.OUT_F32: torch.float32, rb.OUT_BF16: torch.int16, rb.OUT_I32: torch.int32}[out_type]
    c = torch.empty((M, N), dtype=dt, device=cuda)
    if out_type == rb.OUT_I32:
        rb.gemm_i8(aq, wq, rb.B_NK, c, out_type)
    else:
        rb.gemm_i8(aq, wq, rb.B_NK, c, out_type, sa, 1, sw, 1)
    return aq, sa, c


def _fused(rb, torch, xd, wq, sw, out_type, ws, cuda):
    M, K = xd.shape
    N = wq.shape[0]
    aq = torch.full((M, K), 99, dtype=torch.int8, device=cuda)
    sa = torch.full((M,), -1.0, dtype=torch.float32, device=cuda)
    dt = {rb.OUT_F32: torch.float32, rb.OUT_BF16: torch.int16, rb.OUT_I32: torch.int32}[out_type]
    c = torch.full((M, N), 7, dtype=dt, device=cuda)
    rb.w8a8_linear(xd, wq, sw, aq, sa, c, out_type, ws)
    return aq, sa, c


def _bits(t):
    import torch
    a = t.cpu()
    if a.dtype == torch.float32:
        a = a.view(torch.int32)
    return a.numpy()


def _weights(rb, torch, rng, N, K, cuda):
    w = rng.standard_normal((N, K)).astype(np.float32)
    wd = torch.from_numpy(w).to(cuda)
    wq = torch.empty((N, K), dtype=torch.int8, device=cuda)
    sw = torch.empty(N, dtype=torch.float32, device=cuda)
    rb.quantize_i8_rows(wd, sw, wq)
    return wq, sw


@pytest.mark.parametrize("M,N,K,pair", [(4096, 4096, 4096, False), (1000, 1000, 1024, True),
                                        (384, 512, 48, True), (260, 256, 4096, True),
                                        (128, 4096, 256, True), (1, 272, 16, True),
                                        (129, 300, 2064, True), (8192, 2048, 1024, False),
                                        (2560, 4096, 4096, True), (4100, 4096, 1024, True),
                                        (4352, 2816, 384, True), (4096, 4096, 16, True)])
def test_fused_equals_two_calls(rb, orc, cuda, M, N, K, pair):
    import torch
    rng = np.random.default_rng(M * 7 + N + K)
    xd = torch.from_numpy(_x(rng, M, K)).to(cuda)
    wq, sw = _weights(rb, torch, rng, N, K, cuda)
    ws = rb.w8a8_workspace(M, cuda)
    with rb.tile_mode(rb.TILES_PAIR if pair else rb.TILES_AUTO):
        for out_type in (rb.OUT_F32, rb.OUT_BF16, rb.OUT_I32):
            want = _two_calls(rb, torch, xd, wq, sw, out_type, cuda)
            got = _fused(rb, torch, xd, wq, sw, out_type, ws, cuda)
            rb.sync_status()
            for g, w in zip(got, want):
                assert (_bits(g) == _bits(w)).all()
            assert int(ws.abs().sum()) == 0          # the workspace is left zeroed
    # sampled rows against the oracle itself
    rows = np.unique(np.r_[0:6, rng.integers(0, M, 10)])
    rows = rows[rows < M]
    x = xd.cpu().numpy()
    oq, os_ = orc.quantize_i8_rows(x[rows])
    aq, sa, c = got[0], got[1], None
    assert (aq.cpu().numpy()[rows] == oq).all()
    assert (sa.cpu().numpy()[rows].view(np.uint32) == os_.view(np.uint32)).all()
    with rb.tile_mode(rb.TILES_PAIR if pair else rb.TILES_AUTO):
        c = _fused(rb, torch, xd, wq, sw, rb.OUT_F32, ws, cuda)[2]
    rb.sync_status()
    _, oc = orc.gemm_i8(oq, wq.cpu().numpy(), True, os_, 1, sw.cpu().numpy(), 1)
    assert (c.cpu().numpy()[rows].view(np.uint32) == oc.view(np.uint32)).all()


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (4096, 4096, 512)])
def test_repeated_calls_one_workspace(rb, cuda, M, N, K):
    """Back-to-back launches on one stream reuse the workspace: each must
    see it zeroed by the previous one, with inputs that change every call."""
    import torch
    rng = np.random.default_rng(3)
    wq, sw = _weights(rb, torch, rng, N, K, cuda)
    ws = rb.w8a8_workspace(M, cuda)
    xs = [torch.from_numpy(_x(rng, M, K, special=False)).to(cuda) for _ in range(3)]
    with rb.tile_mode(rb.TILES_PAIR):
        outs = []
        for i in range(9):
            outs.append(_fused(rb, torch, xs[i % 3], wq, sw, rb.OUT_F32, ws, cuda))
        rb.sync_status()
        for i in range(3):
            want = _two_calls(rb, torch, xs[i], wq, sw, rb.OUT_F32, cuda)
            for j in (i, i + 3, i + 6):
                for g, w in zip(outs[j], want):
                    assert (_bits(g) == _bits(w)).all()
    assert int(ws.abs().sum()) == 0


def test_one_workspace_for_several_m(rb, cuda):
    """A workspace sized for the largest M serves calls of smaller M in any
    order: each call leaves the counts it used zeroed."""
    import torch
    N, K = 4096, 1024
    rng = np.random.default_rng(5)
    wq, sw = _weights(rb, torch, rng, N, K, cuda)
    ws = rb.w8a8_workspace(8192, cuda)
    with rb.tile_mode(rb.TILES_PAIR):
        for M in (8192, 2560, 4096, 384, 8192, 4352):
            xd = torch.from_numpy(_x(rng, M, K, special=False)).to(cuda)
            got = _fused(rb, torch, xd, wq, sw, rb.OUT_F32, ws, cuda)
            want = _two_calls(rb, torch, xd, wq, sw, rb.OUT_F32, cuda)
            rb.sync_status()
            for g, w in zip(got, want):
                assert (_bits(g) == _bits(w)).all()
            assert int(ws.abs().sum()) == 0


def test_long_rows_take_two_launches(rb, cuda):
    import torch
    M, N, K = 512, 512, 8192
    rng = np.random.default_rng(9)
    xd = torch.from_numpy(_x(rng, M, K)).to(cuda)
    wq, sw = _weights(rb, torch, rng, N, K, cuda)
    ws = rb.w8a8_workspace(M, cuda)
    with rb.tile_mode(rb.TILES_PAIR):
        want = _two_calls(rb, torch, xd, wq, sw, rb.OUT_F32, cuda)
        got = _fused(rb, torch, xd, wq, sw, rb.OUT_F32, ws, cuda)
    rb.sync_status()
    for g, w in zip(got, want):
        assert (_bits(g) == _bits(w)).all()


def test_arguments(rb, cuda):
    import ctypes as C
    import torch
    L = rb.lib()
    x = torch.zeros((256, 64), device=cuda)
    wq = torch.zeros((256, 64), dtype=torch.int8, device=cuda)
    sw = torch.ones(256, device=cuda)
    aq = torch.zeros((256, 64), dtype=torch.int8, device=cuda)
    sa = torch.zeros(256, device=cuda)
    c = torch.zeros((256, 256), device=cuda)
    ws = rb.w8a8_workspace(256, cuda)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    assert L.rouge_b200_w8a8_workspace_bytes(256) == 16 and L.rouge_b200_w8a8_workspace_bytes(0) == 0
    args = [256, 256, 64, P(x), P(wq), P(sw), P(aq), P(sa), P(c), 256, rb.OUT_F32, P(ws), None]
    bad = list(args)
    bad[11] = None                                     # no workspace
    assert L.rouge_b200_w8a8_linear(*bad) == rb.EINVAL
    bad = list(args)
    bad[2] = 40                                        # K % 16 != 0
    assert L.rouge_b200_w8a8_linear(*bad) == rb.EUNSUPPORTED
    assert L.rouge_b200_w8a8_linear(*args) == rb.OK
    assert L.rouge_b200_sync_status(None) == rb.OK
