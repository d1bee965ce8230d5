"""Attention and the transformer block (the GEMM's in-library consumers) on
the GPU against the reference's own code (attention.cpp, attention_gqa.cpp,
transformer.cpp compiled from its sources into oracle/_ref), same host
arrays through the same entry points. The reference sums scores in double
and accumulates in float; ours runs scores and weighted sums on the tf32
tensor cores with split operands (f32-accurate): outputs agree to 1e-5 of
the output scale (the reference test's own bound against a double
reference, test_ai.cpp:185-206)."""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "librouge_ref_shims.so")
_P, _I, _F = C.c_void_p, C.c_int, C.c_float
SIGS = {
    "rouge_attention_f32": [_I, _I, _I, _P, _P, _P, _P, _F, _I, _I],
    "rouge_attention_gqa": [_I, _I, _I, _I, _I, _P, _P, _P, _P, _F, _I, _I, _I],
    "rouge_attention_gqa_fp8kv": [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _F, _I, _I, _I],
    "rouge_rmsnorm": [_P, _I, _P, _F, _P],
    "rouge_rope": [_P, _I, _I, _I, _F],
    "rouge_swiglu": [_P, _P, _I, _P],
    "rouge_transformer_block": [_I] * 6 + [_P] * 10 + [_I, _F, _F, _P],
}


def _bind(lib):
    for n, a in SIGS.items():
        getattr(lib, n).argtypes = a
        getattr(lib, n).restype = None
    return lib


@pytest.fixture(scope="module")
def libs(rb, cuda):
    if not os.path.exists(REF):
        pytest.skip("reference shims library not built")
    return _bind(rb.lib()), _bind(C.CDLL(REF))


def p(a):
    return a.ctypes.data_as(_P)


def _close(got, want, tol=1e-5):
    err = float(np.abs(got.astype(np.float64) - want).max())
    scale = max(1.0, float(np.abs(want).max()))
    assert err <= tol * scale, (err, scale)


@pytest.mark.parametrize("causal,window", [(0, 0), (1, 0), (0, 4), (1, 4)])
def test_gqa_reference_test_shape(libs, causal, window):
    ours, ref = libs
    S, Skv, Dh, Hq, Hkv = 12, 12, 8, 4, 2                 # test_ai.cpp:185-206
    rng = np.random.default_rng(causal * 2 + window)
    Q = rng.uniform(-1, 1, (Hq, S, Dh)).astype(np.float32)
    K = rng.uniform(-1, 1, (Hkv, Skv, Dh)).astype(np.float32)
    V = rng.uniform(-1, 1, (Hkv, Skv, Dh)).astype(np.float32)
    outs = []
    for lib in (ours, ref):
        O = np.full((Hq, S, Dh), np.nan, np.float32)
        lib.rouge_attention_gqa(S, Skv, Dh, Hq, Hkv, p(Q), p(K), p(V), p(O), 0.0, causal, window, 0)
        outs.append(O)
    _close(outs[0], outs[1])


@pytest.mark.parametrize("S,Skv,Dh,Hq,Hkv,causal,window,kv_off", [
    (512, 512, 64, 8, 2, 1, 0, 0),        # bench_ai.cpp:73-84
    (100, 300, 64, 4, 4, 1, 0, 200),      # decode-like: a prefix of 200 cached keys
    (257, 257, 128, 4, 1, 1, 32, 0),      # MQA, sliding window
    (64, 1000, 40, 6, 3, 0, 0, 0),        # odd head size, no mask
    # every group in one batched launch (group * S a multiple of 256) with
    # ragged key counts: the last key tile reads the next head's rows
    (256, 300, 64, 8, 2, 1, 0, 44),
    (128, 200, 40, 4, 2, 0, 8, 0),
])
def test_gqa_shapes(libs, S, Skv, Dh, Hq, Hkv, causal, window, kv_off):
    ours, ref = libs
    rng = np.random.default_rng(S + Skv)
    Q = rng.standard_normal((Hq, S, Dh)).astype(np.float32)
    K = rng.standard_normal((Hkv, Skv, Dh)).astype(np.float32)
    V = rng.standard_normal((Hkv, Skv, Dh)).astype(np.float32)
    outs = []
    for lib in (ours, ref):
        O = np.full((Hq, S, Dh), np.nan, np.float32)
        lib.rouge_attention_gqa(S, Skv, Dh, Hq, Hkv, p(Q), p(K), p(V), p(O), 0.0, causal, window,
                                kv_off)
        outs.append(O)
    _close(outs[0], outs[1])


def test_fp8kv_and_mha(libs):
    ours, ref = libs
    rng = np.random.default_rng(7)
    for S, Skv, Dh, Hq, Hkv in ((10, 10, 16, 4, 4), (200, 333, 64, 8, 2)):  # test_ai.cpp:209-246
        Q = rng.uniform(-1, 1, (Hq, S, Dh)).astype(np.float32)
        Kq = rng.integers(0, 256, (Hkv, Skv, Dh), dtype=np.uint8)
        Vq = rng.integers(0, 256, (Hkv, Skv, Dh), dtype=np.uint8)
        Kq[(Kq & 0x7F) == 0x7F] = 0x38                     # no NaN codes in the cache
        Vq[(Vq & 0x7F) == 0x7F] = 0x38
        sk = rng.uniform(0.001, 0.01, Hkv).astype(np.float32)
        sv = rng.uniform(0.001, 0.01, Hkv).astype(np.float32)
        outs = []
        for lib in (ours, ref):
            O = np.full((Hq, S, Dh), np.nan, np.float32)
            lib.rouge_attention_gqa_fp8kv(S, Skv, Dh, Hq, Hkv, p(Q), p(Kq), p(Vq), p(sk), p(sv),
                                          p(O), 0.0, 1, 0, 0)
            outs.append(O)
        _close(outs[0], outs[1])
    for S, Skv, D, causal, kv_off in ((33, 70, 24, 1, 37), (512, 512, 64, 1, 0)):
        Q = rng.standard_normal((S, D)).astype(np.float32)
        K = rng.standard_normal((Skv, D)).astype(np.float32)
        V = rng.standard_normal((Skv, D)).astype(np.float32)
        outs = []
        for lib in (ours, ref):
            O = np.full((S, D), np.nan, np.float32)
            lib.rouge_attention_f32(S, Skv, D, p(Q), p(K), p(V), p(O), 0.5, causal, kv_off)
            outs.append(O)
        _close(outs[0], outs[1])


def test_vector_helpers(libs):
    ours, ref = libs
    rng = np.random.default_rng(3)
    x = rng.standard_normal(4096).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 4096).astype(np.float32)
    a, b = np.empty_like(x), np.empty_like(x)
    ours.rouge_rmsnorm(p(x), 4096, p(w), 1e-5, p(a))
    ref.rouge_rmsnorm(p(x), 4096, p(w), 1e-5, p(b))
    np.testing.assert_allclose(a, b, rtol=2e-7, atol=0)
    r1 = rng.standard_normal((8, 64)).astype(np.float32)
    r2 = r1.copy()
    ours.rouge_rope(p(r1), 8, 64, 1234, 10000.0)
    ref.rouge_rope(p(r2), 8, 64, 1234, 10000.0)
    np.testing.assert_allclose(r1, r2, rtol=1e-6, atol=1e-6)
    g = (rng.standard_normal(4096) * 4).astype(np.float32)
    u = rng.standard_normal(4096).astype(np.float32)
    ours.rouge_swiglu(p(g), p(u), 4096, p(a))
    ref.rouge_swiglu(p(g), p(u), 4096, p(b))
    np.testing.assert_allclose(a, b, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("S,D,Hq,Hkv,Dq,Dff,wscale", [
    (6, 16, 2, 1, 8, 24, 0.1),             # test_ai.cpp:249-280
    (256, 512, 8, 2, 64, 1376, 0.05),      # bench_ai.cpp:100-126
])
def test_transformer_block(libs, S, D, Hq, Hkv, Dq, Dff, wscale):
    ours, ref = libs
    rng = np.random.default_rng(S + D)
    f = lambda *sh: (rng.standard_normal(sh) * wscale).astype(np.float32)  # noqa: E731
    x = rng.standard_normal((S, D)).astype(np.float32)
    w1 = rng.uniform(0.5, 0.7, D).astype(np.float32)
    w2 = rng.uniform(0.5, 0.7, D).astype(np.float32)
    wq, wk, wv, wo = f(D, Hq * Dq), f(D, Hkv * Dq), f(D, Hkv * Dq), f(Hq * Dq, D)
    wg, wu, wd = f(D, Dff), f(D, Dff), f(Dff, D)
    outs = []
    for lib in (ours, ref):
        out = np.full((S, D), np.nan, np.float32)
        lib.rouge_transformer_block(S, D, Hq, Hkv, Dq, Dq, p(x), p(w1), p(wq), p(wk), p(wv), p(wo),
                                    p(w2), p(wg), p(wu), p(wd), Dff, 10000.0, 1e-5, p(out))
        outs.append(out)
    _close(outs[0], outs[1], 2e-5)
