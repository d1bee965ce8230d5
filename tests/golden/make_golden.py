"""Generate tests/golden/golden.npz from the reference rouge-numerics library.

Runs the unmodified reference functions, compiled from their own sources by
oracle/Makefile into oracle/_ref/librouge_ref.so, on small seeded and
hand-picked inputs, and stores inputs and outputs. The fixtures pin both
the oracle restatement (oracle/rouge_oracle.c) and the GPU kernels without
needing the reference at test time.

    python tests/golden/make_golden.py        # needs oracle/_ref built
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402


def special_floats() -> np.ndarray:
    """Float bit patterns around every rounding / range boundary of the
    f16, bf16 and e4m3 encoders, plus seeded random values."""
    rng = np.random.default_rng(20260101)
    vals = [0.0, -0.0, 1.0, -1.0, 0.5, 448.0, 464.0, 463.99, 480.0, 1000.0, -1000.0,
            65504.0, 65520.0, 65519.99, 1e5, -1e5, np.inf, -np.inf, np.nan,
            2.0 ** -10, -(2.0 ** -10), 2.0 ** -9, -(2.0 ** -9), 2.0 ** -11, 1.5 * 2.0 ** -10,
            2.0 ** -14, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26, 6.1032e-5, -6.1032e-5,
            2.0 ** -6, 2.0 ** -7, 0.875 * 2.0 ** -6, 0.9375 * 2.0 ** -6, 1e-45, 3e38, -3e38]
    bits = np.array(vals, dtype=np.float32).view(np.uint32)
    # Every boundary above +-1 ulp.
    around = np.concatenate([bits - 1, bits, bits + 1]).astype(np.uint32)
    # Near-tie patterns for e4m3 (3 mantissa bits) and f16 (10 bits) roundings.
    ties = []
    for e in range(100, 140):
        for m in (0x080000, 0x07FFFF, 0x080001, 0x180000, 0x001000, 0x003000, 0x000FFF, 0x001001):
            ties.append((e << 23) | m)
            ties.append((1 << 31) | (e << 23) | m)
    rand = np.concatenate([
        rng.standard_normal(2000).astype(np.float32).view(np.uint32),
        (rng.standard_normal(1000) * 1e-3).astype(np.float32).view(np.uint32),
        rng.integers(0, 2 ** 32, 2000, dtype=np.uint64).astype(np.uint32),
    ])
    allb = np.concatenate([around, np.array(ties, np.uint32), rand])
    return allb.view(np.float32)


def main() -> None:
    if not O.Reference.available():
        O.build()
    R = O.Reference()
    out = {}

    # --- formats (fp8.cpp:42-114, fp16.cpp:31-121) ---
    f = special_floats()
    out["fmt_x"] = f
    out["e4m3_codes"] = R.encode_n("e4m3", f)
    out["f16_codes"] = R.encode_n("f16", f)
    out["bf16_codes"] = R.encode_n("bf16", f)
    allc = np.arange(256, dtype=np.uint8)
    out["e4m3_decode_bits"] = R.decode_n("e4m3", allc).view(np.uint32)
    h = np.arange(0, 65536, 7, dtype=np.uint16)
    out["f16_decode_in"] = h
    out["f16_decode_bits"] = R.decode_n("f16", h).view(np.uint32)

    # --- int8 per-row quantization (quant_int8.cpp:72-90) ---
    rng = np.random.default_rng(7)
    X = rng.standard_normal((48, 40)).astype(np.float32)
    X[rng.random(X.shape) < 0.01] *= 20.0           # outliers, as in the W8A8 workload
    X[3] = 0.0                                       # all-zero row -> scale 1.0
    X[4] = np.arange(40, dtype=np.float32) - 19.5    # exact .5 ties after scaling
    X[5, :8] = [127.0, 2.5, 3.5, -2.5, -3.5, 0.5, -0.5, 1.5]  # scale 1.0, RNE ties
    X[5, 8:] = 0.25
    X[6] = 1e-30                                     # tiny but normal
    X[7, 0] = np.nan                                 # NaN is ignored by the max
    X[8] = -7.0
    out["q8_x"] = X
    q, s = R.quantize_i8_channel(X)
    out["q8_codes"], out["q8_scales"] = q, s
    qt, st = R.quantize_i8_tensor(X[:20])
    out["q8t_codes"], out["q8t_scale"] = qt, np.float32(st)

    # --- asymmetric per-group (quant_int8.cpp:94-142, 162-179) ---
    G = rng.standard_normal((12, 64)).astype(np.float32)
    G[0] = np.abs(G[0])            # all >= 0: zero point 0
    G[1] = -np.abs(G[1])           # all <= 0: zero point 255
    G[2] = 0.0                     # constant zero group: scale 1
    G[3, :16] = 2.0                # constant positive group
    G[4, 5] = np.nan
    out["qg_x"] = G
    qg, sg, zg = R.quantize_i8_group(G, 4)
    out["qg_codes"], out["qg_scales"], out["qg_zeros"] = qg, sg, zg
    out["qg_back"] = R.dequantize_i8_group(qg, 4, sg, zg)

    # --- exact int8 GEMM (quant_int8.cpp:189-211) ---
    for tag, (M, N, K) in {"a": (7, 5, 11), "b": (33, 48, 40), "c": (130, 96, 64)}.items():
        A = rng.integers(-127, 128, (M, K), dtype=np.int8)
        B = rng.integers(-127, 128, (K, N), dtype=np.int8)
        sa = rng.uniform(1e-3, 2e-2, M).astype(np.float32)
        sb = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
        out[f"g8{tag}_A"], out[f"g8{tag}_B"] = A, B
        out[f"g8{tag}_sa"], out[f"g8{tag}_sb"] = sa, sb
        out[f"g8{tag}_C"] = R.gemm_i8(A, B, sa, 1, sb, 1)
        out[f"g8{tag}_acc"] = R.gemm_i8_acc(A, B)

    # --- f16 / bf16 / e4m3 GEMMs (fp16.cpp:123-141, fp8.cpp:116-124) ---
    M, N, K = 32, 28, 40  # tests/test_gemm_f16.cpp:63
    Af = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    Bf = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    A16, B16 = R.encode_n("f16", Af), R.encode_n("f16", Bf)
    Ab, Bb = R.encode_n("bf16", Af), R.encode_n("bf16", Bf)
    out["gh_A16"], out["gh_B16"], out["gh_C16"] = A16, B16, R.gemm_f16(A16, B16)
    out["gh_Ab"], out["gh_Bb"], out["gh_Cb"] = Ab, Bb, R.gemm_bf16(Ab, Bb)
    # e4m3 on integers 1..8 is exact (tests/test_gemm_fp8.cpp:73-99)
    M, N, K = 32, 32, 64
    ai = (1 + np.arange(M * K) % 8).astype(np.float32).reshape(M, K)
    bi = (1 + (np.arange(K * N) * 3) % 8).astype(np.float32).reshape(K, N)
    Aq, Bq = R.encode_n("e4m3", ai), R.encode_n("e4m3", bi)
    out["ge_A"], out["ge_B"], out["ge_C"] = Aq, Bq, R.gemm_e4m3(Aq, Bq)

    # --- conv2d (conv.cpp:26-66): NCHW f32 with bias ---
    x = rng.uniform(-1, 1, (2, 8, 7, 9)).astype(np.float32)
    w = rng.standard_normal((16, 8, 3, 3)).astype(np.float32) * 0.2
    b = rng.standard_normal(16).astype(np.float32)
    out["cv_x"], out["cv_w"], out["cv_b"] = x, w, b
    out["cv_y"] = R.conv2d_f32(x, w, b, 1, 1)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), sum(v.nbytes for v in out.values()), "bytes raw")


if __name__ == "__main__":
    main()
