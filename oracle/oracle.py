"""TEST INFRASTRUCTURE ONLY -- numpy front end of the CPU oracle.

Loads oracle/_build/liboracle.so (the C restatement in rouge_oracle.c) and,
when present, oracle/_ref/librouge_ref.so (the reference rouge-numerics
sources compiled by oracle/Makefile). Only tests/, __graft_entry__.smoke()
and bench.py's reference / cpu_baseline legs import this module; the
product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "librouge_ref.so")

_P = C.c_void_p
_I = C.c_int
_F = C.c_float
_SZ = C.c_size_t


def build():
    """Compile the oracle (and the reference, when its sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _ptr(a):
    return a.ctypes.data_as(_P)


class Oracle:
    """The C restatement; every method mirrors one reference function."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        lib = C.CDLL(path)
        self.lib = lib
        for name, res, args in [
            ("or_f16_decode", _F, [C.c_uint16]),
            ("or_f16_encode", C.c_uint16, [_F]),
            ("or_bf16_decode", _F, [C.c_uint16]),
            ("or_bf16_encode", C.c_uint16, [_F]),
            ("or_e4m3_decode", _F, [C.c_uint8]),
            ("or_e4m3_encode", C.c_uint8, [_F]),
            ("or_e4m3_encode_n", None, [_P, _SZ, _P]),
            ("or_e4m3_decode_n", None, [_P, _SZ, _P]),
            ("or_f16_encode_n", None, [_P, _SZ, _P]),
            ("or_f16_decode_n", None, [_P, _SZ, _P]),
            ("or_bf16_encode_n", None, [_P, _SZ, _P]),
            ("or_quantize_i8_rows", _I, [_P, _I, _I, _P, _P]),
            ("or_quantize_i8_tensor", _I, [_P, _I, _P, _P]),
            ("or_dequantize_i8_rows", None, [_P, _I, _I, _P, _P]),
            ("or_quantize_i8_group", _I, [_P, _I, _I, _I, _P, _P, _P]),
            ("or_dequantize_i8_group", None, [_P, _I, _I, _I, _P, _P, _P]),
            ("or_gemm_i8_rows", None, [_I, _I, _P, _P, _I, _P, _I, _P, _I, _P, _I, _P, _P]),
            ("or_gemm_f32_rows", None, [_I, _I, _P, _P, _I, _P, _I, _P]),
            ("or_absmax", _F, [_P, _SZ]),
            ("or_quantize_e4m3_scaled", _F, [_P, _SZ, _F, _P]),
            ("or_conv2d_nhwc", None, [_I] * 9 + [_P, _P, _P, C.c_long, C.c_long, _P]),
            ("or_narrow_encode_n", None, [_P, _SZ, _I, _I, _P]),
            ("or_narrow_decode_n", None, [_P, _SZ, _I, _P]),
            ("or_e8m0_encode", C.c_uint8, [_F]),
            ("or_e8m0_decode", _F, [C.c_uint8]),
            ("or_mx_quantize", _I, [_P, _I, _I, _P, _P]),
            ("or_nvfp4_quantize", _I, [_P, _I, _F, _P, _P]),
            ("or_mx_dequantize", None, [_P, _P, _I, _I, _P]),
        ]:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args

    # -- formats ----------------------------------------------------------
    def e4m3_encode(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, np.uint8)
        self.lib.or_e4m3_encode_n(_ptr(x), x.size, _ptr(out))
        return out

    def e4m3_decode(self, c):
        c = np.ascontiguousarray(c, dtype=np.uint8)
        out = np.empty(c.shape, np.float32)
        self.lib.or_e4m3_decode_n(_ptr(c), c.size, _ptr(out))
        return out

    def f16_encode(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, np.uint16)
        self.lib.or_f16_encode_n(_ptr(x), x.size, _ptr(out))
        return out

    def f16_decode(self, c):
        c = np.ascontiguousarray(c, dtype=np.uint16)
        out = np.empty(c.shape, np.float32)
        self.lib.or_f16_decode_n(_ptr(c), c.size, _ptr(out))
        return out

    def bf16_encode(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, np.uint16)
        self.lib.or_bf16_encode_n(_ptr(x), x.size, _ptr(out))
        return out

    @staticmethod
    def bf16_decode(c):
        return (np.ascontiguousarray(c, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)

    # -- int8 ---------------------------------------------------------------
    def quantize_i8_rows(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = x.shape
        scales = np.empty(rows, np.float32)
        out = np.empty((rows, cols), np.int8)
        assert self.lib.or_quantize_i8_rows(_ptr(x), rows, cols, _ptr(scales), _ptr(out)) == 1
        return out, scales

    def quantize_i8_tensor(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        s = np.zeros(1, np.float32)
        out = np.empty(x.size, np.int8)
        assert self.lib.or_quantize_i8_tensor(_ptr(x), x.size, _ptr(s), _ptr(out)) == 1
        return out, float(s[0])

    def quantize_i8_group(self, x, groups):
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = x.shape
        s = np.empty(rows * groups, np.float32)
        z = np.empty(rows * groups, np.uint8)
        q = np.empty((rows, cols), np.uint8)
        assert self.lib.or_quantize_i8_group(_ptr(x), rows, cols, groups, _ptr(s), _ptr(z), _ptr(q)) == 1
        return q, s, z

    def dequantize_i8_group(self, q, groups, s, z):
        q = np.ascontiguousarray(q, dtype=np.uint8)
        out = np.empty(q.shape, np.float32)
        self.lib.or_dequantize_i8_group(_ptr(q), q.shape[0], q.shape[1], groups,
                                        _ptr(np.ascontiguousarray(s, np.float32)),
                                        _ptr(np.ascontiguousarray(z, np.uint8)), _ptr(out))
        return out

    def dequantize_i8_rows(self, q, scales):
        q = np.ascontiguousarray(q, dtype=np.int8)
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        out = np.empty(q.shape, np.float32)
        self.lib.or_dequantize_i8_rows(_ptr(q), q.shape[0], q.shape[1], _ptr(scales), _ptr(out))
        return out

    def gemm_i8(self, A, B, b_nk, scales_a=None, a_rows=1, scales_b=None, b_cols=1, rows=None):
        """int32 accumulators and (when scales are given) the f32 outputs
        ((float)acc * sa) * sb of the listed rows (all rows if rows is None)."""
        A = np.ascontiguousarray(A, dtype=np.int8)
        B = np.ascontiguousarray(B, dtype=np.int8)
        M, K = A.shape
        N = B.shape[0] if b_nk else B.shape[1]
        ids = np.arange(M, dtype=np.int32) if rows is None else np.ascontiguousarray(rows, np.int32)
        acc = np.empty((ids.size, N), np.int32)
        c = sa = sb = None
        if scales_a is not None:
            sa = np.ascontiguousarray(np.atleast_1d(scales_a), dtype=np.float32)
            sb = np.ascontiguousarray(np.atleast_1d(scales_b), dtype=np.float32)
            c = np.empty((ids.size, N), np.float32)
        self.lib.or_gemm_i8_rows(N, K, _ptr(A), _ptr(B), int(b_nk), _ptr(ids), ids.size,
                                 _ptr(sa) if sa is not None else None, int(a_rows),
                                 _ptr(sb) if sb is not None else None, int(b_cols),
                                 _ptr(acc), _ptr(c) if c is not None else None)
        return acc, c

    def gemm_f32(self, A, B, b_nk, rows=None):
        A = np.ascontiguousarray(A, dtype=np.float32)
        B = np.ascontiguousarray(B, dtype=np.float32)
        M, K = A.shape
        N = B.shape[0] if b_nk else B.shape[1]
        ids = np.arange(M, dtype=np.int32) if rows is None else np.ascontiguousarray(rows, np.int32)
        c = np.empty((ids.size, N), np.float32)
        self.lib.or_gemm_f32_rows(N, K, _ptr(A), _ptr(B), int(b_nk), _ptr(ids), ids.size, _ptr(c))
        return c

    # -- e4m3 per-tensor ------------------------------------------------------
    def absmax(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        return float(self.lib.or_absmax(_ptr(x), x.size))

    def quantize_e4m3_tensor(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        amax = self.absmax(x)
        out = np.empty(x.shape, np.uint8)
        s = self.lib.or_quantize_e4m3_scaled(_ptr(x), x.size, amax, _ptr(out))
        return out, float(np.float32(s)), amax

    # -- narrow formats and MX / NVFP4 blocks (narrow.cpp) -----------------------
    # fmt: 0 e4m3, 1 e5m2, 2 e3m2, 3 e2m3, 4 e2m1 (codes in the low bits)
    NARROW = {"e4m3": 0, "e5m2": 1, "e3m2": 2, "e2m3": 3, "e2m1": 4}

    def narrow_encode(self, x, fmt, nan_to_max=None):
        f = self.NARROW[fmt]
        if nan_to_max is None:
            nan_to_max = f >= 2   # narrow.cpp:172-196: the 6/4-bit formats map NaN to +MAX
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.empty(x.size, np.uint8)
        self.lib.or_narrow_encode_n(_ptr(x), x.size, f, int(nan_to_max), _ptr(out))
        return out

    def narrow_decode(self, c, fmt):
        c = np.ascontiguousarray(c, dtype=np.uint8).ravel()
        out = np.empty(c.size, np.float32)
        self.lib.or_narrow_decode_n(_ptr(c), c.size, self.NARROW[fmt], _ptr(out))
        return out

    def mx_quantize(self, x, fmt):
        """MXFP8 (fmt e4m3 / e5m2) or MXFP4 (e2m1): codes, E8M0 scales per 32."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        q = np.empty(x.size, np.uint8)
        sc = np.empty((x.size + 31) // 32, np.uint8)
        assert self.lib.or_mx_quantize(_ptr(x), x.size, self.NARROW[fmt], _ptr(q), _ptr(sc)) == sc.size
        return q, sc

    def nvfp4_quantize(self, x, gs):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        q = np.empty(x.size, np.uint8)
        sc = np.empty((x.size + 15) // 16, np.uint8)
        assert self.lib.or_nvfp4_quantize(_ptr(x), x.size, gs, _ptr(q), _ptr(sc)) == sc.size
        return q, sc

    def mx_dequantize(self, q, sc, fmt):
        q = np.ascontiguousarray(q, dtype=np.uint8).ravel()
        sc = np.ascontiguousarray(sc, dtype=np.uint8).ravel()
        out = np.empty(q.size, np.float32)
        self.lib.or_mx_dequantize(_ptr(q), _ptr(sc), q.size, self.NARROW[fmt], _ptr(out))
        return out

    # -- conv -------------------------------------------------------------------
    def conv2d_nhwc(self, x, w, bias, stride, pad, p0=0, p1=None):
        """x[N][H][W][Cin] f32, w[Cout][KH][KW][Cin] f32 -> y rows [p1-p0][Cout]."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        N, H, W, Cin = x.shape
        Cout, KH, KW, _ = w.shape
        OH = (H + 2 * pad - KH) // stride + 1
        OW = (W + 2 * pad - KW) // stride + 1
        if p1 is None:
            p1 = N * OH * OW
        y = np.empty((p1 - p0, Cout), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self.lib.or_conv2d_nhwc(N, H, W, Cin, Cout, KH, KW, stride, pad, _ptr(x), _ptr(w),
                                _ptr(b) if b is not None else None, p0, p1, _ptr(y))
        return y


class Reference:
    """The reference library itself (oracle/_ref/librouge_ref.so)."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def __init__(self, path: str = REF_SO):
        lib = C.CDLL(path)
        self.lib = lib
        for name, res, args in [
            ("rouge_quantize_e4m3", C.c_uint8, [_F]),
            ("rouge_dequantize_e4m3", _F, [C.c_uint8]),
            ("rouge_quantize_f16", C.c_uint16, [_F]),
            ("rouge_dequantize_f16", _F, [C.c_uint16]),
            ("rouge_quantize_bf16", C.c_uint16, [_F]),
            ("rouge_dequantize_bf16", _F, [C.c_uint16]),
            ("rouge_quantize_i8_tensor", _I, [_P, _I, _P, _P]),
            ("rouge_quantize_i8_channel", _I, [_P, _I, _I, _P, _P]),
            ("rouge_dequantize_i8_channel", None, [_P, _I, _I, _P, _P]),
            ("rouge_quantize_i8_group", _I, [_P, _I, _I, _I, _P, _P, _P]),
            ("rouge_dequantize_i8_group", None, [_P, _I, _I, _I, _P, _P, _P]),
            ("rouge_gemm_i8", None, [_I, _I, _I, _P, _P, _P, _I, _P, _I, _P]),
            ("rouge_gemm_f32", None, [_I, _I, _I, _P, _P, _P, _P]),
            ("rouge_gemm_f16", None, [_I, _I, _I, _P, _P, _P, _P]),
            ("rouge_gemm_bf16", None, [_I, _I, _I, _P, _P, _P, _P]),
            ("rouge_gemm_e4m3", None, [_I, _I, _I, _P, _P, _P, _P]),
            ("rouge_conv2d_f32", None, [_I] * 9 + [_P, _P, _P, _P, _P]),
            ("rouge_quantize_e5m2", C.c_uint8, [_F]), ("rouge_dequantize_e5m2", _F, [C.c_uint8]),
            ("rouge_quantize_e3m2", C.c_uint8, [_F]), ("rouge_dequantize_e3m2", _F, [C.c_uint8]),
            ("rouge_quantize_e2m3", C.c_uint8, [_F]), ("rouge_dequantize_e2m3", _F, [C.c_uint8]),
            ("rouge_quantize_e2m1", C.c_uint8, [_F]), ("rouge_dequantize_e2m1", _F, [C.c_uint8]),
            ("rouge_mx_quantize_f32", _I, [_P, _I, _I, _P, _P]),
            ("ref_narrow_encode_n", None, [_P, _SZ, _I, _P]),
            ("ref_narrow_decode_n", None, [_P, _SZ, _I, _P]),
            ("rouge_mx_quantize_f32_e2m1", _I, [_P, _I, _P, _P]),
            ("rouge_nvfp4_quantize_f32", _I, [_P, _I, _F, _P, _P]),
            ("rouge_mx_dequantize_f32", None, [_P, _P, _I, _I, _P]),
            ("rouge_mx_dequantize_f32_e2m1", None, [_P, _P, _I, _P]),
            ("ref_hw_threads", _I, []),
            ("ref_quantize_i8_channel_mt", _I, [_P, _I, _I, _P, _P, _I]),
            ("ref_gemm_i8_mt", None, [_I, _I, _I, _P, _P, _P, _I, _P, _I, _P, _I]),
            ("ref_gemm_i8_acc_rows", None, [_I, _I, _P, _P, _I, _I, _P]),
            ("ref_e4m3_encode_n", None, [_P, _SZ, _P]),
            ("ref_f16_encode_n", None, [_P, _SZ, _P]),
            ("ref_bf16_encode_n", None, [_P, _SZ, _P]),
            ("ref_bf16_encode_mt", None, [_P, _SZ, _P, _I]),
            ("ref_synth_uniform", _I, [C.c_uint64, _SZ, _F, _F, _P]),
            ("ref_synth_normal_at", _I, [C.c_uint64, _SZ, _SZ, _F, _F, _P]),
            ("ref_synth_outliers_at", C.c_longlong, [C.c_uint64, _SZ, _SZ, _F, _F, _P]),
            ("ref_e4m3_decode_n", None, [_P, _SZ, _P]),
            ("ref_f16_decode_n", None, [_P, _SZ, _P]),
        ]:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args

    # -- seeded inputs (the benchmark's generator, without its library) -----
    def synth_uniform(self, seed, shape, lo, hi):
        out = np.empty(shape, np.float32)
        assert self.lib.ref_synth_uniform(seed, out.size, lo, hi, _ptr(out)) == 0
        return out

    def synth_normal(self, seed, shape, mean, std, offset=0):
        out = np.empty(shape, np.float32)
        assert self.lib.ref_synth_normal_at(seed, offset, out.size, mean, std, _ptr(out)) == 0
        return out

    def synth_outliers(self, seed, x, frac, mult, offset=0):
        assert x.dtype == np.float32 and x.flags.c_contiguous
        return int(self.lib.ref_synth_outliers_at(seed, offset, x.size, frac, mult, _ptr(x)))

    def bf16_encode(self, x, threads=1):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, np.uint16)
        self.lib.ref_bf16_encode_mt(_ptr(x), x.size, _ptr(out), threads)
        return out

    def quantize_i8_channel(self, x, threads=1):
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = x.shape
        s = np.empty(rows, np.float32)
        q = np.empty((rows, cols), np.int8)
        if threads > 1:
            assert self.lib.ref_quantize_i8_channel_mt(_ptr(x), rows, cols, _ptr(s), _ptr(q), threads)
        else:
            assert self.lib.rouge_quantize_i8_channel(_ptr(x), rows, cols, _ptr(s), _ptr(q)) == 1
        return q, s

    def quantize_i8_tensor(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        s = np.zeros(1, np.float32)
        q = np.empty(x.size, np.int8)
        assert self.lib.rouge_quantize_i8_tensor(_ptr(x), x.size, _ptr(s), _ptr(q)) == 1
        return q, float(s[0])

    def quantize_i8_group(self, x, groups):
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = x.shape
        s = np.empty(rows * groups, np.float32)
        z = np.empty(rows * groups, np.uint8)
        q = np.empty((rows, cols), np.uint8)
        assert self.lib.rouge_quantize_i8_group(_ptr(x), rows, cols, groups, _ptr(s), _ptr(z),
                                                _ptr(q)) == 1
        return q, s, z

    def dequantize_i8_group(self, q, groups, s, z):
        q = np.ascontiguousarray(q, dtype=np.uint8)
        out = np.empty(q.shape, np.float32)
        self.lib.rouge_dequantize_i8_group(_ptr(q), q.shape[0], q.shape[1], groups,
                                           _ptr(np.ascontiguousarray(s, np.float32)),
                                           _ptr(np.ascontiguousarray(z, np.uint8)), _ptr(out))
        return out

    def gemm_i8(self, A, B_kn, sa, a_rows, sb, b_cols, threads=1):
        A = np.ascontiguousarray(A, dtype=np.int8)
        B_kn = np.ascontiguousarray(B_kn, dtype=np.int8)
        M, K = A.shape
        N = B_kn.shape[1]
        sa = np.ascontiguousarray(np.atleast_1d(sa), dtype=np.float32)
        sb = np.ascontiguousarray(np.atleast_1d(sb), dtype=np.float32)
        C_ = np.empty((M, N), np.float32)
        if threads > 1:
            self.lib.ref_gemm_i8_mt(M, N, K, _ptr(A), _ptr(B_kn), _ptr(sa), a_rows, _ptr(sb),
                                    b_cols, _ptr(C_), threads)
        else:
            self.lib.rouge_gemm_i8(M, N, K, _ptr(A), _ptr(B_kn), _ptr(sa), a_rows, _ptr(sb),
                                   b_cols, _ptr(C_))
        return C_

    def gemm_i8_acc(self, A, B_kn, r0=0, r1=None):
        A = np.ascontiguousarray(A, dtype=np.int8)
        B_kn = np.ascontiguousarray(B_kn, dtype=np.int8)
        M, K = A.shape
        N = B_kn.shape[1]
        r1 = M if r1 is None else r1
        acc = np.empty((r1 - r0, N), np.int32)
        self.lib.ref_gemm_i8_acc_rows(N, K, _ptr(A), _ptr(B_kn), r0, r1, _ptr(acc))
        return acc

    def _gemm_codes(self, fn, A, B_kn, dtype):
        A = np.ascontiguousarray(A, dtype=dtype)
        B_kn = np.ascontiguousarray(B_kn, dtype=dtype)
        M, K = A.shape
        N = B_kn.shape[1]
        C_ = np.empty((M, N), np.float32)
        fn(M, N, K, _ptr(A), _ptr(B_kn), _ptr(C_), None)
        return C_

    def gemm_f16(self, A, B_kn):
        return self._gemm_codes(self.lib.rouge_gemm_f16, A, B_kn, np.uint16)

    def gemm_bf16(self, A, B_kn):
        return self._gemm_codes(self.lib.rouge_gemm_bf16, A, B_kn, np.uint16)

    def gemm_e4m3(self, A, B_kn):
        return self._gemm_codes(self.lib.rouge_gemm_e4m3, A, B_kn, np.uint8)

    def gemm_f32(self, A, B_kn):
        return self._gemm_codes(self.lib.rouge_gemm_f32, A, B_kn, np.float32)

    def conv2d_f32(self, x_nchw, w_oihw, bias, stride, pad):
        x = np.ascontiguousarray(x_nchw, dtype=np.float32)
        w = np.ascontiguousarray(w_oihw, dtype=np.float32)
        N, Cin, H, W = x.shape
        Cout, _, KH, KW = w.shape
        OH = (H + 2 * pad - KH) // stride + 1
        OW = (W + 2 * pad - KW) // stride + 1
        y = np.zeros((N, Cout, OH, OW), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self.lib.rouge_conv2d_f32(N, Cin, H, W, Cout, KH, KW, stride, pad, _ptr(x), _ptr(w),
                                  _ptr(b) if b is not None else None, _ptr(y), None)
        return y

    def narrow_encode(self, x, fmt):
        """rouge_quantize_{e5m2,e3m2,e2m3,e2m1} over an array."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.empty(x.size, np.uint8)
        self.lib.ref_narrow_encode_n(_ptr(x), x.size, Oracle.NARROW[fmt], _ptr(out))
        return out

    def narrow_decode(self, c, fmt):
        c = np.ascontiguousarray(c, dtype=np.uint8).ravel()
        out = np.empty(c.size, np.float32)
        self.lib.ref_narrow_decode_n(_ptr(c), c.size, Oracle.NARROW[fmt], _ptr(out))
        return out

    def mx_quantize(self, x, fmt):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        q = np.empty(x.size, np.uint8)
        sc = np.empty((x.size + 31) // 32, np.uint8)
        if fmt == "e2m1":
            nb = self.lib.rouge_mx_quantize_f32_e2m1(_ptr(x), x.size, _ptr(q), _ptr(sc))
        else:
            nb = self.lib.rouge_mx_quantize_f32(_ptr(x), x.size, 1 if fmt == "e4m3" else 2, _ptr(q),
                                                _ptr(sc))
        assert nb == sc.size
        return q, sc

    def nvfp4_quantize(self, x, gs):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        q = np.empty(x.size, np.uint8)
        sc = np.empty((x.size + 15) // 16, np.uint8)
        assert self.lib.rouge_nvfp4_quantize_f32(_ptr(x), x.size, gs, _ptr(q), _ptr(sc)) == sc.size
        return q, sc

    def mx_dequantize(self, q, sc, fmt):
        q = np.ascontiguousarray(q, dtype=np.uint8).ravel()
        sc = np.ascontiguousarray(sc, dtype=np.uint8).ravel()
        out = np.empty(q.size, np.float32)
        if fmt == "e2m1":
            self.lib.rouge_mx_dequantize_f32_e2m1(_ptr(q), _ptr(sc), q.size, _ptr(out))
        else:
            self.lib.rouge_mx_dequantize_f32(_ptr(q), _ptr(sc), q.size, 1 if fmt == "e4m3" else 2,
                                             _ptr(out))
        return out

    def encode_n(self, fmt, x):
        """Bulk reference encode: fmt in {"e4m3", "f16", "bf16"}."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, np.uint8 if fmt == "e4m3" else np.uint16)
        getattr(self.lib, f"ref_{fmt}_encode_n")(_ptr(x), x.size, _ptr(out))
        return out

    def decode_n(self, fmt, c):
        """Bulk reference decode: fmt in {"e4m3", "f16"}."""
        c = np.ascontiguousarray(c, dtype=np.uint8 if fmt == "e4m3" else np.uint16)
        out = np.empty(c.shape, np.float32)
        getattr(self.lib, f"ref_{fmt}_decode_n")(_ptr(c), c.size, _ptr(out))
        return out

    def vec(self, name, x, out_dtype):
        """Apply a scalar reference conversion to every element of x."""
        fn = getattr(self.lib, name)
        flat = np.asarray(x).ravel()
        return np.array([fn(v) for v in flat.tolist()], dtype=out_dtype).reshape(np.shape(x))
