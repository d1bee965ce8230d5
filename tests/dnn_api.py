"""ctypes driver of the cuDNN API subset (include/rouge/cudnn_b200.h and the
reference's cudnn_shim.h): the same calls run against librouge_b200_cudnn.so
and against the reference's shim compiled from its sources
(oracle/_ref/librouge_ref_shims.so), so parity tests compare the two
libraries call for call. Operands are numpy arrays (host memory) or torch
tensors (device memory)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
B200_DNN = os.path.join(ROOT, "rouge-v_b200", "lib", "librouge_b200_cudnn.so")
REF_SHIMS = os.path.join(ROOT, "oracle", "_ref", "librouge_ref_shims.so")

# cudnn_shim.h enum values (the public cuDNN values)
FLOAT, DOUBLE, HALF, INT8, BFLOAT16 = 0, 1, 2, 3, 9
NCHW, NHWC = 0, 1
ALGO_IMPLICIT_GEMM, ALGO_GEMM, ALGO_DIRECT, ALGO_WINOGRAD = 0, 2, 3, 6
SIGMOID, RELU, TANH, CLIPPED_RELU = 0, 1, 2, 3
SOFTMAX_FAST, SOFTMAX_ACCURATE, SOFTMAX_LOG = 0, 1, 2
MODE_INSTANCE, MODE_CHANNEL = 0, 1
BN_SPATIAL, BN_PER_ACTIVATION = 0, 1
SUCCESS, NOT_INITIALIZED, BAD_PARAM, NOT_SUPPORTED = 0, 1, 3, 9

_V = C.c_void_p
_I = C.c_int
_SIGS = {
    "cudnnCreate": [_V], "cudnnDestroy": [_V],
    "cudnnCreateTensorDescriptor": [_V], "cudnnDestroyTensorDescriptor": [_V],
    "cudnnSetTensor4dDescriptor": [_V, _I, _I, _I, _I, _I, _I],
    "cudnnCreateFilterDescriptor": [_V], "cudnnDestroyFilterDescriptor": [_V],
    "cudnnSetFilter4dDescriptor": [_V, _I, _I, _I, _I, _I, _I],
    "cudnnCreateConvolutionDescriptor": [_V], "cudnnDestroyConvolutionDescriptor": [_V],
    "cudnnSetConvolution2dDescriptor": [_V, _I, _I, _I, _I, _I, _I, _I, _I],
    "cudnnGetConvolution2dForwardOutputDim": [_V, _V, _V, _V, _V, _V, _V],
    "cudnnConvolutionForward": [_V, _V, _V, _V, _V, _V, _V, _I, _V, C.c_size_t, _V, _V, _V],
    "cudnnGetConvolutionForwardWorkspaceSize": [_V, _V, _V, _V, _V, _I, _V],
    "cudnnCreateActivationDescriptor": [_V], "cudnnDestroyActivationDescriptor": [_V],
    "cudnnSetActivationDescriptor": [_V, _I, _I, C.c_double],
    "cudnnActivationForward": [_V, _V, _V, _V, _V, _V, _V, _V],
    "cudnnAddTensor": [_V, _V, _V, _V, _V, _V, _V],
    "cudnnSoftmaxForward": [_V, _I, _I, _V, _V, _V, _V, _V, _V],
    "cudnnBatchNormalizationForwardInference":
        [_V, _I, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, C.c_double],
}


def ptr(a):
    """Address of a numpy array (host) or a torch tensor (device)."""
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


class Dnn:
    def __init__(self, path: str):
        self.lib = C.CDLL(path)
        for name, args in _SIGS.items():
            fn = getattr(self.lib, name, None)
            if fn is None:  # the reference's shim has no workspace query
                continue
            fn.argtypes = args
            fn.restype = _I
        self.lib.cudnnGetErrorString.restype = C.c_char_p
        self.lib.cudnnGetErrorString.argtypes = [_I]
        self.lib.cudnnGetVersion.restype = C.c_size_t
        self.h = _V()
        self._descs = []

    def create(self) -> int:
        return self.lib.cudnnCreate(C.byref(self.h))

    def close(self):
        for kind, d in reversed(self._descs):
            getattr(self.lib, f"cudnnDestroy{kind}Descriptor")(d)
        self._descs.clear()
        if self.h:
            self.lib.cudnnDestroy(self.h)
            self.h = _V()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _new(self, kind):
        d = _V()
        assert getattr(self.lib, f"cudnnCreate{kind}Descriptor")(C.byref(d)) == SUCCESS
        self._descs.append((kind, d))
        return d

    def tensor(self, fmt, dtype, n, c, h, w):
        d = self._new("Tensor")
        st = self.lib.cudnnSetTensor4dDescriptor(d, fmt, dtype, n, c, h, w)
        return d, st

    def filter(self, dtype, fmt, k, c, h, w):
        d = self._new("Filter")
        st = self.lib.cudnnSetFilter4dDescriptor(d, dtype, fmt, k, c, h, w)
        return d, st

    def conv(self, pad, stride, dil=1, mode=0, pad_w=None, stride_w=None):
        d = self._new("Convolution")
        st = self.lib.cudnnSetConvolution2dDescriptor(
            d, pad, pad if pad_w is None else pad_w, stride, stride if stride_w is None else stride_w,
            dil, dil, mode, FLOAT)
        return d, st

    def output_dim(self, conv, x, w):
        v = [C.c_int() for _ in range(4)]
        st = self.lib.cudnnGetConvolution2dForwardOutputDim(conv, x, w, *[C.byref(t) for t in v])
        return st, tuple(t.value for t in v)

    def workspace(self, xd, wd, cd, yd, algo=ALGO_IMPLICIT_GEMM):
        n = C.c_size_t(12345)
        st = self.lib.cudnnGetConvolutionForwardWorkspaceSize(self.h, xd, wd, cd, yd, algo,
                                                              C.byref(n))
        return st, n.value

    def conv_forward(self, alpha, xd, x, wd, w, cd, algo, yd, y, beta, ws=None, ws_bytes=0):
        a = C.c_float(alpha)
        b = C.c_float(beta)
        return self.lib.cudnnConvolutionForward(
            self.h, C.byref(a), xd, ptr(x), wd, ptr(w), cd, algo, ws, ws_bytes, C.byref(b), yd, ptr(y))

    def activation(self, mode, coef, alpha, xd, x, beta, yd, y):
        d = self._new("Activation")
        assert self.lib.cudnnSetActivationDescriptor(d, mode, 0, coef) == SUCCESS
        a, b = C.c_float(alpha), C.c_float(beta)
        return self.lib.cudnnActivationForward(self.h, d, C.byref(a), xd, ptr(x), C.byref(b), yd, ptr(y))

    def add(self, a1, ad, A, a2, bd, B):
        x, y = C.c_float(a1), C.c_float(a2)
        return self.lib.cudnnAddTensor(self.h, C.byref(x), ad, ptr(A), C.byref(y), bd, ptr(B))

    def softmax(self, algo, mode, alpha, xd, x, beta, yd, y):
        a, b = C.c_float(alpha), C.c_float(beta)
        return self.lib.cudnnSoftmaxForward(self.h, algo, mode, C.byref(a), xd, ptr(x), C.byref(b),
                                            yd, ptr(y))

    def batchnorm(self, mode, alpha, beta, xd, x, yd, y, bnd, scale, bias, mean, var, eps):
        a, b = C.c_float(alpha), C.c_float(beta)
        return self.lib.cudnnBatchNormalizationForwardInference(
            self.h, mode, C.byref(a), C.byref(b), xd, ptr(x), yd, ptr(y), bnd, ptr(scale),
            ptr(bias), ptr(mean), ptr(var), eps)
