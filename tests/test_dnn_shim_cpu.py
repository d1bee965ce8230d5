"""librouge_b200_cudnn.so without a GPU: it exports every cuDNN entry its
header declares, refuses to create a handle with no device (no CPU
fallback), and its descriptor logic (argument checks, output size) gives
the reference shim's answers call for call (cudnn_shim.cpp:83-186)."""
import ctypes as C
import os
import re

import pytest

import dnn_api as D


@pytest.fixture(scope="module")
def ours(rb):
    assert os.path.exists(D.B200_DNN), "librouge_b200_cudnn.so not built"
    return D.Dnn(D.B200_DNN)


@pytest.fixture(scope="module")
def theirs():
    if not os.path.exists(D.REF_SHIMS):
        pytest.skip("reference shims library not built")
    return D.Dnn(D.REF_SHIMS)


def test_exports_declared_api(ours):
    text = open(os.path.join(D.ROOT, "include", "rouge", "cudnn_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"\b(cudnn\w+)\s*\(", text)))
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(ours.lib, n)]
    assert not missing, missing
    # nothing but cudnn* is defined by the library itself
    import shutil
    import subprocess
    if shutil.which("nm"):
        out = subprocess.run(["nm", "-D", "--defined-only", D.B200_DNN], capture_output=True,
                             text=True, check=True).stdout
        syms = [ln.split()[-1] for ln in out.splitlines() if " T " in ln]
        assert syms and all(s.startswith("cudnn") for s in syms), syms


def test_no_handle_without_device(ours):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    assert ours.lib.cudnnCreate(C.byref(h)) == D.NOT_INITIALIZED
    assert ours.lib.cudnnCreate(None) == D.BAD_PARAM


def test_error_strings_and_version(ours, theirs):
    for s in range(0, 12):
        assert ours.lib.cudnnGetErrorString(s) == theirs.lib.cudnnGetErrorString(s)
    assert ours.lib.cudnnGetVersion() == theirs.lib.cudnnGetVersion()


CONV_ARGS = [  # pad_h, pad_w, stride_h, stride_w, dilation, mode
    (1, 1, 1, 1, 1, 0), (0, 0, 2, 2, 1, 0), (3, 3, 2, 2, 1, 0), (1, 2, 1, 1, 1, 0),
    (1, 1, 1, 2, 1, 0), (1, 1, 1, 1, 2, 0), (1, 1, 1, 1, 1, 1), (-1, -1, 1, 1, 1, 0),
    (1, 1, 0, 0, 1, 0),
]


@pytest.mark.parametrize("args", CONV_ARGS)
def test_conv_descriptor_checks_match_reference(ours, theirs, args):
    ph, pw, sh, sw, dil, mode = args
    got = [lib.conv(ph, sh, dil, mode, pad_w=pw, stride_w=sw)[1] for lib in (ours, theirs)]
    assert got[0] == got[1], (args, got)


@pytest.mark.parametrize("dims", [(1, 2, 8, 8), (0, 2, 8, 8), (3, 1, 1, 1), (2, 3, -1, 5)])
def test_tensor_descriptor_checks_match_reference(ours, theirs, dims):
    a = ours.tensor(D.NCHW, D.FLOAT, *dims)[1]
    b = theirs.tensor(D.NCHW, D.FLOAT, *dims)[1]
    assert a == b


@pytest.mark.parametrize("case", [
    ((1, 2, 8, 8), (3, 2, 3, 3), 1, 1),
    ((2, 3, 224, 224), (64, 3, 7, 7), 3, 2),
    ((4, 16, 9, 7), (8, 16, 5, 5), 0, 1),
    ((1, 1, 4, 4), (1, 1, 5, 5), 0, 1),      # filter larger than the input: BAD_PARAM
    ((1, 1, 4, 4), (1, 1, 3, 3), 0, 3),
])
def test_output_dim_matches_reference(ours, theirs, case):
    xs, ws, pad, stride = case
    res = []
    for lib in (ours, theirs):
        x = lib.tensor(D.NCHW, D.FLOAT, *xs)[0]
        w = lib.filter(D.FLOAT, D.NCHW, *ws)[0]
        cd = lib.conv(pad, stride)[0]
        res.append(lib.output_dim(cd, x, w))
    assert res[0][0] == res[1][0]
    if res[0][0] == D.SUCCESS:
        assert res[0][1] == res[1][1]
