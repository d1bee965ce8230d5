"""C-ABI surface of librouge_b200.so, checked without a GPU: every symbol
declared in include/rouge/numerics_b200.h is exported, the host-side format
converters match the oracle, device entries refuse cleanly with no device,
and the synthetic-data generator is deterministic."""
import ctypes as C

import numpy as np
import pytest


def test_exports_every_declared_symbol(rb):
    names = rb.declared_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(rb.lib(), n)]
    assert not missing, missing


def test_drop_in_names_match_reference_header(rb):
    # The drop-in subset of software/rouge-numerics/include/rouge/numerics.h
    for n in ("rouge_gemm_i8", "rouge_gemm_e4m3", "rouge_gemm_f16", "rouge_gemm_bf16",
              "rouge_quantize_i8_tensor", "rouge_quantize_i8_channel",
              "rouge_dequantize_i8_tensor", "rouge_dequantize_i8_channel",
              "rouge_quantize_e4m3", "rouge_dequantize_e4m3", "rouge_quantize_f16",
              "rouge_dequantize_f16", "rouge_quantize_bf16", "rouge_dequantize_bf16",
              "rouge_gemm_isa_variant", "rouge_gemm_default_config", "rouge_gemm_f32",
              "rouge_gemm_candidate_count", "rouge_gemm_candidate", "rouge_gemm_flops_per_sec",
              "rouge_gemm_tuned"):
        assert n in rb.declared_symbols()
    assert rb.lib().rouge_gemm_isa_variant() == b"sm_100a+tcgen05"


def test_host_converters_match_oracle(rb, orc, golden):
    L = rb.lib()
    x = golden["fmt_x"]
    for enc, fmt in ((L.rouge_quantize_e4m3, "e4m3"), (L.rouge_quantize_f16, "f16"),
                     (L.rouge_quantize_bf16, "bf16")):
        got = np.array([enc(float(v)) for v in x.tolist()])
        want = getattr(orc, f"{fmt}_encode")(x)
        assert (got == want).all(), fmt
    codes = np.arange(256)
    got = np.array([L.rouge_dequantize_e4m3(int(c)) for c in codes], np.float32)
    want = orc.e4m3_decode(codes.astype(np.uint8))
    nan = np.isnan(want)
    assert (np.isnan(got) == nan).all()
    assert (got[~nan].view(np.uint32) == want[~nan].view(np.uint32)).all()
    h = np.arange(0, 65536, 3)
    got = np.array([L.rouge_dequantize_f16(int(c)) for c in h], np.float32)
    want = orc.f16_decode(h.astype(np.uint16))
    nan = np.isnan(want)
    assert (np.isnan(got) == nan).all()
    assert (got[~nan].view(np.uint32) == want[~nan].view(np.uint32)).all()


def test_status_strings(rb):
    L = rb.lib()
    for st in (rb.OK, rb.EINVAL, rb.ENODEV, rb.ECUDA, rb.EUNSUPPORTED, rb.ETIMEOUT, rb.ENOMEM):
        assert L.rouge_b200_status_string(st) != b"unknown status"


def test_invalid_arguments_are_refused(rb):
    L = rb.lib()
    # NULL pointers / bad sizes: no write, EINVAL (reference: silent no-op, quant returns 0)
    assert L.rouge_b200_gemm_i8(0, 4, 16, None, None, 0, None, 1, None, 1, None, 4, 0, None) == rb.EINVAL
    assert L.rouge_b200_quantize_i8_rows(None, 4, 4, None, None, None) == rb.EINVAL
    assert L.rouge_quantize_i8_channel(None, 4, 4, None, None) == 0
    out = np.full(4, 7, np.float32)
    L.rouge_gemm_i8(0, 2, 2, None, None, None, 1, None, 1, out.ctypes.data_as(C.c_void_p))
    assert (out == 7).all()


def test_fused_step_host_checks(rb):
    L = rb.lib()
    # one count per 128-row block, a finished-CTA count and the row counter
    assert L.rouge_b200_w8a8_workspace_bytes(4096) == (32 + 2) * 4
    assert L.rouge_b200_w8a8_workspace_bytes(1000) == (8 + 2) * 4
    assert L.rouge_b200_w8a8_workspace_bytes(0) == 0
    # refused before any device work: no workspace / no input
    assert L.rouge_b200_w8a8_linear(256, 256, 64, None, None, None, None, None, None, 256, 0,
                                    None, None) == rb.EINVAL
    # the wait-limit check refuses limits outside 1 ms .. 2 s (or reports no device)
    st = L.rouge_b200_check_wait_limit(10, None)
    assert st in (rb.EINVAL, rb.ENODEV)
    L.rouge_b200_clear_error()


def test_tile_mode_switch(rb):
    L = rb.lib()
    assert L.rouge_b200_set_tile_mode(7) == rb.EINVAL          # unknown: nothing changed
    prev = L.rouge_b200_set_tile_mode(rb.TILES_PAIR)
    assert prev == rb.TILES_AUTO
    with rb.tile_mode(rb.TILES_SINGLE):
        assert L.rouge_b200_set_tile_mode(rb.TILES_SINGLE) == rb.TILES_SINGLE
    assert L.rouge_b200_set_tile_mode(prev) == rb.TILES_PAIR   # context manager restored it
    L.rouge_b200_clear_error()


def test_no_cpu_fallback_without_device(rb):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = rb.lib()
    assert L.rouge_b200_device_ok() == 0
    L.rouge_b200_clear_error()
    A = np.ones((4, 16), np.int8)
    B = np.ones((16, 4), np.int8)
    s = np.ones(4, np.float32)
    out = np.full((4, 4), -1.0, np.float32)
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    L.rouge_gemm_i8(4, 4, 16, p(A), p(B), p(s), 1, p(s), 1, p(out))
    assert (out == -1.0).all()                       # nothing computed on the CPU
    assert L.rouge_b200_last_error() == rb.ENODEV
    x = np.ones((2, 4), np.float32)
    assert L.rouge_quantize_i8_channel(p(x), 2, 4, p(s), p(A)) == 0


def test_synth_is_deterministic_and_distributed(rb):
    a = rb.synth_normal(42, (1 << 20,), 0.0, 1.0)
    b = rb.synth_normal(42, (1 << 20,), 0.0, 1.0)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
    assert abs(a.mean()) < 5e-3 and abs(a.std() - 1.0) < 5e-3
    u = rb.synth_uniform(0, (1 << 20,), -1.0, 1.0)
    assert u.min() >= -1.0 and u.max() < 1.0 and abs(u.mean()) < 5e-3
    x = np.ones(1 << 20, np.float32)
    n = rb.synth_outliers(1, x, 0.01, 20.0)
    assert abs(n / x.size - 0.01) < 1e-3 and (x == 20.0).sum() == n


def test_cublas_shim_exports_declared_api():
    import ctypes as C
    import os
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    L = C.CDLL(os.path.join(root, "rouge-v_b200", "lib", "librouge_b200_cublas.so"))
    text = open(os.path.join(root, "include", "rouge", "cublas_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"\b(cublas\w+)\s*\(", text)))
    assert len(names) >= 11
    for n in names:
        assert hasattr(L, n), n
    h = C.c_void_p()
    # without an sm_100 device the handle cannot be created (no CPU fallback)
    import torch
    if not torch.cuda.is_available():
        assert L.cublasCreate_v2(C.byref(h)) == 1   # CUBLAS_STATUS_NOT_INITIALIZED


def test_tuner_candidates_and_default_config(rb):
    # numerics.h:307-312: the default configuration, the candidate list, and
    # the default for an index out of range (autotune.cpp:64-66)
    L = rb.lib()
    d = L.rouge_gemm_default_config().astuple()
    assert d == (64, 64, 32, 2, 1)
    n = L.rouge_gemm_candidate_count()
    assert n >= 2
    cands = [L.rouge_gemm_candidate(i).astuple() for i in range(n)]
    assert len(set(cands)) == n and d in cands
    assert L.rouge_gemm_candidate(-1).astuple() == d
    assert L.rouge_gemm_candidate(n).astuple() == d


def test_gemm_f32_entries_without_device_or_arguments(rb):
    import torch
    L = rb.lib()
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    A = np.ones((3, 5), np.float32)
    B = np.ones((5, 4), np.float32)
    out = np.full((3, 4), -7.0, np.float32)
    # invalid sizes / NULL: no-op, zero profile (gemm.cpp:293-294, autotune.cpp:80,101)
    L.rouge_gemm_f32(0, 4, 5, p(A), p(B), p(out), None)
    L.rouge_gemm_f32(3, 4, 5, None, p(B), p(out), None)
    assert (out == -7.0).all()
    assert L.rouge_gemm_flops_per_sec(3, 4, 0, p(A), p(B), p(out), None) == 0.0
    prof = L.rouge_gemm_tuned(3, 4, 5, p(A), None, p(out))
    assert prof.gflops == 0.0 and prof.iters == 0 and prof.cfg.astuple() == (64, 64, 32, 2, 1)
    if torch.cuda.is_available():
        return
    # no device: nothing computed on the CPU, ENODEV kept, zero speed
    L.rouge_b200_clear_error()
    L.rouge_gemm_f32(3, 4, 5, p(A), p(B), p(out), None)
    assert (out == -7.0).all()
    assert L.rouge_b200_last_error() == rb.ENODEV
    assert L.rouge_gemm_flops_per_sec(3, 4, 5, p(A), p(B), p(out), None) == 0.0
    prof = L.rouge_gemm_tuned(3, 4, 5, p(A), p(B), p(out))
    assert prof.gflops == 0.0 and (out == -7.0).all()
    L.rouge_b200_clear_error()
