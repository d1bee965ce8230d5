"""Python binding of librouge_b200.so (the C ABI in include/rouge/numerics_b200.h).

A thin ctypes layer: every function here calls one exported C entry point.
Device-pointer entries take torch CUDA tensors and the current torch stream;
host-pointer (drop-in) entries take numpy arrays, exactly as a C caller of
the reference rouge-numerics API passes host buffers. There is no CPU
fallback: if the shared library is missing or the GPU path fails, calls
raise.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(os.path.dirname(PKG_DIR), "lib")
LIB_PATH = os.path.join(LIB_DIR, "librouge_b200.so")
REPO_ROOT = os.path.dirname(os.path.dirname(PKG_DIR))
HEADER = os.path.join(REPO_ROOT, "include", "rouge", "numerics_b200.h")

OK = 0
EINVAL = -1
ENODEV = -2
ECUDA = -3
EUNSUPPORTED = -4
ETIMEOUT = -5
ENOMEM = -6
ETOOBIG = -7

B_KN = 0
B_NK = 1
OUT_F32 = 0
OUT_BF16 = 1
OUT_I32 = 2
TILES_AUTO = 0
TILES_SINGLE = 1
TILES_PAIR = 2


class RougeB200Error(RuntimeError):
    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: {status} ({msg})")
        self.status = status


def build() -> None:
    """Compile librouge_b200.so in-tree (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", "-C", os.path.dirname(PKG_DIR), "-j8"], check=True)


_P = C.c_void_p
_I = C.c_int
_F = C.c_float
_SZ = C.c_size_t
_U64 = C.c_uint64


class GemmConfig(C.Structure):
    """RougeGemmConfig (numerics.h:35-41)."""
    _fields_ = [("tile_m", _I), ("tile_n", _I), ("tile_k", _I), ("unroll", _I), ("split_k", _I)]

    def astuple(self):
        return (self.tile_m, self.tile_n, self.tile_k, self.unroll, self.split_k)


class GemmProfile(C.Structure):
    """RougeGemmProfile (numerics.h:44-48)."""
    _fields_ = [("cfg", GemmConfig), ("gflops", C.c_double), ("iters", C.c_longlong)]

_SIGS = {
    "rouge_b200_last_error": (_I, []),
    "rouge_b200_clear_error": (None, []),
    "rouge_b200_status_string": (C.c_char_p, [_I]),
    "rouge_gemm_isa_variant": (C.c_char_p, []),
    "rouge_b200_device_ok": (_I, []),
    "rouge_b200_sync_status": (_I, [_P]),
    "rouge_b200_check_wait_limit": (_I, [C.c_ulonglong, _P]),
    "rouge_b200_w8a8_workspace_bytes": (_SZ, [_I]),
    "rouge_b200_w8a8_linear": (_I, [_I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P]),
    "rouge_b200_set_sm_budget": (_I, [_I]),
    "rouge_b200_set_tile_mode": (_I, [_I]),
    "rouge_b200_set_clock_probe": (_I, [_P, _I]),
    "rouge_quantize_e4m3": (C.c_uint8, [_F]),
    "rouge_dequantize_e4m3": (_F, [C.c_uint8]),
    "rouge_quantize_f16": (C.c_uint16, [_F]),
    "rouge_dequantize_f16": (_F, [C.c_uint16]),
    "rouge_quantize_bf16": (C.c_uint16, [_F]),
    "rouge_dequantize_bf16": (_F, [C.c_uint16]),
    "rouge_quantize_i8_tensor": (_I, [_P, _I, _P, _P]),
    "rouge_quantize_i8_channel": (_I, [_P, _I, _I, _P, _P]),
    "rouge_dequantize_i8_tensor": (None, [_P, _I, _F, _P]),
    "rouge_dequantize_i8_channel": (None, [_P, _I, _I, _P, _P]),
    "rouge_quantize_i8_group": (_I, [_P, _I, _I, _I, _P, _P, _P]),
    "rouge_dequantize_i8_group": (None, [_P, _I, _I, _I, _P, _P, _P]),
    "rouge_b200_quantize_i8_group": (_I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "rouge_b200_dequantize_i8_group": (_I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "rouge_gemm_i8": (None, [_I, _I, _I, _P, _P, _P, _I, _P, _I, _P]),
    "rouge_gemm_i8_noalloc": (_I, [_I, _I, _I, _P, _P, _P, _I, _P, _I, _P]),
    "rouge_gemm_e4m3": (None, [_I, _I, _I, _P, _P, _P, _P]),
    "rouge_gemm_f32": (None, [_I, _I, _I, _P, _P, _P, _P]),
    "rouge_gemm_default_config": (GemmConfig, []),
    "rouge_gemm_candidate_count": (_I, []),
    "rouge_gemm_candidate": (GemmConfig, [_I]),
    "rouge_gemm_flops_per_sec": (C.c_double, [_I, _I, _I, _P, _P, _P, _P]),
    "rouge_gemm_tuned": (GemmProfile, [_I, _I, _I, _P, _P, _P]),
    "rouge_gemm_f16": (None, [_I, _I, _I, _P, _P, _P, _P]),
    "rouge_gemm_bf16": (None, [_I, _I, _I, _P, _P, _P, _P]),
    "rouge_conv2d_f32": (None, [_I] * 9 + [_P, _P, _P, _P, _P]),
    "rouge_conv_implicit_f32": (None, [_I] * 9 + [_P, _P, _P, _P, _P]),
    "rouge_b200_quantize_i8_rows": (_I, [_P, _I, _I, _P, _P, _P]),
    "rouge_b200_dequantize_i8_rows": (_I, [_P, _I, _I, _P, _F, _P, _P]),
    "rouge_b200_absmax_f32": (_I, [_P, _SZ, _P, _P]),
    "rouge_b200_quantize_e4m3_scaled": (_I, [_P, _SZ, _P, _P, _P, _P]),
    "rouge_b200_quantize_e4m3_tensor": (_I, [_P, _SZ, _P, _P, _P, _P]),
    "rouge_b200_mx_quantize": (_I, [_P, _SZ, _I, _P, _P, _P]),
    "rouge_b200_nvfp4_quantize": (_I, [_P, _SZ, C.c_float, _P, _P, _P]),
    "rouge_b200_mx_dequantize": (_I, [_P, _P, _SZ, _I, _P, _P]),
    "rouge_b200_mx_scale_atoms_bytes": (_SZ, [_I, _I]),
    "rouge_b200_mx_scale_atoms": (_I, [_P, _I, _I, _P, _P]),
    "rouge_b200_gemm_mx": (_I, [_I, _I, _I, _P, _I, _P, _P, _I, _P, _P, _I, _I, _P]),
    "rouge_b200_nvfp4_scale_atoms_bytes": (_SZ, [_I, _I]),
    "rouge_b200_nvfp4_scale_atoms": (_I, [_P, _I, _I, _P, _P]),
    "rouge_b200_fp4_pack": (_I, [_P, _SZ, _P, _P]),
    "rouge_b200_nvfp4_quantize_packed": (_I, [_P, _SZ, C.c_float, _P, _P, _P]),
    "rouge_b200_gemm_nvfp4": (_I, [_I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P]),
    "rouge_b200_attention_workspace": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "rouge_b200_attention_gqa": (_I, [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P,
                                      C.c_float, _I, _I, _I, _P, _SZ, _P]),
    "rouge_b200_transformer_block_workspace": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "rouge_b200_transformer_block": (_I, [_I] * 6 + [_P] * 10 + [_I, C.c_float, C.c_float, _P, _P,
                                                                  _SZ, _P]),
    "rouge_b200_mxfp4_scale_atoms_bytes": (_SZ, [_I, _I]),
    "rouge_b200_mxfp4_scale_atoms": (_I, [_P, _I, _I, _P, _P]),
    "rouge_b200_gemm_mxfp4": (_I, [_I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _P]),
    "rouge_quantize_e5m2": (C.c_uint8, [C.c_float]), "rouge_dequantize_e5m2": (C.c_float, [C.c_uint8]),
    "rouge_quantize_e3m2": (C.c_uint8, [C.c_float]), "rouge_dequantize_e3m2": (C.c_float, [C.c_uint8]),
    "rouge_quantize_e2m3": (C.c_uint8, [C.c_float]), "rouge_dequantize_e2m3": (C.c_float, [C.c_uint8]),
    "rouge_quantize_e2m1": (C.c_uint8, [C.c_float]), "rouge_dequantize_e2m1": (C.c_float, [C.c_uint8]),
    "rouge_mx_quantize_f32": (_I, [_P, _I, _I, _P, _P]),
    "rouge_mx_quantize_f32_e2m1": (_I, [_P, _I, _P, _P]),
    "rouge_nvfp4_quantize_f32": (_I, [_P, _I, C.c_float, _P, _P]),
    "rouge_mx_dequantize_f32": (None, [_P, _P, _I, _I, _P]),
    "rouge_mx_dequantize_f32_e2m1": (None, [_P, _P, _I, _P]),
    "rouge_b200_convert_f32_to_f16": (_I, [_P, _SZ, _P, _P]),
    "rouge_b200_convert_f32_to_bf16": (_I, [_P, _SZ, _P, _P]),
    "rouge_b200_convert_e4m3_to_f32": (_I, [_P, _SZ, _P, _P]),
    "rouge_b200_gemm_i8": (_I, [_I, _I, _I, _P, _P, _I, _P, _I, _P, _I, _P, _I, _I, _P]),
    "rouge_b200_gemm_i8_bcast": (_I, [_I, _I, _I, _P, _P, _I, _P, _I, _P, _I, _P, _P, _I,
                                      C.c_longlong, _I, _I, _P]),
    "rouge_b200_gemm_e4m3": (_I, [_I, _I, _I, _P, _P, _I, _P, _P, _P, _I, _I, _P]),
    "rouge_b200_gemm_f16": (_I, [_I, _I, _I, _P, _P, _I, _I, _P, _I, _I, _P]),
    "rouge_b200_conv2d_nhwc_f16": (_I, [_I] * 9 + [_P, _P, _P, _P, _I, _P]),
    "rouge_b200_synth_uniform": (_I, [_U64, _SZ, _F, _F, _P]),
    "rouge_b200_synth_normal": (_I, [_U64, _SZ, _F, _F, _P]),
    "rouge_b200_synth_outliers": (C.c_longlong, [_U64, _SZ, _F, _F, _P]),
    "rouge_b200_synth_normal_at": (_I, [_U64, _SZ, _SZ, _F, _F, _P]),
    "rouge_b200_synth_outliers_at": (C.c_longlong, [_U64, _SZ, _SZ, _F, _F, _P]),
    "rouge_b200_unshard_columns": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded shared library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() or "
                               f"make -C rouge-v_b200")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def declared_symbols() -> list[str]:
    """Names of every function declared in include/rouge/numerics_b200.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rouge_\w+)\s*\(", text)))


def _check(fn: str, status: int) -> None:
    if status != OK:
        msg = lib().rouge_b200_status_string(status).decode()
        raise RougeB200Error(fn, status, msg)


def _stream():
    """The current CUDA stream of the current device, as a handle. torch's
    raw-handle accessor costs ~0.1 us against ~3 us for building a Stream
    object; the public call is the fallback where the accessor is absent."""
    import torch
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return C.c_void_p(raw(torch.cuda.current_device()))
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _hp(a):
    return a.ctypes.data_as(_P)


# ----------------------------------------------------------------- device API

def quantize_i8_rows(x, scales, out):
    _check("rouge_b200_quantize_i8_rows", lib().rouge_b200_quantize_i8_rows(
        _dp(x), x.shape[0], x.shape[1], _dp(scales), _dp(out), _stream()))


def dequantize_i8_rows(q, scales, out, scale=0.0):
    _check("rouge_b200_dequantize_i8_rows", lib().rouge_b200_dequantize_i8_rows(
        _dp(q), q.shape[0], q.shape[1], _dp(scales), scale, _dp(out), _stream()))


def quantize_i8_group(x, groups, scales, zeros, out):
    _check("rouge_b200_quantize_i8_group", lib().rouge_b200_quantize_i8_group(
        _dp(x), x.shape[0], x.shape[1], groups, _dp(scales), _dp(zeros), _dp(out), _stream()))


def dequantize_i8_group(q, groups, scales, zeros, out):
    _check("rouge_b200_dequantize_i8_group", lib().rouge_b200_dequantize_i8_group(
        _dp(q), q.shape[0], q.shape[1], groups, _dp(scales), _dp(zeros), _dp(out), _stream()))


def absmax(x, amax):
    _check("rouge_b200_absmax_f32", lib().rouge_b200_absmax_f32(_dp(x), x.numel(), _dp(amax), _stream()))


def quantize_e4m3_scaled(x, amax, scale_out, out):
    _check("rouge_b200_quantize_e4m3_scaled", lib().rouge_b200_quantize_e4m3_scaled(
        _dp(x), x.numel(), _dp(amax), _dp(scale_out), _dp(out), _stream()))


def quantize_e4m3_tensor(x, amax_out, scale_out, out):
    _check("rouge_b200_quantize_e4m3_tensor", lib().rouge_b200_quantize_e4m3_tensor(
        _dp(x), x.numel(), _dp(amax_out), _dp(scale_out), _dp(out), _stream()))


FMT_E4M3, FMT_E5M2, FMT_E2M1 = 0, 1, 4


def mx_quantize(x, fmt, codes, scales):
    """MXFP8 / MXFP4 block quantization of a flat f32 tensor (blocks of 32)."""
    _check("rouge_b200_mx_quantize", lib().rouge_b200_mx_quantize(
        _dp(x), x.numel(), fmt, _dp(codes), _dp(scales), _stream()))


def nvfp4_quantize(x, global_scale, codes, scales):
    _check("rouge_b200_nvfp4_quantize", lib().rouge_b200_nvfp4_quantize(
        _dp(x), x.numel(), global_scale, _dp(codes), _dp(scales), _stream()))


def mx_dequantize(codes, scales, fmt, out):
    _check("rouge_b200_mx_dequantize", lib().rouge_b200_mx_dequantize(
        _dp(codes), _dp(scales), codes.numel(), fmt, _dp(out), _stream()))


def mx_scale_atoms(scales, rows, K, atoms):
    """[rows][K/32] E8M0 scales -> the tensor-core atom layout of gemm_mx."""
    _check("rouge_b200_mx_scale_atoms", lib().rouge_b200_mx_scale_atoms(
        _dp(scales), rows, K, _dp(atoms), _stream()))


def mx_scale_atoms_bytes(rows, K):
    return lib().rouge_b200_mx_scale_atoms_bytes(rows, K)


def gemm_mx(A, fmt_a, sfa, B, fmt_b, sfb, C, out_type):
    """C[M][N] = (A x 2^sfa) . (B x 2^sfb)^T, A [M][K], B [N][K] e4m3/e5m2 codes."""
    M, K = A.shape
    N = B.shape[0]
    _check("rouge_b200_gemm_mx", lib().rouge_b200_gemm_mx(
        M, N, K, _dp(A), fmt_a, _dp(sfa), _dp(B), fmt_b, _dp(sfb), _dp(C), C.shape[1], out_type,
        _stream()))


def nvfp4_scale_atoms_bytes(rows, K):
    return lib().rouge_b200_nvfp4_scale_atoms_bytes(rows, K)


def nvfp4_scale_atoms(scales, rows, K, atoms):
    """[rows][K/16] UE4M3 scales -> the tensor-core atom layout of gemm_nvfp4."""
    _check("rouge_b200_nvfp4_scale_atoms", lib().rouge_b200_nvfp4_scale_atoms(
        _dp(scales), rows, K, _dp(atoms), _stream()))


def nvfp4_quantize_packed(x, global_scale, packed, scales):
    _check("rouge_b200_nvfp4_quantize_packed", lib().rouge_b200_nvfp4_quantize_packed(
        _dp(x), x.numel(), global_scale, _dp(packed), _dp(scales), _stream()))


def fp4_pack(codes, packed):
    """e2m1 codes (one per byte) -> two per byte, lower index in the low nibble."""
    _check("rouge_b200_fp4_pack", lib().rouge_b200_fp4_pack(
        _dp(codes), codes.numel(), _dp(packed), _stream()))


def gemm_nvfp4(A, sfa, gs_a, B, sfb, gs_b, C, out_type):
    """C[M][N] = gs_a gs_b (A x sfa) . (B x sfb)^T, A [M][K/2], B [N][K/2] packed e2m1."""
    M, K = A.shape[0], 2 * A.shape[1]
    N = B.shape[0]
    _check("rouge_b200_gemm_nvfp4", lib().rouge_b200_gemm_nvfp4(
        M, N, K, _dp(A), _dp(sfa), None if gs_a is None else _dp(gs_a), _dp(B), _dp(sfb),
        None if gs_b is None else _dp(gs_b), _dp(C), C.shape[1], out_type, _stream()))


def mxfp4_scale_atoms_bytes(rows, K):
    return lib().rouge_b200_mxfp4_scale_atoms_bytes(rows, K)


def mxfp4_scale_atoms(scales, rows, K, atoms):
    _check("rouge_b200_mxfp4_scale_atoms", lib().rouge_b200_mxfp4_scale_atoms(
        _dp(scales), rows, K, _dp(atoms), _stream()))


def gemm_mxfp4(A, sfa, B, sfb, C, out_type):
    """C[M][N] = (A x 2^sfa) . (B x 2^sfb)^T, A [M][K/2], B [N][K/2] packed e2m1."""
    M, K = A.shape[0], 2 * A.shape[1]
    N = B.shape[0]
    _check("rouge_b200_gemm_mxfp4", lib().rouge_b200_gemm_mxfp4(
        M, N, K, _dp(A), _dp(sfa), _dp(B), _dp(sfb), _dp(C), C.shape[1], out_type, _stream()))


def attention_gqa(Q, K, V, O, scale=0.0, causal=1, window=0, kv_off=0, Kq=None, Vq=None,
                  scales_k=None, scales_v=None, workspace=None):
    """O[Hq][S][Dh] from Q[Hq][S][Dh] and K/V[Hkv][Skv][Dh] (f32, or e4m3 Kq/Vq with
    per-head scales); workspace: a uint8 tensor of attention_workspace() bytes."""
    Hq, S, Dh = Q.shape
    src = K if Kq is None else Kq
    Hkv, Skv = src.shape[0], src.shape[1]
    if workspace is None:
        import torch
        workspace = torch.empty(attention_workspace(S, Skv, Dh, Hq, Hkv, Kq is not None),
                                dtype=torch.uint8, device=Q.device)
    d = lambda t: None if t is None else _dp(t)  # noqa: E731
    _check("rouge_b200_attention_gqa", lib().rouge_b200_attention_gqa(
        S, Skv, Dh, Hq, Hkv, _dp(Q), d(K), d(V), d(Kq), d(Vq), d(scales_k), d(scales_v), _dp(O),
        scale, causal, window, kv_off, _dp(workspace), workspace.numel(), _stream()))


def attention_workspace(S, Skv, Dh, Hq, Hkv, fp8_kv=False):
    return lib().rouge_b200_attention_workspace(S, Skv, Dh, Hq, Hkv, int(bool(fp8_kv)))


def transformer_block_workspace(S, D, Hq, Hkv, Dq, Dff):
    return lib().rouge_b200_transformer_block_workspace(S, D, Hq, Hkv, Dq, Dff)


def transformer_block(x, wrms1, wq, wk, wv, wo, wrms2, wgate, wup, wdown, Hq, Hkv, Dq, out,
                      rope_theta=10000.0, rms_eps=1e-5, workspace=None):
    S, D = x.shape
    Dff = wgate.shape[1]
    if workspace is None:
        import torch
        workspace = torch.empty(transformer_block_workspace(S, D, Hq, Hkv, Dq, Dff),
                                dtype=torch.uint8, device=x.device)
    _check("rouge_b200_transformer_block", lib().rouge_b200_transformer_block(
        S, D, Hq, Hkv, Dq, Dq, _dp(x), _dp(wrms1), _dp(wq), _dp(wk), _dp(wv), _dp(wo), _dp(wrms2),
        _dp(wgate), _dp(wup), _dp(wdown), Dff, rope_theta, rms_eps, _dp(out), _dp(workspace),
        workspace.numel(), _stream()))


def convert_f32_to_f16(x, out):
    _check("rouge_b200_convert_f32_to_f16", lib().rouge_b200_convert_f32_to_f16(
        _dp(x), x.numel(), _dp(out), _stream()))


def convert_f32_to_bf16(x, out):
    _check("rouge_b200_convert_f32_to_bf16", lib().rouge_b200_convert_f32_to_bf16(
        _dp(x), x.numel(), _dp(out), _stream()))


def convert_e4m3_to_f32(x, out):
    _check("rouge_b200_convert_e4m3_to_f32", lib().rouge_b200_convert_e4m3_to_f32(
        _dp(x), x.numel(), _dp(out), _stream()))


def gemm_i8(A, B, b_layout, C_, out_type, scales_a=None, a_rows=1, scales_b=None, b_cols=1):
    M, K = A.shape
    N = B.shape[1] if b_layout == B_KN else B.shape[0]
    _check("rouge_b200_gemm_i8", lib().rouge_b200_gemm_i8(
        M, N, K, _dp(A), _dp(B), b_layout, _dp(scales_a), a_rows, _dp(scales_b), b_cols,
        _dp(C_), C_.stride(0), out_type, _stream()))


def gemm_i8_bcast(A, B, b_layout, out_type, scales_a, a_rows, scales_b, b_cols, mc_ptr=0,
                  peer_ptrs=(), ldc=0, col_off=0):
    """rouge_b200_gemm_i8_bcast: this rank's M x N block written to column
    col_off of every rank's [M][ldc] output, through the multicast address
    mc_ptr (an int) or the list of peer pointers peer_ptrs (ints)."""
    M, K = A.shape
    N = B.shape[0] if b_layout == B_NK else B.shape[1]
    peers = (C.c_void_p * 8)(*[C.c_void_p(p) for p in peer_ptrs]) if not mc_ptr else None
    _check("rouge_b200_gemm_i8_bcast", lib().rouge_b200_gemm_i8_bcast(
        M, N, K, _dp(A), _dp(B), b_layout, _dp(scales_a), a_rows, _dp(scales_b), b_cols,
        C.c_void_p(mc_ptr) if mc_ptr else None, peers, 0 if mc_ptr else len(peer_ptrs), ldc,
        col_off, out_type, _stream()))


def w8a8_workspace(M, device):
    """Zeroed workspace of rouge_b200_w8a8_linear for M rows (every call
    leaves it zeroed)."""
    import torch
    n = lib().rouge_b200_w8a8_workspace_bytes(M)
    return torch.zeros((n + 3) // 4, dtype=torch.int32, device=device)


def w8a8_linear(X, Wq, sw, Aq, sa, C_, out_type, ws):
    """Aq, sa = per-row int8 quantization of X[M][K]; C = dequant(Aq . Wq^T)
    with Wq[N][K] codes and sw[N] scales (one fused launch when it applies)."""
    M, K = X.shape
    N = Wq.shape[0]
    _check("rouge_b200_w8a8_linear", lib().rouge_b200_w8a8_linear(
        M, N, K, _dp(X), _dp(Wq), _dp(sw), _dp(Aq), _dp(sa), _dp(C_), C_.stride(0), out_type,
        _dp(ws), _stream()))


def gemm_e4m3(A, B, b_layout, C_, out_type, scale_a=None, scale_b=None):
    M, K = A.shape
    N = B.shape[1] if b_layout == B_KN else B.shape[0]
    _check("rouge_b200_gemm_e4m3", lib().rouge_b200_gemm_e4m3(
        M, N, K, _dp(A), _dp(B), b_layout, _dp(scale_a), _dp(scale_b), _dp(C_), C_.stride(0),
        out_type, _stream()))


def gemm_f16(A, B, b_layout, C_, out_type, is_bf16=False):
    M, K = A.shape
    N = B.shape[1] if b_layout == B_KN else B.shape[0]
    _check("rouge_b200_gemm_f16", lib().rouge_b200_gemm_f16(
        M, N, K, _dp(A), _dp(B), b_layout, int(is_bf16), _dp(C_), C_.stride(0), out_type,
        _stream()))


def conv2d_nhwc_f16(X, Wt, bias, Y, stride, pad, is_bf16=False):
    """X[N][H][W][Cin], Wt[Cout][KH][KW][Cin] (16-bit codes), Y[N][OH][OW][Cout] f32."""
    N, H, W, Cin = X.shape
    Cout, KH, KW, _ = Wt.shape
    _check("rouge_b200_conv2d_nhwc_f16", lib().rouge_b200_conv2d_nhwc_f16(
        N, H, W, Cin, Cout, KH, KW, stride, pad, _dp(X), _dp(Wt), _dp(bias), _dp(Y),
        int(is_bf16), _stream()))


def sync_status():
    _check("rouge_b200_sync_status", lib().rouge_b200_sync_status(_stream()))


def check_wait_limit(limit_ns):
    """Launches the never-completing bounded wait (limit_ns) on the current
    stream and returns the status rouge_b200_sync_status then reports
    (ROUGE_B200_ETIMEOUT when the limit works)."""
    L = lib()
    _check("rouge_b200_check_wait_limit", L.rouge_b200_check_wait_limit(int(limit_ns), _stream()))
    return L.rouge_b200_sync_status(_stream())


class tile_mode:
    """Context manager selecting the GEMM / convolution tile shapes
    (TILES_AUTO, TILES_SINGLE or TILES_PAIR) and restoring the previous mode."""

    def __init__(self, mode: int):
        self.mode = mode

    def __enter__(self):
        prev = lib().rouge_b200_set_tile_mode(self.mode)
        if prev < 0:
            raise RougeB200Error("rouge_b200_set_tile_mode", prev, "unknown mode")
        self.prev = prev
        return self

    def __exit__(self, *exc):
        lib().rouge_b200_set_tile_mode(self.prev)
        return False


class clock_probe:
    """Context manager recording, for every GEMM / convolution launch on the
    current device while it is active, each of the first `ctas` CTAs'
    %clock64 and %globaltimer at its start and end
    (rouge_b200_set_clock_probe). After the launch of interest,
    `sm_mhz()` gives the SM clock each CTA ran at, from those stamps."""

    def __init__(self, ctas: int, device=None):
        import torch
        self.ctas = int(ctas)
        self.stamps = torch.zeros(4 * self.ctas, dtype=torch.int64, device=device or "cuda")

    def __enter__(self):
        _check("rouge_b200_set_clock_probe",
               lib().rouge_b200_set_clock_probe(_dp(self.stamps), self.ctas))
        return self

    def __exit__(self, *exc):
        lib().rouge_b200_set_clock_probe(None, 0)
        return False

    def sm_mhz(self):
        """Per-CTA SM clock in MHz of the last launch (CTAs that wrote no
        stamps are left out)."""
        import numpy as np
        w = self.stamps.view(-1, 4).cpu().numpy().astype(np.float64)
        ok = (w[:, 3] > w[:, 1]) & (w[:, 2] > w[:, 0])
        return (w[ok, 2] - w[ok, 0]) / (w[ok, 3] - w[ok, 1]) * 1000.0


# ------------------------------------------------------------- host drop-in API

def _last_error(fn):
    st = lib().rouge_b200_last_error()
    lib().rouge_b200_clear_error()
    if st != OK:
        raise RougeB200Error(fn, st, lib().rouge_b200_status_string(st).decode())


def host_quantize_i8_channel(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    s = np.empty(rows, np.float32)
    q = np.empty((rows, cols), np.int8)
    lib().rouge_b200_clear_error()
    if lib().rouge_quantize_i8_channel(_hp(x), rows, cols, _hp(s), _hp(q)) != 1:
        _last_error("rouge_quantize_i8_channel")
        raise RougeB200Error("rouge_quantize_i8_channel", EINVAL, "returned 0")
    return q, s


def host_quantize_i8_tensor(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32).ravel()
    s = np.zeros(1, np.float32)
    q = np.empty(x.size, np.int8)
    lib().rouge_b200_clear_error()
    if lib().rouge_quantize_i8_tensor(_hp(x), x.size, _hp(s), _hp(q)) != 1:
        _last_error("rouge_quantize_i8_tensor")
        raise RougeB200Error("rouge_quantize_i8_tensor", EINVAL, "returned 0")
    return q, float(s[0])


def host_quantize_i8_group(x: np.ndarray, groups: int):
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    s = np.empty(rows * groups, np.float32)
    z = np.empty(rows * groups, np.uint8)
    q = np.empty((rows, cols), np.uint8)
    lib().rouge_b200_clear_error()
    if lib().rouge_quantize_i8_group(_hp(x), rows, cols, groups, _hp(s), _hp(z), _hp(q)) != 1:
        _last_error("rouge_quantize_i8_group")
        raise RougeB200Error("rouge_quantize_i8_group", EINVAL, "returned 0")
    return q, s, z


def host_dequantize_i8_group(q: np.ndarray, groups: int, s: np.ndarray, z: np.ndarray):
    q = np.ascontiguousarray(q, np.uint8)
    s = np.ascontiguousarray(s, np.float32)
    z = np.ascontiguousarray(z, np.uint8)
    out = np.empty(q.shape, np.float32)
    lib().rouge_b200_clear_error()
    lib().rouge_dequantize_i8_group(_hp(q), q.shape[0], q.shape[1], groups, _hp(s), _hp(z), _hp(out))
    _last_error("rouge_dequantize_i8_group")
    return out


def host_dequantize_i8_channel(q: np.ndarray, scales: np.ndarray):
    q = np.ascontiguousarray(q, np.int8)
    scales = np.ascontiguousarray(scales, np.float32)
    out = np.empty(q.shape, np.float32)
    lib().rouge_b200_clear_error()
    lib().rouge_dequantize_i8_channel(_hp(q), q.shape[0], q.shape[1], _hp(scales), _hp(out))
    _last_error("rouge_dequantize_i8_channel")
    return out


def host_dequantize_i8_tensor(q: np.ndarray, scale: float):
    q = np.ascontiguousarray(q, np.int8).ravel()
    out = np.empty(q.size, np.float32)
    lib().rouge_b200_clear_error()
    lib().rouge_dequantize_i8_tensor(_hp(q), q.size, scale, _hp(out))
    _last_error("rouge_dequantize_i8_tensor")
    return out


def host_gemm_i8(A, B_kn, sa, a_rows, sb, b_cols, out=None):
    A = np.ascontiguousarray(A, np.int8)
    B_kn = np.ascontiguousarray(B_kn, np.int8)
    sa = np.ascontiguousarray(np.atleast_1d(sa), np.float32)
    sb = np.ascontiguousarray(np.atleast_1d(sb), np.float32)
    M, K = A.shape
    N = B_kn.shape[1]
    out = np.empty((M, N), np.float32) if out is None else out
    lib().rouge_b200_clear_error()
    lib().rouge_gemm_i8(M, N, K, _hp(A), _hp(B_kn), _hp(sa), a_rows, _hp(sb), b_cols, _hp(out))
    _last_error("rouge_gemm_i8")
    return out


def _host_gemm_codes(name, A, B_kn, dtype):
    A = np.ascontiguousarray(A, dtype)
    B_kn = np.ascontiguousarray(B_kn, dtype)
    M, K = A.shape
    N = B_kn.shape[1]
    out = np.empty((M, N), np.float32)
    lib().rouge_b200_clear_error()
    getattr(lib(), name)(M, N, K, _hp(A), _hp(B_kn), _hp(out), None)
    _last_error(name)
    return out


def host_gemm_e4m3(A, B_kn):
    return _host_gemm_codes("rouge_gemm_e4m3", A, B_kn, np.uint8)


def host_gemm_f32(A, B_kn, cfg=None, out=None):
    """rouge_gemm_f32: A[M][K] . B[K][N] (f32, host arrays); cfg a
    GemmConfig or None."""
    A = np.ascontiguousarray(A, np.float32)
    B_kn = np.ascontiguousarray(B_kn, np.float32)
    M, K = A.shape
    N = B_kn.shape[1]
    out = np.empty((M, N), np.float32) if out is None else out
    lib().rouge_b200_clear_error()
    lib().rouge_gemm_f32(M, N, K, _hp(A), _hp(B_kn), _hp(out),
                         None if cfg is None else C.cast(C.pointer(cfg), _P))
    _last_error("rouge_gemm_f32")
    return out


def gemm_candidates():
    """The tuner's candidate configurations (rouge_gemm_candidate)."""
    return [lib().rouge_gemm_candidate(i) for i in range(lib().rouge_gemm_candidate_count())]


def gemm_tuned(A, B_kn, out):
    """rouge_gemm_tuned on host arrays; returns the GemmProfile."""
    M, K = A.shape
    N = B_kn.shape[1]
    return lib().rouge_gemm_tuned(M, N, K, _hp(A), _hp(B_kn), _hp(out))


def gemm_flops_per_sec(A, B_kn, out, cfg=None):
    M, K = A.shape
    N = B_kn.shape[1]
    return lib().rouge_gemm_flops_per_sec(M, N, K, _hp(A), _hp(B_kn), _hp(out),
                                          None if cfg is None else C.cast(C.pointer(cfg), _P))


def host_conv2d_f32(x, w, bias, stride, pad, implicit=False):
    """rouge_conv2d_f32 / rouge_conv_implicit_f32: x[N][Cin][H][W],
    w[Cout][Cin][KH][KW], bias[Cout] or None; returns y[N][Cout][OH][OW]."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    N, Cin, H, W = x.shape
    Cout, _, KH, KW = w.shape
    OH = (H + 2 * pad - KH) // stride + 1
    OW = (W + 2 * pad - KW) // stride + 1
    y = np.full((N, Cout, OH, OW), np.nan, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    fn = lib().rouge_conv_implicit_f32 if implicit else lib().rouge_conv2d_f32
    lib().rouge_b200_clear_error()
    fn(N, Cin, H, W, Cout, KH, KW, stride, pad, _hp(x), _hp(w), None if b is None else _hp(b),
       _hp(y), None)
    _last_error("rouge_conv_implicit_f32" if implicit else "rouge_conv2d_f32")
    return y


def host_gemm_f16(A, B_kn):
    return _host_gemm_codes("rouge_gemm_f16", A, B_kn, np.uint16)


def host_gemm_bf16(A, B_kn):
    return _host_gemm_codes("rouge_gemm_bf16", A, B_kn, np.uint16)


# ------------------------------------------------------------------ synthetic data

def synth_uniform(seed: int, shape, lo: float, hi: float, out=None) -> np.ndarray:
    out = np.empty(shape, np.float32) if out is None else out
    assert lib().rouge_b200_synth_uniform(seed, out.size, lo, hi, _hp(out)) == 0
    return out


def synth_normal(seed: int, shape, mean: float, std: float, out=None) -> np.ndarray:
    out = np.empty(shape, np.float32) if out is None else out
    assert lib().rouge_b200_synth_normal(seed, out.size, mean, std, _hp(out)) == 0
    return out


def synth_outliers(seed: int, x: np.ndarray, frac: float, mult: float, offset: int = 0) -> int:
    return int(lib().rouge_b200_synth_outliers_at(seed, offset, x.size, frac, mult, _hp(x)))


def synth_normal_at(seed: int, offset: int, shape, mean: float, std: float) -> np.ndarray:
    out = np.empty(shape, np.float32)
    assert lib().rouge_b200_synth_normal_at(seed, offset, out.size, mean, std, _hp(out)) == 0
    return out


def unshard_columns(src, dst, M, N, g, ns, R):
    """src[M/R][g][R][ns] (all-gathered bands) -> dst[M][ldd] row-major."""
    _check("rouge_b200_unshard_columns", lib().rouge_b200_unshard_columns(
        _dp(src), _dp(dst), M, N, g, ns, R, dst.stride(0), src.element_size(), _stream()))
