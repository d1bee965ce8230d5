"""Block-scaled MXFP8 and NVFP4 GEMMs (tcgen05 kind::mxf8f6f4 / mxf4nvf4
.block_scale, CTA pairs)
against the oracle: operands quantized by the MX block quantizer (bit-exact
with the reference), decoded exactly by the oracle (narrow.cpp:304-331) and
multiplied in double. The tensor cores multiply exactly and accumulate in
f32, so the relative L2 error is bounded by f32 accumulation (<= 1e-5).
Also checks the scale-atom layout against its definition."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FMT = {"e4m3": 0, "e5m2": 1}


def _quantize(rb, torch, x, fmt, cuda):
    rows, K = x.shape
    q = torch.empty((rows, K), dtype=torch.uint8, device=cuda)
    s = torch.empty((rows, K // 32), dtype=torch.uint8, device=cuda)
    rb.mx_quantize(x, FMT[fmt], q, s)
    atoms = torch.empty(rb.mx_scale_atoms_bytes(rows, K), dtype=torch.uint8, device=cuda)
    rb.mx_scale_atoms(s, rows, K, atoms)
    return q, s, atoms


def test_scale_atom_layout(rb, cuda):
    import torch
    rows, K = 300, 416
    s = torch.randint(0, 255, (rows, K // 32), dtype=torch.uint8, device=cuda)
    atoms = torch.empty(rb.mx_scale_atoms_bytes(rows, K), dtype=torch.uint8, device=cuda)
    rb.mx_scale_atoms(s, rows, K, atoms)
    a = atoms.cpu().numpy().reshape(-1, 512)
    sh = s.cpu().numpy()
    kb128 = (K + 127) // 128
    for rb_ in range((rows + 127) // 128):
        for kb in range(kb128):
            atom = a[rb_ * kb128 + kb]
            for r in range(128):
                for j in range(4):
                    row, col = rb_ * 128 + r, kb * 4 + j
                    want = sh[row, col] if row < rows and col < K // 32 else 127
                    assert atom[16 * (r % 32) + 4 * (r // 32) + j] == want


# (4096, 4096, 256): 256 tiles on 74 CTA pairs, the last round's 34 tiles cut
# into 68 half-width units: full tiles and units share one launch
@pytest.mark.parametrize("M,N,K", [(256, 128, 128), (512, 256, 1024), (300, 200, 96),
                                   (1000, 384, 544), (2048, 2048, 4096), (4096, 4096, 256)])
@pytest.mark.parametrize("fa,fb", [("e4m3", "e4m3"), ("e5m2", "e5m2"), ("e4m3", "e5m2")])
def test_gemm_mx_against_oracle(rb, orc, cuda, M, N, K, fa, fb):
    import torch
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    # rows and K-blocks of very different magnitudes exercise the scales
    xa = torch.randn((M, K), device=cuda, generator=g) * torch.exp2(
        torch.randint(-8, 9, (M, K // 32), device=cuda, generator=g).float()).repeat_interleave(32, 1)
    xb = torch.randn((N, K), device=cuda, generator=g) * torch.exp2(
        torch.randint(-8, 9, (N, 1), device=cuda, generator=g).float())
    qa, sa, ta = _quantize(rb, torch, xa, fa, cuda)
    qb, sb, tb = _quantize(rb, torch, xb, fb, cuda)
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    rb.gemm_mx(qa, FMT[fa], ta, qb, FMT[fb], tb, C, rb.OUT_F32)
    rb.sync_status()
    A = orc.mx_dequantize(qa.cpu().numpy(), sa.cpu().numpy(), fa).reshape(M, K).astype(np.float64)
    B = orc.mx_dequantize(qb.cpu().numpy(), sb.cpu().numpy(), fb).reshape(N, K).astype(np.float64)
    rows = np.unique(np.linspace(0, M - 1, min(M, 64)).astype(int))
    want = A[rows] @ B.T
    got = C.cpu().numpy()[rows].astype(np.float64)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-5, err


def test_gemm_mx_bf16_out(rb, orc, cuda):
    import torch
    M, N, K = 512, 256, 512
    xa = torch.randn((M, K), device=cuda)
    xb = torch.randn((N, K), device=cuda)
    qa, sa, ta = _quantize(rb, torch, xa, "e4m3", cuda)
    qb, sb, tb = _quantize(rb, torch, xb, "e4m3", cuda)
    C = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    rb.gemm_mx(qa, 0, ta, qb, 0, tb, C, rb.OUT_BF16)
    A = orc.mx_dequantize(qa.cpu().numpy(), sa.cpu().numpy(), "e4m3").reshape(M, K).astype(np.float64)
    B = orc.mx_dequantize(qb.cpu().numpy(), sb.cpu().numpy(), "e4m3").reshape(N, K).astype(np.float64)
    want = A @ B.T
    got = C.float().cpu().numpy()
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 4e-3


def _nvfp4(rb, torch, x, gs, cuda):
    rows, K = x.shape
    q = torch.empty((rows, K), dtype=torch.uint8, device=cuda)
    s = torch.empty((rows, K // 16), dtype=torch.uint8, device=cuda)
    rb.nvfp4_quantize(x, gs, q, s)
    packed = torch.empty((rows, K // 2), dtype=torch.uint8, device=cuda)
    rb.fp4_pack(q, packed)
    atoms = torch.empty(rb.nvfp4_scale_atoms_bytes(rows, K), dtype=torch.uint8, device=cuda)
    rb.nvfp4_scale_atoms(s, rows, K, atoms)
    return q, s, packed, atoms


def _nvfp4_decode(orc, q, s, gs, rows, K):
    """x = e2m1(q) * e4m3(scale) * gs (narrow.cpp:270-300: codes of x / (scale gs))."""
    v = orc.narrow_decode(q.cpu().numpy().ravel(), "e2m1").astype(np.float64)
    sc = orc.narrow_decode(s.cpu().numpy().ravel(), "e4m3").astype(np.float64)
    return (v.reshape(rows, K // 16, 16) * sc.reshape(rows, K // 16, 1)).reshape(rows, K) * gs


def test_fp4_pack(rb, cuda):
    import torch
    c = torch.randint(0, 16, (4096,), dtype=torch.uint8, device=cuda)
    p = torch.empty(2048, dtype=torch.uint8, device=cuda)
    rb.fp4_pack(c, p)
    ch = c.cpu().numpy()
    assert (p.cpu().numpy() == (ch[0::2] | (ch[1::2] << 4))).all()


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (512, 256, 1024), (300, 200, 96),
                                   (1000, 384, 544), (2048, 2048, 4096), (4096, 4096, 512)])
@pytest.mark.parametrize("gsa,gsb", [(1.0, 1.0), (0.37, 4.0)])
def test_gemm_nvfp4_against_oracle(rb, orc, cuda, M, N, K, gsa, gsb):
    import torch
    g = torch.Generator(device=cuda).manual_seed(M + 3 * N + K)
    xa = torch.randn((M, K), device=cuda, generator=g) * torch.exp2(
        torch.randint(-6, 7, (M, K // 16), device=cuda, generator=g).float()).repeat_interleave(16, 1)
    xb = torch.randn((N, K), device=cuda, generator=g)
    qa, sa, pa, ta = _nvfp4(rb, torch, xa, gsa, cuda)
    qb, sb, pb, tb = _nvfp4(rb, torch, xb, gsb, cuda)
    ga = torch.tensor([gsa], device=cuda)
    gb = torch.tensor([gsb], device=cuda)
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    rb.gemm_nvfp4(pa, ta, ga, pb, tb, gb, C, rb.OUT_F32)
    rb.sync_status()
    rows = np.unique(np.linspace(0, M - 1, min(M, 64)).astype(int))
    A = _nvfp4_decode(orc, qa[rows.tolist()], sa[rows.tolist()], gsa, rows.size, K)
    B = _nvfp4_decode(orc, qb, sb, gsb, N, K)
    want = A @ B.T
    got = C.cpu().numpy()[rows].astype(np.float64)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-5, err


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (512, 256, 1024), (300, 200, 96),
                                   (1000, 384, 544), (4096, 4096, 512)])
def test_gemm_mxfp4_against_oracle(rb, orc, cuda, M, N, K):
    import torch
    g = torch.Generator(device=cuda).manual_seed(M + 5 * N + K)
    xa = torch.randn((M, K), device=cuda, generator=g) * torch.exp2(
        torch.randint(-6, 7, (M, K // 32), device=cuda, generator=g).float()).repeat_interleave(32, 1)
    xb = torch.randn((N, K), device=cuda, generator=g)
    out = []
    for x, rows in ((xa, M), (xb, N)):
        q = torch.empty((rows, K), dtype=torch.uint8, device=cuda)
        s = torch.empty((rows, K // 32), dtype=torch.uint8, device=cuda)
        rb.mx_quantize(x, rb.FMT_E2M1, q, s)
        p = torch.empty((rows, K // 2), dtype=torch.uint8, device=cuda)
        rb.fp4_pack(q, p)
        t = torch.empty(rb.mxfp4_scale_atoms_bytes(rows, K), dtype=torch.uint8, device=cuda)
        rb.mxfp4_scale_atoms(s, rows, K, t)
        out.append((q, s, p, t))
    (qa, sa, pa, ta), (qb, sb, pb, tb) = out
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    rb.gemm_mxfp4(pa, ta, pb, tb, C, rb.OUT_F32)
    rb.sync_status()
    rows = np.unique(np.linspace(0, M - 1, min(M, 64)).astype(int))
    A = orc.mx_dequantize(qa[rows.tolist()].cpu().numpy(), sa[rows.tolist()].cpu().numpy(),
                          "e2m1").reshape(rows.size, K).astype(np.float64)
    B = orc.mx_dequantize(qb.cpu().numpy(), sb.cpu().numpy(), "e2m1").reshape(N, K).astype(np.float64)
    want = A @ B.T
    got = C.cpu().numpy()[rows].astype(np.float64)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-5, err
