"""BASELINE configs 3 and 5 at their full sizes on the GPU, through the C
ABI, against the oracle.

Config 3: e4m3 codes of an 8192 x 8192 N(0,1) operand under its per-tensor
absmax scale, bit-exact over the whole tensor (fp8.cpp:75-106 with
s = amax / 448, tests/test_ai.cpp:225-231), then the 8192^3 e4m3 GEMM with
bf16 output (B in the reference's [K][N] layout) within 1e-2 relative L2 on
sampled rows.

Config 5: the GEMM one rank of eight computes (M=16384, K=8192, its 3584
output columns of N=28672) through the broadcast-epilogue kernel the fused
sharded path runs, with this GPU's own full-width C as the only
destination: every column of the shard bit-exact on rows at both ends and
at the 128/256/2048-row band edges, columns of the other shards untouched."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_config3_codes_whole_tensor_and_gemm(rb, orc, cuda):
    n = 8192
    A = rb.synth_normal(3, (n, n), 0.0, 1.0)
    B = rb.synth_normal(4, (n, n), 0.0, 1.0)
    ad, bd = torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)
    qa = torch.empty((n, n), dtype=torch.uint8, device=cuda)
    qb = torch.empty((n, n), dtype=torch.uint8, device=cuda)
    sc = torch.zeros(4, dtype=torch.float32, device=cuda)  # amaxA, sA, amaxB, sB
    rb.quantize_e4m3_tensor(ad, sc[0:1], sc[1:2], qa)
    rb.quantize_e4m3_tensor(bd, sc[2:3], sc[3:4], qb)
    rb.sync_status()
    del ad, bd
    oa, sa, amax_a = orc.quantize_e4m3_tensor(A)
    got = qa.cpu().numpy()
    bad = np.count_nonzero(got != oa)
    assert bad == 0, f"{bad} of {n * n} e4m3 codes differ"
    assert np.float32(sc[0].item()) == np.float32(amax_a)
    assert np.float32(sc[1].item()).view(np.uint32) == np.float32(sa).view(np.uint32)
    ob, sb, _ = orc.quantize_e4m3_tensor(B)
    assert (qb.cpu().numpy() == ob).all()
    del A, B
    c = torch.empty((n, n), dtype=torch.int16, device=cuda)
    qb_kn = qb.t().contiguous()                      # the reference's B[K][N] layout
    rb.gemm_e4m3(qa, qb_kn, rb.B_KN, c, rb.OUT_BF16, sc[1:2], sc[3:4])
    rb.sync_status()
    rows = np.array([0, 1, 127, 128, 255, 256, 4095, 8191], np.int32)
    want = orc.gemm_f32(orc.e4m3_decode(oa[rows]), orc.e4m3_decode(ob), True) * \
        np.float32(np.float32(sa) * np.float32(sb))
    gotb = orc.bf16_decode(c[rows.tolist()].cpu().numpy().view(np.uint16))
    err = np.linalg.norm(gotb - want) / np.linalg.norm(want)
    assert err <= 1e-2, err


def test_config5_one_rank_shard_full_size(rb, orc, cuda):
    from rouge_b200.sharded import shard_columns
    M, N, K, g, r = 16384, 28672, 8192, 8, 3
    ns, ranges = shard_columns(N, g)
    n0, n1 = ranges[r]
    assert n1 - n0 == ns == 3584
    x = rb.synth_normal(8, (M, K), 0.0, 1.0)
    rb.synth_outliers(8, x, 0.01, 20.0)
    xd = torch.from_numpy(x).to(cuda)
    del x
    qx = torch.empty((M, K), dtype=torch.int8, device=cuda)
    sx = torch.empty(M, dtype=torch.float32, device=cuda)
    rb.quantize_i8_rows(xd, sx, qx)
    del xd
    wd = torch.from_numpy(rb.synth_normal_at(9, n0 * K, (ns, K), 0.0, 0.02)).to(cuda)
    qw = torch.empty((ns, K), dtype=torch.int8, device=cuda)
    sw = torch.empty(ns, dtype=torch.float32, device=cuda)
    rb.quantize_i8_rows(wd, sw, qw)
    del wd
    out = torch.full((M, N), 0x7B7B, dtype=torch.int16, device=cuda)  # sentinel
    rb.gemm_i8_bcast(qx, qw, rb.B_NK, rb.OUT_BF16, sx, 1, sw, 1, peer_ptrs=(out.data_ptr(),),
                     ldc=N, col_off=n0)
    rb.sync_status()
    rows = np.array([0, 1, 127, 128, 255, 256, 2047, 2048, 8191, 8192, 16127, 16128, 16383],
                    np.int32)
    _, c = orc.gemm_i8(qx[rows.tolist()].cpu().numpy(), qw.cpu().numpy(), True,
                       sx[rows.tolist()].cpu().numpy(), 1, sw.cpu().numpy(), 1)
    got = out[rows.tolist()].cpu().numpy().view(np.uint16)
    assert (got[:, n0:n1] == orc.bf16_encode(c)).all()
    assert (got[:, :n0] == 0x7B7B).all() and (got[:, n1:] == 0x7B7B).all()
    # every row written: the shard's column block holds no sentinel left
    assert not bool((out[:, n0:n1] == 0x7B7B).all(dim=1).any())
