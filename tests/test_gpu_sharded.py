"""GPU side of the N-sharded W8A8 GEMM: the unshard
kernel, a one-GPU run of the whole path, and (with two or more GPUs) a
two-rank NCCL run. Outputs are bf16 codes of ((float)acc*sa)*sb and must
equal the oracle bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_unshard_columns(rb, cuda):
    nb, g, R, ns = 3, 4, 128, 48
    M, N = nb * R, g * ns - 8
    src = torch.randint(-30000, 30000, (nb, g, R, ns), dtype=torch.int16, device=cuda)
    dst = torch.full((M, N + 8), 7, dtype=torch.int16, device=cuda)
    rb.unshard_columns(src, dst, M, N, g, ns, R)   # ldd = N + 8
    rb.sync_status()
    want = src.permute(0, 2, 1, 3).reshape(M, g * ns)[:, :N]
    assert torch.equal(dst[:, :N], want)
    assert (dst[:, N:] == 7).all()   # columns past N untouched


def _problem(M, N, K, seed=11):
    rng = np.random.default_rng(seed)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sa = rng.uniform(1e-3, 1e-2, M).astype(np.float32)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    return A, W, sa, sw


def _run_rank(rank, world, device, M, N, K, R):
    from rouge_b200.sharded import ShardedW8A8
    A, W, sa, sw = _problem(M, N, K)
    sh = ShardedW8A8(M, N, K, rank, world, device, R=R)
    n0, n1 = sh.columns
    w_shard = np.zeros((sh.ns, K), np.int8)
    w_shard[: n1 - n0] = W[n0:n1]
    sw_shard = np.zeros(sh.ns, np.float32)
    sw_shard[: n1 - n0] = sw[n0:n1]
    d = torch.device(device)
    out = sh(torch.from_numpy(A).to(d), torch.from_numpy(sa).to(d), torch.from_numpy(w_shard).to(d),
             torch.from_numpy(sw_shard).to(d))
    torch.cuda.synchronize(d)
    return out.view(torch.int16).cpu().numpy().view(np.uint16), (A, W, sa, sw)


def test_sharded_one_gpu(rb, orc, cuda):
    got, (A, W, sa, sw) = _run_rank(0, 1, "cuda:0", 512, 1024, 512, 128)
    rb.sync_status()
    _, c = orc.gemm_i8(A, W, True, sa, 1, sw, 1)
    assert (got == orc.bf16_encode(c)).all()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_rank(rank, world, port, M, N, K, R, q):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [here, os.path.join(root, "rouge-v_b200"), os.path.join(root, "oracle")]
    import torch.distributed as dist
    import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        got, (A, W, sa, sw) = _run_rank(rank, world, f"cuda:{rank}", M, N, K, R)
        orc = O.Oracle()
        rows = np.arange(0, M, 37, dtype=np.int32)
        _, c = orc.gemm_i8(A, W, True, sa, 1, sw, 1, rows=rows)
        q.put((rank, bool((got[rows] == orc.bf16_encode(c)).all())))
    finally:
        dist.destroy_process_group()


def test_sharded_two_gpus(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    args = (world, port, 1024, 2048, 1024, 256, q)
    procs = [ctx.Process(target=_nccl_rank, args=(r,) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert all(res.values()), res


# ------------------------------------------------------ all-gather fused into the GEMM

def test_gemm_bcast_peer_stores_one_gpu(rb, orc, cuda):
    # rouge_b200_gemm_i8_bcast through its peer-pointer form with two
    # destinations on this GPU: both receive the block at column col_off,
    # bit-exact, and nothing outside it is written.
    M, N, K, ldc, col_off = 384, 96, 256, 256, 64
    A, W, sa, sw = _problem(M, N, K, seed=5)
    outs = [torch.full((M, ldc), 7, dtype=torch.int16, device=cuda) for _ in range(2)]
    d = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    rb.gemm_i8_bcast(d(A), d(W), rb.B_NK, rb.OUT_BF16, d(sa), 1, d(sw), 1,
                     peer_ptrs=[o.data_ptr() for o in outs], ldc=ldc, col_off=col_off)
    rb.sync_status()
    _, c = orc.gemm_i8(A, W, True, sa, 1, sw, 1)
    want = orc.bf16_encode(c)
    for o in outs:
        g = o.cpu().numpy().view(np.uint16)
        assert (g[:, col_off:col_off + N] == want).all()
        assert (g[:, :col_off] == 7).all() and (g[:, col_off + N:] == 7).all()


def test_fused_sharded_one_gpu(rb, orc, cuda):
    from rouge_b200.sharded import FusedShardedW8A8
    M, N, K = 512, 1024, 512
    A, W, sa, sw = _problem(M, N, K)
    sh = FusedShardedW8A8(M, N, K, 0, 1, "cuda:0")
    d = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    out = sh(d(A), d(sa), d(W), d(sw))
    rb.sync_status()
    _, c = orc.gemm_i8(A, W, True, sa, 1, sw, 1)
    assert (out.view(torch.int16).cpu().numpy().view(np.uint16) == orc.bf16_encode(c)).all()


def _fused_rank(rank, world, port, M, N, K, use_mc, q):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [here, os.path.join(root, "rouge-v_b200"), os.path.join(root, "oracle")]
    import torch.distributed as dist
    import oracle as O
    from rouge_b200.sharded import FusedShardedW8A8
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    sh = None
    try:
        A, W, sa, sw = _problem(M, N, K)
        sh = FusedShardedW8A8(M, N, K, rank, world, f"cuda:{rank}", use_multicast=use_mc)
        n0, n1 = sh.columns
        w_shard = np.zeros((sh.ns, K), np.int8)
        w_shard[: n1 - n0] = W[n0:n1]
        sw_shard = np.zeros(sh.ns, np.float32)
        sw_shard[: n1 - n0] = sw[n0:n1]
        d = lambda a: torch.from_numpy(a).to(f"cuda:{rank}")  # noqa: E731
        out = sh(d(A), d(sa), d(w_shard), d(sw_shard))
        torch.cuda.synchronize()
        got = out.view(torch.int16).cpu().numpy().view(np.uint16)
        orc = O.Oracle()
        rows = np.arange(0, M, 37, dtype=np.int32)
        _, c = orc.gemm_i8(A, W, True, sa, 1, sw, 1, rows=rows)
        q.put((rank, sh.mode, bool((got[rows] == orc.bf16_encode(c)).all())))
        dist.barrier()
    finally:
        if sh is not None:
            sh.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("use_mc", [True, False])
def test_fused_sharded_two_gpus(cuda, use_mc):
    # Every rank's full output (both ranks' column blocks) equals the oracle:
    # the epilogue's broadcast placed each tile on every GPU.
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    args = (world, port, 1024, 2048, 1024, use_mc, q)
    procs = [ctx.Process(target=_fused_rank, args=(r,) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = [q.get(timeout=10) for _ in range(world)]
    assert all(p.exitcode == 0 for p in procs)
    assert all(ok for _, _, ok in res), res
