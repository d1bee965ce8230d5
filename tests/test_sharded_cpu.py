"""Host-side logic of the N-sharded W8A8 GEMM on CPU:
column shards, band rows, and the band-wise all-gather + unshard through
two gloo ranks. The local GEMM and the unshard step are CPU stand-ins
injected by the test (the oracle's exact int8 GEMM, a torch permute); the
GPU versions are covered by tests/test_gpu_sharded.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rouge_b200.sharded import ShardedW8A8, band_rows, shard_columns


def test_shard_columns():
    ns, r = shard_columns(28672, 8)
    assert ns == 3584 and r[0] == (0, 3584) and r[-1] == (25088, 28672)
    ns, r = shard_columns(100, 3)           # ns rounded up to 16: last shard short
    assert ns == 48 and r == [(0, 48), (48, 96), (96, 100)]
    ns, r = shard_columns(16, 4)
    assert ns == 16 and r == [(0, 16), (16, 16), (16, 16), (16, 16)]   # empty shards allowed


def test_band_rows():
    assert band_rows(16384) == 2048
    assert band_rows(4096) == 2048
    assert band_rows(384) == 384
    assert band_rows(200) == 200            # no multiple-of-128 divisor: one band


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_gemm(orc):
    from conftest import ROOT  # noqa: F401  (paths)

    def gemm(a, sa, w, sw, out):
        _, c = orc.gemm_i8(a.numpy(), w.numpy(), True, sa.numpy(), 1, sw.numpy(), 1)
        out.copy_(torch.from_numpy(orc.bf16_encode(c).view(np.int16)).view(torch.bfloat16))
    return gemm


def _cpu_unshard(src, out, M, N, g, ns, R):
    nb = M // R
    full = src.reshape(nb, g, R, ns).permute(0, 2, 1, 3).reshape(M, g * ns)
    out.copy_(full[:, :N])


def _rank(rank, world, port, M, N, K, R, q):
    import sys
    sys.path[:0] = [os.path.join(os.path.dirname(__file__)), os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle")]
    import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc = O.Oracle()
        rng = np.random.default_rng(7)
        A = rng.integers(-127, 128, (M, K), dtype=np.int8)
        W = rng.integers(-127, 128, (N, K), dtype=np.int8)
        sa = rng.uniform(1e-3, 1e-2, M).astype(np.float32)
        sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
        sh = ShardedW8A8(M, N, K, rank, world, "cpu", R=R, local_gemm=_cpu_gemm(orc),
                         unshard=_cpu_unshard)
        n0, n1 = sh.columns
        w_shard = np.zeros((sh.ns, K), np.int8)
        w_shard[: n1 - n0] = W[n0:n1]
        sw_shard = np.zeros(sh.ns, np.float32)
        sw_shard[: n1 - n0] = sw[n0:n1]
        out = sh(torch.from_numpy(A), torch.from_numpy(sa), torch.from_numpy(w_shard),
                 torch.from_numpy(sw_shard))
        _, full = orc.gemm_i8(A, W, True, sa, 1, sw, 1)
        want = orc.bf16_encode(full)
        got = out.view(torch.int16).numpy().view(np.uint16)
        q.put((rank, bool((got == want).all())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M,N,K,R", [(2, 256, 96, 64, 128), (3, 128, 100, 32, 64)])
def test_sharded_gather_gloo(world, M, N, K, R):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, M, N, K, R, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert all(results[r] for r in range(world)), results


def _failing_rank(rank, world, port, q):
    """Rank 1's local GEMM fails the way a device entry reports a bounded
    wait that ran out (the binding raises); rank 1 leaves without joining
    the band's all-gather. Rank 0 must get an error from that collective
    within the process group's short timeout instead of waiting for good."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    M, N, K, R = 256, 64, 32, 128

    def gemm(a, sa, w, sw, out):
        if rank == 1:
            raise RuntimeError("rouge_b200_gemm_i8: device-side wait timed out (-5)")
        out.zero_()

    sh = ShardedW8A8(M, N, K, rank, world, "cpu", R=R, local_gemm=gemm, unshard=_cpu_unshard)
    a = torch.zeros((M, K), dtype=torch.int8)
    sa = torch.ones(M)
    w = torch.zeros((sh.ns, K), dtype=torch.int8)
    sw = torch.ones(sh.ns)
    t0 = time.monotonic()
    try:
        sh(a, sa, w, sw)
        q.put((rank, "completed", time.monotonic() - t0))
    except RuntimeError as e:
        q.put((rank, "timed out" if "timed out" in str(e) else "error", time.monotonic() - t0))
        if rank == 1:
            raise
    finally:
        if rank == 0:
            try:
                dist.destroy_process_group()
            except Exception:  # the peer is gone; nothing left to tear down
                pass


def test_rank_failure_ends_peer_collective_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank waited past every timeout"
    res = {}
    while not q.empty():
        r, what, dt = q.get(timeout=5)
        res[r] = (what, dt)
    assert res[1][0] == "timed out"              # the failing call raised on rank 1
    assert procs[1].exitcode != 0                # and the rank left
    assert res[0][0] != "completed"              # rank 0's all-gather ended with an error
    assert res[0][1] < 60.0, res
