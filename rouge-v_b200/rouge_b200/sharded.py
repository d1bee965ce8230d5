"""N-sharded W8A8 GEMM across the GPUs of one node.

Rank r of g holds the full int8 activations A[M][K] (with per-token scales)
and the rows [n0, n1) of the int8 weights W[N][K] (per-output-channel
scales): its own block of output columns. It computes C[:, n0:n1] with the
tcgen05 GEMM (int32 accumulation, dequant to bf16 in the epilogue) in bands
of R rows; as soon as band b is finished its shard is all-gathered over
NVLink (NCCL, on a separate stream), so the exchange of band b overlaps the
GEMM of band b+1. The gathered bands arrive as [M/R][g][R][ns] and one
HBM-bound kernel writes them row-major into C[M][N] on every rank.

The reference has no multi-GPU code; this is the one sharded path of the
build. Every rank issues the same collectives in the same order.
"""
from __future__ import annotations

import math
from typing import Callable, List, Optional, Tuple


def shard_columns(N: int, world: int, align: int = 16) -> Tuple[int, List[Tuple[int, int]]]:
    """Shard width ns (a multiple of `align`) and each rank's [n0, n1)."""
    ns = int(math.ceil(math.ceil(N / world) / align) * align)
    return ns, [(min(N, r * ns), min(N, (r + 1) * ns)) for r in range(world)]


def band_rows(M: int, target: int = 2048, multiple: int = 128) -> int:
    """Largest divisor of M that is a multiple of `multiple` and <= target
    (M itself when no such divisor exists)."""
    best = 0
    for r in range(multiple, min(M, target) + 1, multiple):
        if M % r == 0:
            best = r
    return best or M


class ShardedW8A8:
    """C[M][N] = dequant(A . W^T) with W's rows sharded over the ranks.

    local_gemm(a_rows, sa_rows, w_shard, sw_shard, out_rows) and
    unshard(gathered, out, M, N, g, ns, R) default to the sm_100a kernels;
    tests inject CPU versions to exercise the rank and collective logic
    with gloo.
    """

    def __init__(self, M: int, N: int, K: int, rank: int, world: int, device, group=None,
                 R: Optional[int] = None, local_gemm: Optional[Callable] = None,
                 unshard: Optional[Callable] = None):
        import torch
        import torch.distributed as dist

        self.M, self.N, self.K = M, N, K
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device)
        self.ns, self.ranges = shard_columns(N, world)
        self.R = R or band_rows(M)
        assert M % self.R == 0
        self.nbands = M // self.R
        self.dist = dist if world > 1 else None
        dt = torch.bfloat16
        self.shard = torch.empty((M, self.ns), dtype=dt, device=self.device)
        self.gathered = (torch.empty((self.nbands, world, self.R, self.ns), dtype=dt,
                                     device=self.device) if world > 1 else None)
        # One rank: the shard is the output (ns == N), no layout step.
        self.out = self.shard if world == 1 else torch.empty((M, N), dtype=dt, device=self.device)
        self.cuda = self.device.type == "cuda"
        if self.cuda:
            self.comm = torch.cuda.Stream(device=self.device)
            self.done = [torch.cuda.Event() for _ in range(self.nbands)]
        if local_gemm is None or unshard is None:
            from . import (OUT_BF16, B_NK, gemm_i8, unshard_columns)
            if local_gemm is None:
                def local_gemm(a, sa, w, sw, out):
                    gemm_i8(a, w, B_NK, out, OUT_BF16, sa, 1, sw, 1)
            if unshard is None:
                unshard = unshard_columns
        self.local_gemm, self.unshard = local_gemm, unshard

    @property
    def columns(self) -> Tuple[int, int]:
        return self.ranges[self.rank]

    def weight_rows(self) -> int:
        """Rows of W this rank must hold (its shard, zero-padded to ns)."""
        return self.ns

    def __call__(self, a, sa, w_shard, sw_shard, events=None):
        """a[M][K] int8, sa[M] f32, w_shard[ns][K] int8, sw_shard[ns] f32.
        events, if given, is a dict receiving 'gemm_done' (CUDA event
        recorded after the last GEMM band on the current stream)."""
        import torch
        R = self.R
        cur = torch.cuda.current_stream(self.device) if self.cuda else None
        for b in range(self.nbands):
            rows = slice(b * R, (b + 1) * R)
            self.local_gemm(a[rows], sa[rows], w_shard, sw_shard, self.shard[rows])
            if self.world == 1:
                continue  # nothing to exchange: the shard is the whole output
            # rank-concatenated output of band b: [g*R][ns] = [g][R][ns]
            dst = self.gathered[b].view(self.world * R, self.ns)
            if self.cuda:
                self.done[b].record(cur)
                with torch.cuda.stream(self.comm):
                    self.comm.wait_event(self.done[b])
                    self.dist.all_gather_into_tensor(dst, self.shard[rows], group=self.group)
            else:
                self.dist.all_gather_into_tensor(dst, self.shard[rows], group=self.group)
        if events is not None and self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(cur)
            events["gemm_done"] = ev
        if self.world == 1:
            return self.out
        if self.cuda:
            cur.wait_stream(self.comm)
        self.unshard(self.gathered, self.out, self.M, self.N, self.world, self.ns, R)
        return self.out
