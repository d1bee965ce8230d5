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


class FusedShardedW8A8:
    """The same product as ShardedW8A8 with the all-gather fused into the
    GEMM: every rank's output C[M][N] is a symmetric-memory buffer (one
    allocation per rank, mapped into every rank's address space), and the
    GEMM epilogue writes each tile of this rank's column block [n0, n1) into
    every rank's C at once -- either one TMA store of a 64-column line
    (128-byte rows) per rank through the peer pointers (the default), or
    multimem stores (16 bytes each, staged so that every store instruction
    covers whole 128-byte row segments) to the buffer's NVLink multicast
    address, which the NVSwitch replicates to every GPU. No separate
    exchange, no layout step: the
    tiles land row-major at their final place. A device-side barrier across
    the ranks (signal pads, system scope) ends each call, after which every
    rank's C is complete.

    Requires N % 16 == 0 (16-byte vectors at every shard's column offset).
    """

    def __init__(self, M: int, N: int, K: int, rank: int, world: int, device, group=None,
                 use_multicast: Optional[bool] = None):
        import torch
        import torch.distributed as dist
        from . import OUT_BF16, B_NK, gemm_i8, gemm_i8_bcast

        assert N % 16 == 0, "fused sharding needs N % 16 == 0"
        self.M, self.N, self.K = M, N, K
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.ns, self.ranges = shard_columns(N, world)
        self._gemm, self._bcast, self._bf16, self._nk = gemm_i8, gemm_i8_bcast, OUT_BF16, B_NK
        self.handle = None
        self.mc = 0
        self.peers = ()
        if world == 1:
            self.out = torch.empty((M, N), dtype=torch.bfloat16, device=self.device)
            self.mode = "local"
            return
        import torch.distributed._symmetric_memory as symm
        g = group if group is not None else dist.group.WORLD
        self.out = symm.empty((M, N), dtype=torch.bfloat16, device=self.device)
        self.handle = symm.rendezvous(self.out, g)
        if use_multicast is None:
            use_multicast = self.default_multicast(world)
        has_mc = use_multicast and bool(symm._SymmetricMemory.has_multicast_support(
            symm.DeviceType.CUDA, self.device.index or 0))
        # The handle's pointers address the start of each rank's allocation;
        # the tensor starts `delta` bytes into it (0 when it owns the whole
        # allocation). Every store stays inside [delta, delta + M*N*2).
        delta = self.out.data_ptr() - int(self.handle.buffer_ptrs[rank])
        if delta < 0 or delta + M * N * 2 > int(self.handle.buffer_size):
            raise RuntimeError("symmetric buffer does not cover the output")
        mc = int(self.handle.multicast_ptr) if has_mc else 0
        if mc:
            self.mc, self.mode = mc + delta, "multimem"
        else:
            self.peers = tuple(int(p) + delta for p in self.handle.buffer_ptrs)
            self.mode = "peer-stores"

    @staticmethod
    def default_multicast(world: int) -> bool:
        """The form used unless the caller chooses: peer TMA stores. A
        multicast store is written into every bound GPU, the sender's own
        copy included, so each GPU receives all of C over NVLink; peer
        stores send a tile world - 1 times but each GPU receives only the
        other ranks' (world - 1) / world of C. With whole 128-byte lines per
        row the peer form is the faster one at 2 and at 8 ranks."""
        del world
        return False

    @property
    def columns(self) -> Tuple[int, int]:
        return self.ranges[self.rank]

    def __call__(self, a, sa, w_shard, sw_shard, events=None):
        """a[M][K] int8, sa[M] f32, w_shard[ns][K] int8 (rows beyond this
        rank's columns ignored), sw_shard[ns] f32. Returns C[M][N] bf16."""
        import torch
        n0, n1 = self.columns
        ncols = n1 - n0
        cur = torch.cuda.current_stream(self.device)
        if self.world == 1:
            self._gemm(a, w_shard[:ncols], self._nk, self.out, self._bf16, sa, 1, sw_shard[:ncols], 1)
        elif ncols > 0:
            self._bcast(a, w_shard[:ncols], self._nk, self._bf16, sa, 1, sw_shard[:ncols], 1,
                        mc_ptr=self.mc, peer_ptrs=self.peers, ldc=self.N, col_off=n0)
        if events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(cur)
            events["gemm_done"] = ev
        if self.handle is not None:
            self.handle.barrier(channel=0, timeout_ms=10000)
        return self.out

    def close(self):
        """Drop the symmetric-memory buffer (every rank, after the last call)."""
        self.handle = None
        self.out = None
