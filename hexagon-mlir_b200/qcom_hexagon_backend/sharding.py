"""Column (N) sharding of a linear layer across the GPUs of one box.

The reference has no multi-device path (its only parallelism is the
4-thread split of FormVirtualThreadsPass.cpp:51-202 on one DSP).  The B200
build shards the large output projections (the LM head of BASELINE config 5)
by output column: rank r holds W[n0_r:n1_r, :] and the full activation A,
computes C[:, n0_r:n1_r] with no communication inside the GEMM, and, when
the caller wants full rows, one NCCL all-gather over NVLink assembles
C[M, N].

The host logic here only uses torch.distributed collectives and the C-ABI
kernels, so the partition and the gather assembly are tested with gloo
ranks on the CPU; the GEMM itself only runs on sm_100 GPUs.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib, ops


def shard_width(N: int, world: int, align: int = 8) -> int:
    """Columns per rank: ceil(N / world) rounded up to `align` (keeps every
    shard's rows 16-byte aligned for TMA with 16-bit outputs)."""
    if world < 1 or N < 0:
        raise ValueError("world must be >= 1 and N >= 0")
    ns = -(-N // world)
    return -(-ns // align) * align


def shard_range(N: int, world: int, rank: int, align: int = 8) -> Tuple[int, int]:
    """[n0, n1) output columns owned by `rank` (the last shards may be short or empty)."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    ns = shard_width(N, world, align)
    n0 = min(N, rank * ns)
    return n0, min(N, n0 + ns)


def rows_from_shards(gathered: torch.Tensor, N: int) -> torch.Tensor:
    """[world, M, Ns] rank-major gather result -> [M, N] row-major.

    On CUDA tensors this is the hx_shards_to_rows kernel; on CPU tensors (the
    gloo tests) the same reordering is written with torch ops."""
    world, M, ns = gathered.shape
    if gathered.is_cuda:
        out = ops.shards_to_rows(gathered.contiguous(), world)
    else:
        out = gathered.permute(1, 0, 2).reshape(M, world * ns)
    return out[:, :N] if world * ns != N else out


def gather_columns(local: torch.Tensor, N: int, group=None) -> torch.Tensor:
    """All-gather every rank's [M, Ns] shard (torch.distributed) and assemble [M, N]."""
    world = dist.get_world_size(group)
    M, ns = local.shape
    gathered = torch.empty((world, M, ns), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(gathered.view(world * M, ns), local.contiguous(), group=group)
    return rows_from_shards(gathered, N)


class NcclComm:
    """An NCCL communicator owned by libhx_gemm (for hx_sharded_gemm_allgather).
    Rank 0 creates the unique id; torch.distributed broadcasts it."""

    def __init__(self, group=None):
        lib = _lib.load()
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        size = lib.hx_nccl_unique_id_size()
        buf = (ctypes.c_uint8 * size)()
        if self.rank == 0:
            _lib.check(lib.hx_nccl_get_unique_id(buf), "hx_nccl_get_unique_id")
        dev = torch.device("cuda", torch.cuda.current_device())
        t = torch.tensor(list(bytes(buf)), dtype=torch.uint8, device=dev)
        dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        ctypes.memmove(buf, bytes(t.cpu().numpy().tobytes()), size)
        comm = ctypes.c_void_p()
        _lib.check(lib.hx_nccl_comm_init(ctypes.byref(comm), self.world, buf, self.rank), "hx_nccl_comm_init")
        self.handle = comm

    def close(self):
        if self.handle:
            _lib.load().hx_nccl_comm_destroy(self.handle)
            self.handle = None


class ColumnShardedLinear:
    """y = x @ W.T (+ bias) with W split by output column across ranks.

    weight: this rank's shard [n1-n0, K], or the full [N, K] with full=True.
    forward(x, gather=False) returns the local [M, Ns] shard (vocab-parallel
    layout); gather=True returns the full [M, N] on every rank.
    """

    def __init__(self, weight: torch.Tensor, N: int, rank: int, world: int, *, full: bool = False,
                 bias: Optional[torch.Tensor] = None, group=None, comm: Optional[NcclComm] = None):
        self.N, self.rank, self.world, self.group, self.comm = N, rank, world, group, comm
        self.ns = shard_width(N, world)
        n0, n1 = shard_range(N, world, rank)
        w = weight[n0:n1] if full else weight
        if w.shape[0] != n1 - n0:
            raise ValueError(f"rank {rank} weight shard has {w.shape[0]} rows, expected {n1 - n0}")
        if n1 - n0 < self.ns:  # pad the short last shard with zero rows: equal gather sizes
            pad = torch.zeros((self.ns - (n1 - n0), w.shape[1]), dtype=w.dtype, device=w.device)
            w = torch.cat([w, pad], 0)
        self.weight = w.contiguous()
        self.bias = None
        if bias is not None:
            b = bias[n0:n1] if full else bias
            if b.shape[0] < self.ns:
                b = torch.cat([b, torch.zeros(self.ns - b.shape[0], dtype=b.dtype, device=b.device)])
            self.bias = b.contiguous()

    def forward(self, x: torch.Tensor, gather: bool = True, out: Optional[torch.Tensor] = None):
        x2 = x.reshape(-1, x.shape[-1])
        if not gather:
            return ops.linear(x2, self.weight, self.bias, out=out)
        if self.comm is None:
            local = ops.linear(x2, self.weight, self.bias, out=out)
            return gather_columns(local, self.N, self.group)
        # One C call: the sharded GEMM, then the NCCL all-gather on the same stream.
        d, local, dev = ops.make_desc(x2, self.weight, out=out, bias=self.bias,
                                      epilogue="bias" if self.bias is not None else "none")
        gathered = torch.empty((self.world, x2.shape[0], self.ns), dtype=local.dtype, device=dev)
        lib = _lib.load()
        with torch.cuda.device(dev):
            rc = lib.hx_sharded_gemm_allgather(ctypes.byref(d), self.rank, self.world, self.comm.handle,
                                               ctypes.c_void_p(gathered.data_ptr()),
                                               ctypes.c_void_p(ops._stream_ptr(dev)))
        _lib.check(rc, "hx_sharded_gemm_allgather")
        return rows_from_shards(gathered, self.N)
