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


def vocab_parallel_softmax(local: torch.Tensor, n_valid: Optional[int] = None, group=None, *,
                           log: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Softmax over the full vocabulary of column-sharded logits, without
    gathering them: local is this rank's [M, Ns] shard (its first n_valid
    columns are real; the padding of a short last shard is left out).  Each
    rank reduces its rows to {max, sum exp}, the ranks all-gather those
    [M, 2] floats (8 bytes a row), every rank combines them into the global
    pair and normalises its own columns.  Returns this rank's [M, n_valid]
    probabilities (log-probabilities with log=True); out may be `local`
    itself (in place)."""
    x = local if n_valid is None or n_valid == local.shape[1] else local[:, :n_valid]
    st = ops.softmax_stats(x)
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world > 1:
        all_st = torch.empty((world,) + tuple(st.shape), dtype=st.dtype, device=st.device)
        dist.all_gather_into_tensor(all_st, st, group=group)
    else:
        all_st = st.unsqueeze(0)
    glob = ops.softmax_combine(all_st)
    if out is not None and out.shape != x.shape:
        out = out[:, : x.shape[1]]
    return ops.softmax_apply(x, glob, log=log, out=out)


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


def ce_chunk_count(M: int, chunks: int = 0) -> int:
    """Row chunks hx_sharded_gemm_gather_ce runs for M rows and a requested count."""
    if chunks == 0:
        chunks = min(6, max(1, M // 2048))
    rows = -(-M // chunks)
    rows = max(256, -(-rows // 256) * 256)
    return -(-M // rows)


class P2PGather:
    """Sharded GEMM + all-gather over NVLink into peer-mapped buffers.

    transfer="epilogue": one fused launch (hx_sharded_gemm_gather_p2p) whose
    GEMM epilogue stores each output chunk into every rank's buffer;
    transfer="copy_engine": the GEMM in row chunks with each finished chunk
    copied to the peers by DMA (hx_sharded_gemm_gather_ce), overlapping the
    next chunk.

    Every rank owns a [world, M, ns] gather buffer and a flag array in its own
    GPU memory; the buffers are exported as CUDA IPC handles, exchanged with
    torch.distributed and mapped by every other rank.  run(x, w) computes this
    rank's shard x @ w.T and its GEMM epilogue writes each output chunk into
    all ranks' buffers at [rank], so when it returns (stream-ordered) the
    buffer holds every rank's shard.  All ranks must call run() the same
    number of times (it synchronises them on the GPU, with bounded waits).

    If a bounded wait runs out, error_flag reads 41 and the contents of every
    rank's gather buffer are undefined for that call: the GEMM still runs and
    still stores into the peers' buffers, which a late peer may be reading.
    The caller should treat the gather as failed on all ranks.
    """

    def __init__(self, M: int, ns: int, dtype: torch.dtype, group=None, transfer: str = "epilogue",
                 chunks: int = 0):
        if transfer not in ("epilogue", "copy_engine"):
            raise ValueError("transfer must be 'epilogue' or 'copy_engine'")
        self.transfer, self.chunks = transfer, chunks
        lib = _lib.load()
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the fused gather takes at most 8 ranks")
        self.M, self.ns, self.dtype, self.group = M, ns, dtype, group
        self.device = torch.device("cuda", torch.cuda.current_device())
        esz = torch.empty(0, dtype=dtype).element_size()
        hsz = lib.hx_peer_handle_size()
        self._mine = []
        self._opened = []
        handles = []
        # Every step that can fail on one rank alone is followed by a
        # collective vote, so either all ranks construct the gather or all
        # raise: a rank that fell back alone would leave its peers waiting.
        err = None
        try:
            for nbytes in (self.world * M * ns * esz, 256):  # gather buffer, flags
                ptr, h = ctypes.c_void_p(), (ctypes.c_uint8 * hsz)()
                _lib.check(lib.hx_peer_alloc(nbytes, ctypes.byref(ptr), h), "hx_peer_alloc")
                self._mine.append(ptr.value)
                handles.append(bytes(h))
        except Exception as ex:  # noqa: BLE001 - re-raised after the vote
            err = ex
        self._vote(err, "peer buffer allocation")
        blob = torch.tensor(list(b"".join(handles)), dtype=torch.uint8, device=self.device)
        allb = torch.empty(self.world * blob.numel(), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allb, blob, group=group)
        allb = bytes(allb.cpu().numpy().tobytes())
        bufs, flags = [], []
        try:
            for r in range(self.world):
                if r == self.rank:
                    bufs.append(self._mine[0])
                    flags.append(self._mine[1])
                    continue
                ptrs = []
                for j in range(2):
                    off = (r * 2 + j) * hsz
                    h = (ctypes.c_uint8 * hsz).from_buffer_copy(allb[off:off + hsz])
                    p = ctypes.c_void_p()
                    _lib.check(lib.hx_peer_open(h, ctypes.byref(p)), "hx_peer_open")
                    self._opened.append(p.value)
                    ptrs.append(p.value)
                bufs.append(ptrs[0])
                flags.append(ptrs[1])
        except Exception as ex:  # noqa: BLE001
            err = ex
        self._vote(err, "peer buffer mapping")
        self._bufs = (ctypes.c_void_p * self.world)(*bufs)
        self._flags = (ctypes.c_void_p * self.world)(*flags)
        self.epoch = 0
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._local_view = _device_view(self._mine[0], (self.world, M, ns), dtype, self.device)

    @property
    def last_chunks(self) -> int:
        """GEMM launches per run() of the copy-engine transfer (the library's
        chunking rule: whole 256-row tiles, up to 6 automatic chunks)."""
        return ce_chunk_count(self.M, self.chunks)

    def _vote(self, err, what):
        """All ranks agree that `what` succeeded everywhere, or all release what
        they hold and raise."""
        ok = torch.tensor([0 if err is not None else 1], dtype=torch.int32, device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if int(ok.item()) == 1:
            return
        self._release()
        raise RuntimeError(f"fused gather unavailable: {what} failed on "
                           + (f"this rank ({err})" if err is not None else "another rank"))

    def _release(self):
        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            lib.hx_peer_close(ctypes.c_void_p(p))
        self._opened = []
        dist.barrier(group=self.group)  # peers unmapped before the memory goes
        for p in self._mine:
            lib.hx_peer_free(ctypes.c_void_p(p))
        self._mine = []

    def run(self, x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Returns this rank's [world, M, ns] buffer holding all shards."""
        d, _, dev = ops.make_desc(x, w, out=self._local_view[self.rank], bias=bias,
                                  epilogue="bias" if bias is not None else "none", b_const=True)
        lib = _lib.load()
        with torch.cuda.device(dev):
            if self.transfer == "epilogue":
                rc = lib.hx_sharded_gemm_gather_p2p(ctypes.byref(d), self.rank, self.world, self._bufs,
                                                    self._flags, self.epoch,
                                                    ctypes.c_void_p(self.error_flag.data_ptr()),
                                                    ctypes.c_void_p(ops._stream_ptr(dev)))
            else:
                rc = lib.hx_sharded_gemm_gather_ce(ctypes.byref(d), self.rank, self.world, self._bufs,
                                                   self._flags, self.epoch,
                                                   ctypes.c_void_p(self.error_flag.data_ptr()), self.chunks,
                                                   ctypes.c_void_p(ops._stream_ptr(dev)))
        _lib.check(rc, "hx_sharded_gemm_gather_" + ("p2p" if self.transfer == "epilogue" else "ce"))
        self.epoch += 1
        return self._local_view

    def close(self):
        self._release()


def _device_view(ptr: int, shape, dtype, device) -> torch.Tensor:
    """A tensor over device memory the library allocated (no copy, not owned)."""
    class _Holder:
        pass

    h = _Holder()
    numel = 1
    for s in shape:
        numel *= s
    esz = torch.empty(0, dtype=dtype).element_size()
    h.__cuda_array_interface__ = {"shape": (numel,), "typestr": {1: "|u1", 2: "<u2", 4: "<u4"}[esz],
                                  "data": (ptr, False), "version": 3, "strides": None}
    flat = torch.as_tensor(h, device=device)
    return flat.view(dtype).view(*shape)
