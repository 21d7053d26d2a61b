"""Multi-rank host logic of the column-sharded GEMM on CPU gloo ranks
(world size 2 and 3): shard partition, padded all-gather, and the
rank-major -> row-major reassembly.  Each rank's GEMM here is the test's own
torch matmul (the kernels need an sm_100 GPU)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qcom_hexagon_backend import sharding as S


def test_shard_ranges_cover_exactly():
    for N in (1, 7, 64, 100, 50304):
        for world in (1, 2, 3, 4, 8):
            spans = [S.shard_range(N, world, r) for r in range(world)]
            assert [c for a, b in spans for c in range(a, b)] == list(range(N))
            assert all(b - a <= S.shard_width(N, world) for a, b in spans)
    assert S.shard_width(50304, 8) == 6288
    with pytest.raises(ValueError):
        S.shard_range(10, 2, 2)


def test_rows_from_shards_cpu():
    world, M, ns = 3, 5, 4
    g = torch.arange(world * M * ns).reshape(world, M, ns)
    out = S.rows_from_shards(g, N=10)
    assert out.shape == (M, 10)
    for r in range(world):
        for c in range(ns):
            if r * ns + c < 10:
                assert torch.equal(out[:, r * ns + c], g[r, :, c])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, N, K, M, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        x = torch.randn(M, K, generator=g)
        w = torch.randn(N, K, generator=g)
        n0, n1 = S.shard_range(N, world, rank)
        local = torch.zeros(M, S.shard_width(N, world))
        local[:, : n1 - n0] = x @ w[n0:n1].T
        full = S.gather_columns(local, N)
        q.put((rank, bool(torch.allclose(full, x @ w.T, atol=1e-4)), tuple(full.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,N", [(2, 64), (3, 100)])
def test_gather_columns_gloo(world, N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, N, 16, 6, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=60) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res)
    assert all(shape == (6, N) for _, _, shape in res)
