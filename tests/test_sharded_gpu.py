"""Multi-GPU parity of the column-sharded GEMM (BASELINE config 5 shape,
scaled down): every rank computes its column shard with hx kernels and the
full logits are assembled (a) with torch.distributed NCCL all-gather, (b)
with the library's own NCCL communicator (hx_sharded_gemm_allgather) and (c)
by the fused GEMM whose epilogue stores into every rank's buffer over NVLink
(hx_sharded_gemm_gather_p2p).
Needs >= 2 GPUs; runs as child processes, one per GPU."""

import os
import socket
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = textwrap.dedent(r'''
    import os, sys
    sys.path.insert(0, os.path.join(ROOT, "hexagon-mlir_b200")); sys.path.insert(0, ROOT)
    import numpy as np, torch, torch.distributed as dist
    from qcom_hexagon_backend import sharding as S
    from oracle import gemm_oracle as O
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    M, K, N = 512, 256, 1000
    g = torch.Generator().manual_seed(9)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    ref = O.matmul_f32(a.float().numpy(), w.float().numpy())
    lin = S.ColumnShardedLinear(w.cuda(), N, rank, world, full=True)
    y1 = lin.forward(a.cuda()).float().cpu().numpy()
    comm = S.NcclComm()
    lin2 = S.ColumnShardedLinear(w.cuda(), N, rank, world, full=True, comm=comm)
    y2 = lin2.forward(a.cuda()).float().cpu().numpy()
    local = lin.forward(a.cuda(), gather=False).float().cpu().numpy()
    n0, n1 = S.shard_range(N, world, rank)
    e1, e2 = O.max_rel_err(y1, ref), O.max_rel_err(y2, ref)
    e3 = O.max_rel_err(local[:, : n1 - n0], ref[:, n0:n1])
    assert y1.shape == (M, N) and y2.shape == (M, N), (y1.shape, y2.shape)
    assert e1 <= 1e-2 and e2 <= 1e-2 and e3 <= 1e-2, (e1, e2, e3)
    # (c) the fused GEMM + NVLink all-gather: several calls in a row
    pg = S.P2PGather(M, lin.ns, torch.bfloat16)
    for it in range(3):
        buf = pg.run(a.cuda() * (it + 1), lin.weight)
        torch.cuda.synchronize()
        assert int(pg.error_flag.item()) == 0, int(pg.error_flag.item())
        y4 = S.rows_from_shards(buf, N).float().cpu().numpy()
        e4 = O.max_rel_err(y4, ref * (it + 1))
        assert y4.shape == (M, N) and e4 <= 1e-2, (it, e4)
    pg.close()
    # (d) the same through the copy engines, GEMM in row chunks
    for chunks in (0, 3):
        pg = S.P2PGather(M, lin.ns, torch.bfloat16, transfer="copy_engine", chunks=chunks)
        for it in range(3):
            buf = pg.run(a.cuda() * (it + 1), lin.weight)
            torch.cuda.synchronize()
            assert int(pg.error_flag.item()) == 0, int(pg.error_flag.item())
            y5 = S.rows_from_shards(buf, N).float().cpu().numpy()
            e5 = O.max_rel_err(y5, ref * (it + 1))
            assert y5.shape == (M, N) and e5 <= 1e-2, (chunks, it, e5)
        pg.close()
    # (e) vocab-parallel softmax of the local shards: no logit gather
    local = lin.forward(a.cuda(), gather=False)
    sm = S.vocab_parallel_softmax(local, n1 - n0)
    torch.cuda.synchronize()
    refp = O.softmax_ref(ref)[:, n0:n1]
    got = sm.float().cpu().numpy()
    assert (np.abs(got - refp) <= 1e-2 * np.abs(refp) + 1e-6).all(), "vocab-parallel softmax"
    torch.cuda.synchronize(); comm.close(); dist.destroy_process_group()
    print("rank", rank, "ok", e1, e2, e3, e4)
''')


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_lmhead_multi_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _port()
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
               NCCL_NVLS_ENABLE="0")
    code = f"ROOT = {ROOT!r}\n" + WORKER
    procs = [subprocess.Popen([sys.executable, "-c", code], env=dict(env, RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(world)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    for r, (p, out) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {r} failed:\n{out[-3000:]}"
        assert f"rank {r} ok" in out


DEVICE_WORKER = textwrap.dedent(r'''
    import os, sys
    sys.path.insert(0, os.path.join(ROOT, "hexagon-mlir_b200")); sys.path.insert(0, ROOT)
    import numpy as np, torch
    import qcom_hexagon_backend as q
    from oracle import gemm_oracle as O
    # One process, two GPUs, the same tile plans (one-CTA 198 KB-smem tiles, CTA
    # pairs, split-K clusters): each kernel's shared-memory limit is a per-device
    # attribute, so the second device must be configured too.
    g = torch.Generator().manual_seed(77)
    cases = [(1024, 768, 768, {}), (4096, 4096, 1024, {}), (256, 384, 2048, {"split_k": 2, "tile_n": 128})]
    for M, N, K, kw in cases:
        a = torch.randn(M, K, generator=g).half()
        w = (torch.randn(N, K, generator=g) * 0.02).half()
        ref = O.matmul_f32(a.float().numpy(), w.float().numpy())
        for dev in (0, 1, 0):
            with torch.cuda.device(dev):
                out = q.gemm(a.to(f"cuda:{dev}"), w.to(f"cuda:{dev}"), **kw)
                torch.cuda.synchronize(dev)
            e = O.max_rel_err(out.float().cpu().numpy(), ref)
            assert e <= 1e-2, (M, N, K, dev, e)
    print("two devices ok")
''')


def test_one_process_two_devices():
    """A process that drives two GPUs launches the same kernels on both."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    code = f"ROOT = {ROOT!r}\n" + DEVICE_WORKER
    p = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=240)
    assert p.returncode == 0 and "two devices ok" in p.stdout, (p.stdout + p.stderr)[-3000:]
