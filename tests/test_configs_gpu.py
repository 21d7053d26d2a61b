"""GPU parity at the benchmark configurations' real shapes, through the C ABI,
against the CPU oracle (fp32 accumulate of upcast operands; the golden of
test/python/triton/test_matmul.py:90).

  * config 3 (Qwen2.5-0.5B prefill, bf16, 2048 tokens): fused gate/up
    896 -> 2x4864 with SwiGLU, down 4864 -> 896 +residual, QKV 896 -> 1152 +bias;
  * config 5 (LM head, M=16384 x K=2048 x N=50304): bf16 and int8 W8A8
    bit-exact, the full launch with a sample of rows checked, and every
    column-shard width the 2/4/8-way split produces (25152, 12576, 6288; 6288
    leaves a partial 256-column tile);
  * the fused all-gather's peer-store epilogue (hx_sharded_gemm_gather_p2p) on
    one GPU: two ranks' buffers on the same device, the simulated peer's flags
    pre-published so that no kernel waits on another; and the bounded wait
    running out on a flag that nothing sets.

Tolerance: max |out - ref| / max |ref| <= 1e-2 for bf16 (plus the elementwise
bound of test_gemm_gpu.assert_close); int8 with int32 output is bit-exact.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O
from test_gemm_gpu import assert_close, to_np32

pytestmark = pytest.mark.gpu

LM_M, LM_K, LM_N = 16384, 2048, 50304


def hx():
    import qcom_hexagon_backend as q

    return q


def _bf16(shape, g, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


# ---------------------------------------------------------------- config 3
def test_config3_gate_up_swiglu(cuda_device):
    q = hx()
    g = torch.Generator().manual_seed(300)
    x = _bf16((2048, 896), g)
    w = _bf16((2 * 4864, 896), g, 0.02)  # [gate; up]
    out = q.gemm(x.to(cuda_device), w.to(cuda_device), epilogue="swiglu")
    torch.cuda.synchronize()
    assert out.shape == (2048, 4864) and out.dtype == torch.bfloat16
    assert_close(to_np32(out), O.linear_ref(to_np32(x), to_np32(w), epilogue="swiglu"))


def test_config3_down_residual(cuda_device):
    q = hx()
    g = torch.Generator().manual_seed(301)
    h = _bf16((2048, 4864), g)
    w = _bf16((896, 4864), g, 0.02)
    res = _bf16((2048, 896), g)
    d = cuda_device
    out = q.gemm(h.to(d), w.to(d), epilogue="residual", residual=res.to(d))
    torch.cuda.synchronize()
    assert_close(to_np32(out), O.linear_ref(to_np32(h), to_np32(w), epilogue="residual",
                                            residual=to_np32(res)))


def test_config3_qkv_bias(cuda_device):
    q = hx()
    g = torch.Generator().manual_seed(302)
    x = _bf16((2048, 896), g)
    w = _bf16((896 + 2 * 128, 896), g, 0.02)
    b = _bf16((896 + 2 * 128,), g, 0.02)
    d = cuda_device
    out = q.gemm(x.to(d), w.to(d), epilogue="bias", bias=b.to(d))
    torch.cuda.synchronize()
    assert_close(to_np32(out), O.linear_ref(to_np32(x), to_np32(w), epilogue="bias", bias=to_np32(b)))


# ---------------------------------------------------------------- config 5
def _rows(M, n, seed):
    r = np.random.default_rng(seed).choice(M, size=n, replace=False)
    return np.sort(np.concatenate([r, [0, M - 1]]))


def _lm_bf16(seed, N):
    g = torch.Generator().manual_seed(seed)
    return _bf16((LM_M, LM_K), g), _bf16((N, LM_K), g, 0.02)


def _lm_int8(seed, N):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (LM_M, LM_K), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (N, LM_K), generator=g, dtype=torch.int8)
    return a, w


def _exact_int8_rows(a_rows: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Exact int32 products through fp64 BLAS: |acc| <= 2048 * 127^2 < 2^53."""
    c = a_rows.astype(np.float64) @ w.astype(np.float64).T
    return c.astype(np.int64).astype(np.int32)


def test_config5_lmhead_bf16_full(cuda_device):
    """The full 16384 x 50304 launch (the bench's kernel plan); 258 rows checked."""
    q = hx()
    a, w = _lm_bf16(500, LM_N)
    out = q.gemm(a.to(cuda_device), w.to(cuda_device))
    torch.cuda.synchronize()
    rows = _rows(LM_M, 256, 0)
    got = out[torch.from_numpy(rows).to(cuda_device)].float().cpu().numpy()
    ref = O.matmul_f32(to_np32(a[torch.from_numpy(rows)]), to_np32(w))
    assert_close(got, ref)


def test_config5_lmhead_int8_full_exact(cuda_device):
    q = hx()
    a, w = _lm_int8(501, LM_N)
    out = q.gemm(a.to(cuda_device), w.to(cuda_device))
    torch.cuda.synchronize()
    assert out.dtype == torch.int32 and out.shape == (LM_M, LM_N)
    rows = _rows(LM_M, 128, 1)
    got = out[torch.from_numpy(rows).to(cuda_device)].cpu().numpy()
    np.testing.assert_array_equal(got, _exact_int8_rows(a.numpy()[rows], w.numpy()))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("kind", ["bf16", "int8"])
def test_config5_shard_widths(cuda_device, world, kind):
    """Every rank's column shard of the 50304-wide LM head at 2/4/8 ranks
    (shard_width pads the last shard; 6288 columns leave a partial tile).
    Rank world-1's shard is run (the same width as every other at these N)."""
    from qcom_hexagon_backend.sharding import shard_range, shard_width

    q = hx()
    ns = shard_width(LM_N, world)
    assert ns == LM_N // world
    n0, n1 = shard_range(LM_N, world, world - 1)
    d = cuda_device
    if kind == "bf16":
        a, w = _lm_bf16(510 + world, LM_N)
    else:
        a, w = _lm_int8(520 + world, LM_N)
    ws = w[n0:n1].contiguous()
    out = q.gemm(a.to(d), ws.to(d))
    torch.cuda.synchronize()
    assert out.shape == (LM_M, ns)
    rows = _rows(LM_M, 256, world)
    got = out[torch.from_numpy(rows).to(d)].cpu()
    if kind == "bf16":
        assert_close(got.float().numpy(), O.matmul_f32(to_np32(a[torch.from_numpy(rows)]), to_np32(ws)))
    else:
        np.testing.assert_array_equal(got.numpy(), _exact_int8_rows(a.numpy()[rows], ws.numpy()))


# ---------------------------------------------------------------- fused gather, one GPU
def _p2p_call(q, a, w, bufs, flags, world, rank, epoch, err, odt=torch.bfloat16, ce_chunks=None):
    from qcom_hexagon_backend import _lib, ops

    lib = _lib.load()
    ns = w.shape[0]
    view = bufs[rank].view(odt).view(world, a.shape[0], ns)[rank]
    d, _, dev = ops.make_desc(a, w, out=view, b_const=True)
    cb = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
    cf = (ctypes.c_void_p * world)(*[f.data_ptr() for f in flags])
    with torch.cuda.device(dev):
        if ce_chunks is not None:
            return lib.hx_sharded_gemm_gather_ce(ctypes.byref(d), rank, world, cb, cf, epoch,
                                                 ctypes.c_void_p(err.data_ptr()), ce_chunks,
                                                 ctypes.c_void_p(ops._stream_ptr(dev)))
        return lib.hx_sharded_gemm_gather_p2p(ctypes.byref(d), rank, world, cb, cf, epoch,
                                              ctypes.c_void_p(err.data_ptr()),
                                              ctypes.c_void_p(ops._stream_ptr(dev)))


@pytest.mark.parametrize("transfer", ["epilogue", "ce_auto", "ce_3"])
@pytest.mark.parametrize("world,rank", [(2, 0), (2, 1), (4, 2), (8, 5)])
@pytest.mark.parametrize("kind", ["bf16", "int8"])
def test_peer_store_epilogue_one_gpu(cuda_device, world, rank, kind, transfer):
    """The GEMM's epilogue stores this rank's shard into every rank's gather
    buffer.  All `world` buffers live on this GPU; the other ranks' flags are
    pre-published (value 1000 >= every barrier value used here), so both
    barriers pass at once and no kernel waits on another kernel."""
    from qcom_hexagon_backend import _lib

    q = hx()
    d = cuda_device
    M, K, ns = 1000, 512, 1576  # a partial 256-column tile; 16-byte aligned rows
    g = torch.Generator().manual_seed(600 + world * 10 + rank)
    if kind == "bf16":
        a, w = _bf16((M, K), g), _bf16((ns, K), g, 0.02)
        odt, ref = torch.bfloat16, None
    else:
        a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        w = torch.randint(-127, 128, (ns, K), generator=g, dtype=torch.int8)
        odt = torch.int32
    esz = torch.empty(0, dtype=odt).element_size()
    bufs = [torch.full((world * M * ns * esz,), 0x7F, dtype=torch.uint8, device=d) for _ in range(world)]
    flags = [torch.zeros(64, dtype=torch.int32, device=d) for _ in range(world)]
    flags[rank][:world] = 1000
    err = torch.zeros(1, dtype=torch.int32, device=d)
    for epoch in range(3):
        ad = (a.to(d) if kind == "int8" else (a.float() * (epoch + 1)).to(torch.bfloat16).to(d))
        ce = None if transfer == "epilogue" else (0 if transfer == "ce_auto" else 3)
        rc = _p2p_call(q, ad, w.to(d), bufs, flags, world, rank, epoch, err, odt, ce)
        assert rc == 0, _lib.load().hx_last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        if kind == "bf16":
            ref = O.matmul_f32(to_np32(ad), to_np32(w))
        else:
            ref = _exact_int8_rows(a.numpy(), w.numpy())
        for r in range(world):
            slot = bufs[r].view(odt).view(world, M, ns)[rank].cpu()
            if kind == "bf16":
                assert_close(slot.float().numpy(), ref)
            else:
                np.testing.assert_array_equal(slot.numpy(), ref)
        # the barrier published this rank's arrival in every peer's array
        for r in range(world):
            if r != rank:
                assert int(flags[r][rank].item()) == 2 * epoch + 2
    # other ranks' slots are untouched
    for r in range(world):
        other = (rank + 1) % world
        raw = bufs[r].view(world, M * ns * esz)[other]
        assert bool((raw == 0x7F).all())


def test_peer_barrier_timeout_sets_status(cuda_device):
    """The peer's flag is never set: both bounded waits run out (about 2 s
    each), the error word reads 41, the call still returns and the context
    stays usable (a later GEMM is correct)."""
    q = hx()
    d = cuda_device
    g = torch.Generator().manual_seed(700)
    a, w = _bf16((256, 256), g), _bf16((512, 256), g, 0.02)
    bufs = [torch.zeros(2 * 256 * 512 * 2, dtype=torch.uint8, device=d) for _ in range(2)]
    flags = [torch.zeros(64, dtype=torch.int32, device=d) for _ in range(2)]
    err = torch.zeros(1, dtype=torch.int32, device=d)
    rc = _p2p_call(q, a.to(d), w.to(d), bufs, flags, 2, 0, 0, err)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 41
    out = q.gemm(a.to(d), w.to(d))
    torch.cuda.synchronize()
    assert_close(to_np32(out), O.matmul_f32(to_np32(a), to_np32(w)))
