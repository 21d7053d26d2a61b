"""Row kernels either side of the linear layer, against the CPU oracle:

  * softmax / log-softmax over rows (hx_softmax), including the LM head's
    50304-wide vocabulary rows, one pass (row in shared memory) and two;
  * the vocab-parallel softmax (hx_softmax_stats -> combine -> apply) with
    the vocabulary split into 2, 4 and 8 column shards of one GPU's logits
    (the same arithmetic each rank runs; the cross-rank exchange is only of
    the [M, 2] stats);
  * LayerNorm / RMSNorm row statistics and the GEMMs that fold them in
    (hx_gemm_norm), with bias, GELU, residual and SwiGLU epilogues.

Tolerances: softmax probabilities |y - ref| <= 2e-3 * max(ref) + the output
dtype's rounding (fp16 / bf16 / fp32 outputs), log-softmax <= 1e-4 absolute
for fp32 outputs; normalised linears max rel err <= 1e-2 as every other
fp16 / bf16 GEMM test, and a max abs error within 1.5x that of the unfused
pipeline in the same dtype (normalised activation rounded, then the GEMM).  Reference goldens: test/python/triton/test_softmax.py,
test_online_softmax.py (atol 1e-5 on fp32 128x128), test_layer_norm.py,
test_rms_norm.py.
"""

import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O
from test_gemm_gpu import assert_close, to_np32

pytestmark = pytest.mark.gpu


def hx():
    import qcom_hexagon_backend as q

    return q


RTOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 1e-2}


def _check_probs(out, ref, dtype):
    err = np.abs(to_np32(out).astype(np.float64) - ref)
    bound = RTOL[dtype] * np.abs(ref) + 1e-6 * np.abs(ref).max(axis=-1, keepdims=True) + 1e-7
    assert (err <= bound).all(), float((err / np.maximum(np.abs(ref), 1e-30)).max())


@pytest.mark.parametrize("shape", [(128, 128), (300, 1000), (64, 50304), (8, 70000), (3, 130000)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
def test_softmax_rows(cuda_device, shape, dtype):
    q = hx()
    g = torch.Generator().manual_seed(900 + shape[1])
    x = (torch.randn(*shape, generator=g) * 3).to(dtype)
    out = q.ops.softmax(x.to(cuda_device), out_dtype=torch.float32)
    torch.cuda.synchronize()
    _check_probs(out, O.softmax_ref(to_np32(x)), torch.float32)
    y = q.ops.softmax(x.to(cuda_device))  # output in the input dtype
    torch.cuda.synchronize()
    _check_probs(y, O.softmax_ref(to_np32(x)), dtype)


def test_log_softmax_and_strided_rows(cuda_device):
    q = hx()
    g = torch.Generator().manual_seed(910)
    big = (torch.randn(64, 1100, generator=g) * 4).to(torch.bfloat16).to(cuda_device)
    x = big[:, :1000]  # ldx 1100
    out = q.ops.softmax(x, log=True, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = O.softmax_ref(to_np32(x), log=True)
    assert np.abs(to_np32(out) - ref).max() <= 1e-4


def test_softmax_masked_rows(cuda_device):
    """-inf entries (masked vocabulary) contribute nothing; a row of one
    finite value is a one-hot."""
    q = hx()
    x = torch.randn(4, 512)
    x[0, 100:] = float("-inf")
    x[1, :] = float("-inf")
    x[1, 7] = 2.0
    out = q.ops.softmax(x.to(cuda_device), out_dtype=torch.float32).cpu().numpy()
    ref = O.softmax_ref(x.numpy())
    assert np.isfinite(out).all()
    assert np.abs(out - ref).max() <= 1e-6
    assert out[1, 7] == 1.0


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("log", [False, True])
def test_vocab_parallel_softmax_shards(cuda_device, world, log):
    """The LM head's 50304-wide rows split into `world` column shards (the
    sharded GEMM's layout): per-shard stats, combine, per-shard apply."""
    from qcom_hexagon_backend.sharding import shard_range

    q = hx()
    g = torch.Generator().manual_seed(920 + world)
    M, N = 256, 50304
    x = (torch.randn(M, N, generator=g) * 2).to(torch.bfloat16).to(cuda_device)
    parts, stats = [], []
    for r in range(world):
        n0, n1 = shard_range(N, world, r)
        parts.append(x[:, n0:n1])
        stats.append(q.ops.softmax_stats(x[:, n0:n1]))
    glob = q.ops.softmax_combine(torch.stack(stats).contiguous())
    ys = [q.ops.softmax_apply(p, glob, log=log, out_dtype=torch.float32) for p in parts]
    torch.cuda.synchronize()
    y = torch.cat(ys, 1).cpu().numpy()
    ref = O.softmax_ref(to_np32(x), log=log)
    if log:
        assert np.abs(y - ref).max() <= 1e-4
    else:
        _check_probs(torch.from_numpy(y), ref, torch.float32)


@pytest.mark.parametrize("kind", ["layer", "rms"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32], ids=["f16", "bf16", "f32"])
def test_row_norm_stats(cuda_device, kind, dtype):
    q = hx()
    g = torch.Generator().manual_seed(930)
    x = (torch.randn(333, 896, generator=g) * 2 + 5).to(dtype)  # offset mean: shifted sums
    st = q.ops.row_norm_stats(x.to(cuda_device), kind, 1e-5).cpu().numpy()
    X = to_np32(x).astype(np.float64)
    if kind == "layer":
        mu, var = X.mean(-1), X.var(-1)
        assert np.abs(st[:, 0] - mu).max() <= 1e-4 * np.abs(mu).max()
    else:
        var = (X * X).mean(-1)
        assert (st[:, 0] == 0).all()
    np.testing.assert_allclose(st[:, 1], 1 / np.sqrt(var + 1e-5), rtol=1e-4)


NORM_CASES = [("layer", "bias", torch.float16), ("layer", "bias_gelu_tanh", torch.float16),
              ("layer", "bias_residual", torch.bfloat16), ("layer", "none", torch.bfloat16),
              ("rms", "none", torch.bfloat16), ("rms", "swiglu", torch.bfloat16),
              ("layer", "swiglu", torch.float16), ("rms", "bias_silu", torch.float16)]


@pytest.mark.parametrize("kind,epilogue,dtype", NORM_CASES, ids=lambda v: str(v).replace("torch.", ""))
@pytest.mark.parametrize("shape", [(1024, 2304, 768), (200, 300, 136)], ids=["gpt2qkv", "tails"])
def test_gemm_with_folded_norm(cuda_device, kind, epilogue, dtype, shape):
    q = hx()
    M, N, K = shape
    d = cuda_device
    g = torch.Generator().manual_seed(940 + M)
    x = (torch.randn(M, K, generator=g) + 0.5).to(dtype)
    rows = 2 * N if epilogue == "swiglu" else N
    w = (torch.randn(rows, K, generator=g) * 0.02).to(dtype)
    gamma = (1 + 0.1 * torch.randn(K, generator=g)).to(dtype)
    beta = (0.1 * torch.randn(K, generator=g)).to(dtype) if kind == "layer" else None
    bias = (torch.randn(N, generator=g) * 0.02).to(dtype) if "bias" in epilogue else None
    res = torch.randn(M, N, generator=g).to(dtype) if "residual" in epilogue else None
    if epilogue == "swiglu" and beta is not None:
        beta = None  # a bias after the fold has nowhere to go in SwiGLU
    wf, cs, bf = q.ops.fold_norm_weight(w.to(d), bias.to(d) if bias is not None else None, gamma.to(d),
                                        beta.to(d) if beta is not None else None, kind)
    stats = q.ops.row_norm_stats(x.to(d), kind, 1e-5)
    act = {"bias_gelu_tanh": "gelu_tanh", "bias_silu": "silu", "swiglu": "swiglu"}.get(epilogue)
    out = q.ops.linear_norm(x.to(d), wf, cs, bf, stats, kind, activation=act,
                            residual=res.to(d) if res is not None else None)
    torch.cuda.synchronize()
    ref = O.norm_linear_ref(to_np32(x), to_np32(w), kind=kind, gamma=to_np32(gamma),
                            beta=to_np32(beta) if beta is not None else None, epilogue=epilogue,
                            bias=to_np32(bias) if bias is not None else None,
                            residual=to_np32(res) if res is not None else None)
    got = to_np32(out)
    assert O.max_rel_err(got, ref) <= 1e-2
    # Folding may not cost accuracy against the unfused pipeline in the same
    # dtype (the normalised activation rounded to it, then the same GEMM).
    xn = O.norm_ref(to_np32(x), kind, to_np32(gamma), to_np32(beta) if beta is not None else None)
    unfused = q.gemm(torch.from_numpy(xn.astype(np.float32)).to(dtype).to(d), w.to(d), epilogue=epilogue,
                     bias=bias.to(d) if bias is not None else None, residual=res.to(d) if res is not None else None)
    torch.cuda.synchronize()
    e_fused = np.abs(got - ref).max()
    e_unfused = np.abs(to_np32(unfused) - ref).max()
    assert e_fused <= 1.5 * e_unfused + 1e-3 * np.abs(ref).max(), (e_fused, e_unfused)
