"""Batched GEMM (hx_gemm_batched through ops.bmm / ops.matmul_batched) against
the CPU oracle: linalg.batch_matmul (B[K,N] items) and
batch_matmul_transpose_b (B[N,K] items), the two batched forms
ScheduleMatmulForHVXPass.cpp:105-167 produces.

Attention shapes: GPT-2's 12 heads, S = 1024, head dim 64, fp16 — scores
q @ k^T (K = 64, N = 1024, k read as a transposed view) and context p @ v
(K = 1024, N = 64).  Plus item tails (M not a multiple of 128: one launch per
item), N / K tails, strided items, a shared B, bf16, int8 (exact) and an
epilogue.  Tolerance as the other fp16/bf16 tests: max |out - ref| / max |ref|
<= 1e-2 (plus the elementwise bound); int8 bit-exact.
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


def _rand(shape, g, dtype, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_attention_scores_gpt2_heads(cuda_device, dtype):
    """q @ k^T for 12 heads x 1024 x 64: k is a transposed view -> W[N,K] items."""
    q = hx()
    g = torch.Generator().manual_seed(800)
    Q = _rand((1, 12, 1024, 64), g, dtype)
    Kt = _rand((1, 12, 1024, 64), g, dtype)
    out = q.matmul_batched(Q.to(cuda_device), Kt.to(cuda_device).transpose(-1, -2))
    torch.cuda.synchronize()
    assert out.shape == (1, 12, 1024, 1024)
    ref = O.batch_matmul_f32(to_np32(Q.reshape(12, 1024, 64)), to_np32(Kt.reshape(12, 1024, 64)), "nk")
    assert_close(to_np32(out).reshape(12, 1024, 1024), ref)


def test_attention_context_gpt2_heads(cuda_device):
    """p @ v for 12 heads: [1024 x 1024] . [1024 x 64] -> B[K,N] items."""
    q = hx()
    g = torch.Generator().manual_seed(801)
    P = torch.softmax(torch.randn(12, 1024, 1024, generator=g), -1).half()
    V = _rand((12, 1024, 64), g, torch.float16)
    out = q.bmm(P.to(cuda_device), V.to(cuda_device), b_layout="kn")
    torch.cuda.synchronize()
    assert_close(to_np32(out), O.batch_matmul_f32(to_np32(P), to_np32(V), "kn"))


@pytest.mark.parametrize("shape", [(3, 256, 200, 72), (5, 128, 64, 512), (2, 100, 130, 40), (4, 200, 96, 64)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_bmm_shapes(cuda_device, shape, layout):
    """One launch when M % 128 == 0, item by item otherwise; N and K tails."""
    q = hx()
    nb, M, N, K = shape
    g = torch.Generator().manual_seed(810 + M + N)
    a = _rand((nb, M, K), g, torch.float16)
    b = _rand((nb, K, N) if layout == "kn" else (nb, N, K), g, torch.float16, 0.1)
    out = q.bmm(a.to(cuda_device), b.to(cuda_device), b_layout=layout)
    torch.cuda.synchronize()
    assert_close(to_np32(out), O.batch_matmul_f32(to_np32(a), to_np32(b), layout))


def test_bmm_strided_items_and_epilogue(cuda_device):
    """Items of A and B are slices of larger buffers (item strides > rows x ld);
    bias + residual epilogue with a batched residual."""
    q = hx()
    d = cuda_device
    g = torch.Generator().manual_seed(820)
    big_a = _rand((4, 384, 320), g, torch.bfloat16)
    big_b = _rand((4, 300, 200), g, torch.bfloat16, 0.1)
    a = big_a.to(d)[:, :256, :192]          # lda 320, item stride 384 * 320
    b = big_b.to(d)[:, :264, :192]          # W[N,K] items, ldb 200
    bias = _rand((264,), g, torch.bfloat16, 0.1).to(d)
    res = _rand((4, 256, 264), g, torch.bfloat16).to(d)
    out = q.bmm(a, b, b_layout="nk", epilogue="bias_residual", bias=bias, residual=res)
    torch.cuda.synchronize()
    ref = O.batch_matmul_f32(to_np32(a), to_np32(b), "nk") + to_np32(bias)[None, None, :] + to_np32(res)
    assert_close(to_np32(out), ref)


def test_bmm_shared_b(cuda_device):
    """A 2-D B shared by every item (stride_b = 0): one GEMM over batch x M rows."""
    q = hx()
    g = torch.Generator().manual_seed(830)
    a = _rand((6, 128, 96), g, torch.float16)
    w = _rand((80, 96), g, torch.float16, 0.1)
    out = q.bmm(a.to(cuda_device), w.to(cuda_device), b_layout="nk")
    torch.cuda.synchronize()
    assert_close(to_np32(out), O.batch_matmul_f32(to_np32(a), to_np32(w), "nk"))


def test_bmm_int8_exact(cuda_device):
    q = hx()
    g = torch.Generator().manual_seed(840)
    a = torch.randint(-127, 128, (3, 256, 512), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (3, 384, 512), generator=g, dtype=torch.int8)
    out = q.bmm(a.to(cuda_device), b.to(cuda_device), b_layout="nk")
    torch.cuda.synchronize()
    for i in range(3):
        np.testing.assert_array_equal(out[i].cpu().numpy(), O.int8_gemm_exact(a[i].numpy(), b[i].numpy()))


def test_matmul_batched_broadcast(cuda_device):
    """Broadcast batch dimensions: [2, 1, M, K] @ [3, K, N]."""
    q = hx()
    g = torch.Generator().manual_seed(850)
    x = _rand((2, 1, 128, 64), g, torch.float16)
    y = _rand((3, 64, 72), g, torch.float16, 0.1)
    out = q.matmul_batched(x.to(cuda_device), y.to(cuda_device))
    torch.cuda.synchronize()
    ref = np.matmul(to_np32(x), to_np32(y))
    assert out.shape == (2, 3, 128, 72)
    assert_close(to_np32(out), ref)


def test_bmm_empty_batch(cuda_device):
    q = hx()
    a = torch.empty(0, 128, 64, dtype=torch.float16, device=cuda_device)
    b = torch.empty(0, 64, 32, dtype=torch.float16, device=cuda_device)
    assert q.bmm(a, b).shape == (0, 128, 32)


def test_fx_attention_module(cuda_device):
    """An eager attention block (scores, softmax, context) through the FX
    backend: both batched products and both projections run on the kernels."""
    from qcom_hexagon_backend import fx_backend as FX

    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.qkv = torch.nn.Linear(768, 3 * 768)
            self.o = torch.nn.Linear(768, 768)

        def forward(self, x):
            B, S, _ = x.shape
            q, k, v = self.qkv(x).split(768, dim=-1)
            q = q.view(B, S, 12, 64).transpose(1, 2)
            k = k.view(B, S, 12, 64).transpose(1, 2)
            v = v.view(B, S, 12, 64).transpose(1, 2)
            p = torch.softmax(torch.matmul(q, k.transpose(-1, -2)) * 0.125, dim=-1)
            ctx = torch.matmul(p, v).transpose(1, 2).reshape(B, S, 768)
            return self.o(ctx)

    torch.manual_seed(860)
    m = Attn().half().eval()
    x = torch.randn(1, 256, 768).half()
    with torch.no_grad():
        ref = m.float()(x.float()).numpy()
    m.half()
    gm = FX.compile_module(m, cuda_device, example_inputs=[x], mode="export")
    assert sum(1 for n in gm.graph.nodes if n.target is FX.hx_bmm) == 2
    assert FX.count_hx_calls(gm) == 4
    with torch.no_grad():
        out = gm(x.to(cuda_device))
    torch.cuda.synchronize()
    assert_close(to_np32(out), ref, tol=2e-2)
