"""Convolution as a GEMM (hx_conv2d through ops.conv2d_nhwc / ops.conv2d)
against the CPU oracle (fp32 sum over filter taps; the golden of
benchmark_models/micro_bench/test_conv_benchmark.py, torch nn.Conv2d on the
CPU, which MatmulToConvPass.cpp's conv_2d_nhwc_fhwc mirrors).

The reference benchmark's configurations (batch 1, 3x3 filters, padding 1)
run in fp16: those with C a multiple of 64 take the implicit GEMM (4-D TMA
boxes at tap-shifted coordinates, zero fill as padding), the others
(C = 16, 32) the im2col workspace path.  Plus batch > 1, stride 2,
dilation 2, 1x1 and 5x5 filters, bf16, fused bias / GELU / residual, and the
FX route of nn.Conv2d.  Tolerance as every fp16 / bf16 GEMM test:
max |out - ref| / max |ref| <= 1e-2 plus the elementwise bound.
"""

import pytest
import torch

from oracle import gemm_oracle as O
from test_gemm_gpu import assert_close, to_np32

pytestmark = pytest.mark.gpu

# (batch, in_channels, out_channels, height, width, kernel) of test_conv_benchmark.py
REF_CONFIGS = [(1, 16, 32, 32, 32, 3), (1, 32, 64, 16, 16, 3), (1, 64, 64, 16, 16, 3),
               (1, 128, 128, 8, 8, 3), (1, 256, 256, 8, 8, 3), (1, 512, 512, 4, 4, 3),
               (1, 1024, 1024, 4, 4, 3), (1, 2048, 2048, 4, 4, 3)]


def hx():
    import qcom_hexagon_backend as q

    return q


def _inputs(N, C, OC, H, W, K, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).to(dtype)
    w = (torch.randn(OC, K, K, C, generator=g) / (K * (C ** 0.5))).to(dtype)
    b = (torch.randn(OC, generator=g) * 0.1).to(dtype)
    return x, w, b


def _workspace(q, **kw):
    """Bytes of im2col workspace the library asks for (0 = implicit GEMM)."""
    import ctypes
    from qcom_hexagon_backend import _lib

    d = _lib.HxConv2dDesc()
    for k, v in kw.items():
        setattr(d, k, v)
    n = ctypes.c_int64()
    _lib.check(_lib.load().hx_conv2d_workspace_size(ctypes.byref(d), ctypes.byref(n)), "ws")
    return n.value


@pytest.mark.parametrize("cfg", REF_CONFIGS, ids=lambda c: "x".join(map(str, c)))
def test_reference_benchmark_configs(cuda_device, cfg):
    q = hx()
    N, C, OC, H, W, K = cfg
    x, w, b = _inputs(N, C, OC, H, W, K, torch.float16, sum(cfg))
    y = q.ops.conv2d_nhwc(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), padding=K // 2)
    torch.cuda.synchronize()
    ref = O.conv2d_nhwc_ref(to_np32(x), to_np32(w), padding=(K // 2, K // 2), bias=to_np32(b))
    assert y.shape == ref.shape
    assert_close(to_np32(y), ref)
    ws = _workspace(q, N=N, H=H, W=W, C=C, OC=OC, KH=K, KW=K, stride_h=1, stride_w=1, pad_h=K // 2,
                    pad_w=K // 2, dil_h=1, dil_w=1, dtype=1, x=64, w=64)
    assert (ws == 0) == (C % 64 == 0 and 128 // min(W, 128) <= H), ws


@pytest.mark.parametrize("case", [
    dict(N=4, C=64, OC=96, H=16, W=16, K=3, s=1, p=1, d=1),     # implicit, batch 4 (H*W = 256)
    dict(N=2, C=128, OC=200, H=32, W=32, K=1, s=1, p=0, d=1),   # 1x1: a plain GEMM through the 4-D map
    dict(N=1, C=64, OC=64, H=20, W=16, K=5, s=1, p=2, d=1),     # 5x5, tall image
    dict(N=1, C=64, OC=72, H=8, W=256, K=3, s=1, p=1, d=1),     # wide rows (OW % 128 == 0)
    dict(N=2, C=64, OC=64, H=17, W=17, K=3, s=2, p=1, d=1),     # stride 2: im2col
    dict(N=1, C=64, OC=64, H=16, W=16, K=3, s=1, p=2, d=2),     # dilation 2: im2col
    dict(N=3, C=24, OC=40, H=10, W=12, K=3, s=1, p=0, d=1),     # C % 8 == 0, no padding: im2col
    dict(N=1, C=3, OC=16, H=15, W=15, K=3, s=1, p=1, d=1),      # C = 3 (scalar im2col)
], ids=lambda c: "n{N}c{C}o{OC}h{H}w{W}k{K}s{s}p{p}d{d}".format(**c))
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_conv_shapes(cuda_device, case, dtype):
    q = hx()
    c = case
    x, w, b = _inputs(c["N"], c["C"], c["OC"], c["H"], c["W"], c["K"], dtype, 1000 + c["C"] + c["H"])
    y = q.ops.conv2d_nhwc(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), stride=c["s"],
                          padding=c["p"], dilation=c["d"])
    torch.cuda.synchronize()
    ref = O.conv2d_nhwc_ref(to_np32(x), to_np32(w), stride=(c["s"],) * 2, padding=(c["p"],) * 2,
                            dilation=(c["d"],) * 2, bias=to_np32(b))
    assert_close(to_np32(y), ref)


def test_conv_fused_epilogues(cuda_device):
    q = hx()
    d = cuda_device
    x, w, b = _inputs(1, 64, 64, 16, 16, 3, torch.float16, 1100)
    ref = O.conv2d_nhwc_ref(to_np32(x), to_np32(w), padding=(1, 1), bias=to_np32(b))
    y = q.ops.conv2d_nhwc(x.to(d), w.to(d), b.to(d), padding=1, epilogue="bias_gelu_tanh")
    torch.cuda.synchronize()
    assert_close(to_np32(y), O.gelu_tanh(ref))
    res = x.to(d)  # same shape as y: [1, 16, 16, 64]
    y2 = q.ops.conv2d_nhwc(x.to(d), w.to(d), b.to(d), padding=1, epilogue="bias_residual", residual=res)
    torch.cuda.synchronize()
    assert_close(to_np32(y2), ref + to_np32(x))


def test_conv_nchw_and_fx(cuda_device):
    """ops.conv2d on NCHW tensors and an nn.Conv2d module through the FX backend."""
    from qcom_hexagon_backend import fx_backend as FX

    q = hx()
    torch.manual_seed(1200)
    m = torch.nn.Sequential(torch.nn.Conv2d(64, 128, 3, padding=1), torch.nn.ReLU(),
                            torch.nn.Conv2d(128, 64, 3, padding=1)).eval()
    x = torch.randn(2, 64, 16, 16)
    with torch.no_grad():
        ref = m(x).numpy()
    m16 = m.half()
    y1 = q.ops.conv2d(x.half().to(cuda_device), m16[0].weight.to(cuda_device), m16[0].bias.to(cuda_device), padding=1)
    torch.cuda.synchronize()
    with torch.no_grad():
        r1 = torch.nn.functional.conv2d(x, m[0].weight.float(), m[0].bias.float(), padding=1).numpy()
    assert_close(to_np32(y1), r1, tol=1e-2)
    gm = FX.compile_module(m16, cuda_device, example_inputs=[x.half()], mode="trace")
    assert sum(1 for n in gm.graph.nodes if n.target is FX.hx_conv2d) == 2
    with torch.no_grad():
        y = gm(x.half().to(cuda_device))
    torch.cuda.synchronize()
    assert_close(to_np32(y), ref, tol=2e-2)
