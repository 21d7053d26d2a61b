"""CPU oracle for the linear-layer GEMM path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this module, and only as the checker or the timed CPU
baseline.  The product path (qcom_hexagon_backend) never calls it.

What it restates.  The reference (hustc12/hexagon-mlir) checks every matmul
against PyTorch on the host CPU, in fp32:
  * test/python/triton/test_matmul.py:90   reference = torch.matmul(A, B)
  * test/python/torch-mlir/utils.py:54     golden = self.model(*inputs)
  * test/python/mlir/hexkl_linalg_matmul/wrapper.cpp:47-66
        acc(float) += (float)act[row*K+k] * W[k*M+col]   (fp32 accumulation
        of fp16 products, |diff| <= 1e-2)
  * epilogues: F.gelu(approximate="tanh") (test/python/triton/test_gelu.py:72),
    F.silu (test/python/triton/test_silu.py:63), bias / residual adds as in
    aten.linear / aten.addmm lowered by torch-mlir
    (benchmark_models/run_gpt2lmheadmodel.py:75-82).
This module computes the same functions in numpy fp32 (inputs upcast
exactly, fp32 accumulation, epilogue in fp32).  int8 W8A8 is exact int32
(numpy int64 matmul, then checked to fit int32); W8A16 is dequantise-then-
fp32-matmul, the lowering the reference applies to quantised ops
(lib/Conversion/LinalgToLLVM/LinalgToLLVMPass.cpp:203-209).

Parity pin: tests/golden/ holds fixtures produced by PyTorch CPU (the
reference's own golden path) by tests/golden/make_golden.py; test_oracle.py
checks this oracle against them.  The reference's compiled Hexagon kernel
cannot run here (no Hexagon SDK/simulator), so the pin is to its golden, not
to its device output.  The int8 paths have no reference test (the reference
has no int8 GEMM); they are pinned only to exact integer arithmetic.
"""

from __future__ import annotations

import numpy as np

GELU_K0 = np.float32(0.7978845608028654)  # sqrt(2/pi)
GELU_K1 = np.float32(0.044715)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """F.gelu(x, approximate="tanh") in fp32."""
    x = x.astype(np.float32)
    return (np.float32(0.5) * x * (np.float32(1) + np.tanh(GELU_K0 * (x + GELU_K1 * x * x * x)))).astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    """F.silu(x) = x * sigmoid(x) in fp32."""
    x = x.astype(np.float32)
    return (x / (np.float32(1) + np.exp(-x))).astype(np.float32)


def as_f32(a: np.ndarray) -> np.ndarray:
    return np.asarray(a).astype(np.float32)


def matmul_f32(a: np.ndarray, b: np.ndarray, b_layout: str = "nk") -> np.ndarray:
    """fp32-accumulated product of upcast operands.  b is W[N,K] ("nk") or B[K,N] ("kn")."""
    A = as_f32(a)
    B = as_f32(b)
    return (A @ (B.T if b_layout == "nk" else B)).astype(np.float32)


def linear_ref(a, b, *, b_layout="nk", epilogue="none", bias=None, residual=None, scale=None):
    """fp32 oracle of epilogue(a @ B) for every fused epilogue the kernels implement.

    For "swiglu", b is W[2N,K] = [gate; up] and the result has N columns.
    """
    if epilogue == "swiglu":
        w = as_f32(b)
        n = w.shape[0] // 2
        g = as_f32(a) @ w[:n].T
        u = as_f32(a) @ w[n:].T
        return (silu(g) * u).astype(np.float32)
    acc = matmul_f32(a, b, b_layout)
    if epilogue == "dequant_scale":
        acc = acc * as_f32(scale)[None, :]
    if bias is not None and epilogue in ("bias", "bias_gelu_tanh", "bias_residual", "dequant_scale", "bias_silu"):
        acc = acc + as_f32(bias)[None, :]
    if epilogue in ("bias_residual", "residual"):
        acc = acc + as_f32(residual)
    if epilogue == "bias_gelu_tanh":
        acc = gelu_tanh(acc)
    elif epilogue == "bias_silu":
        acc = silu(acc)
    return acc.astype(np.float32)


def int8_gemm_exact(a_s8: np.ndarray, w_s8: np.ndarray, b_layout: str = "nk") -> np.ndarray:
    """Exact int32 C = A . B for int8 operands (W8A8, int32 accumulate)."""
    A = np.asarray(a_s8).astype(np.int64)
    B = np.asarray(w_s8).astype(np.int64)
    C = A @ (B.T if b_layout == "nk" else B)
    if C.size and (C.max() > np.iinfo(np.int32).max or C.min() < np.iinfo(np.int32).min):
        raise OverflowError("int8 product does not fit int32")
    return C.astype(np.int32)


def w8a16_ref(x_f16, w_s8, scale_f16, bias_f16=None) -> np.ndarray:
    """fp32 y = x . (W * scale[:, None])^T (+ bias): dequantise, then fp32 matmul."""
    Wd = as_f32(w_s8) * as_f32(scale_f16)[:, None]
    y = as_f32(x_f16) @ Wd.T
    if bias_f16 is not None:
        y = y + as_f32(bias_f16)[None, :]
    return y.astype(np.float32)


def max_rel_err(out, ref) -> float:
    """max |out - ref| / max |ref|: the normwise relative error the tolerance
    (<= 1e-2 for fp16/bf16 with fp32 accumulate) is stated on."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = max(np.abs(ref).max(initial=0.0), 1e-30)
    return float(np.abs(out - ref).max(initial=0.0) / denom)


def bf16_to_f32(bits_u16: np.ndarray) -> np.ndarray:
    """Decode bf16 values stored as raw uint16 bits."""
    return (np.asarray(bits_u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (finite inputs)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    return ((u + rounding) >> 16).astype(np.uint16)


def batch_matmul_f32(a, b, b_layout: str = "kn") -> np.ndarray:
    """fp32 batched product of upcast operands: a [B,M,K]; b [B,K,N] ("kn",
    linalg.batch_matmul) or [B,N,K] ("nk", batch_matmul_transpose_b, the
    transpose fold of ScheduleMatmulForHVXPass.cpp:105-167); a 2-D b is
    shared by every item.  Same arithmetic as matmul_f32, per item."""
    A = as_f32(a)
    B = as_f32(b)
    if B.ndim == 2:
        B = np.broadcast_to(B, (A.shape[0],) + B.shape)
    Bk = np.swapaxes(B, -1, -2) if b_layout == "nk" else B
    return np.matmul(A, Bk).astype(np.float32)


def softmax_ref(x, log: bool = False) -> np.ndarray:
    """Row softmax (or log-softmax) in fp64 of upcast x: the golden of
    test/python/triton/test_softmax.py / test_online_softmax.py
    (torch.nn.functional.softmax(x, dim=1))."""
    X = np.asarray(x, dtype=np.float64)
    mx = X.max(axis=-1, keepdims=True)
    e = np.exp(X - mx)
    s = e.sum(axis=-1, keepdims=True)
    return (X - mx - np.log(s)) if log else e / s


def norm_ref(x, kind: str = "layer", gamma=None, beta=None, eps: float = 1e-5) -> np.ndarray:
    """F.layer_norm (biased variance) or F.rms_norm over the last dimension, in
    fp64: the goldens of test/python/triton/test_layer_norm.py and
    test_rms_norm.py."""
    X = np.asarray(x, dtype=np.float64)
    if kind == "layer":
        mu = X.mean(-1, keepdims=True)
        var = ((X - mu) ** 2).mean(-1, keepdims=True)
        Y = (X - mu) / np.sqrt(var + eps)
    else:
        Y = X / np.sqrt((X * X).mean(-1, keepdims=True) + eps)
    if gamma is not None:
        Y = Y * np.asarray(gamma, np.float64)
    if beta is not None:
        Y = Y + np.asarray(beta, np.float64)
    return Y


def norm_linear_ref(x, w, *, kind="layer", gamma=None, beta=None, eps=1e-5, epilogue="none", bias=None,
                    residual=None) -> np.ndarray:
    """epilogue(norm(x) @ W^T): the norm in fp64, rounded to nothing, then the
    fp32 linear oracle.  (Unfused reference order: norm pass, then matmul.)"""
    y = norm_ref(x, kind, gamma, beta, eps).astype(np.float32)
    return linear_ref(y, w, epilogue=epilogue, bias=bias, residual=residual)


def conv2d_nhwc_ref(x, w, *, stride=(1, 1), padding=(0, 0), dilation=(1, 1), bias=None) -> np.ndarray:
    """fp32 2-D convolution of upcast operands, NHWC activations and OHWI
    filters, zero padding: the golden of
    benchmark_models/micro_bench/test_conv_benchmark.py (torch nn.Conv2d on
    the CPU), written as a sum over filter taps of [pixels, C] @ [C, OC]."""
    X = as_f32(x)
    Wt = as_f32(w)
    N, H, W, C = X.shape
    OC, KH, KW, _ = Wt.shape
    sh, sw = stride
    ph, pw = padding
    dh, dw = dilation
    OH = (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1
    OW = (W + 2 * pw - dw * (KW - 1) - 1) // sw + 1
    Xp = np.zeros((N, H + 2 * ph, W + 2 * pw, C), np.float32)
    Xp[:, ph:ph + H, pw:pw + W, :] = X
    out = np.zeros((N, OH, OW, OC), np.float32)
    for kh in range(KH):
        for kw in range(KW):
            patch = Xp[:, kh * dh: kh * dh + (OH - 1) * sh + 1: sh, kw * dw: kw * dw + (OW - 1) * sw + 1: sw, :]
            out += (patch.reshape(-1, C) @ Wt[:, kh, kw, :].T).reshape(N, OH, OW, OC)
    if bias is not None:
        out += as_f32(bias)
    return out
