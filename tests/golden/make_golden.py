"""Generate the golden fixtures in this directory from PyTorch CPU.

PyTorch on the host CPU is the reference's own golden for this path
(test/python/triton/test_matmul.py:90 `torch.matmul`,
test/python/torch-mlir/utils.py:54 the model's PyTorch forward,
test/python/mlir/hexkl_linalg_matmul/wrapper.cpp:47-66 fp32 accumulation).
Each case stores its seeded inputs and the PyTorch-CPU fp32 output, so the
oracle and the GPU kernels can be checked against the same numbers without
PyTorch's CPU kernels in the loop.

    python tests/golden/make_golden.py      # rewrites golden_*.npz

Inputs follow the value distributions of the benchmark configs, at sizes
small enough to keep the files to a few hundred KB: N(0,1) activations,
N(0,0.02) weights and biases, U{-127..127} int8, U(0.001,0.02) scales.
Shapes deliberately include tails (dimensions not multiples of the tiles).
"""

from __future__ import annotations

import os

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def fp_case(seed, M, N, K, dtype, epilogue, b_layout="nk"):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(dtype)
    if epilogue == "swiglu":
        w = (torch.randn(2 * N, K, generator=g) * 0.02).to(dtype)
    elif b_layout == "nk":
        w = (torch.randn(N, K, generator=g) * 0.02).to(dtype)
    else:
        w = (torch.randn(K, N, generator=g) * 0.02).to(dtype)
    bias = (torch.randn(N, generator=g) * 0.02).to(dtype)
    res = torch.randn(M, N, generator=g).to(dtype)
    af, wf, bf, rf = a.float(), w.float(), bias.float(), res.float()
    if epilogue == "swiglu":
        out = F.silu(af @ wf[:N].T) * (af @ wf[N:].T)
    else:
        acc = af @ (wf.T if b_layout == "nk" else wf)
        if epilogue == "none":
            out = acc
        elif epilogue == "bias":
            out = acc + bf
        elif epilogue == "bias_gelu_tanh":
            out = F.gelu(acc + bf, approximate="tanh")
        elif epilogue == "bias_silu":
            out = F.silu(acc + bf)
        elif epilogue == "bias_residual":
            out = acc + bf + rf
        elif epilogue == "residual":
            out = acc + rf
        else:
            raise ValueError(epilogue)
    return dict(a=_bits(a), w=_bits(w), bias=_bits(bias), residual=_bits(res),
                out=out.numpy().astype(np.float32),
                meta=np.array([M, N, K, seed]), dtype=str(dtype).split(".")[-1],
                epilogue=epilogue, b_layout=b_layout)


def int8_case(seed, M, N, K):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int64).to(torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int64).to(torch.int8)
    out = a.to(torch.int64) @ w.to(torch.int64).T
    return dict(a=a.numpy(), w=w.numpy(), out=out.to(torch.int32).numpy(), meta=np.array([M, N, K, seed]))


def w8a16_case(seed, M, N, K):
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int64).to(torch.int8)
    scale = (torch.rand(N, generator=g) * 0.019 + 0.001).to(torch.float16)
    x = torch.randn(M, K, generator=g).to(torch.float16)
    y = F.linear(x.float(), w.float() * scale.float()[:, None])
    return dict(x=x.numpy(), w=w.numpy(), scale=scale.numpy(), out=y.numpy().astype(np.float32),
                meta=np.array([M, N, K, seed]))


def main():
    cases = []
    seed = 1000
    for dtype in (torch.float16, torch.bfloat16):
        for epi in ("none", "bias", "bias_gelu_tanh", "bias_silu", "bias_residual", "residual", "swiglu"):
            seed += 1
            cases.append((f"fp_{str(dtype).split('.')[-1]}_{epi}", fp_case(seed, 96, 80, 72, dtype, epi)))
        seed += 1
        cases.append((f"fp_{str(dtype).split('.')[-1]}_none_kn", fp_case(seed, 64, 136, 48, dtype, "none", "kn")))
    # the reference's own Triton test shape (test_matmul.py:22-24), scaled down in M
    seed += 1
    cases.append(("fp_float16_none_kn_refshape", fp_case(seed, 128, 512, 64, torch.float16, "none", "kn")))
    for i, (M, N, K) in enumerate([(64, 96, 128), (33, 50, 160)]):
        cases.append((f"int8_{i}", int8_case(2000 + i, M, N, K)))
    for i, M in enumerate([1, 8]):
        cases.append((f"w8a16_m{M}", w8a16_case(3000 + i, M, 48, 256)))
    for name, c in cases:
        np.savez_compressed(os.path.join(HERE, f"golden_{name}.npz"), **c)
    print(f"wrote {len(cases)} fixtures to {HERE}")


if __name__ == "__main__":
    main()
