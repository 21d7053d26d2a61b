"""The benchmark workloads of this path, as plain PyTorch modules.

These are the model shapes the reference's benchmark scripts feed through
torch-mlir (benchmark_models/run_gpt2lmheadmodel.py, run_qwen2.5-0.5b.py,
run_tinyllama.py, run_falcon_rw_1b.py), reduced to the linear layers that
reach `linalg.matmul` + epilogue.  They are ordinary nn.Modules (no calls
into this package): the reference arm runs them on the CPU with PyTorch,
and the B200 path compiles the very same module through fx_backend.

Weights are random-init from a seeded CPU generator (no checkpoints are
available offline); the layers between the linears (attention, norms) are
not on this path and are left out.  Each forward consumes every GEMM's
output, so no GEMM is dead code.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


def _init_linear(lin: nn.Linear, g: torch.Generator, std: float = 0.02) -> nn.Linear:
    with torch.no_grad():
        lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * std)
        if lin.bias is not None:
            lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * std)
    return lin


# ---------------------------------------------------------------- config 2
class GPT2LinearBlock(nn.Module):
    """GPT-2-small block's four linears: c_attn (QKV, +bias), attn c_proj
    (+bias +residual), mlp c_fc (+bias +GELU-tanh), mlp c_proj (+bias +residual).
    The attention core is not on the path; c_proj reads the first `hidden`
    columns of QKV in its place."""

    def __init__(self, hidden: int, g: torch.Generator):
        super().__init__()
        self.hidden = hidden
        self.c_attn = _init_linear(nn.Linear(hidden, 3 * hidden), g)
        self.attn_proj = _init_linear(nn.Linear(hidden, hidden), g)
        self.c_fc = _init_linear(nn.Linear(hidden, 4 * hidden), g)
        self.mlp_proj = _init_linear(nn.Linear(4 * hidden, hidden), g)

    def forward(self, h):
        qkv = self.c_attn(h)
        a = self.attn_proj(qkv[:, : self.hidden]) + h
        u = F.gelu(self.c_fc(a), approximate="tanh")
        return self.mlp_proj(u) + a


class GPT2LinearStack(nn.Module):
    def __init__(self, layers: int = 12, hidden: int = 768, seed: int = 1236):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.blocks = nn.ModuleList([GPT2LinearBlock(hidden, g) for _ in range(layers)])

    def forward(self, h):
        for b in self.blocks:
            h = b(h)
        return h


# ---------------------------------------------------------------- config 3
class QwenLinearBlock(nn.Module):
    """Qwen2.5-0.5B prefill linears: fused QKV (+bias), fused gate/up with a
    SwiGLU epilogue, down (+residual).  Attention is not on the path: each
    layer's QKV output is summed into a running [M, hidden+2kv] accumulator
    (a fused residual add), which joins the output once at the end."""

    def __init__(self, hidden: int, inter: int, kv: int, g: torch.Generator):
        super().__init__()
        self.hidden = hidden
        self.qkv = _init_linear(nn.Linear(hidden, hidden + 2 * kv), g)
        self.gate = _init_linear(nn.Linear(hidden, inter, bias=False), g)
        self.up = _init_linear(nn.Linear(hidden, inter, bias=False), g)
        self.down = _init_linear(nn.Linear(inter, hidden, bias=False), g)

    def forward(self, h, acc):
        acc = self.qkv(h) + acc
        u = F.silu(self.gate(h)) * self.up(h)
        return self.down(u) + h, acc


class QwenLinearStack(nn.Module):
    def __init__(self, layers: int = 24, hidden: int = 896, inter: int = 4864, kv: int = 128,
                 seed: int = 1237):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.blocks = nn.ModuleList([QwenLinearBlock(hidden, inter, kv, g) for _ in range(layers)])

    def forward(self, h):
        acc = h.new_zeros(h.shape[0], self.blocks[0].qkv.out_features)
        for b in self.blocks:
            h, acc = b(h, acc)
        return h + acc[:, : h.shape[1]]


# ---------------------------------------------------------------- config 4
@dataclass
class W8A16Linear:
    """int8 per-output-channel weight: W ~ U{-127..127}, fp16 scale ~ U(0.001, 0.02)."""

    weight: torch.Tensor  # int8 [N, K]
    scale: torch.Tensor   # fp16 [N]

    @staticmethod
    def make(n: int, k: int, g: torch.Generator) -> "W8A16Linear":
        w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int64).to(torch.int8)
        s = (torch.rand(n, generator=g) * 0.019 + 0.001).to(torch.float16)
        return W8A16Linear(w, s)


TINYLLAMA_PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def tinyllama_shapes(hidden: int = 2048, inter: int = 5632, kv: int = 256):
    """(N, K) of each decode projection (32 heads, 4 KV heads, head_dim 64)."""
    return {"q": (hidden, hidden), "k": (kv, hidden), "v": (kv, hidden), "o": (hidden, hidden),
            "gate": (inter, hidden), "up": (inter, hidden), "down": (hidden, inter)}


def make_tinyllama_w8a16(layers: int = 22, seed: int = 1238):
    g = torch.Generator().manual_seed(seed)
    shapes = tinyllama_shapes()
    return [{p: W8A16Linear.make(*shapes[p], g) for p in TINYLLAMA_PROJ} for _ in range(layers)]


def tinyllama_decode_bytes(M: int, layers: int = 22) -> int:
    """Algorithmic HBM bytes of one decode step: int8 weights + fp16 scales +
    fp16 activations in and out, each once."""
    tot = 0
    for n, k in tinyllama_shapes().values():
        tot += n * k + 2 * n + 2 * M * k + 2 * M * n
    return tot * layers


# ---------------------------------------------------------------- config 5
LMHEAD_M, LMHEAD_K, LMHEAD_N = 16384, 2048, 50304


def gpt2_stack_flops(M: int = 1024, layers: int = 12, hidden: int = 768) -> int:
    return 2 * M * hidden * (3 * hidden + hidden + 4 * hidden) * layers + 2 * M * 4 * hidden * hidden * layers


def qwen_stack_flops(M: int = 2048, layers: int = 24, hidden: int = 896, inter: int = 4864, kv: int = 128) -> int:
    return 2 * M * hidden * (2 * inter + inter + hidden + 2 * kv) * layers


def gpt2_stack_bytes(M: int = 1024, layers: int = 12, hidden: int = 768) -> int:
    """Algorithmic bytes: each GEMM's A, W, bias, residual and C once (fp16)."""
    per = 0
    for (k, n, res) in ((hidden, 3 * hidden, False), (hidden, hidden, True),
                        (hidden, 4 * hidden, False), (4 * hidden, hidden, True)):
        per += 2 * (M * k + n * k + n + M * n + (M * n if res else 0))
    return per * layers
