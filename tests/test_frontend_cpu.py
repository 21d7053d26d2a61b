"""CPU tests of the host-side front end: HexagonOptions, the FX rewrite of
linear(+epilogue) patterns, and the run_torch_mlir surface."""

import dataclasses
import math

import pytest
import torch
import torch.fx as fx
import torch.nn as nn
import torch.nn.functional as F

from qcom_hexagon_backend import fx_backend as FX
from qcom_hexagon_backend import workloads as WL
from qcom_hexagon_backend.backend import HexagonOptions, TorchMLIRHexagonLauncher
from qcom_hexagon_backend.backend.hexagon_options import IGNORED_ON_B200

# Field names of the reference dataclass (qcom_hexagon_backend/backend/hexagon_options.py:17-88).
REFERENCE_FIELDS = [
    "allow_fp8e4nv", "allowed_dot_input_precisions", "arch_triple", "arch_features", "vectorize",
    "vector_length", "num_threads", "data_layout", "num_warps", "num_stages", "num_ctas", "shared",
    "cluster_dims", "supported_fp8_dtypes", "sanitize_overflow", "debug", "name", "htp_kernel_gen",
    "target_artifact", "iterations", "fusion", "fusionAllowRecompute", "fusionDoMultiUse",
    "enableBufferization", "enableCollapseAddressSpace", "enableConvTiling", "enableDoubleBuffering",
    "convTilingFactor", "convTileHeightDim", "convTileOCDim", "enableConvertToHexagonmem",
    "enableHexagonmemCopyToDMA", "enableHexKL", "enableMultiThreading", "enableSCFThreading",
    "enableSplitReduction", "enableVectorization", "enableVTCMTiling", "enableHVXInlining",
    "enableSeedLayoutConversions", "tileSizes", "lowerConstantsInSeparateSharedObjects", "enableLWP",
    "disableLWPLoop", "LWPloopDepth",
]


def test_options_keep_reference_fields():
    names = [f.name for f in dataclasses.fields(HexagonOptions)]
    assert names[: len(REFERENCE_FIELDS)] == REFERENCE_FIELDS
    assert set(IGNORED_ON_B200) <= set(names)


def test_options_validation_and_override():
    with pytest.raises(ValueError):
        HexagonOptions(target_artifact="exe")
    with pytest.raises(ValueError):
        HexagonOptions(tileSizes="100")
    with pytest.raises(ValueError):
        HexagonOptions(tileSizes="128,9")
    assert HexagonOptions(tileSizes="256, 4").tile_override() == (256, 4)
    assert HexagonOptions(tileSizes="192").tile_override() == (192, 0)
    assert HexagonOptions().tile_override() == (0, 0)
    o = HexagonOptions.from_dict(HexagonOptions().__dict__)
    assert o.hash() == HexagonOptions().hash()
    with pytest.raises(TypeError):
        HexagonOptions.from_dict({"notAnOption": 1})
    with pytest.raises(dataclasses.FrozenInstanceError):
        o.iterations = 3


def _fx_targets(gm):
    return [n.target for n in gm.graph.nodes if n.op == "call_function"]


def test_rewrite_gpt2_block_patterns():
    gm = FX.rewrite(fx.symbolic_trace(WL.GPT2LinearStack(layers=2)))
    calls = [n for n in gm.graph.nodes if n.op == "call_function" and n.target is FX.hx_linear]
    assert len(calls) == 8
    assert [n.kwargs.get("activation") for n in calls] == [None, None, "gelu_tanh", None] * 2
    assert [n.kwargs.get("residual") is not None for n in calls] == [False, True, False, True] * 2
    assert F.gelu not in _fx_targets(gm)


def test_rewrite_qwen_swiglu():
    m = WL.QwenLinearStack(layers=2, hidden=64, inter=96, kv=16)
    gm = FX.rewrite(fx.symbolic_trace(m))
    sw = [n for n in gm.graph.nodes if n.op == "call_function" and n.target is FX.hx_swiglu]
    assert len(sw) == 2
    w = getattr(gm, sw[0].args[1].target)
    assert tuple(w.shape) == (192, 64)
    assert torch.equal(w[:96], m.blocks[0].gate.weight) and torch.equal(w[96:], m.blocks[0].up.weight)
    assert FX.count_hx_calls(gm) == 6


def test_rewrite_functional_linear_multi_user_not_fused():
    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.w = nn.Parameter(torch.randn(8, 4))

        def forward(self, x):
            y = F.linear(x, self.w)
            return y * 2 + y

    gm = FX.rewrite(fx.symbolic_trace(M()))
    assert _fx_targets(gm).count(FX.hx_linear) == 1
    node = [n for n in gm.graph.nodes if n.target is FX.hx_linear][0]
    assert "residual" not in node.kwargs


def test_rewritten_graph_has_no_cpu_path():
    gm = FX.rewrite(fx.symbolic_trace(WL.GPT2LinearStack(layers=1, hidden=64)))
    with pytest.raises(ValueError, match="CUDA"):
        gm(torch.randn(4, 64))


def test_run_torch_mlir_rejects_mlir_paths():
    with pytest.raises(NotImplementedError):
        TorchMLIRHexagonLauncher().run_torch_mlir("model.mlirbc", [torch.zeros(1)], "f")


def test_workload_counts():
    assert WL.gpt2_stack_flops() == 173946175488
    assert abs(WL.qwen_stack_flops() / 1e12 - 1.387) < 1e-3
    assert abs(WL.tinyllama_decode_bytes(1) / 1e6 - 971.2) < 0.5


# ---------------------------------------------------------------- aten / addmm / mm routes
def _ref_linear(x, weight, bias=None, residual=None, activation=None, weight_const=False, b_layout="nk"):
    """Torch stand-in for hx_linear with the same argument meaning (checks the
    rewritten graph's wiring on the CPU; the kernel itself is tested on GPU)."""
    w = weight if b_layout == "kn" else weight.t()
    y = x @ w
    if bias is not None:
        y = y + bias
    if activation == "gelu_tanh":
        y = F.gelu(y, approximate="tanh")
    elif activation == "silu":
        y = F.silu(y)
    if residual is not None:
        y = y + residual.reshape(y.shape)
    return y


def _run_with_ref(gm, *args):
    for n in gm.graph.nodes:
        if n.op == "call_function" and n.target is FX.hx_linear:
            n.target = _ref_linear
    gm.recompile()
    return gm(*args)


class _Conv1DBlock(nn.Module):
    """HF GPT-2's Conv1D form: addmm(bias, x2d, W[K,N]) then view, dropout, residual,
    and the NewGELU expression written out with pow/tanh."""

    def __init__(self, d=16, f=24):
        super().__init__()
        self.w1 = nn.Parameter(torch.randn(d, f) * 0.1)
        self.b1 = nn.Parameter(torch.randn(f) * 0.1)
        self.w2 = nn.Parameter(torch.randn(f, d) * 0.1)
        self.b2 = nn.Parameter(torch.randn(d) * 0.1)
        self.drop = nn.Dropout(0.1)

    def forward(self, x):
        h = torch.addmm(self.b1, x.view(-1, x.size(-1)), self.w1).view(x.shape[0], x.shape[1], -1)
        h = 0.5 * h * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (h + 0.044715 * torch.pow(h, 3.0))))
        y = torch.addmm(self.b2, h.view(-1, h.size(-1)), self.w2).view(x.shape)
        return x + self.drop(y)


def test_rewrite_addmm_newgelu_residual_export():
    """torch.export graph (aten ops): both addmm fold their constant W[K,N] into a
    transposed W[N,K] buffer; the GELU expression and the residual add fuse."""
    m = _Conv1DBlock().eval()
    x = torch.randn(2, 5, 16)
    gm = FX.rewrite(FX.capture(m, [x], "export"))
    calls = [n for n in gm.graph.nodes if n.op == "call_function" and n.target is FX.hx_linear]
    assert len(calls) == 2
    assert calls[0].kwargs.get("activation") == "gelu_tanh" and "b_layout" not in calls[0].kwargs
    assert calls[1].kwargs.get("residual") is not None
    tg = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert not any("tanh" in t or "pow" in t or "addmm" in t for t in tg)
    w0 = getattr(gm, calls[0].args[1].target)
    assert torch.equal(w0, m.w1.detach().t())
    torch.testing.assert_close(_run_with_ref(gm, x), m(x), rtol=1e-5, atol=1e-5)


def test_rewrite_addmm_symbolic_trace():
    m = _Conv1DBlock().eval()
    x = torch.randn(2, 5, 16)
    gm = FX.rewrite(FX.capture(m, [x], "trace"))
    assert FX.count_hx_calls(gm) == 2
    torch.testing.assert_close(_run_with_ref(gm, x), m(x), rtol=1e-5, atol=1e-5)


class _MatmulForms(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Parameter(torch.randn(16, 8))
        self.b = nn.Parameter(torch.randn(8, 12))

    def forward(self, x, wdyn):
        y = torch.mm(x, self.a)                 # constant B[K,N]
        y = F.silu(y @ self.b)                  # operator.matmul + SiLU
        z = torch.matmul(y, wdyn)               # a non-constant B[K,N]: runs as kn
        return z + x[:, :4]


@pytest.mark.parametrize("mode", ["trace", "export"])
def test_rewrite_mm_matmul_forms(mode):
    m = _MatmulForms()
    x, wd = torch.randn(6, 16), torch.randn(12, 4)
    gm = FX.rewrite(FX.capture(m, [x, wd], mode))
    calls = [n for n in gm.graph.nodes if n.op == "call_function" and n.target is FX.hx_linear]
    # a symbolic trace has no shape for the input `wdyn`, so that product stays a torch op
    assert len(calls) == (3 if mode == "export" else 2)
    assert calls[1].kwargs.get("activation") == "silu"
    if mode == "export":
        assert calls[2].kwargs.get("b_layout") == "kn" and calls[2].kwargs.get("residual") is not None
    torch.testing.assert_close(_run_with_ref(gm, x, wd), m(x, wd), rtol=1e-5, atol=1e-5)


def test_batched_matmul_is_not_a_linear():
    class B(nn.Module):
        def forward(self, q, k):
            return torch.matmul(q, k.transpose(-1, -2))

    q = torch.randn(2, 3, 5, 4)
    gm = FX.rewrite(FX.capture(B(), [q, q], "export"))
    assert not any(n.target is FX.hx_linear for n in gm.graph.nodes)
    assert sum(1 for n in gm.graph.nodes if n.target is FX.hx_bmm) == 1


def test_training_dropout_blocks_fusion():
    class D(nn.Module):
        def __init__(self):
            super().__init__()
            self.l = nn.Linear(8, 8)

        def forward(self, x):
            return x + F.dropout(self.l(x), 0.5)  # training=True by default: not transparent

    gm = FX.rewrite(fx.symbolic_trace(D()))
    node = [n for n in gm.graph.nodes if n.target is FX.hx_linear][0]
    assert "residual" not in node.kwargs


def test_hf_gpt2_lmhead_routes_every_linear():
    """Random-init HF GPT2LMHeadModel (GPT2Config(), 12 layers, fp16) through the
    export capture: every Conv1D addmm (4 per layer) and the LM head become
    fused kernel calls, with GELU and both residual adds in the epilogue."""
    transformers = pytest.importorskip("transformers")
    cfg = transformers.GPT2Config()
    cfg.use_cache = False
    torch.manual_seed(0)
    m = transformers.GPT2LMHeadModel(cfg).eval().half()
    ids = torch.randint(0, cfg.vocab_size, (1, 8))
    gm = FX.rewrite(FX.capture(m, [ids], "auto"))
    calls = [n for n in gm.graph.nodes if n.op == "call_function" and n.target is FX.hx_linear]
    assert len(calls) == 12 * 4 + 1
    assert sum(n.kwargs.get("activation") == "gelu_tanh" for n in calls) == 12
    assert sum(n.kwargs.get("residual") is not None for n in calls) == 24
    assert not any("addmm" in str(n.target) for n in gm.graph.nodes)


class _Attn(nn.Module):
    def __init__(self, d=32, h=4):
        super().__init__()
        self.d, self.h = d, h
        self.qkv = nn.Linear(d, 3 * d)
        self.o = nn.Linear(d, d)

    def forward(self, x):
        B, S, _ = x.shape
        q, k, v = self.qkv(x).split(self.d, dim=-1)
        q = q.view(B, S, self.h, -1).transpose(1, 2)
        k = k.view(B, S, self.h, -1).transpose(1, 2)
        v = v.view(B, S, self.h, -1).transpose(1, 2)
        p = torch.softmax(torch.matmul(q, k.transpose(-1, -2)), dim=-1)
        return self.o(torch.matmul(p, v).transpose(1, 2).reshape(B, S, self.d))


def test_rewrite_batched_matmuls_export():
    """Attention's q @ k^T and p @ v (rank-4 operands) become hx_bmm calls; the
    rewritten graph, with torch stand-ins for the kernels, computes the same."""
    m = _Attn().eval()
    x = torch.randn(2, 8, 32)
    gm = FX.rewrite(FX.capture(m, [x], "export"))
    assert sum(1 for n in gm.graph.nodes if n.op == "call_function" and n.target is FX.hx_bmm) == 2
    assert FX.count_hx_calls(gm) == 4
    for n in gm.graph.nodes:
        if n.op == "call_function" and n.target is FX.hx_bmm:
            n.target = torch.matmul
    torch.testing.assert_close(_run_with_ref(gm, x), m(x), rtol=1e-5, atol=1e-5)


def test_rewrite_torch_bmm_trace():
    class M(nn.Module):
        def forward(self, a, b):
            return torch.bmm(a, b)

    gm = FX.rewrite(fx.symbolic_trace(M()))
    assert FX.count_hx_calls(gm) == 1


def _ref_stats(x, kind, eps):
    x2 = x.reshape(-1, x.shape[-1]).float()
    mu = x2.mean(-1) if kind == "layer" else torch.zeros(x2.shape[0])
    var = x2.var(-1, unbiased=False) if kind == "layer" else (x2 * x2).mean(-1)
    return torch.stack([mu, torch.rsqrt(var + eps)], -1)


def _ref_linear_norm(x, weight, bias=None, residual=None, activation=None, weight_const=False, b_layout="nk",
                     norm_kind=None, norm_stats=None, col_sum=None):
    x2 = x.reshape(-1, x.shape[-1]).float()
    y = x2 @ (weight.float() if b_layout == "kn" else weight.float().t())
    if norm_kind is not None:
        y = y * norm_stats[:, 1:2]
        if norm_kind == "layer":
            y = y - (norm_stats[:, 1:2] * norm_stats[:, 0:1]) * col_sum[None, :]
    if bias is not None:
        y = y + bias.float()
    if activation == "gelu_tanh":
        y = F.gelu(y, approximate="tanh")
    elif activation == "swiglu":
        n = y.shape[-1] // 2
        y = F.silu(y[:, :n]) * y[:, n:]
    if residual is not None:
        y = y + residual.reshape(y.shape).float()
    return y.reshape(*x.shape[:-1], y.shape[-1])


def _run_norm_ref(gm, *args):
    for n in gm.graph.nodes:
        if n.op == "call_function" and n.target is FX.hx_linear:
            n.target = _ref_linear_norm
        elif n.op == "call_function" and n.target is FX.hx_norm_stats:
            n.target = _ref_stats
        elif n.op == "call_function" and n.target is FX.hx_swiglu:
            n.target = lambda x, w, norm_kind=None, norm_stats=None, col_sum=None: _ref_linear_norm(
                x, w, activation="swiglu", norm_kind=norm_kind, norm_stats=norm_stats, col_sum=col_sum)
    gm.recompile()
    return gm(*args)


class _LNBlock(nn.Module):
    def __init__(self, d=32):
        super().__init__()
        self.ln = nn.LayerNorm(d)
        self.up = nn.Linear(d, 64)
        self.qkv = nn.Linear(d, 48)
        with torch.no_grad():
            self.ln.weight.uniform_(0.5, 1.5)
            self.ln.bias.uniform_(-0.3, 0.3)

    def forward(self, x):
        h = self.ln(x)
        return F.gelu(self.up(h), approximate="tanh").sum(-1) + self.qkv(h).sum(-1)


@pytest.mark.parametrize("mode", ["trace", "export"])
def test_fold_layernorm_into_linears(mode):
    m = _LNBlock().eval()
    x = torch.randn(3, 7, 32) * 2 + 1
    gm = FX.rewrite(FX.capture(m, [x], mode))
    assert sum(1 for n in gm.graph.nodes if n.target is FX.hx_norm_stats) == 1
    assert not any("layer_norm" in str(n.target) or (n.op == "call_module" and "ln" in str(n.target))
                   for n in gm.graph.nodes)
    folded = [n for n in gm.graph.nodes if n.target is FX.hx_linear]
    assert len(folded) == 2 and all(n.kwargs.get("norm_kind") == "layer" for n in folded)
    torch.testing.assert_close(_run_norm_ref(gm, x), m(x), rtol=1e-4, atol=1e-4)


def test_fold_rmsnorm_into_swiglu():
    class Qwenish(nn.Module):
        def __init__(self, d=32, f=40):
            super().__init__()
            self.norm = nn.RMSNorm(d, eps=1e-6)
            self.gate = nn.Linear(d, f, bias=False)
            self.up = nn.Linear(d, f, bias=False)
            with torch.no_grad():
                self.norm.weight.uniform_(0.5, 1.5)

        def forward(self, x):
            h = self.norm(x)
            return F.silu(self.gate(h)) * self.up(h)

    m = Qwenish().eval()
    x = torch.randn(5, 32)
    gm = FX.rewrite(fx.symbolic_trace(m))
    sw = [n for n in gm.graph.nodes if n.target is FX.hx_swiglu]
    assert len(sw) == 1 and sw[0].kwargs.get("norm_kind") == "rms"
    torch.testing.assert_close(_run_norm_ref(gm, x), m(x), rtol=1e-4, atol=1e-4)


def test_norm_with_other_user_not_folded():
    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.ln = nn.LayerNorm(16)
            self.l = nn.Linear(16, 16)

        def forward(self, x):
            h = self.ln(x)
            return self.l(h) + h  # h itself is needed: the norm stays

    gm = FX.rewrite(fx.symbolic_trace(M()))
    assert not any(n.target is FX.hx_norm_stats for n in gm.graph.nodes)


@pytest.mark.parametrize("mode", ["trace", "export"])
def test_rewrite_conv2d(mode):
    class Net(nn.Module):
        def __init__(self):
            super().__init__()
            self.c1 = nn.Conv2d(8, 16, 3, padding=1)
            self.c2 = nn.Conv2d(16, 4, 3, stride=2, bias=False)

        def forward(self, x):
            return self.c2(F.relu(self.c1(x)))

    m = Net().eval()
    x = torch.randn(2, 8, 9, 9)
    gm = FX.rewrite(FX.capture(m, [x], mode))
    convs = [n for n in gm.graph.nodes if n.op == "call_function" and n.target is FX.hx_conv2d]
    assert len(convs) == 2
    for n in convs:  # torch stand-in with the same argument meaning
        n.target = lambda x, w, b, s, p, d: F.conv2d(x, w.permute(0, 3, 1, 2), b, s, p, d)
    gm.recompile()
    torch.testing.assert_close(gm(x), m(x), rtol=1e-5, atol=1e-5)
