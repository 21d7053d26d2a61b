"""CPU tests of the host-side front end: HexagonOptions, the FX rewrite of
linear(+epilogue) patterns, and the run_torch_mlir surface."""

import dataclasses

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
