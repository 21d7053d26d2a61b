"""Reference-compatible launch surface (qcom_hexagon_backend/backend/)."""

from .hexagon_options import HexagonOptions
from .torch_mlir_hexagon_launcher import CompiledGraph, TestReport, TorchMLIRHexagonLauncher

__all__ = ["HexagonOptions", "TorchMLIRHexagonLauncher", "CompiledGraph", "TestReport"]
