"""Reference-compatible launch surface (qcom_hexagon_backend/backend/)."""

from .compiler import HexagonBackend, translate_linalg_to_obj
from .driver import HexagonDriver, HexagonLauncher, MatmulProgram, matmul
from .hexagon_options import HexagonOptions
from .torch_mlir_hexagon_launcher import CompiledGraph, TestReport, TorchMLIRHexagonLauncher

__all__ = ["HexagonOptions", "TorchMLIRHexagonLauncher", "CompiledGraph", "TestReport",
           "HexagonDriver", "HexagonLauncher", "HexagonBackend", "MatmulProgram", "matmul",
           "translate_linalg_to_obj"]
