"""qcom_hexagon_backend — B200 (sm_100a) drop-in for hexagon-mlir's
linear-layer matmul path.

Same package name and surface as the reference's Python backend
(qcom_hexagon_backend/backend/: HexagonOptions, TorchMLIRHexagonLauncher,
HexagonDriver); underneath, hand-written tcgen05/TMA kernels in
lib/libhx_gemm.so instead of the MLIR -> Hexagon LLVM -> DSP pipeline.
"""

from . import _lib
from . import ops
from .ops import (W8A16Group, bmm, gemm, gemv_w8a16, linear, matmul, matmul_batched, matmul_f16f16_f32,
                  shards_to_rows)

__all__ = ["bmm", "matmul_batched", "gemm", "gemv_w8a16", "linear", "matmul", "matmul_f16f16_f32", "shards_to_rows", "_lib"]
