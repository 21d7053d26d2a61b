"""HexagonOptions — the reference's option dataclass, kept as the drop-in
configuration surface (qcom_hexagon_backend/backend/hexagon_options.py:17-101).

Every field the reference defines is accepted with the same name, type and
default, so existing call sites (Triton kwargs, `options=HexagonOptions().__dict__`
for run_torch_mlir) keep working.  Hexagon-only code-generation knobs
(HVX vector width, VTCM tiling, DMA lowering, LWP profiling, ...) have no
meaning on the B200 and are accepted and ignored; `tileSizes` keeps its
role as the tile override.  The B200-specific fields at the end select the
kernel configuration.
"""

from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass, fields
from typing import Tuple

# Fields of the reference dataclass that steer Hexagon code generation only.
IGNORED_ON_B200 = (
    "arch_triple", "arch_features", "vectorize", "vector_length", "num_threads", "data_layout",
    "num_warps", "num_stages", "num_ctas", "shared", "cluster_dims", "htp_kernel_gen",
    "target_artifact", "fusion", "fusionAllowRecompute", "fusionDoMultiUse",
    "enableBufferization", "enableCollapseAddressSpace", "enableConvTiling",
    "enableDoubleBuffering", "convTilingFactor", "convTileHeightDim", "convTileOCDim",
    "enableConvertToHexagonmem", "enableHexagonmemCopyToDMA", "enableHexKL",
    "enableMultiThreading", "enableSCFThreading", "enableSplitReduction", "enableVectorization",
    "enableVTCMTiling", "enableHVXInlining", "enableSeedLayoutConversions",
    "lowerConstantsInSeparateSharedObjects", "enableLWP", "disableLWPLoop", "LWPloopDepth",
)


@dataclass(frozen=True)
class HexagonOptions:
    # ---- fields of the reference (same names, types, defaults) ----
    allow_fp8e4nv: bool = False
    allowed_dot_input_precisions: Tuple[str] = ("ieee",)
    arch_triple: str = "hexagon"
    arch_features: str = f'+hvxv{os.getenv("HEXAGON_ARCH_VERSION")},+hvx-length128b'
    vectorize: int = 1
    vector_length: int = 32
    num_threads: int = 4
    data_layout: str = (
        "e-m:e-p:32:32:32-a:0-n16:32-i64:64:64-i32:32:32-i16:16:16-i1:8:8-f32:32:"
        "32-f64:64:64-v32:32:32-v64:64:64-v512:512:512-v1024:1024:1024-v2048:2048:2048"
    )
    num_warps: int = 1
    num_stages: int = 1
    num_ctas: int = 1
    shared: bool = False
    cluster_dims: tuple = (1, 1, 1)
    supported_fp8_dtypes: Tuple[str, ...] = ()
    sanitize_overflow: bool = True
    debug: bool = False
    name: str = "Hexagon"
    htp_kernel_gen: bool = False
    target_artifact: str = "o"
    iterations: int = 10
    fusion: bool = True
    fusionAllowRecompute: bool = False
    fusionDoMultiUse: bool = True
    enableBufferization: bool = True
    enableCollapseAddressSpace: bool = True
    enableConvTiling: bool = False
    enableDoubleBuffering: bool = False
    convTilingFactor: int = -1
    convTileHeightDim: bool = False
    convTileOCDim: bool = False
    enableConvertToHexagonmem: bool = True
    enableHexagonmemCopyToDMA: bool = False
    enableHexKL: bool = False
    enableMultiThreading: bool = False
    enableSCFThreading: bool = False
    enableSplitReduction: bool = False
    enableVectorization: bool = True
    enableVTCMTiling: bool = True
    enableHVXInlining: bool = False
    enableSeedLayoutConversions: bool = False
    tileSizes: str = ""  # B200: "N" or "N,stages" tile override (N in 64/96/128/192/256)
    lowerConstantsInSeparateSharedObjects: bool = False
    enableLWP: bool = False
    disableLWPLoop: bool = False
    LWPloopDepth: int = 1

    # ---- B200 additions ----
    device: int = -1                # CUDA device index; -1 = the current device at compile time
    fuse_epilogue: bool = True      # fold bias/GELU/SiLU/SwiGLU/residual into the GEMM
    use_cuda_graph: bool = True     # capture the compiled graph's launches once, replay
    chain_gemms: bool = False       # run consecutive linears as one persistent launch
    world_size: int = 1             # column-sharding degree (LM-head style GEMMs)
    shard_dim: str = "n"            # only "n" (output columns) is supported
    capture: str = "auto"           # FX capture: "trace", "export" (torch.export, aten ops) or "auto"

    def __post_init__(self):
        valid_artifacts = {"o", "llir", "so"}
        if self.target_artifact not in valid_artifacts:
            raise ValueError(
                f"Invalid target_artifact '{self.target_artifact}'. "
                f"Must be one of: {', '.join(sorted(valid_artifacts))}"
            )
        if self.shard_dim != "n":
            raise ValueError("shard_dim must be 'n' (column sharding)")
        if self.world_size < 1:
            raise ValueError("world_size must be >= 1")
        if self.capture not in ("auto", "trace", "export"):
            raise ValueError("capture must be 'auto', 'trace' or 'export'")
        self.tile_override()  # validates tileSizes

    def cuda_device(self):
        """The torch.device this configuration runs on (device -1: torch's current device)."""
        import torch

        return torch.device("cuda", self.device if self.device >= 0 else torch.cuda.current_device())

    def tile_override(self) -> Tuple[int, int]:
        """(tile_n, stages) from tileSizes; 0 means automatic."""
        if not self.tileSizes:
            return 0, 0
        parts = [p.strip() for p in self.tileSizes.split(",") if p.strip()]
        try:
            vals = [int(p) for p in parts]
        except ValueError:
            raise ValueError(f"tileSizes must be 'N' or 'N,stages', got {self.tileSizes!r}") from None
        if not vals or len(vals) > 2 or vals[0] not in (64, 96, 128, 192, 256):
            raise ValueError(f"tileSizes must be 'N' or 'N,stages' with N in 64/96/128/192/256, got {self.tileSizes!r}")
        stages = vals[1] if len(vals) == 2 else 0
        if stages and not 2 <= stages <= 8:
            raise ValueError("stages must be in [2, 8]")
        return vals[0], stages

    @classmethod
    def from_dict(cls, d: dict | None) -> "HexagonOptions":
        """Build from a (possibly partial) dict such as HexagonOptions().__dict__;
        unknown keys raise, like the reference's frozen dataclass would."""
        if not d:
            return cls()
        names = {f.name for f in fields(cls)}
        unknown = set(d) - names
        if unknown:
            raise TypeError(f"unknown HexagonOptions fields: {sorted(unknown)}")
        return cls(**d)

    def hash(self):
        key = "_".join([f"{name}-{val}" for name, val in self.__dict__.items()])
        return hashlib.md5(key.encode("utf-8")).hexdigest()
