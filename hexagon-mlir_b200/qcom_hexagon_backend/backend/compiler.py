"""Compile-side names of the reference's Triton backend (backend/compiler.py,
triton_qcom_hexagon_backend.cc:91-101), kept so imports resolve.

The reference lowers Triton IR through MLIR to Hexagon objects.  This B200
build has no MLIR: the matmul path runs hand-written sm_100a kernels, reached
through ``backend.driver.matmul``, ``qcom_hexagon_backend.linear`` or the
torch.fx rewrite.  The compile entry points therefore validate options and
refuse linalg input with the reference's error type for unsupported input.
"""

from __future__ import annotations

from dataclasses import fields
from typing import Any

from .hexagon_options import HexagonOptions


def translate_linalg_to_obj(module: Any, options: dict) -> list:
    """Reference: linalg module -> list of object files.  No B200 analogue."""
    raise NotImplementedError("linalg input not supported; pass torch tensors")


class HexagonBackend:
    """Backend object with the reference's option handling."""

    binary_ext = "so"

    def __init__(self, target: Any = None) -> None:
        self.target = target

    @staticmethod
    def supports_target(target: Any) -> bool:
        backend = getattr(target, "backend", target[0] if isinstance(target, tuple) else target)
        return backend in ("cuda", "hexagon")

    def parse_options(self, opts: dict) -> HexagonOptions:
        """The HexagonOptions fields present in `opts` (others are ignored,
        as in the reference's parse_options)."""
        names = {f.name for f in fields(HexagonOptions)}
        return HexagonOptions(**{k: v for k, v in opts.items() if k in names})

    def add_stages(self, stages: dict, options: HexagonOptions, language: Any = None) -> None:
        raise NotImplementedError("no IR stages on the B200 build: the matmul path runs "
                                  "hand-written kernels (backend.driver.matmul)")

    def pack_metadata(self, metadata: Any) -> tuple:
        return (getattr(metadata, "name", "matmul"),)
