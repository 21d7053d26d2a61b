"""Triton-side launch surface of the reference, for the matmul path.

The reference registers a Triton driver (``HexagonDriver``, backend/driver.py)
whose launcher class is called by Triton's ``CompiledKernel`` as
``launcher(gx, gy, gz, stream, function, packed_metadata, launch_metadata,
enter_hook, exit_hook, *args)`` (backend/driver.py:34-76).  Its tests launch a
``tl.dot`` program as ``matmul[(1,)](A, B, C, n_rows, n_cols, n_inner,
**HexagonOptions)`` (test/python/triton/test_matmul.py:67-87) and read the
result back from ``C``.

This build has no tracing compiler: there is no MLIR to lower.  What it keeps
is the call surface for the one program on its hot path:

* ``HexagonDriver`` with the reference's method names; its ``launcher_cls``
  takes the same positional arguments, where ``function`` is a
  ``MatmulProgram`` (the stand-in for a compiled ``tl.dot`` kernel);
* ``matmul``, a kernel object indexable by a launch grid, with the argument
  order and options of the reference test's kernel, running ``hx_gemm``.

Errors follow the reference: ``ValueError`` for an empty launch grid or bad
arguments, ``NotImplementedError`` for programs other than the matmul.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, fields
from typing import Any, Optional, Sequence

import torch

from .. import ops
from .hexagon_options import HexagonOptions

_OPTION_NAMES = {f.name for f in fields(HexagonOptions)}


def _check_grid(grid: Sequence[int]) -> None:
    if math.prod(int(g) for g in grid) < 1:
        raise ValueError("Must set at least 1 program in the launch grid; to launch once, "
                         "invoke the kernel as kernel[(1,)](...)")


def _options(kwargs: dict) -> HexagonOptions:
    unknown = sorted(k for k in kwargs if k not in _OPTION_NAMES)
    if unknown:
        raise ValueError(f"unknown HexagonOptions field(s): {unknown}")
    return HexagonOptions(**kwargs)


def run_matmul(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, n_rows: int, n_cols: int,
               n_inner: int, options: Optional[HexagonOptions] = None) -> None:
    """C[n_rows, n_cols] = A[n_rows, n_inner] . B[n_inner, n_cols] (row-major,
    B in [K, N] layout as in the reference kernel), fp32 accumulation,
    stored in C's dtype.  Host tensors are copied to the GPU and the result is
    written back into C, as the reference writes results into its pointer
    arguments (backend/triton_hexagon_launcher.py:424-427)."""
    opts = options or HexagonOptions()
    for t, name, shape in ((A, "A", (n_rows, n_inner)), (B, "B", (n_inner, n_cols)), (C, "C", (n_rows, n_cols))):
        if not isinstance(t, torch.Tensor):
            raise ValueError(f"{name} must be a torch.Tensor")
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {shape}")
    dev = opts.cuda_device()
    tile_n, stages = opts.tile_override()
    a = A.to(dev).contiguous()
    b = B.to(dev).contiguous()
    c = C.to(dev) if C.device == dev and C.is_contiguous() else torch.empty(C.shape, dtype=C.dtype, device=dev)
    ops.gemm(a, b, b_layout="kn", out=c, tile_n=tile_n, stages=stages)
    if c.data_ptr() != C.data_ptr():
        C.copy_(c)


@dataclass(frozen=True)
class MatmulProgram:
    """Stand-in for a compiled ``tl.dot`` program (the ``function`` argument
    the launcher receives): C = A . B, arguments (A, B, C, n_rows, n_cols,
    n_inner)."""

    name: str = "matmul"
    options: HexagonOptions = field(default_factory=HexagonOptions)

    def __call__(self, A, B, C, n_rows, n_cols, n_inner):
        run_matmul(A, B, C, int(n_rows), int(n_cols), int(n_inner), self.options)


class HexagonLauncher:
    """Callable with the argument list Triton's CompiledKernel passes."""

    def __init__(self, src: Any = None, metadata: Any = None):
        self.src, self.metadata = src, metadata

    def __call__(self, gx, gy, gz, stream, function, packed_metadata, launch_metadata,
                 enter_hook, exit_hook, *args):
        _check_grid((gx, gy, gz))
        if not isinstance(function, MatmulProgram):
            raise NotImplementedError("this B200 build runs only the linalg.matmul program "
                                      "(pass a MatmulProgram, or call qcom_hexagon_backend.linear)")
        if enter_hook is not None:
            enter_hook(launch_metadata)
        function(*args)
        if exit_hook is not None:
            exit_hook(launch_metadata)


class HexagonDriver:
    """Driver object with the reference's method names; register it with
    ``triton.runtime.driver.set_active(HexagonDriver())`` where Triton is used."""

    def __init__(self, device_type: str = "cuda"):
        self.backend = "HEXAGON"
        self.device_type = device_type
        self.launcher_cls = HexagonLauncher
        self.binary_ext = "so"

    @staticmethod
    def is_active() -> bool:
        return torch.cuda.is_available()

    def map_python_to_cpp_type(self, ty: str) -> str:
        table = {"i1": "int32_t", "i8": "int8_t", "i16": "int16_t", "i32": "int32_t", "i64": "int64_t",
                 "u1": "uint32_t", "u8": "uint8_t", "u16": "uint16_t", "u32": "uint32_t",
                 "u64": "uint64_t", "fp16": "float", "bf16": "float", "fp32": "float",
                 "f32": "float", "fp64": "double"}
        return table[ty]

    def get_benchmarker(self):
        def bench(fn, reps: int = 20):
            fn()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(reps):
                fn()
            e.record()
            e.synchronize()
            return s.elapsed_time(e) / reps
        return bench

    def get_current_target(self):
        return ("cuda", 100, 32)  # (backend, sm_100, warp size)

    def get_current_device(self):
        return torch.cuda.current_device()

    def get_active_torch_device(self):
        return torch.device("cuda", torch.cuda.current_device())

    def get_current_stream(self, device=None):
        return torch.cuda.current_stream(device).cuda_stream


class _GridLaunch:
    def __init__(self, grid):
        self.grid = tuple(grid) if isinstance(grid, (tuple, list)) else (grid,)

    def __call__(self, A, B, C, n_rows, n_cols, n_inner, **options):
        _check_grid(self.grid + (1,) * (3 - len(self.grid)))
        prog = MatmulProgram(options=_options(options))
        HexagonLauncher()(*(self.grid + (1,) * (3 - len(self.grid))), None, prog, None, None, None, None,
                          A, B, C, n_rows, n_cols, n_inner)


class _MatmulKernel:
    """``matmul[grid](A, B, C, n_rows, n_cols, n_inner, **HexagonOptions)``"""

    def __getitem__(self, grid):
        return _GridLaunch(grid)


matmul = _MatmulKernel()
