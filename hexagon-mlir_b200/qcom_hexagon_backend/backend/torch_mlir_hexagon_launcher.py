"""TorchMLIRHexagonLauncher — the reference's PyTorch entry point, on B200.

Reference: qcom_hexagon_backend/backend/torch_mlir_hexagon_launcher.py:258-306
    run_torch_mlir(mlir_bytecode_path, inputs, func_name,
                   base_dir_for_artifacts=None, iterations=1, options=None,
                   enable_etm=False) -> list[Tensor]
There, the MLIR is compiled to a Hexagon .so, the host inputs are written to
files, the kernel runs `iterations` times on the DSP inside
benchmark_time_us (test/utils/dsp/include/hexagon_benchmark.h:20-29), and the
outputs come back as fresh host tensors.

Here the "compile" step traces the model with torch.fx, rewrites its linear
layers onto the B200 kernels (fx_backend) and captures the whole forward in
a CUDA graph; "run" copies the host inputs into the graph's device buffers,
replays it `iterations` times and copies the outputs back to the host.
There is no MLIR on this path: pass the PyTorch module itself where the
reference took the torch-mlir bytecode path (a str path raises
NotImplementedError).  Same argument meaning and same return type: a list of
host tensors.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
import torch.nn as nn

from .. import fx_backend, ops
from .hexagon_options import HexagonOptions


@dataclass
class TestReport:
    """Name / Result / Perf / Units, as the reference's perf.txt report
    (test/utils/dsp/include/test_report.h:35-71)."""

    name: str
    result: str
    perf: float
    units: str = "us"

    def line(self) -> str:
        return f"Name:{self.name} Result:{self.result} Perf:{self.perf:.3f} Units:{self.units}"


def _leaves(out) -> list:
    """The forward's output tensors in pytree order (tuples, lists, dicts and
    HF ModelOutput all flatten; the reference's launcher likewise returns the
    flat list of the function's results, logits first for GPT2LMHeadModel)."""
    import torch.utils._pytree as pytree

    return [t for t in pytree.tree_leaves(out) if isinstance(t, torch.Tensor)]


class CompiledGraph:
    """A model compiled for one input signature: rewritten FX module, static
    device buffers, and (optionally) the CUDA graph of one forward."""

    def __init__(self, module: nn.Module, example_inputs: Sequence[torch.Tensor], options: HexagonOptions):
        self.options = options
        self.device = options.cuda_device()
        self.gm = fx_backend.compile_module(module, self.device, chain=options.chain_gemms,
                                            example_inputs=example_inputs, mode=options.capture)
        self.n_hx_calls = fx_backend.count_hx_calls(self.gm)
        self.static_in = [torch.empty(t.shape, dtype=t.dtype, device=self.device) for t in example_inputs]
        for s, t in zip(self.static_in, example_inputs):
            s.copy_(t)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.stream = torch.cuda.Stream(self.device)
        with torch.cuda.device(self.device), torch.no_grad():
            # Warm-up on a side stream (first calls set kernel attributes).
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.stream):
                out = self._forward()
                out = self._forward()
            torch.cuda.current_stream(self.device).wait_stream(self.stream)
            torch.cuda.synchronize(self.device)
            if options.use_cuda_graph:
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph, stream=self.stream):
                    out = self._forward()
        self.static_out = _leaves(out)

    def _forward(self):
        if self.options.chain_gemms:
            with ops.chained(self.device):
                return self.gm(*self.static_in)
        return self.gm(*self.static_in)

    def launch(self) -> None:
        """Run one forward on the current stream over the static buffers."""
        if self.graph is not None:
            self.graph.replay()
        else:
            outs = _leaves(self._forward())
            for s, o in zip(self.static_out, outs):
                s.copy_(o)

    def run(self, inputs: Sequence[torch.Tensor], iterations: int = 1,
            outputs: Optional[Sequence[torch.Tensor]] = None) -> list[torch.Tensor]:
        """Host inputs in, host outputs out.  Pinned host tensors are copied
        asynchronously; `outputs` may supply preallocated (pinned) host
        tensors to receive the results."""
        if len(inputs) != len(self.static_in):
            raise ValueError(f"expected {len(self.static_in)} inputs, got {len(inputs)}")
        with torch.cuda.device(self.device):
            for s, t in zip(self.static_in, inputs):
                if tuple(t.shape) != tuple(s.shape) or t.dtype != s.dtype:
                    raise ValueError("input signature differs from the compiled one")
                s.copy_(t, non_blocking=t.is_pinned() or t.is_cuda)
            for _ in range(max(1, iterations)):
                self.launch()
            if outputs is None:
                outputs = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in self.static_out]
            for h, o in zip(outputs, self.static_out):
                h.copy_(o, non_blocking=h.is_pinned())
            torch.cuda.current_stream(self.device).synchronize()
        return list(outputs)


class TorchMLIRHexagonLauncher:
    def __init__(self):
        self._cache: dict = {}
        self.last_report: Optional[TestReport] = None

    def compile_torch_mlir(self, model, inputs: Sequence[torch.Tensor], func_name: str = "forward",
                           options=None) -> CompiledGraph:
        if isinstance(model, (str, bytes)):
            raise NotImplementedError(
                "linalg/MLIR input is not supported on the B200 backend; pass the torch module")
        if not isinstance(model, nn.Module):
            raise TypeError("model must be a torch.nn.Module")
        opts = options if isinstance(options, HexagonOptions) else HexagonOptions.from_dict(options)
        key = (id(model), func_name, opts.hash(), opts.cuda_device().index,
               tuple((tuple(t.shape), t.dtype) for t in inputs))
        cg = self._cache.get(key)
        if cg is None:
            cg = CompiledGraph(model, inputs, opts)
            self._cache[key] = cg
        return cg

    def run_torch_mlir(
        self,
        mlir_bytecode_path,
        inputs: list[torch.Tensor],
        func_name: str,
        base_dir_for_artifacts: Optional[str] = None,
        iterations: int = 1,
        options: dict = None,
        enable_etm=False,
        outputs: Optional[Sequence[torch.Tensor]] = None,
    ) -> list[torch.Tensor]:
        """Compile (cached) and run `mlir_bytecode_path` — here, the nn.Module —
        on host `inputs`; returns host output tensors."""
        if enable_etm:
            raise NotImplementedError("ETM profiling is a Hexagon feature")
        cg = self.compile_torch_mlir(mlir_bytecode_path, inputs, func_name, options)
        t0 = time.perf_counter()
        outs = cg.run(inputs, iterations=iterations, outputs=outputs)
        dt_us = (time.perf_counter() - t0) * 1e6 / max(1, iterations)
        self.last_report = TestReport(func_name, "Pass", dt_us, "us")
        return outs
