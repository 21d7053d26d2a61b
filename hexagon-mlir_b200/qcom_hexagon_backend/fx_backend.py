"""FX graph rewriter: route a PyTorch model's linear layers (+ epilogue)
to the B200 kernels.

The reference takes a PyTorch model through torch-mlir
(`torch_mlir.fx.export_and_import(..., LINALG_ON_TENSORS)`,
benchmark_models/run_gpt2lmheadmodel.py:70-88), which turns each
aten.linear / aten.addmm into linalg.transpose + linalg.matmul + an
elementwise linalg.generic, then folds the transpose into
matmul_transpose_b (lib/Transforms/ScheduleMatmulForHVXPass.cpp:84-93).
Here the same graph-level decision is made on a torch.fx graph: each
linear node, together with the elementwise op that consumes it, becomes one
call of the fused GEMM kernel.

Patterns (the producer must have the consumer as its only user):
  linear(x)                          -> hx linear (bias if present)
  gelu(linear(x), approximate=tanh)  -> bias + GELU-tanh epilogue
  silu(linear(x))                    -> bias + SiLU epilogue
  linear(x) + r   /   r + linear(x)  -> bias + residual epilogue
  silu(linear_g(x)) * linear_u(x)    -> SwiGLU epilogue over [W_g; W_u]
                                        (both without bias, same x)
Everything else in the graph runs unchanged (on the GPU, as torch ops).
"""

from __future__ import annotations

import copy
import operator
from typing import Callable, Optional

import torch
import torch.fx as fx
import torch.nn as nn
import torch.nn.functional as F

from . import ops

_LINEAR_FNS = (F.linear, torch._C._nn.linear)
_GELU_FNS = (F.gelu, torch._C._nn.gelu)
_SILU_FNS = (F.silu,)
_ADD_FNS = (operator.add, torch.add, operator.iadd)
_MUL_FNS = (operator.mul, torch.mul)


def hx_linear(x, weight, bias=None, residual=None, activation=None, weight_const=False):
    """Fused linear used as the call_function target of rewritten nodes.
    weight_const: the weight is a module parameter/buffer (constant while the
    compiled forward runs), so the kernel may prefetch it early."""
    if residual is not None:
        out_shape = (*x.shape[:-1], weight.shape[0])
        if tuple(residual.shape) != out_shape or residual.dtype != x.dtype:
            # Broadcasting residual: not an epilogue the kernel fuses.
            y = ops.linear(x, weight, bias, activation=activation, b_const=weight_const)
            ops.chain_flush()  # the add below reads y
            return y + residual
    return ops.linear(x, weight, bias, activation=activation, residual=residual, b_const=weight_const)


def hx_swiglu(x, weight_gate_up):
    # the fused [gate; up] weight is a buffer the rewrite registered: constant
    return ops.linear(x, weight_gate_up, None, activation="swiglu", b_const=True)


def _users(n: fx.Node):
    return list(n.users.keys())


class _LinearSite:
    """A linear call in the graph: its input node and weight / bias sources."""

    def __init__(self, node, x, weight, bias):
        self.node, self.x, self.weight, self.bias = node, x, weight, bias


def _as_linear(gm: fx.GraphModule, n: fx.Node) -> Optional[_LinearSite]:
    if n.op == "call_module":
        mod = gm.get_submodule(n.target)
        if isinstance(mod, nn.Linear) and len(n.args) == 1 and not n.kwargs:
            return _LinearSite(n, n.args[0], ("attr", n.target + ".weight"),
                               ("attr", n.target + ".bias") if mod.bias is not None else None)
    if n.op == "call_function" and n.target in _LINEAR_FNS:
        args = list(n.args) + [None] * (3 - len(n.args))
        x, w, b = args[0], n.kwargs.get("weight", args[1]), n.kwargs.get("bias", args[2])
        return _LinearSite(n, x, ("node", w), ("node", b) if b is not None else None)
    return None


def _is_gelu_tanh(n: fx.Node) -> bool:
    if n.op == "call_function" and n.target in _GELU_FNS:
        return n.kwargs.get("approximate", n.args[1] if len(n.args) > 1 else "none") == "tanh"
    return False


def _is_silu(gm, n: fx.Node) -> bool:
    if n.op == "call_function" and n.target in _SILU_FNS and not n.kwargs.get("inplace", False):
        return True
    if n.op == "call_module" and isinstance(gm.get_submodule(n.target), nn.SiLU):
        return True
    return False


def _src(graph: fx.Graph, src):
    """Materialise a weight/bias source as a node."""
    if src is None:
        return None
    kind, val = src
    return graph.get_attr(val) if kind == "attr" else val


def rewrite(gm: fx.GraphModule) -> fx.GraphModule:
    """Rewrite linear(+epilogue) patterns in place; returns the module."""
    graph = gm.graph
    sites = {}
    for n in list(graph.nodes):
        s = _as_linear(gm, n)
        if s is not None:
            sites[n] = s
    done = set()

    # SwiGLU: mul(silu(lin_g(x)), lin_u(x)), both bias-free, weights constant.
    fused_count = 0
    for n in list(graph.nodes):
        if not (n.op == "call_function" and n.target in _MUL_FNS and len(n.args) == 2):
            continue
        a, b = n.args
        for sil, lin_u in ((a, b), (b, a)):
            if not (isinstance(sil, fx.Node) and isinstance(lin_u, fx.Node)):
                continue
            if not _is_silu(gm, sil) or len(_users(sil)) != 1:
                continue
            lin_g = sil.args[0] if sil.args else None
            if lin_g not in sites or lin_u not in sites or lin_g in done or lin_u in done:
                continue
            sg, su = sites[lin_g], sites[lin_u]
            if sg.x is not su.x or sg.bias or su.bias or len(_users(lin_g)) != 1 or len(_users(lin_u)) != 1:
                continue
            if sg.weight[0] != "attr" or su.weight[0] != "attr":
                continue
            wg = gm.get_parameter(sg.weight[1]) if _has_param(gm, sg.weight[1]) else None
            wu = gm.get_parameter(su.weight[1]) if _has_param(gm, su.weight[1]) else None
            if wg is None or wu is None or wg.shape != wu.shape:
                continue
            name = f"_hx_swiglu_w{fused_count}"
            fused_count += 1
            gm.register_buffer(name, torch.cat([wg.detach(), wu.detach()], 0))
            with graph.inserting_before(n):
                w = graph.get_attr(name)
                new = graph.call_function(hx_swiglu, (sg.x, w))
            n.replace_all_uses_with(new)
            for dead in (n, sil, lin_g, lin_u):
                graph.erase_node(dead)
            done.update((lin_g, lin_u))
            break

    for n in list(sites):
        if n in done:
            continue
        s = _as_linear(gm, n)  # re-read: earlier rewrites may have replaced its inputs
        users = _users(n)
        act, residual, tail = None, None, n
        if len(users) == 1:
            u = users[0]
            if _is_gelu_tanh(u):
                act, tail = "gelu_tanh", u
            elif _is_silu(gm, u):
                act, tail = "silu", u
            elif u.op == "call_function" and u.target in _ADD_FNS and len(u.args) == 2 and not u.kwargs:
                other = u.args[1] if u.args[0] is n else u.args[0]
                if isinstance(other, fx.Node) and other is not n:
                    residual, tail = other, u
        with graph.inserting_before(tail):
            w = _src(graph, s.weight)
            b = _src(graph, s.bias)
            kwargs = {}
            if s.weight[0] == "attr":
                kwargs["weight_const"] = True
            if act:
                kwargs["activation"] = act
            if residual is not None:
                kwargs["residual"] = residual
            new = graph.call_function(hx_linear, (s.x, w, b), kwargs)
        tail.replace_all_uses_with(new)
        if tail is not n:
            graph.erase_node(tail)
        graph.erase_node(n)
    graph.lint()
    gm.recompile()
    return gm


def insert_chain_flushes(gm: fx.GraphModule) -> fx.GraphModule:
    """Before every node that may read tensor data and is not a fused linear,
    insert ops.chain_flush(), so GEMMs queued by ops.chained() have run.
    Fused linears queue themselves; getitem (views) reads nothing."""
    graph = gm.graph
    for n in list(graph.nodes):
        if n.op in ("placeholder", "get_attr"):
            continue
        if n.op == "call_function" and (n.target in (hx_linear, hx_swiglu, ops.chain_flush)
                                        or n.target is operator.getitem):
            continue
        with graph.inserting_before(n):
            graph.call_function(ops.chain_flush, ())
    graph.lint()
    gm.recompile()
    return gm


def _has_param(gm, qualname):
    try:
        gm.get_parameter(qualname)
        return True
    except AttributeError:
        return False


def count_hx_calls(gm: fx.GraphModule) -> int:
    return sum(1 for n in gm.graph.nodes if n.op == "call_function" and n.target in (hx_linear, hx_swiglu))


def compile_module(module: nn.Module, device: torch.device | str = "cuda",
                   chain: bool = False) -> fx.GraphModule:
    """Trace `module`, move its parameters to `device` and rewrite its linear
    layers onto the B200 kernels.  With `chain`, flush points are inserted so
    the graph can run under ops.chained() (consecutive linears become one
    hx_gemm_chain launch).  The original module is not modified."""
    gm = fx.symbolic_trace(copy.deepcopy(module))  # the GraphModule would share parameters
    gm = gm.to(device)
    gm = rewrite(gm)
    return insert_chain_flushes(gm) if chain else gm


def hexagon_backend(gm: fx.GraphModule, example_inputs) -> Callable:
    """torch.compile backend: `torch.compile(model, backend=hexagon_backend)`.

    The graph Dynamo hands over keeps module parameters as get_attr/call_module
    nodes or as inputs; linear patterns are rewritten either way (weights that
    arrive as inputs skip only the SwiGLU weight concatenation)."""
    return rewrite(gm).forward
