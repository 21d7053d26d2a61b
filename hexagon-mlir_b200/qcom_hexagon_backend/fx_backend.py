"""FX graph rewriter: route a PyTorch model's linear layers (+ epilogue)
to the B200 kernels.

The reference takes a PyTorch model through torch-mlir
(`torch_mlir.fx.export_and_import(..., LINALG_ON_TENSORS)`,
benchmark_models/run_gpt2lmheadmodel.py:70-88), which turns each
aten.linear / aten.addmm / aten.mm into linalg.transpose + linalg.matmul + an
elementwise linalg.generic, then folds the transpose into
matmul_transpose_b (lib/Transforms/ScheduleMatmulForHVXPass.cpp:84-93).
Here the same graph-level decision is made on a torch.fx graph, either a
symbolic trace (torch-level ops) or a torch.export graph (aten ops, the
graph export_and_import starts from): each linear node, together with the
elementwise op that consumes it, becomes one call of the fused GEMM kernel.

Linear nodes: F.linear / nn.Linear / aten.linear (W[N,K]); torch.addmm /
aten.addmm (bias + x @ W[K,N], beta = alpha = 1, as HF Conv1D computes);
torch.mm / aten.mm / torch.matmul / aten.matmul / `@` with a 2-D right
operand (x @ W[K,N]).  A constant W[K,N] (a module parameter or buffer) is
transposed once at compile time into a W[N,K] buffer, the transpose fold of
ScheduleMatmulForHVXPass; a non-constant one runs as the B[K,N] layout.

Epilogue patterns (each intermediate node must have one user).  Between
the linear and its consumer the rewriter looks through views / reshapes and
inference-mode dropout, which it re-applies to the fused result:
  linear(x)                          -> hx linear (bias if present)
  gelu(linear(x), approximate=tanh)  -> bias + GELU-tanh epilogue
  0.5*y*(1+tanh(c*(y+0.044715*y^3))) -> the same (HF NewGELU written out)
  silu(linear(x))                    -> bias + SiLU epilogue
  linear(x) + r   /   r + linear(x)  -> bias + residual epilogue
  silu(linear_g(x)) * linear_u(x)    -> SwiGLU epilogue over [W_g; W_u]
                                        (both without bias, same x)
Convolutions (nn.Conv2d / aten.conv2d, groups 1, constant filters) become
the implicit-GEMM convolution (hx_conv2d), filters permuted once to
[OC, KH, KW, C]: the conv consumer of HMX in MatmulToConvPass.cpp.
Batched products (torch.bmm / aten.bmm, and matmul with both operands of
rank >= 3, e.g. attention's q @ k^T and p @ v) become one batched GEMM
(hx_bmm), the batch_matmul / batch_matmul_transpose_b of
ScheduleMatmulForHVXPass.cpp:105-167.
Everything else in the graph runs unchanged (on the GPU, as torch ops).
"""

from __future__ import annotations

import copy
import math
import operator
from typing import Callable, Optional

import torch
import torch.fx as fx
import torch.nn as nn
import torch.nn.functional as F

from . import ops

aten = torch.ops.aten
_LINEAR_FNS = (F.linear, torch._C._nn.linear, aten.linear.default)
_ADDMM_FNS = (torch.addmm, aten.addmm.default)
_MM_FNS = (torch.mm, aten.mm.default)
_MATMUL_FNS = (torch.matmul, operator.matmul, aten.matmul.default)
_BMM_FNS = (torch.bmm, aten.bmm.default)
_GELU_FNS = (F.gelu, torch._C._nn.gelu, aten.gelu.default)
_SILU_FNS = (F.silu, aten.silu.default)
_ADD_FNS = (operator.add, torch.add, operator.iadd, aten.add.Tensor)
_MUL_FNS = (operator.mul, torch.mul, aten.mul.Tensor)
_TANH_FNS = (torch.tanh, aten.tanh.default)
_POW_FNS = (torch.pow, operator.pow, aten.pow.Tensor_Scalar)
_VIEW_FNS = (aten.view.default, aten.reshape.default, aten._unsafe_view.default, aten.alias.default,
             torch.reshape)
_VIEW_METHODS = ("view", "reshape")
_DROPOUT_FNS = (F.dropout, aten.dropout.default)


def hx_norm_stats(x, kind, eps):
    """Row statistics of a LayerNorm / RMSNorm folded into the linears after it."""
    ops.chain_flush()
    return ops.row_norm_stats(x, kind, eps)


def hx_linear(x, weight, bias=None, residual=None, activation=None, weight_const=False, b_layout="nk",
              norm_kind=None, norm_stats=None, col_sum=None):
    """Fused linear used as the call_function target of rewritten nodes.
    weight: W[N,K] (b_layout "nk") or B[K,N] ("kn").  residual may have any
    shape whose last dimension is N and whose size is x's rows x N (the
    rewriter passes the consumer's operand, which can be the viewed shape).
    weight_const: the weight is a module parameter/buffer (constant while the
    compiled forward runs), so the kernel may prefetch it early.
    norm_kind / norm_stats / col_sum: a LayerNorm / RMSNorm of x folded in
    (weight and bias are then the folded ones, see ops.fold_norm_weight)."""
    if norm_kind is not None:
        return ops.linear(x, weight, bias, activation=activation, residual=residual, b_const=weight_const,
                          b_layout=b_layout, norm=(norm_kind, norm_stats, col_sum))
    if residual is not None:
        n = weight.shape[0] if b_layout == "nk" else weight.shape[1]
        rows = x.numel() // x.shape[-1] if x.shape[-1] else 0
        if residual.shape[-1] != n or residual.numel() != rows * n or residual.dtype != x.dtype \
                or not residual.is_contiguous():
            # Broadcasting or strided residual: not an epilogue the kernel fuses.
            y = ops.linear(x, weight, bias, activation=activation, b_const=weight_const, b_layout=b_layout)
            ops.chain_flush()  # the add below reads y
            return y + residual.reshape(y.shape) if residual.numel() == y.numel() else y + residual
        residual = residual.reshape(*x.shape[:-1], n)
    return ops.linear(x, weight, bias, activation=activation, residual=residual, b_const=weight_const,
                      b_layout=b_layout)


def hx_bmm(x, y):
    """Batched product (torch.bmm / torch.matmul of rank >= 3 operands) on the
    batched GEMM kernel: linalg.batch_matmul, or batch_matmul_transpose_b when
    y is a transposed view."""
    ops.chain_flush()
    return ops.matmul_batched(x, y)


def hx_conv2d(x, weight_ohwi, bias, stride, padding, dilation):
    """nn.Conv2d / aten.conv2d (groups 1) as the implicit-GEMM convolution:
    NCHW in and out, computed channels-last with the filters pre-permuted to
    [OC, KH, KW, C] once at compile time."""
    ops.chain_flush()
    y = ops.conv2d_nhwc(x.permute(0, 2, 3, 1), weight_ohwi, bias, stride=stride, padding=padding,
                        dilation=dilation)
    return y.permute(0, 3, 1, 2)


def hx_swiglu(x, weight_gate_up, norm_kind=None, norm_stats=None, col_sum=None):
    # the fused [gate; up] weight is a buffer the rewrite registered: constant
    if norm_kind is not None:
        return ops.linear(x, weight_gate_up, None, activation="swiglu", b_const=True,
                          norm=(norm_kind, norm_stats, col_sum))
    return ops.linear(x, weight_gate_up, None, activation="swiglu", b_const=True)


def _users(n: fx.Node):
    return list(n.users.keys())


class _LinearSite:
    """A linear call in the graph: its input node, weight / bias sources and
    the weight's layout ("nk" = W[N,K], "kn" = B[K,N])."""

    def __init__(self, node, x, weight, bias, layout="nk"):
        self.node, self.x, self.weight, self.bias, self.layout = node, x, weight, bias, layout


def _rank(gm, v) -> Optional[int]:
    """Tensor rank of a graph value when known (export metadata or a parameter)."""
    if isinstance(v, fx.Node):
        val = v.meta.get("val", v.meta.get("example_value"))
        if isinstance(val, torch.Tensor):
            return val.dim()
        if v.op == "get_attr":
            try:
                t = _get_attr(gm, v.target)
            except AttributeError:
                return None
            return t.dim() if isinstance(t, torch.Tensor) else None
    return None


def _get_attr(gm, qualname):
    obj = gm
    for part in qualname.split("."):
        obj = getattr(obj, part)
    return obj


def _weight_src(w):
    if isinstance(w, fx.Node) and w.op == "get_attr":
        return ("attr", w.target)
    return ("node", w)


def _as_linear(gm: fx.GraphModule, n: fx.Node) -> Optional[_LinearSite]:
    if n.op == "call_module":
        mod = gm.get_submodule(n.target)
        if isinstance(mod, nn.Linear) and len(n.args) == 1 and not n.kwargs:
            return _LinearSite(n, n.args[0], ("attr", n.target + ".weight"),
                               ("attr", n.target + ".bias") if mod.bias is not None else None)
        return None
    if n.op != "call_function":
        return None
    if n.target in _LINEAR_FNS:
        args = list(n.args) + [None] * (3 - len(n.args))
        x, w, b = args[0], n.kwargs.get("weight", args[1]), n.kwargs.get("bias", args[2])
        return _LinearSite(n, x, _weight_src(w), _weight_src(b) if b is not None else None)
    if n.target in _ADDMM_FNS:
        if len(n.args) != 3 or any(n.kwargs.get(k, 1) != 1 for k in ("beta", "alpha")):
            return None
        if set(n.kwargs) - {"beta", "alpha"}:
            return None
        b, x, w = n.args
        if _rank(gm, b) not in (None, 1) or _rank(gm, w) not in (None, 2):
            return None
        return _LinearSite(n, x, _weight_src(w), _weight_src(b), "kn")
    if n.target in _MM_FNS or n.target in _MATMUL_FNS:
        if len(n.args) != 2 or n.kwargs:
            return None
        x, w = n.args
        rw, rx = _rank(gm, w), _rank(gm, x)
        if n.target in _MATMUL_FNS and (rw != 2 or (rx is not None and rx < 1)):
            return None  # only x[..., K] @ W[K, N] with W known 2-D; batched products are not linears
        return _LinearSite(n, x, _weight_src(w), None, "kn")
    return None


def _is_transparent(gm, n: fx.Node) -> bool:
    """A node that only reshapes its first input, or is inference-mode dropout."""
    if n.op == "call_function" and n.target in _VIEW_FNS:
        return True
    if n.op == "call_method" and n.target in _VIEW_METHODS:
        return True
    if n.op == "call_function" and n.target in _DROPOUT_FNS:
        train = n.kwargs.get("train", n.kwargs.get("training", n.args[2] if len(n.args) > 2 else
                                                    (n.target is F.dropout)))
        return train is False
    if n.op == "call_module" and isinstance(gm.get_submodule(n.target), nn.Dropout):
        return not gm.get_submodule(n.target).training
    return False


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


def _fn(n, fns):
    return isinstance(n, fx.Node) and n.op == "call_function" and n.target in fns and not n.kwargs


def _scalar_pair(n: fx.Node, fns, value, tol=1e-6):
    """(tensor operand) if n is fn(t, value) or fn(value, t) with a Python scalar."""
    if not _fn(n, fns) or len(n.args) != 2:
        return None
    a, b = n.args
    for t, c in ((a, b), (b, a)):
        if isinstance(t, fx.Node) and isinstance(c, (int, float)) and abs(c - value) <= tol * max(1.0, abs(value)):
            return t
    return None


def _gelu_tanh_expr(y: fx.Node) -> Optional[tuple]:
    """Match 0.5*y*(1 + tanh(sqrt(2/pi)*(y + 0.044715*y^3))) written with
    elementwise ops (HF NewGELUActivation / gelu_new), grouped as
    (0.5*y)*(1 + tanh(...)), scalars on either side.  Returns (final node,
    the expression's nodes) or None."""
    users = _users(y)
    if len(users) != 3:
        return None
    half = cube = inner = None
    for u in users:
        if _scalar_pair(u, _MUL_FNS, 0.5) is y:
            half = u
        elif _scalar_pair(u, _POW_FNS, 3.0) is y:
            cube = u
        elif _fn(u, _ADD_FNS) and len(u.args) == 2 and y in u.args:
            inner = u
    if half is None or cube is None or inner is None:
        return None
    nodes = [half, cube, inner]
    cu = _users(cube)
    if len(cu) != 1 or _scalar_pair(cu[0], _MUL_FNS, 0.044715) is not cube:
        return None
    k = cu[0]
    nodes.append(k)
    if k not in inner.args:
        return None
    iu = _users(inner)
    if len(iu) != 1 or _scalar_pair(iu[0], _MUL_FNS, math.sqrt(2.0 / math.pi), 1e-5) is not inner:
        return None
    sc = iu[0]
    nodes.append(sc)
    su = _users(sc)
    if len(su) != 1 or not (_fn(su[0], _TANH_FNS) and su[0].args[0] is sc):
        return None
    th = su[0]
    nodes.append(th)
    tu = _users(th)
    if len(tu) != 1 or _scalar_pair(tu[0], _ADD_FNS, 1.0) is not th:
        return None
    one = tu[0]
    nodes.append(one)
    ou = _users(one)
    hu = _users(half)
    if len(ou) != 1 or len(hu) != 1 or ou[0] is not hu[0]:
        return None
    fin = ou[0]
    if not (_fn(fin, _MUL_FNS) and set(fin.args) == {half, one}):
        return None
    nodes.append(fin)
    return fin, nodes


def _src(graph: fx.Graph, src):
    """Materialise a weight/bias source as a node."""
    if src is None:
        return None
    kind, val = src
    return graph.get_attr(val) if kind == "attr" else val


def _has_param(gm, qualname):
    try:
        t = _get_attr(gm, qualname)
    except AttributeError:
        return False
    return isinstance(t, torch.Tensor)


def _transposed_const(gm, qualname, cache):
    """Register (once) W[N,K] = B[K,N]^T for a constant weight; returns its attribute name."""
    if qualname not in cache:
        name = f"_hx_wT{len(cache)}"
        gm.register_buffer(name, _get_attr(gm, qualname).detach().t().contiguous())
        cache[qualname] = name
    return cache[qualname]


def _fuse_swiglu(gm: fx.GraphModule, sites: dict, done: set) -> None:
    """mul(silu(lin_g(x)), lin_u(x)), both bias-free W[N,K] constants -> one SwiGLU GEMM."""
    graph = gm.graph
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
            if sg.weight[0] != "attr" or su.weight[0] != "attr" or sg.layout != "nk" or su.layout != "nk":
                continue
            if not (_has_param(gm, sg.weight[1]) and _has_param(gm, su.weight[1])):
                continue
            wg, wu = _get_attr(gm, sg.weight[1]), _get_attr(gm, su.weight[1])
            if wg.shape != wu.shape:
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


def _consumer(gm, cur: fx.Node):
    """The epilogue that consumes `cur`: (activation, residual, tail, nodes) or None."""
    us = _users(cur)
    if len(us) == 1:
        u = us[0]
        if _is_gelu_tanh(u) and u.args[0] is cur:
            return "gelu_tanh", None, u, [u]
        if _is_silu(gm, u) and u.args and u.args[0] is cur:
            return "silu", None, u, [u]
        if (u.op == "call_function" and u.target in _ADD_FNS and len(u.args) == 2 and not u.kwargs):
            other = u.args[1] if u.args[0] is cur else u.args[0]
            if isinstance(other, fx.Node) and other is not cur:
                return None, other, u, [u]
    elif len(us) == 3:
        m = _gelu_tanh_expr(cur)
        if m is not None:
            return "gelu_tanh", None, m[0], m[1]
    return None


def rewrite(gm: fx.GraphModule) -> fx.GraphModule:
    """Rewrite linear(+epilogue) patterns in place; returns the module."""
    graph = gm.graph
    sites = {}
    for n in list(graph.nodes):
        s = _as_linear(gm, n)
        if s is not None:
            sites[n] = s
    done = set()
    _fuse_swiglu(gm, sites, done)
    tcache = {}
    for n in list(sites):
        if n in done:
            continue
        s = _as_linear(gm, n)  # re-read: earlier rewrites may have replaced its inputs
        if s is None:
            continue
        chain, cur = [], n
        while True:  # views / reshapes / inference dropout between the linear and its consumer
            us = _users(cur)
            if len(us) == 1 and _is_transparent(gm, us[0]) and us[0].args and us[0].args[0] is cur:
                cur = us[0]
                chain.append(cur)
            else:
                break
        c = _consumer(gm, cur)
        act, residual, tail, expr = c if c is not None else (None, None, cur, [])
        with graph.inserting_before(tail):
            layout = s.layout
            if s.weight[0] == "attr" and layout == "kn" and _has_param(gm, s.weight[1]):
                w = graph.get_attr(_transposed_const(gm, s.weight[1], tcache))
                layout = "nk"
            else:
                w = _src(graph, s.weight)
            b = _src(graph, s.bias)
            kwargs = {}
            if s.weight[0] == "attr":
                kwargs["weight_const"] = True
            if layout != "nk":
                kwargs["b_layout"] = layout
            if act:
                kwargs["activation"] = act
            if residual is not None:
                kwargs["residual"] = residual
            new = graph.call_function(hx_linear, (s.x, w, b), kwargs)
            mapping, last = {n: new}, new
            for cn in chain:  # re-apply the reshapes to the fused result
                last = graph.node_copy(cn, lambda a: mapping.get(a, a))
                mapping[cn] = last
        tail.replace_all_uses_with(last)
        pending = list(expr)
        while pending:  # users before producers (the expression's nodes are not in graph order)
            free = [d for d in pending if not d.users]
            if not free:
                raise RuntimeError("fused epilogue nodes still in use")
            for d in free:
                graph.erase_node(d)
                pending.remove(d)
        for dead in reversed(chain):
            graph.erase_node(dead)
        graph.erase_node(n)
    _rewrite_batched(gm)
    _rewrite_convs(gm)
    _fold_norms(gm)
    graph.lint()
    gm.recompile()
    return gm


_LN_FNS = (F.layer_norm, aten.layer_norm.default)
_RMS_FNS = (aten.rms_norm.default,) + ((F.rms_norm,) if hasattr(F, "rms_norm") else ())


def _norm_site(gm, n: fx.Node):
    """(kind, x, gamma, beta, eps) of a LayerNorm / RMSNorm over the last
    dimension whose affine parameters are constants (get_attr names or None)."""
    def attr_or_none(v):
        if v is None:
            return True, None
        if isinstance(v, fx.Node) and v.op == "get_attr":
            return True, v.target
        return False, None

    if n.op == "call_module":
        mod = gm.get_submodule(n.target)
        if isinstance(mod, nn.LayerNorm) and len(mod.normalized_shape) == 1 and len(n.args) == 1:
            return ("layer", n.args[0], n.target + ".weight" if mod.weight is not None else None,
                    n.target + ".bias" if mod.bias is not None else None, float(mod.eps))
        if hasattr(nn, "RMSNorm") and isinstance(mod, nn.RMSNorm) and len(mod.normalized_shape) == 1 \
                and mod.eps is not None and len(n.args) == 1:
            return ("rms", n.args[0], n.target + ".weight" if mod.weight is not None else None, None, float(mod.eps))
        return None
    if n.op != "call_function":
        return None
    if n.target in _LN_FNS:
        args = list(n.args) + [None] * (5 - len(n.args))
        x, shape = args[0], n.kwargs.get("normalized_shape", args[1])
        w, b = n.kwargs.get("weight", args[2]), n.kwargs.get("bias", args[3])
        eps = n.kwargs.get("eps", args[4] if args[4] is not None else 1e-5)
        kind = "layer"
    elif n.target in _RMS_FNS:
        args = list(n.args) + [None] * (4 - len(n.args))
        x, shape = args[0], n.kwargs.get("normalized_shape", args[1])
        w, b, eps = n.kwargs.get("weight", args[2]), None, n.kwargs.get("eps", args[3])
        kind = "rms"
        if eps is None:
            return None  # dtype-dependent default: not known from the graph
    else:
        return None
    if not isinstance(shape, (list, tuple)) or len(shape) != 1 or not isinstance(eps, (int, float)):
        return None
    ok_w, wname = attr_or_none(w)
    ok_b, bname = attr_or_none(b)
    if not (ok_w and ok_b):
        return None
    return kind, x, wname, bname, float(eps)


def _fold_norms(gm: fx.GraphModule) -> None:
    """norm(x) whose every use reaches (through reshapes) the activation input
    of a fused linear with constant W[N,K] weights -> row statistics of x plus
    linears over x with gamma / beta folded into their weights and bias; the
    normalised activation is never materialised."""
    graph = gm.graph
    cache = {}
    for n in list(graph.nodes):
        site = _norm_site(gm, n)
        if site is None:
            continue
        kind, x, gname, bname, eps = site
        uses = []  # (chain of reshapes, consumer)
        ok = True
        for u in _users(n):
            chain, cur = [], u
            while _is_transparent(gm, cur) and len(_users(cur)) == 1 and cur.args and \
                    (cur.args[0] is n or (chain and cur.args[0] is chain[-1])):
                chain.append(cur)
                cur = _users(cur)[0]
            src = chain[-1] if chain else n
            if src in cur.args[1:] or any(v is src for v in cur.kwargs.values()):
                ok = False  # the normalised value is needed itself (e.g. as a residual)
                break
            if cur.op == "call_function" and cur.target is hx_linear and cur.args[0] is src and \
                    cur.kwargs.get("b_layout", "nk") == "nk" and cur.kwargs.get("norm_kind") is None and \
                    isinstance(cur.args[1], fx.Node) and cur.args[1].op == "get_attr" and \
                    (cur.args[2] is None or (isinstance(cur.args[2], fx.Node) and cur.args[2].op == "get_attr")):
                uses.append((chain, cur))
            elif cur.op == "call_function" and cur.target is hx_swiglu and cur.args[0] is src and \
                    len(cur.args) == 2 and isinstance(cur.args[1], fx.Node) and cur.args[1].op == "get_attr":
                uses.append((chain, cur))
            else:
                ok = False
                break
        if not ok or not uses:
            continue
        gamma = _get_attr(gm, gname).detach() if gname else None
        beta = _get_attr(gm, bname).detach() if bname else None
        with graph.inserting_before(n):
            stats = graph.call_function(hx_norm_stats, (x, kind, eps))
        for chain, lin in uses:
            wname = lin.args[1].target
            bias_node = lin.args[2] if lin.target is hx_linear else None
            key = (wname, bias_node.target if bias_node is not None else None, gname, bname, kind)
            if key not in cache:
                w = _get_attr(gm, wname).detach()
                b = _get_attr(gm, bias_node.target).detach() if bias_node is not None else None
                wf, cs, bf = ops.fold_norm_weight(w, b, gamma, beta, kind)
                i = len(cache)
                gm.register_buffer(f"_hx_nw{i}", wf)
                if cs is not None:
                    gm.register_buffer(f"_hx_ncs{i}", cs)
                if bf is not None:
                    gm.register_buffer(f"_hx_nb{i}", bf)
                cache[key] = (f"_hx_nw{i}", f"_hx_ncs{i}" if cs is not None else None,
                              f"_hx_nb{i}" if bf is not None else None)
            wn, csn, bn = cache[key]
            with graph.inserting_before(lin):
                mapping, last = {n: x}, x
                for cn in chain:
                    last = graph.node_copy(cn, lambda a: mapping.get(a, a))
                    mapping[cn] = last
                wnode = graph.get_attr(wn)
                csnode = graph.get_attr(csn) if csn else None
                bnode = graph.get_attr(bn) if bn else None
            new_args = list(lin.args)
            new_args[0] = last
            new_args[1] = wnode
            if lin.target is hx_linear:
                new_args[2] = bnode
            lin.args = tuple(new_args)
            lin.kwargs = dict(lin.kwargs, norm_kind=kind, norm_stats=stats, col_sum=csnode)
            for cn in reversed(chain):
                graph.erase_node(cn)
        graph.erase_node(n)


_CONV_FNS = (F.conv2d, aten.conv2d.default)


def _rewrite_convs(gm: fx.GraphModule) -> None:
    """Conv2d with constant filters, groups 1, numeric padding -> hx_conv2d."""
    graph = gm.graph
    done = {}
    for n in list(graph.nodes):
        if n.op == "call_module":
            mod = gm.get_submodule(n.target)
            if not (isinstance(mod, nn.Conv2d) and mod.groups == 1 and not isinstance(mod.padding, str)
                    and mod.padding_mode == "zeros" and len(n.args) == 1 and not n.kwargs):
                continue
            x, wname = n.args[0], n.target + ".weight"
            bname = n.target + ".bias" if mod.bias is not None else None
            stride, padding, dilation = tuple(mod.stride), tuple(mod.padding), tuple(mod.dilation)
        elif n.op == "call_function" and n.target in _CONV_FNS:
            args = list(n.args) + [None] * (7 - len(n.args))
            names = ["input", "weight", "bias", "stride", "padding", "dilation", "groups"]
            vals = {k: n.kwargs.get(k, a) for k, a in zip(names, args)}
            w, b = vals["weight"], vals["bias"]
            groups = vals["groups"] if vals["groups"] is not None else 1
            if groups != 1 or isinstance(vals["padding"], str):
                continue
            if not (isinstance(w, fx.Node) and w.op == "get_attr"):
                continue
            if b is not None and not (isinstance(b, fx.Node) and b.op == "get_attr"):
                continue
            x, wname, bname = vals["input"], w.target, (b.target if b is not None else None)
            pr = lambda v, d: tuple(v) if isinstance(v, (list, tuple)) else ((v, v) if v is not None else (d, d))
            stride, padding, dilation = pr(vals["stride"], 1), pr(vals["padding"], 0), pr(vals["dilation"], 1)
            if len(stride) != 2 or len(padding) != 2 or len(dilation) != 2:
                continue
        else:
            continue
        weight = _get_attr(gm, wname)
        if not isinstance(weight, torch.Tensor) or weight.dim() != 4:
            continue
        if wname not in done:
            name = f"_hx_conv_w{len(done)}"
            gm.register_buffer(name, weight.detach().permute(0, 2, 3, 1).contiguous())
            done[wname] = name
        with graph.inserting_before(n):
            wnode = graph.get_attr(done[wname])
            bnode = graph.get_attr(bname) if bname else None
            new = graph.call_function(hx_conv2d, (x, wnode, bnode, stride, padding, dilation))
        n.replace_all_uses_with(new)
        graph.erase_node(n)


def _rewrite_batched(gm: fx.GraphModule) -> None:
    """bmm / matmul nodes whose operands are both batched (rank >= 3 known
    from export metadata, or bmm itself) -> hx_bmm."""
    graph = gm.graph
    for n in list(graph.nodes):
        if n.op != "call_function" or len(n.args) != 2 or n.kwargs:
            continue
        x, y = n.args
        if n.target in _BMM_FNS:
            pass
        elif n.target in _MATMUL_FNS:
            rx, ry = _rank(gm, x), _rank(gm, y)
            if rx is None or ry is None or rx < 3 or ry < 3:
                continue
        else:
            continue
        with graph.inserting_before(n):
            new = graph.call_function(hx_bmm, (x, y))
        n.replace_all_uses_with(new)
        graph.erase_node(n)


def insert_chain_flushes(gm: fx.GraphModule) -> fx.GraphModule:
    """Before every node that may read tensor data and is not a fused linear,
    insert ops.chain_flush(), so GEMMs queued by ops.chained() have run.
    Fused linears queue themselves; getitem (views) reads nothing."""
    graph = gm.graph
    for n in list(graph.nodes):
        if n.op in ("placeholder", "get_attr"):
            continue
        if n.op == "call_function" and (n.target in (hx_linear, hx_swiglu, hx_bmm, hx_conv2d, hx_norm_stats,
                                                     ops.chain_flush)
                                        or n.target is operator.getitem):
            continue
        with graph.inserting_before(n):
            graph.call_function(ops.chain_flush, ())
    graph.lint()
    gm.recompile()
    return gm


def count_hx_calls(gm: fx.GraphModule) -> int:
    return sum(1 for n in gm.graph.nodes
               if n.op == "call_function" and n.target in (hx_linear, hx_swiglu, hx_bmm, hx_conv2d))


def capture(module: nn.Module, example_inputs=None, mode: str = "auto") -> fx.GraphModule:
    """The module as an FX graph.  "trace": torch.fx.symbolic_trace (torch-level
    ops); "export": torch.export (aten ops, the graph torch-mlir's
    export_and_import lowers); "auto": trace, and export when the module does
    not trace (data-dependent Python, as in HF transformers models).  Export
    needs example inputs on the module's device, since it records the devices
    of tensors the forward creates."""
    if mode not in ("auto", "trace", "export"):
        raise ValueError("capture mode must be 'auto', 'trace' or 'export'")
    if mode in ("auto", "trace"):
        try:
            return fx.symbolic_trace(module)
        except Exception:  # noqa: BLE001 - untraceable Python control flow
            if mode == "trace":
                raise
    if example_inputs is None:
        raise ValueError("torch.export capture needs example inputs")
    with torch.no_grad():
        ep = torch.export.export(module, tuple(example_inputs))
    return ep.module()


def compile_module(module: nn.Module, device: torch.device | str = "cuda",
                   chain: bool = False, example_inputs=None, mode: str = "auto") -> fx.GraphModule:
    """Capture `module` (see capture()), on `device`, and rewrite its linear
    layers onto the B200 kernels.  With `chain`, flush points are inserted so
    the graph can run under ops.chained() (consecutive linears become one
    hx_gemm_chain launch).  The original module is not modified."""
    mod = copy.deepcopy(module).to(device)  # the GraphModule would share parameters
    ex = None
    if example_inputs is not None:
        ex = [t.to(device) if isinstance(t, torch.Tensor) else t for t in example_inputs]
    gm = capture(mod, ex, mode).to(device)
    gm = rewrite(gm)
    return insert_chain_flushes(gm) if chain else gm


def hexagon_backend(gm: fx.GraphModule, example_inputs) -> Callable:
    """torch.compile backend: `torch.compile(model, backend=hexagon_backend)`.

    The graph Dynamo hands over keeps module parameters as get_attr/call_module
    nodes or as inputs; linear patterns are rewritten either way (weights that
    arrive as inputs skip only the SwiGLU weight concatenation)."""
    return rewrite(gm).forward
