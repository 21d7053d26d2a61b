"""Torch-tensor front end of the B200 linear-layer kernels.

Each function checks its tensors, fills the C descriptor and calls the
library on the current CUDA stream.  The tensors must already be on an
sm_100 GPU; nothing here computes on the CPU and nothing falls back to
torch.matmul.

Reference behaviour mirrored: a linear layer is `linalg.matmul` on
`matmul_transpose_b` operands (W[N,K], folded by
lib/Transforms/ScheduleMatmulForHVXPass.cpp:84-93) followed by an
elementwise `linalg.generic` (bias, GELU-tanh, SiLU, residual add, cast;
lowered separately in lib/Conversion/LinalgToLLVM/FusionPass.cpp:163-179).
Here both run in one kernel.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_DT = {
    torch.float16: _lib.HX_F16,
    torch.bfloat16: _lib.HX_BF16,
    torch.int8: _lib.HX_S8,
    torch.int32: _lib.HX_S32,
    torch.float32: _lib.HX_F32,
}


def _dtype_code(t: torch.Tensor, what: str) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"{what}: unsupported dtype {t.dtype}") from None


def _check_cuda(t: torch.Tensor, what: str, device: Optional[torch.device] = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{what} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor (there is no CPU path)")
    if device is not None and t.device != device:
        raise ValueError(f"{what} is on {t.device}, expected {device}")


def _row_major_2d(t: torch.Tensor, what: str) -> int:
    """Return the leading dimension of a 2-D tensor with unit column stride."""
    if t.dim() != 2:
        raise ValueError(f"{what} must be 2-D, got shape {tuple(t.shape)}")
    if t.stride(1) != 1 and t.shape[1] > 1:
        raise ValueError(f"{what} must have unit stride along its last dimension")
    return max(t.stride(0), t.shape[1], 1)


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    b_layout: str = "nk",
    out: Optional[torch.Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
    epilogue: str = "none",
    bias: Optional[torch.Tensor] = None,
    residual: Optional[torch.Tensor] = None,
    scale: Optional[torch.Tensor] = None,
    tile_n: int = 0,
    stages: int = 0,
    max_ctas: int = 0,
    force_simt: bool = False,
    error_flag: Optional[torch.Tensor] = None,
    timeout_cycles: int = 0,
    split_k: int = 0,
    b_const: bool = False,
    norm: Optional[tuple] = None,
) -> torch.Tensor:
    """out = epilogue(a @ B) with B = b.T (b_layout "nk", b is W[N,K]) or
    B = b (b_layout "kn", b is [K,N]).

    norm: (kind, row_stats, col_sum) folds a LayerNorm / RMSNorm of a's rows
    into the GEMM (hx_gemm_norm): b is then the folded weight W * gamma,
    row_stats the [M, 2] float32 output of row_norm_stats(a) and col_sum the
    float32 row sums of b (see fold_norm_weight).

    For epilogue "swiglu", b is the fused [gate; up] weight of 2N rows and
    out = silu(a @ gate.T) * (a @ up.T) has N columns.  b_const: b is a
    constant (model weights) nothing earlier in the stream writes, so the
    kernel may start fetching it before the previous kernel ends.
    """
    d, out, dev = make_desc(a, b, b_layout=b_layout, out=out, out_dtype=out_dtype, epilogue=epilogue,
                            bias=bias, residual=residual, scale=scale, tile_n=tile_n, stages=stages,
                            max_ctas=max_ctas, force_simt=force_simt, error_flag=error_flag,
                            timeout_cycles=timeout_cycles, split_k=split_k, b_const=b_const)
    if norm is not None:
        kind, stats, col_sum = norm
        kind = _NORM_KINDS[kind] if isinstance(kind, str) else int(kind)
        _check_cuda(stats, "row_stats", dev)
        if stats.dtype != torch.float32 or tuple(stats.shape) != (a.shape[0], 2) or not stats.is_contiguous():
            raise ValueError("row_stats must be a contiguous float32 [M, 2] tensor")
        if kind == _lib.HX_NORM_LAYER:
            want = 2 * d.N if epilogue == "swiglu" else d.N
            _check_cuda(col_sum, "col_sum", dev)
            if col_sum.dtype != torch.float32 or col_sum.numel() != want or not col_sum.is_contiguous():
                raise ValueError(f"col_sum must be a contiguous float32 vector of {want}")
        chain_flush()
        lib = _lib.load()
        with torch.cuda.device(dev):
            rc = lib.hx_gemm_norm(ctypes.byref(d), kind, ctypes.c_void_p(stats.data_ptr()),
                                  ctypes.c_void_p(col_sum.data_ptr() if col_sum is not None else 0),
                                  ctypes.c_void_p(_stream_ptr(dev)))
        _lib.check(rc, "hx_gemm_norm")
        return out
    rec = _recorder
    if rec is not None and rec.device == dev:
        if rec.accepts(d, a, b, residual, b_layout, tile_n, stages, max_ctas, force_simt):
            rec.add(d, a, b, out, residual, bias, scale)
            return out
        rec.flush()
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.hx_gemm(ctypes.byref(d), ctypes.c_void_p(_stream_ptr(dev)))
    _lib.check(rc, "hx_gemm")
    return out


class ChainRecorder:
    """Collects consecutive fused GEMMs and runs them as one hx_gemm_chain
    launch, so consecutive linear layers overlap on the GPU.

    Inside `with ops.chained():` every eligible gemm()/linear() call returns
    its (not yet computed) output and is queued; its A operand and residual
    are matched against queued outputs (views such as a column slice count)
    to find the dependencies.  flush() launches the queue; it runs when the
    scope ends, before an ineligible call, and wherever the caller reads the
    data (fx_backend inserts ops.chain_flush before every node that is not a
    fused linear or a view).
    """

    MAX = 64

    def __init__(self, device):
        self.device = torch.device(device)
        self.descs, self.a_dep, self.r_dep, self.outs, self.keep = [], [], [], [], []

    def _producer(self, t):
        if t is None:
            return -1
        p = t.data_ptr()
        for i in range(len(self.outs) - 1, -1, -1):
            o = self.outs[i]
            lo = o.data_ptr()
            if lo <= p < lo + o.numel() * o.element_size():
                return i
        return -1

    def accepts(self, d, a, b, residual, b_layout, tile_n, stages, max_ctas, force_simt):
        if b_layout != "nk" or tile_n or stages or max_ctas or force_simt:
            return False
        if a.dtype not in (torch.float16, torch.bfloat16) or d.K == 0 or d.M == 0 or d.N == 0 or d.K % 64:
            return False
        if d.epilogue == _lib.HX_EPI_DEQUANT_SCALE:
            return False
        if a.data_ptr() % 16 or b.data_ptr() % 16 or (d.lda * 2) % 16 or (d.ldb * 2) % 16:
            return False
        for t in (a, residual):
            i = self._producer(t)
            if i >= 0 and self.descs[i].M != d.M:
                return False
        return True

    def add(self, d, a, b, out, residual, bias, scale):
        if len(self.descs) == self.MAX:
            self.flush()
        self.a_dep.append(self._producer(a))
        self.r_dep.append(self._producer(residual))
        self.descs.append(d)
        self.outs.append(out)
        self.keep.append((a, b, residual, bias, scale))

    def flush(self):
        n = len(self.descs)
        if n == 0:
            return
        arr = (_lib.HxGemmDesc * n)(*self.descs)
        ad = (ctypes.c_int32 * n)(*self.a_dep)
        rd = (ctypes.c_int32 * n)(*self.r_dep)
        nctr = sum((d.M + 127) // 128 for d in self.descs)
        counters = torch.empty(nctr, dtype=torch.int32, device=self.device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            rc = lib.hx_gemm_chain(arr, ad, rd, n, ctypes.c_void_p(counters.data_ptr()), nctr, None,
                                   ctypes.c_void_p(_stream_ptr(self.device)))
        self.keep.append(counters)
        keep = self.keep
        self.descs, self.a_dep, self.r_dep, self.outs, self.keep = [], [], [], [], []
        _lib.check(rc, "hx_gemm_chain")
        # Operands may be freed now: any reuse of their memory is stream-ordered
        # after this launch.
        del keep


_recorder: Optional[ChainRecorder] = None


class chained:
    """Context manager: queue eligible GEMMs and run them as hx_gemm_chain launches."""

    def __init__(self, device):
        self.device = device

    def __enter__(self):
        global _recorder
        if _recorder is not None:
            raise RuntimeError("ops.chained() does not nest")
        _recorder = ChainRecorder(self.device)
        return _recorder

    def __exit__(self, *exc):
        global _recorder
        rec, _recorder = _recorder, None
        if exc[0] is None:
            rec.flush()
        return False


def chain_flush(*args):
    """Run any queued chained GEMMs (a no-op outside ops.chained()); returns
    its first argument so it can sit in an FX graph before a data read."""
    if _recorder is not None:
        _recorder.flush()
    return args[0] if args else None


def make_desc(a, b, *, b_layout="nk", out=None, out_dtype=None, epilogue="none", bias=None,
              residual=None, scale=None, tile_n=0, stages=0, max_ctas=0, force_simt=False,
              error_flag=None, timeout_cycles=0, split_k=0, b_const=False):
    """Validate the tensors and fill an hx_gemm_desc; returns (desc, out, device).
    The tensors must stay alive while the descriptor is in use."""
    _check_cuda(a, "a")
    dev = a.device
    _check_cuda(b, "b", dev)
    if epilogue not in _lib.EPILOGUES:
        raise ValueError(f"unknown epilogue {epilogue!r}; one of {sorted(_lib.EPILOGUES)}")
    epi = _lib.EPILOGUES[epilogue]
    lda = _row_major_2d(a, "a")
    ldb = _row_major_2d(b, "b")
    M, K = a.shape
    if b_layout == "nk":
        nb, kb = b.shape
        N = nb // 2 if epi == _lib.HX_EPI_SWIGLU else nb
        if epi == _lib.HX_EPI_SWIGLU and nb % 2:
            raise ValueError("swiglu weight must have an even number of rows")
        layout = _lib.HX_B_NK
    elif b_layout == "kn":
        kb, N = b.shape
        layout = _lib.HX_B_KN
    else:
        raise ValueError("b_layout must be 'nk' or 'kn'")
    if kb != K:
        raise ValueError(f"inner dimensions differ: a has K={K}, b has K={kb}")
    if a.dtype != b.dtype:
        raise TypeError(f"a and b dtypes differ ({a.dtype} vs {b.dtype})")
    if out is None:
        if out_dtype is None:
            out_dtype = torch.int32 if (a.dtype == torch.int8 and epi == _lib.HX_EPI_NONE) else (
                torch.float16 if a.dtype == torch.int8 else a.dtype)
        out = torch.empty((M, N), dtype=out_dtype, device=dev)
    else:
        _check_cuda(out, "out", dev)
        if tuple(out.shape) != (M, N):
            raise ValueError(f"out has shape {tuple(out.shape)}, expected {(M, N)}")
    ldc = _row_major_2d(out, "out")

    d = _lib.HxGemmDesc()
    d.M, d.N, d.K = M, N, K
    d.a_dtype = d.b_dtype = _dtype_code(a, "a")
    d.c_dtype = _dtype_code(out, "out")
    d.b_layout = layout
    d.A, d.lda = a.data_ptr(), lda
    d.B, d.ldb = b.data_ptr(), ldb
    d.C, d.ldc = out.data_ptr(), ldc
    d.epilogue = epi
    if bias is not None:
        _check_cuda(bias, "bias", dev)
        if bias.dim() != 1 or bias.shape[0] != N or bias.stride(0) != 1:
            raise ValueError(f"bias must be a contiguous vector of {N}")
        d.bias, d.bias_dtype = bias.data_ptr(), _dtype_code(bias, "bias")
    if residual is not None:
        _check_cuda(residual, "residual", dev)
        if tuple(residual.shape) != (M, N) or residual.dtype != out.dtype:
            raise ValueError("residual must match out in shape and dtype")
        d.residual, d.ldr = residual.data_ptr(), _row_major_2d(residual, "residual")
    if scale is not None:
        _check_cuda(scale, "scale", dev)
        if scale.dim() != 1 or scale.shape[0] != N or scale.stride(0) != 1:
            raise ValueError(f"scale must be a contiguous vector of {N}")
        d.scale, d.scale_dtype = scale.data_ptr(), _dtype_code(scale, "scale")
    d.tile_n, d.stages, d.max_ctas = tile_n, stages, max_ctas
    d.force_simt = 1 if force_simt else 0
    if error_flag is not None:
        _check_cuda(error_flag, "error_flag", dev)
        if error_flag.dtype != torch.int32 or error_flag.numel() < 1:
            raise ValueError("error_flag must be an int32 CUDA tensor")
        d.error_flag = error_flag.data_ptr()
    d.timeout_cycles = timeout_cycles
    d.split_k = split_k
    d.flags = _lib.HX_GEMM_B_CONST if b_const else 0
    return d, out, dev


def linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    activation: Optional[str] = None,
    residual: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    b_layout: str = "nk",
    **kw,
) -> torch.Tensor:
    """nn.Linear forward with a fused epilogue: act(x @ W.T + bias) + residual.

    activation: None | "gelu_tanh" | "silu" | "swiglu" (weight = [gate; up]).
    b_layout "kn" takes the weight as B[K,N] (x @ B + bias, aten.addmm's form).
    Leading dimensions of x are flattened, as aten.linear does.
    """
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    r2 = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
    if activation is None:
        if bias is not None and residual is not None:
            epi = "bias_residual"
        elif bias is not None:
            epi = "bias"
        elif residual is not None:
            epi = "residual"
        else:
            epi = "none"
    elif activation == "gelu_tanh":
        if residual is not None:
            raise ValueError("gelu_tanh epilogue takes no residual")
        epi = "bias_gelu_tanh"
    elif activation == "silu":
        if residual is not None:
            raise ValueError("silu epilogue takes no residual")
        epi = "bias_silu"
    elif activation == "swiglu":
        if residual is not None or bias is not None:
            raise ValueError("swiglu epilogue takes no bias or residual")
        epi = "swiglu"
    else:
        raise ValueError(f"unknown activation {activation!r}")
    o2 = out.reshape(-1, out.shape[-1]) if out is not None else None
    if b_layout == "kn" and activation == "swiglu":
        raise ValueError("swiglu takes the weight as [gate; up] W[2N,K]")
    y = gemm(x2, weight, b_layout=b_layout, out=o2, epilogue=epi, bias=bias, residual=r2, **kw)
    return y.reshape(*lead, y.shape[-1])


def matmul(a: torch.Tensor, b: torch.Tensor, *, out: Optional[torch.Tensor] = None,
           out_dtype: Optional[torch.dtype] = None, **kw) -> torch.Tensor:
    """C = A @ B with B stored [K, N] (plain linalg.matmul / tl.dot)."""
    return gemm(a, b, b_layout="kn", out=out, out_dtype=out_dtype, **kw)


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


def conv2d_nhwc(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, *, stride=1, padding=0,
                dilation=1, epilogue: Optional[str] = None, residual: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """2-D convolution as a GEMM (hx_conv2d): x [N, H, W, C] (channels
    innermost), w [OC, KH, KW, C]; returns y [N, OH, OW, OC].  epilogue
    defaults to "bias" with a bias, else "none"; "bias_gelu_tanh",
    "bias_silu", "residual", "bias_residual" are fused too.  The im2col
    workspace, when the shape needs one, is allocated here on x's device."""
    _check_cuda(x, "x")
    _check_cuda(w, "w", x.device)
    if x.dim() != 4 or w.dim() != 4 or x.shape[3] != w.shape[3]:
        raise ValueError(f"x must be [N,H,W,C] and w [OC,KH,KW,C], got {tuple(x.shape)} and {tuple(w.shape)}")
    if x.dtype != w.dtype or x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("conv2d takes f16 or bf16 x and w of the same dtype")
    x = x.contiguous()
    w = w.contiguous()
    (sh, sw), (ph, pw), (dh, dw) = _pair(stride), _pair(padding), _pair(dilation)
    N, H, W, C = x.shape
    OC, KH, KW, _ = w.shape
    OH = (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1
    OW = (W + 2 * pw - dw * (KW - 1) - 1) // sw + 1
    if epilogue is None:
        epilogue = "bias" if bias is not None else "none"
    if out is None:
        out = torch.empty((N, OH, OW, OC), dtype=x.dtype, device=x.device)
    d = _lib.HxConv2dDesc()
    d.N, d.H, d.W, d.C, d.OC, d.KH, d.KW = N, H, W, C, OC, KH, KW
    d.stride_h, d.stride_w, d.pad_h, d.pad_w, d.dil_h, d.dil_w = sh, sw, ph, pw, dh, dw
    d.dtype = _dtype_code(x, "x")
    d.x, d.w, d.y = x.data_ptr(), w.data_ptr(), out.data_ptr()
    if bias is not None:
        _check_cuda(bias, "bias", x.device)
        bias = bias.contiguous()
        d.bias, d.bias_dtype = bias.data_ptr(), _dtype_code(bias, "bias")
    d.epilogue = _lib.EPILOGUES[epilogue]
    if residual is not None:
        _check_cuda(residual, "residual", x.device)
        if tuple(residual.shape) != tuple(out.shape) or not residual.is_contiguous() or residual.dtype != out.dtype:
            raise ValueError("residual must be a contiguous [N, OH, OW, OC] tensor of y's dtype")
        d.residual = residual.data_ptr()
    lib = _lib.load()
    nbytes = ctypes.c_int64()
    _lib.check(lib.hx_conv2d_workspace_size(ctypes.byref(d), ctypes.byref(nbytes)), "hx_conv2d_workspace_size")
    ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=x.device) if nbytes.value else None
    with torch.cuda.device(x.device):
        rc = lib.hx_conv2d(ctypes.byref(d), ctypes.c_void_p(ws.data_ptr() if ws is not None else 0), nbytes.value,
                           ctypes.c_void_p(_stream_ptr(x.device)))
    _lib.check(rc, "hx_conv2d")
    return out


def conv2d(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, stride=1, padding=0,
           dilation=1, groups: int = 1) -> torch.Tensor:
    """F.conv2d on NCHW tensors (groups == 1) through conv2d_nhwc: x is read
    as channels-last (no copy when x is already torch.channels_last) and the
    result is returned as an NCHW-shaped channels-last tensor."""
    if groups != 1:
        raise ValueError("conv2d: groups must be 1")
    if isinstance(padding, str):
        raise ValueError("conv2d: string padding is not supported")
    x_nhwc = x.permute(0, 2, 3, 1)
    w_ohwi = weight.permute(0, 2, 3, 1)
    y = conv2d_nhwc(x_nhwc, w_ohwi, bias, stride=stride, padding=padding, dilation=dilation)
    return y.permute(0, 3, 1, 2)


_NORM_KINDS = {"layer": _lib.HX_NORM_LAYER, "rms": _lib.HX_NORM_RMS}


def row_norm_stats(x: torch.Tensor, kind: str = "layer", eps: float = 1e-5) -> torch.Tensor:
    """[M, 2] float32 per-row {mean, 1/sqrt(var + eps)} (kind "layer",
    F.layer_norm's statistics) or {0, 1/sqrt(mean(x^2) + eps)} ("rms") of the
    last dimension of x (hx_row_norm_stats)."""
    _check_cuda(x, "x")
    x2 = x.reshape(-1, x.shape[-1])
    ld = _row_major_2d(x2, "x")
    stats = torch.empty((x2.shape[0], 2), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.hx_row_norm_stats(ctypes.c_void_p(x2.data_ptr()), _dtype_code(x2, "x"), x2.shape[0], x2.shape[1],
                                   ld, _NORM_KINDS[kind], ctypes.c_float(eps), ctypes.c_void_p(stats.data_ptr()),
                                   ctypes.c_void_p(_stream_ptr(x.device)))
    _lib.check(rc, "hx_row_norm_stats")
    return stats


def fold_norm_weight(weight: torch.Tensor, bias: Optional[torch.Tensor], gamma: Optional[torch.Tensor],
                     beta: Optional[torch.Tensor], kind: str = "layer"):
    """Fold a norm's affine parameters into the linear layer after it (done
    once, at compile time): returns (W' = W * gamma in W's dtype, col_sum =
    float32 row sums of W' as stored, bias' = bias + W @ beta in float32, or
    None).  With these, linear(norm(x)) = linear_norm(x, W', col_sum, bias')."""
    w32 = weight.float()
    if gamma is not None:
        w32 = w32 * gamma.float()[None, :]
    wf = w32.to(weight.dtype).contiguous()
    col_sum = wf.float().sum(1).contiguous() if kind == "layer" else None
    b = bias.float() if bias is not None else None
    if beta is not None and kind == "layer":
        wb = weight.float() @ beta.float()
        b = wb if b is None else b + wb
    return wf, col_sum, (b.contiguous() if b is not None else None)


def linear_norm(x: torch.Tensor, weight: torch.Tensor, col_sum: Optional[torch.Tensor],
                bias: Optional[torch.Tensor], stats: torch.Tensor, kind: str = "layer", *,
                activation: Optional[str] = None, residual: Optional[torch.Tensor] = None,
                **kw) -> torch.Tensor:
    """linear(norm(x)) with the norm folded (weights from fold_norm_weight,
    stats from row_norm_stats(x))."""
    return linear(x, weight, bias, activation=activation, residual=residual, norm=(kind, stats, col_sum), **kw)


def _softmax_dtypes(x, out, out_dtype):
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    return out


def softmax(x: torch.Tensor, *, log: bool = False, out: Optional[torch.Tensor] = None,
            out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Softmax (log-softmax with log=True) over the last dimension (hx_softmax)."""
    _check_cuda(x, "x")
    x2 = x.reshape(-1, x.shape[-1])
    ldx = _row_major_2d(x2, "x")
    out = _softmax_dtypes(x, out, out_dtype)
    o2 = out.view(-1, out.shape[-1])
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.hx_softmax(ctypes.c_void_p(x2.data_ptr()), _dtype_code(x2, "x"), x2.shape[0], x2.shape[1], ldx,
                            ctypes.c_void_p(o2.data_ptr()), _dtype_code(o2, "out"), _row_major_2d(o2, "out"),
                            1 if log else 0, ctypes.c_void_p(_stream_ptr(x.device)))
    _lib.check(rc, "hx_softmax")
    return out


def softmax_stats(x: torch.Tensor) -> torch.Tensor:
    """[M, 2] float32 {row max, sum of exp(x - max)} of a 2-D x (hx_softmax_stats)."""
    _check_cuda(x, "x")
    ldx = _row_major_2d(x, "x")
    st = torch.empty((x.shape[0], 2), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.hx_softmax_stats(ctypes.c_void_p(x.data_ptr()), _dtype_code(x, "x"), x.shape[0], x.shape[1], ldx,
                                  ctypes.c_void_p(st.data_ptr()), ctypes.c_void_p(_stream_ptr(x.device)))
    _lib.check(rc, "hx_softmax_stats")
    return st


def softmax_combine(stats_all: torch.Tensor) -> torch.Tensor:
    """[world, M, 2] per-rank pairs -> [M, 2] global {max, sum} (hx_softmax_combine)."""
    _check_cuda(stats_all, "stats_all")
    if stats_all.dtype != torch.float32 or stats_all.dim() != 3 or not stats_all.is_contiguous():
        raise ValueError("stats_all must be a contiguous float32 [world, M, 2] tensor")
    world, M, _ = stats_all.shape
    st = torch.empty((M, 2), dtype=torch.float32, device=stats_all.device)
    lib = _lib.load()
    with torch.cuda.device(stats_all.device):
        rc = lib.hx_softmax_combine(ctypes.c_void_p(stats_all.data_ptr()), world, M, ctypes.c_void_p(st.data_ptr()),
                                    ctypes.c_void_p(_stream_ptr(stats_all.device)))
    _lib.check(rc, "hx_softmax_combine")
    return st


def softmax_apply(x: torch.Tensor, stats: torch.Tensor, *, log: bool = False, out: Optional[torch.Tensor] = None,
                  out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Softmax of a 2-D x with given [M, 2] row {max, sum} (hx_softmax_apply)."""
    _check_cuda(x, "x")
    ldx = _row_major_2d(x, "x")
    if stats.dtype != torch.float32 or tuple(stats.shape) != (x.shape[0], 2) or not stats.is_contiguous():
        raise ValueError("stats must be a contiguous float32 [M, 2] tensor")
    out = _softmax_dtypes(x, out, out_dtype)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.hx_softmax_apply(ctypes.c_void_p(x.data_ptr()), _dtype_code(x, "x"), x.shape[0], x.shape[1], ldx,
                                  ctypes.c_void_p(stats.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                  _dtype_code(out, "out"), _row_major_2d(out, "out"), 1 if log else 0,
                                  ctypes.c_void_p(_stream_ptr(x.device)))
    _lib.check(rc, "hx_softmax_apply")
    return out


def bmm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    b_layout: str = "kn",
    out: Optional[torch.Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
    epilogue: str = "none",
    bias: Optional[torch.Tensor] = None,
    residual: Optional[torch.Tensor] = None,
    **kw,
) -> torch.Tensor:
    """Batched product out[i] = epilogue(a[i] @ B[i]) (hx_gemm_batched).

    a: [batch, M, K] with unit stride along K (any row and item strides).
    b: [batch, K, N] ("kn", linalg.batch_matmul) or [batch, N, K] ("nk",
    batch_matmul_transpose_b), unit stride along the last dimension; a 2-D b
    is shared by every item.  residual: [batch, M, N]; bias: [N], shared.
    """
    _check_cuda(a, "a")
    if a.dim() != 3:
        raise ValueError(f"a must be 3-D [batch, M, K], got {tuple(a.shape)}")
    nb = a.shape[0]
    shared = b.dim() == 2
    if not shared and (b.dim() != 3 or b.shape[0] != nb):
        raise ValueError(f"b must be [batch, ...] with batch {nb}, or 2-D, got {tuple(b.shape)}")
    b0 = b if shared else b[0] if nb > 0 else b.new_empty(b.shape[1:])
    M = a.shape[1]
    N = (b0.shape[1] if b_layout == "kn" else b0.shape[0])
    if out is None:
        if out_dtype is None:
            out_dtype = torch.int32 if (a.dtype == torch.int8 and epilogue == "none") else (
                torch.float16 if a.dtype == torch.int8 else a.dtype)
        out = torch.empty((nb, M, N), dtype=out_dtype, device=a.device)
    elif tuple(out.shape) != (nb, M, N):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(nb, M, N)}")
    if nb == 0:
        return out
    if residual is not None and tuple(residual.shape) != (nb, M, N):
        raise ValueError("residual must be [batch, M, N]")
    d, _, dev = make_desc(a[0], b0, b_layout=b_layout, out=out[0], epilogue=epilogue, bias=bias,
                          residual=residual[0] if residual is not None else None, **kw)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.hx_gemm_batched(ctypes.byref(d), nb, a.stride(0), 0 if shared else b.stride(0),
                                 out.stride(0), residual.stride(0) if residual is not None else 0,
                                 ctypes.c_void_p(_stream_ptr(dev)))
    _lib.check(rc, "hx_gemm_batched")
    return out


def matmul_batched(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """torch.matmul for x [..., M, K] and y [..., K, N] with broadcast batch
    dimensions.  A y whose K dimension has unit stride (a transposed view,
    as in q @ k.transpose(-1, -2)) is read as W[N, K] items without a copy."""
    if x.dim() < 2 or y.dim() < 2:
        raise ValueError("matmul_batched needs operands of rank >= 2")
    batch = torch.broadcast_shapes(x.shape[:-2], y.shape[:-2])
    M, K = x.shape[-2], x.shape[-1]
    N = y.shape[-1]
    x3 = x.expand(*batch, M, K).reshape(-1, M, K)
    if x3.stride(-1) != 1:
        x3 = x3.contiguous()
    if y.stride(-2) == 1 and y.stride(-1) != 1:  # [.., K, N] view of [.., N, K] memory
        y3 = y.transpose(-1, -2).expand(*batch, N, K).reshape(-1, N, K)
        layout = "nk"
    else:
        y3 = y.expand(*batch, K, N).reshape(-1, K, N)
        layout = "kn"
    if y3.stride(-1) != 1:
        y3 = y3.contiguous()
    out = bmm(x3, y3, b_layout=layout)
    return out.reshape(*batch, M, N)


def matmul_f16f16_f32(act: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """HexKL drop-in (hexkl_matmul_f16f16_f32, bin/runtime/src/HexKLAPI.cpp:15):
    out[f32, n_row x n_col] = act[f16, n_row x n_inner] @ W[f16, n_inner x n_col]."""
    _check_cuda(act, "act")
    _check_cuda(w, "W", act.device)
    if act.dtype != torch.float16 or w.dtype != torch.float16:
        raise TypeError("hexkl matmul takes f16 operands")
    if not (act.is_contiguous() and w.is_contiguous()):
        raise ValueError("hexkl matmul takes contiguous operands")
    n_row, n_inner = act.shape
    k2, n_col = w.shape
    if k2 != n_inner:
        raise ValueError("inner dimensions differ")
    if out is None:
        out = torch.empty((n_row, n_col), dtype=torch.float32, device=act.device)
    lib = _lib.load()
    with torch.cuda.device(act.device):
        rc = lib.hx_matmul_f16f16_f32(n_row, n_col, n_inner, out.data_ptr(), act.data_ptr(),
                                      w.data_ptr(), ctypes.c_void_p(_stream_ptr(act.device)))
    _lib.check(rc, "hx_matmul_f16f16_f32")
    return out


def gemv_w8a16(x: torch.Tensor, w_int8: torch.Tensor, scale: torch.Tensor,
               bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None, *,
               weights_const: bool = False, force_cuda_core: bool = False) -> torch.Tensor:
    """y[M,N] = x[M,K] @ (w_int8[N,K] * scale[N,None]).T (+ bias), f16 in/out.

    weights_const: the weight/scale are model constants that no kernel still
    running before this call writes; their loads then overlap that kernel."""
    _check_cuda(x, "x")
    dev = x.device
    _check_cuda(w_int8, "w_int8", dev)
    _check_cuda(scale, "scale", dev)
    if x.dtype != torch.float16 or w_int8.dtype != torch.int8 or scale.dtype != torch.float16:
        raise TypeError("gemv_w8a16 takes f16 x, int8 weight, f16 scale")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    M, K = x2.shape
    N, K2 = w_int8.shape
    if K2 != K:
        raise ValueError("inner dimensions differ")
    if scale.numel() != N or not scale.is_contiguous():
        raise ValueError("scale must be a contiguous vector of N")
    if bias is not None:
        _check_cuda(bias, "bias", dev)
        if bias.dtype != torch.float16 or bias.numel() != N or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous f16 vector of N")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=dev)
    o2 = out.reshape(-1, N)
    lib = _lib.load()
    with torch.cuda.device(dev):
        flags = (_lib.HX_GEMV_WEIGHTS_CONST if weights_const else 0) | (
            _lib.HX_GEMV_FORCE_CUDA_CORE if force_cuda_core else 0)
        rc = lib.hx_gemv_w8a16_ex(
            M, N, K, x2.data_ptr(), _row_major_2d(x2, "x"), w_int8.data_ptr(),
            _row_major_2d(w_int8, "w_int8"), scale.data_ptr(),
            bias.data_ptr() if bias is not None else None, o2.data_ptr(),
            _row_major_2d(o2, "out"), flags, ctypes.c_void_p(_stream_ptr(dev)))
    _lib.check(rc, "hx_gemv_w8a16")
    return out.reshape(*lead, N)


class W8A16Group:
    """A list of W8A16 projections run as one persistent launch
    (hx_gemv_w8a16_grouped): the linears of a decode step.

    add() returns the projection's index; pass it as `dep` of a later
    projection whose x is that projection's y.  run() launches the group on
    the current stream.  All tensors must stay alive while the group is used.
    """

    def __init__(self, M: int, device):
        self.M = M
        self.device = torch.device(device)
        self._items = []
        self._keep = []
        self._arr = None
        self.counters = None
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)

    def add(self, x, w_int8, scale, y, bias=None, dep: int = -1) -> int:
        for t, nm in ((x, "x"), (w_int8, "w_int8"), (scale, "scale"), (y, "y")):
            _check_cuda(t, nm, self.device)
        if x.dtype != torch.float16 or y.dtype != torch.float16 or w_int8.dtype != torch.int8:
            raise TypeError("W8A16 projection takes f16 x/y and an int8 weight")
        N, K = w_int8.shape
        if tuple(x.shape) != (self.M, K) or tuple(y.shape) != (self.M, N) or scale.numel() != N:
            raise ValueError("projection shapes do not match M, N, K")
        if not (-1 <= dep < len(self._items)):
            raise ValueError("dep must be -1 or the index of an earlier projection")
        it = _lib.HxW8A16Proj()
        it.N, it.K = N, K
        it.x, it.ldx = x.data_ptr(), _row_major_2d(x, "x")
        it.W, it.ldw = w_int8.data_ptr(), _row_major_2d(w_int8, "w_int8")
        it.scale = scale.data_ptr()
        it.bias = bias.data_ptr() if bias is not None else None
        it.y, it.ldy = y.data_ptr(), _row_major_2d(y, "y")
        it.dep = dep
        self._items.append(it)
        self._keep += [x, w_int8, scale, y, bias]
        self._arr = None
        return len(self._items) - 1

    def run(self):
        n = len(self._items)
        if self._arr is None:
            self._arr = (_lib.HxW8A16Proj * n)(*self._items)
            self.counters = torch.zeros(max(n, 1), dtype=torch.int32, device=self.device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            rc = lib.hx_gemv_w8a16_grouped(self.M, n, self._arr, ctypes.c_void_p(self.counters.data_ptr()),
                                           ctypes.c_void_p(self.error_flag.data_ptr()),
                                           ctypes.c_void_p(_stream_ptr(self.device)))
        _lib.check(rc, "hx_gemv_w8a16_grouped")


def shards_to_rows(gathered: torch.Tensor, world: int) -> torch.Tensor:
    """[world, M, Ns] rank-major all-gather result -> row-major [M, world*Ns]."""
    _check_cuda(gathered, "gathered")
    if gathered.dim() != 3 or gathered.shape[0] != world or not gathered.is_contiguous():
        raise ValueError("gathered must be a contiguous [world, M, Ns] tensor")
    _, M, ns = gathered.shape
    out = torch.empty((M, world * ns), dtype=gathered.dtype, device=gathered.device)
    lib = _lib.load()
    with torch.cuda.device(gathered.device):
        rc = lib.hx_shards_to_rows(gathered.data_ptr(), out.data_ptr(), world, M, ns,
                                   gathered.element_size(),
                                   ctypes.c_void_p(_stream_ptr(gathered.device)))
    _lib.check(rc, "hx_shards_to_rows")
    return out
