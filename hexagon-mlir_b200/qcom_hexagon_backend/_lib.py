"""ctypes binding of the C ABI in include/hx_gemm.h (libhx_gemm.so).

This is the only way Python reaches the kernels.  There is no CPU or
PyTorch fallback: if the shared library is missing, every op raises.
The reference's equivalent bridge is the pybind module
qcom_hexagon_backend/python/triton_qcom_hexagon_backend.cc:52-102, which
hands MLIR to the compiler; here the bridge hands device pointers to
pre-compiled sm_100a kernels.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libhx_gemm.so"
LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)

# status codes (include/hx_gemm.h)
HX_OK = 0
HX_E_INVALID_ARG = -1
HX_E_UNSUPPORTED = -2
HX_E_CUDA = -3
HX_E_TIMEOUT = -4
HX_E_NCCL = -5
HX_E_NO_DEVICE = -6
HX_E_TOO_LARGE = -7

# element types
HX_F16, HX_BF16, HX_S8, HX_S32, HX_F32 = 0, 1, 2, 3, 4
# B layouts
HX_B_NK, HX_B_KN = 0, 1
# hx_gemv_w8a16_ex flags
HX_GEMM_B_CONST = 1
HX_GEMV_WEIGHTS_CONST = 1
HX_GEMV_FORCE_CUDA_CORE = 2
# epilogues
HX_NORM_LAYER = 0
HX_NORM_RMS = 1
HX_EPI_NONE = 0
HX_EPI_BIAS = 1
HX_EPI_BIAS_GELU_TANH = 2
HX_EPI_BIAS_RESIDUAL = 3
HX_EPI_RESIDUAL = 4
HX_EPI_SWIGLU = 5
HX_EPI_DEQUANT_SCALE = 6
HX_EPI_BIAS_SILU = 7

EPILOGUES = {
    "none": HX_EPI_NONE,
    "bias": HX_EPI_BIAS,
    "bias_gelu_tanh": HX_EPI_BIAS_GELU_TANH,
    "bias_residual": HX_EPI_BIAS_RESIDUAL,
    "residual": HX_EPI_RESIDUAL,
    "swiglu": HX_EPI_SWIGLU,
    "dequant_scale": HX_EPI_DEQUANT_SCALE,
    "bias_silu": HX_EPI_BIAS_SILU,
}


class HxGemmDesc(ctypes.Structure):
    """Mirror of `hx_gemm_desc` (field order and types must match)."""

    _fields_ = [
        ("M", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("a_dtype", ctypes.c_int32),
        ("b_dtype", ctypes.c_int32),
        ("c_dtype", ctypes.c_int32),
        ("b_layout", ctypes.c_int32),
        ("A", ctypes.c_void_p),
        ("lda", ctypes.c_int64),
        ("B", ctypes.c_void_p),
        ("ldb", ctypes.c_int64),
        ("C", ctypes.c_void_p),
        ("ldc", ctypes.c_int64),
        ("epilogue", ctypes.c_int32),
        ("bias_dtype", ctypes.c_int32),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("ldr", ctypes.c_int64),
        ("scale_dtype", ctypes.c_int32),
        ("scale", ctypes.c_void_p),
        ("tile_n", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32),
        ("force_simt", ctypes.c_int32),
        ("error_flag", ctypes.c_void_p),
        ("timeout_cycles", ctypes.c_uint64),
        ("split_k", ctypes.c_int32),
        ("flags", ctypes.c_int32),
    ]


class HxConv2dDesc(ctypes.Structure):
    """Mirror of `hx_conv2d_desc`."""

    _fields_ = [
        ("N", ctypes.c_int64), ("H", ctypes.c_int64), ("W", ctypes.c_int64), ("C", ctypes.c_int64),
        ("OC", ctypes.c_int64), ("KH", ctypes.c_int64), ("KW", ctypes.c_int64),
        ("stride_h", ctypes.c_int32), ("stride_w", ctypes.c_int32),
        ("pad_h", ctypes.c_int32), ("pad_w", ctypes.c_int32),
        ("dil_h", ctypes.c_int32), ("dil_w", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("y", ctypes.c_void_p),
        ("bias", ctypes.c_void_p), ("bias_dtype", ctypes.c_int32), ("epilogue", ctypes.c_int32),
        ("residual", ctypes.c_void_p), ("error_flag", ctypes.c_void_p),
    ]


class HxW8A16Proj(ctypes.Structure):
    """Mirror of `hx_w8a16_proj`."""

    _fields_ = [
        ("N", ctypes.c_int64), ("K", ctypes.c_int64),
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("W", ctypes.c_void_p), ("ldw", ctypes.c_int64),
        ("scale", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("dep", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


# Every function the header declares, with its ctypes signature.
_I64, _I32, _VP = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
SIGNATURES = {
    "hx_gemm": (_I32, [ctypes.POINTER(HxGemmDesc), _VP]),
    "hx_gemm_batched": (_I32, [ctypes.POINTER(HxGemmDesc), _I64, _I64, _I64, _I64, _I64, _VP]),
    "hx_conv2d_workspace_size": (_I32, [ctypes.POINTER(HxConv2dDesc), ctypes.POINTER(_I64)]),
    "hx_conv2d": (_I32, [ctypes.POINTER(HxConv2dDesc), _VP, _I64, _VP]),
    "hx_gemm_norm": (_I32, [ctypes.POINTER(HxGemmDesc), _I32, _VP, _VP, _VP]),
    "hx_softmax": (_I32, [_VP, _I32, _I64, _I64, _I64, _VP, _I32, _I64, _I32, _VP]),
    "hx_softmax_stats": (_I32, [_VP, _I32, _I64, _I64, _I64, _VP, _VP]),
    "hx_softmax_combine": (_I32, [_VP, _I32, _I64, _VP, _VP]),
    "hx_softmax_apply": (_I32, [_VP, _I32, _I64, _I64, _I64, _VP, _VP, _I32, _I64, _I32, _VP]),
    "hx_row_norm_stats": (_I32, [_VP, _I32, _I64, _I64, _I64, _I32, ctypes.c_float, _VP, _VP]),
    "hx_sharded_gemm_gather_p2p": (_I32, [ctypes.POINTER(HxGemmDesc), _I32, _I32, _VP, _VP, _I32, _VP, _VP]),
    "hx_sharded_gemm_gather_ce": (_I32, [ctypes.POINTER(HxGemmDesc), _I32, _I32, _VP, _VP, _I32, _VP, _I32, _VP]),
    "hx_peer_handle_size": (_I32, []),
    "hx_peer_alloc": (_I32, [_I64, ctypes.POINTER(_VP), _VP]),
    "hx_peer_open": (_I32, [_VP, ctypes.POINTER(_VP)]),
    "hx_peer_close": (_I32, [_VP]),
    "hx_peer_free": (_I32, [_VP]),
    "hx_matmul_f16f16_f32": (_I32, [_I64, _I64, _I64, _VP, _VP, _VP, _VP]),
    "hx_gemv_w8a16": (_I32, [_I64, _I64, _I64, _VP, _I64, _VP, _I64, _VP, _VP, _VP, _I64, _VP]),
    "hx_gemv_w8a16_ex": (_I32, [_I64, _I64, _I64, _VP, _I64, _VP, _I64, _VP, _VP, _VP, _I64, _I32, _VP]),
    "hx_gemv_w8a16_grouped": (_I32, [_I64, _I32, ctypes.POINTER(HxW8A16Proj), _VP, _VP, _VP]),
    "hx_gemv_w8a16_grouped_noalloc": (_I32, [_I64, _I32, ctypes.POINTER(HxW8A16Proj), _VP, _VP]),
    "hx_gemm_chain": (_I32, [ctypes.POINTER(HxGemmDesc), _VP, _VP, _I32, _VP, _I64, _VP, _VP]),
    "hx_sharded_gemm_allgather": (_I32, [ctypes.POINTER(HxGemmDesc), _I32, _I32, _VP, _VP, _VP]),
    "hx_shards_to_rows": (_I32, [_VP, _VP, _I32, _I64, _I64, _I32, _VP]),
    "hx_nccl_unique_id_size": (_I32, []),
    "hx_nccl_get_unique_id": (_I32, [_VP]),
    "hx_nccl_comm_init": (_I32, [ctypes.POINTER(_VP), _I32, _VP, _I32]),
    "hx_nccl_comm_destroy": (_I32, [_VP]),
    "hx_query_workspace": (_I32, [ctypes.POINTER(HxGemmDesc), ctypes.POINTER(_I64)]),
    "hx_status_str": (ctypes.c_char_p, [_I32]),
    "hx_last_error": (ctypes.c_char_p, []),
    "hx_version": (_I32, []),
}

_lib = None
_lock = threading.Lock()


class HexagonB200Error(RuntimeError):
    """A kernel call returned a non-zero HX_E_* status."""

    def __init__(self, status: int, what: str, detail: str = ""):
        self.status = status
        super().__init__(f"{what} failed: {status_name(status)}" + (f" ({detail})" if detail else ""))


def load() -> ctypes.CDLL:
    """Load libhx_gemm.so once; raise if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                "(there is no CPU fallback)"
            )
        lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_name(status: int) -> str:
    return load().hx_status_str(status).decode()


def last_error() -> str:
    return load().hx_last_error().decode()


def check(status: int, what: str) -> None:
    if status == HX_OK:
        return
    detail = last_error()
    if status == HX_E_INVALID_ARG:
        raise ValueError(f"{what}: invalid argument ({detail})")
    raise HexagonB200Error(status, what, detail)
