"""CPU tests of the C-ABI boundary: the library loads, exports every
function include/hx_gemm.h declares, its descriptor layout matches the
ctypes mirror, and argument validation answers without touching a GPU."""

import ctypes
import os
import re
import subprocess

import pytest

from qcom_hexagon_backend import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def header_functions():
    names = set()
    for h in HEADERS:
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(hx_\w+)\s*\(", src, flags=re.M))
    return sorted(names)


def test_header_declares_entry_points():
    names = header_functions()
    for must in ("hx_gemm", "hx_matmul_f16f16_f32", "hx_gemv_w8a16", "hx_sharded_gemm_allgather",
                 "hx_status_str", "hx_query_workspace"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in header_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_ctypes_table_covers_header():
    assert set(header_functions()) <= set(_lib.SIGNATURES)


@pytest.mark.parametrize("cname,cls", [("hx_gemm_desc", _lib.HxGemmDesc), ("hx_conv2d_desc", _lib.HxConv2dDesc),
                                       ("hx_w8a16_proj", _lib.HxW8A16Proj)])
def test_desc_layout_matches_c(tmp_path, cname, cls):
    """sizeof/offsetof of each C descriptor from the C compiler == the ctypes mirror."""
    fields = [f for f, _ in cls._fields_]
    prog = ["#include <stdio.h>", "#include <stddef.h>", '#include "hx_gemm.h"', "int main(void){",
            f'printf("%zu\\n", sizeof({cname}));']
    prog += [f'printf("%zu\\n", offsetof({cname}, {f}));' for f in fields]
    prog += ["return 0;}"]
    c = tmp_path / "layout.c"
    c.write_text("\n".join(prog))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(c), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(cls)
    for f, off in zip(fields, vals[1:]):
        assert getattr(cls, f).offset == off, f


def test_status_strings():
    assert _lib.status_name(0) == "HX_OK"
    assert _lib.status_name(-1) == "HX_E_INVALID_ARG"
    assert _lib.status_name(-4) == "HX_E_TIMEOUT"
    assert _lib.status_name(-99) == "HX_E_UNKNOWN"


def _desc(**kw):
    d = _lib.HxGemmDesc()
    d.M, d.N, d.K = 16, 16, 16
    d.a_dtype = d.b_dtype = d.c_dtype = _lib.HX_F16
    d.lda = d.ldb = d.ldc = 16
    d.A, d.B, d.C = 0x1000, 0x2000, 0x3000
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,code", [
    (dict(M=-1), _lib.HX_E_INVALID_ARG),
    (dict(b_dtype=_lib.HX_BF16), _lib.HX_E_UNSUPPORTED),
    (dict(a_dtype=_lib.HX_F32, b_dtype=_lib.HX_F32), _lib.HX_E_UNSUPPORTED),
    (dict(c_dtype=_lib.HX_S32), _lib.HX_E_UNSUPPORTED),
    (dict(lda=8), _lib.HX_E_INVALID_ARG),
    (dict(ldc=8), _lib.HX_E_INVALID_ARG),
    (dict(epilogue=_lib.HX_EPI_BIAS), _lib.HX_E_INVALID_ARG),
    (dict(epilogue=_lib.HX_EPI_RESIDUAL), _lib.HX_E_INVALID_ARG),
    (dict(epilogue=_lib.HX_EPI_DEQUANT_SCALE), _lib.HX_E_INVALID_ARG),
    (dict(epilogue=99), _lib.HX_E_INVALID_ARG),
    (dict(b_layout=5), _lib.HX_E_INVALID_ARG),
    (dict(C=0), _lib.HX_E_INVALID_ARG),
    (dict(epilogue=_lib.HX_EPI_SWIGLU, b_layout=_lib.HX_B_KN), _lib.HX_E_UNSUPPORTED),
])
def test_validation_without_gpu(kw, code):
    lib = _lib.load()
    d = _desc(**kw)
    assert lib.hx_gemm(ctypes.byref(d), None) == code
    assert _lib.last_error() != ""


def test_empty_problem_is_ok_without_gpu():
    lib = _lib.load()
    assert lib.hx_gemm(ctypes.byref(_desc(M=0)), None) == _lib.HX_OK


def test_gemv_validation():
    lib = _lib.load()
    assert lib.hx_gemv_w8a16(-1, 4, 4, None, 4, None, 4, None, None, None, 4, None) == _lib.HX_E_INVALID_ARG
    assert lib.hx_gemv_w8a16(1, 4, 4, None, 4, None, 4, None, None, None, 4, None) == _lib.HX_E_INVALID_ARG
    assert lib.hx_gemv_w8a16(0, 4, 4, None, 4, None, 4, None, None, None, 4, None) == _lib.HX_OK


def test_check_raises():
    with pytest.raises(ValueError):
        _lib.check(_lib.HX_E_INVALID_ARG, "x")
    with pytest.raises(_lib.HexagonB200Error):
        _lib.check(_lib.HX_E_CUDA, "x")


def test_workspace_query():
    lib = _lib.load()
    n = ctypes.c_int64(-1)
    assert lib.hx_query_workspace(ctypes.byref(_desc()), ctypes.byref(n)) == 0 and n.value == 0


def test_ops_reject_cpu_tensors():
    import torch

    from qcom_hexagon_backend import ops

    with pytest.raises(ValueError, match="CUDA"):
        ops.gemm(torch.zeros(4, 4, dtype=torch.float16), torch.zeros(4, 4, dtype=torch.float16))
