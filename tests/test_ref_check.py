"""The oracle and the HexKL drop-in checked by the reference's own compiled
CPU check: `check()` of test/python/mlir/hexkl_linalg_matmul/wrapper.cpp
(fp32-accumulated fp16 matmul, |diff| <= 1e-2 per element), built by
oracle/Makefile into oracle/_ref/libref_check.so where the reference tree is
present.  Skipped where that library was not built."""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "_ref", "libref_check.so")

pytestmark = pytest.mark.skipif(not os.path.exists(LIB), reason="oracle/_ref/libref_check.so not built")


def _lib():
    lib = ctypes.CDLL(LIB)
    lib.hx_ref_check.restype = ctypes.c_int
    lib.hx_ref_check.argtypes = [ctypes.c_void_p] * 3
    return lib


def _sizes(lib):
    n, k, m = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
    lib.hx_ref_check_sizes(ctypes.byref(n), ctypes.byref(k), ctypes.byref(m))
    return n.value, k.value, m.value


def _inputs(n, k, m, seed):
    # the reference's set_pointer_random: N(0, 0.5) rounded to 4 decimals, fp16
    rng = np.random.default_rng(seed)
    act = np.round(rng.normal(0.0, 0.5, (n, k)) * 1e4) / 1e4
    w = np.round(rng.normal(0.0, 0.5, (k, m)) * 1e4) / 1e4
    return np.ascontiguousarray(act.astype(np.float16)), np.ascontiguousarray(w.astype(np.float16))


def _check(lib, out, act, w):
    out = np.ascontiguousarray(out, dtype=np.float32)
    return lib.hx_ref_check(out.ctypes.data, act.view(np.uint16).ctypes.data, w.view(np.uint16).ctypes.data)


def test_oracle_passes_reference_check():
    lib = _lib()
    n, k, m = _sizes(lib)
    act, w = _inputs(n, k, m, 3)
    ref = O.matmul_f32(act, w, "kn")
    assert _check(lib, ref, act, w) == 1
    bad = ref.copy()
    bad[n // 2, m // 3] += 0.05  # beyond the 1e-2 bound: the reference check must reject it
    assert _check(lib, bad, act, w) == 0


@pytest.mark.gpu
def test_hexkl_dropin_passes_reference_check(cuda_device):
    import qcom_hexagon_backend as q

    lib = _lib()
    n, k, m = _sizes(lib)
    act, w = _inputs(n, k, m, 4)
    out = q.matmul_f16f16_f32(torch.from_numpy(act).to(cuda_device), torch.from_numpy(w).to(cuda_device))
    torch.cuda.synchronize()
    assert _check(lib, out.cpu().numpy(), act, w) == 1
