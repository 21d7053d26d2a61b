"""CPU tests: the plain-C oracle (oracle/gemm_ref.c) against the golden
fixtures.  Test infrastructure only."""

import ctypes
import glob
import os
import subprocess

import numpy as np
import pytest

from oracle import gemm_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "golden_*.npz")))
EPI = {"none": 0, "bias": 1, "bias_gelu_tanh": 2, "bias_residual": 3, "residual": 4, "swiglu": 5,
       "dequant_scale": 6, "bias_silu": 7}


@pytest.fixture(scope="module")
def cref():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "liboracle.so"))
    P, I = ctypes.c_void_p, ctypes.c_int64
    lib.hx_ref_gemm.argtypes = [I, I, I, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, P]
    lib.hx_ref_gemm_s8.argtypes = [I, I, I, P, P, ctypes.c_int, P]
    lib.hx_ref_w8a16.argtypes = [I, I, I, P, P, P, P]
    lib.hx_ref_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.hx_ref_f16_to_f32.restype = ctypes.c_float
    return lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def test_f16_decode(cref):
    bits = np.arange(0, 1 << 16, 97, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([cref.hx_ref_f16_to_f32(int(b)) for b in bits], dtype=np.float32)
    fin = np.isfinite(ref)
    np.testing.assert_array_equal(got[fin], ref[fin])
    assert np.all(np.isnan(got[np.isnan(ref)]))


@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_fp_" in p], ids=os.path.basename)
def test_c_oracle_matches_golden(cref, path):
    z = np.load(path)
    dt, epi = str(z["dtype"]), str(z["epilogue"])
    layout = 0 if str(z["b_layout"]) == "nk" else 1
    a = np.ascontiguousarray(z["a"].view(np.uint16))
    w = np.ascontiguousarray(z["w"].view(np.uint16))
    M, N, K, _ = [int(v) for v in z["meta"]]
    dec = O.bf16_to_f32 if dt == "bfloat16" else (lambda x: x.astype(np.float32))
    bias = np.ascontiguousarray(dec(z["bias"]), dtype=np.float32)
    res = np.ascontiguousarray(dec(z["residual"]), dtype=np.float32)
    out = np.zeros((M, N), np.float32)
    cref.hx_ref_gemm(M, N, K, _ptr(a), _ptr(w), 1 if dt == "bfloat16" else 0, layout, EPI[epi],
                     _ptr(bias), _ptr(res), None, _ptr(out))
    assert O.max_rel_err(out, z["out"]) < 1e-5


@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_int8_" in p], ids=os.path.basename)
def test_c_oracle_int8_exact(cref, path):
    z = np.load(path)
    M, N, K, _ = [int(v) for v in z["meta"]]
    out = np.zeros((M, N), np.int32)
    cref.hx_ref_gemm_s8(M, N, K, _ptr(np.ascontiguousarray(z["a"])), _ptr(np.ascontiguousarray(z["w"])),
                        0, _ptr(out))
    np.testing.assert_array_equal(out, z["out"])


@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_w8a16_" in p], ids=os.path.basename)
def test_c_oracle_w8a16(cref, path):
    z = np.load(path)
    M, N, K, _ = [int(v) for v in z["meta"]]
    out = np.zeros((M, N), np.float32)
    cref.hx_ref_w8a16(M, N, K, _ptr(np.ascontiguousarray(z["x"].view(np.uint16))),
                      _ptr(np.ascontiguousarray(z["w"])),
                      _ptr(np.ascontiguousarray(z["scale"].view(np.uint16))), _ptr(out))
    assert O.max_rel_err(out, z["out"]) < 1e-5
