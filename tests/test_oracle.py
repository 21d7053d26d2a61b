"""CPU tests: the numpy oracle against the PyTorch-CPU golden fixtures.

The fixtures (tests/golden/golden_*.npz, made by tests/golden/make_golden.py)
hold the reference's own golden: PyTorch CPU in fp32
(test/python/triton/test_matmul.py:90, test/python/torch-mlir/utils.py:54).
"""

import glob
import os

import numpy as np
import pytest

from oracle import gemm_oracle as O

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


def _decode(arr, dtype):
    return O.bf16_to_f32(arr) if dtype == "bfloat16" else arr.astype(np.float32)


def test_fixtures_present():
    assert len(GOLDEN) >= 20


@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_fp_" in p], ids=os.path.basename)
def test_oracle_matches_golden_fp(path):
    z = np.load(path)
    dt = str(z["dtype"])
    epi = str(z["epilogue"])
    layout = str(z["b_layout"])
    a, w = _decode(z["a"], dt), _decode(z["w"], dt)
    bias, res = _decode(z["bias"], dt), _decode(z["residual"], dt)
    out = O.linear_ref(a, w, b_layout=layout, epilogue=epi, bias=bias, residual=res)
    # same fp32 math, different summation order: agreement to fp32 rounding
    assert O.max_rel_err(out, z["out"]) < 1e-5


@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_int8_" in p], ids=os.path.basename)
def test_oracle_matches_golden_int8_exact(path):
    z = np.load(path)
    out = O.int8_gemm_exact(z["a"], z["w"])
    np.testing.assert_array_equal(out, z["out"])


@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_w8a16_" in p], ids=os.path.basename)
def test_oracle_matches_golden_w8a16(path):
    z = np.load(path)
    out = O.w8a16_ref(z["x"], z["w"], z["scale"])
    assert O.max_rel_err(out, z["out"]) < 1e-5


def test_gelu_silu_values():
    x = np.array([-3.0, -1.0, 0.0, 0.5, 2.0], dtype=np.float32)
    np.testing.assert_allclose(O.silu(x), x / (1 + np.exp(-x)), rtol=1e-6)
    np.testing.assert_allclose(O.gelu_tanh(np.float32([0.0]))[0], 0.0)
    assert abs(float(O.gelu_tanh(np.float32([2.0]))[0]) - 1.9545977) < 1e-5


def test_bf16_roundtrip():
    x = np.float32([1.0, -2.5, 3.14159, 1e-3, 65504.0])
    y = O.bf16_to_f32(O.f32_to_bf16_bits(x))
    assert np.all(np.abs(y - x) <= np.abs(x) * 2 ** -8)


def test_int8_overflow_guard():
    a = np.full((1, 200000), 127, np.int8)
    with pytest.raises(OverflowError):
        O.int8_gemm_exact(a, a)
