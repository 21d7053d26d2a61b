"""The reference's Triton-side surface for the matmul path
(backend/driver.py, backend/compiler.py, test/python/triton/test_matmul.py)."""

import numpy as np
import pytest
import torch

from qcom_hexagon_backend.backend import (HexagonBackend, HexagonDriver, HexagonLauncher, HexagonOptions,
                                          MatmulProgram, matmul, translate_linalg_to_obj)


def test_empty_grid_raises_value_error():
    with pytest.raises(ValueError):
        HexagonLauncher()(0, 1, 1, None, MatmulProgram(), None, None, None, None)
    with pytest.raises(ValueError):
        matmul[(0,)](None, None, None, 1, 1, 1)


def test_non_matmul_program_not_implemented():
    with pytest.raises(NotImplementedError):
        HexagonLauncher()(1, 1, 1, None, object(), None, None, None, None)


def test_unknown_option_rejected():
    with pytest.raises(ValueError):
        matmul[(1,)](None, None, None, 1, 1, 1, notAnOption=True)


def test_linalg_input_refused():
    with pytest.raises(NotImplementedError):
        translate_linalg_to_obj(object(), {})


def test_backend_options_and_driver_names():
    be = HexagonBackend(("cuda", 100, 32))
    assert HexagonBackend.supports_target(HexagonDriver().get_current_target())
    opts = be.parse_options({"enableVTCMTiling": False, "tileSizes": "128", "bogus": 1})
    assert isinstance(opts, HexagonOptions) and opts.tileSizes == "128" and not opts.enableVTCMTiling
    drv = HexagonDriver()
    assert drv.launcher_cls is HexagonLauncher
    assert drv.map_python_to_cpp_type("fp16") == "float"


def test_bad_shapes_rejected():
    a = torch.zeros(4, 8, dtype=torch.float16)
    with pytest.raises(ValueError):
        MatmulProgram()(a, torch.zeros(8, 4, dtype=torch.float16), torch.zeros(4, 5, dtype=torch.float16), 4, 4, 8)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1024, 512, 64), (1024, 1024, 1024), (100, 72, 40)])
def test_reference_style_matmul_launch(cuda_device, shape):
    """Same call as the reference test: host fp16 tensors, result read back from C."""
    import oracle.gemm_oracle as O

    n_rows, n_cols, n_inner = shape
    g = torch.Generator().manual_seed(70)
    A = torch.rand((n_rows, n_inner), generator=g, dtype=torch.float32).half()
    B = torch.rand((n_inner, n_cols), generator=g, dtype=torch.float32).half()
    C = torch.zeros((n_rows, n_cols), dtype=torch.float16)
    matmul[(1,)](A, B, C, n_rows, n_cols, n_inner, enableMultiThreading=True, enableVTCMTiling=True,
                 enableConvertToHexagonmem=True, enableHexagonmemCopyToDMA=True)
    assert C.device.type == "cpu"
    ref = O.linear_ref(A.float().numpy(), B.float().numpy(), b_layout="kn")
    assert torch.allclose(C.float(), torch.from_numpy(np.asarray(ref, np.float32)), atol=2e-1)
    err = np.abs(C.float().numpy() - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert err <= 1e-2
