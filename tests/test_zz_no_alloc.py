"""GPU test of hx_gemv_w8a16_grouped_noalloc, the grouped W8A16 entry point
for callers that cannot allocate device memory (a serving engine whose pool
owns the GPU, a decode loop that must not synchronise on cudaMalloc, a
foreign-function host that only passes pointers it owns).

It is called through the C ABI and checked against the allocating entry
point, hx_gemv_w8a16_grouped, on the same inputs, with the tolerance the
other parity tests use, on two calls in a row (the second call must clear
the counters the first one left behind).  The file is named so that pytest
collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _projections(M, device):
    """Four projections, one of them dependent on another (y of #0 feeds #2)."""
    g = torch.Generator().manual_seed(77 + M)
    keep, projs = [], []
    from qcom_hexagon_backend import _lib

    specs = [(2048, 2048, -1, 0.0015), (256, 2048, -1, 0.02), (512, 2048, 0, 0.02), (300, 64, -1, 0.02)]
    ys = []
    for n, k, dep, s_hi in specs:
        w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int64).to(torch.int8).to(device)
        s = (torch.rand(n, generator=g) * (s_hi - 0.001) + 0.001).half().to(device)
        x = ys[dep] if dep >= 0 else torch.randn(M, k, generator=g).half().to(device)
        y = torch.full((M, n), float("nan"), dtype=torch.float16, device=device)
        ys.append(y)
        p = _lib.HxW8A16Proj()
        p.N, p.K = n, k
        p.x, p.ldx = x.data_ptr(), k
        p.W, p.ldw = w.data_ptr(), k
        p.scale, p.bias = s.data_ptr(), None
        p.y, p.ldy = y.data_ptr(), n
        p.dep = dep
        projs.append(p)
        keep += [w, s, x, y]
    arr = (_lib.HxW8A16Proj * len(projs))(*projs)
    return arr, ys, keep


@pytest.mark.parametrize("M", [1, 4])
def test_noalloc_matches_allocating_entry_point(cuda_device, M):
    from qcom_hexagon_backend import _lib

    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    arr_a, ys_a, keep_a = _projections(M, cuda_device)
    counters = torch.zeros(len(arr_a), dtype=torch.int32, device=cuda_device)
    flag_a = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    rc = lib.hx_gemv_w8a16_grouped(M, len(arr_a), arr_a, ctypes.c_void_p(counters.data_ptr()),
                                   ctypes.c_void_p(flag_a.data_ptr()), stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize(cuda_device)
    ref = [y.float().cpu().numpy() for y in ys_a]

    arr_b, ys_b, keep_b = _projections(M, cuda_device)  # same seeds -> same inputs
    flag_b = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for call in range(2):
        for y in ys_b:
            y.fill_(float("nan"))
        rc = lib.hx_gemv_w8a16_grouped_noalloc(M, len(arr_b), arr_b, ctypes.c_void_p(flag_b.data_ptr()), stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize(cuda_device)
        assert int(flag_b.item()) == 0, f"call {call}: a bounded wait ran out"
        for got, want in zip(ys_b, ref):
            got = got.float().cpu().numpy()
            assert np.isfinite(got).all(), f"call {call}: output not written"
            assert O.max_rel_err(got, want) <= TOL, f"call {call}"


def test_noalloc_rejects_too_many_projections(cuda_device):
    from qcom_hexagon_backend import _lib

    lib = _lib.load()
    arr = (_lib.HxW8A16Proj * 257)()
    rc = lib.hx_gemv_w8a16_grouped_noalloc(1, 257, arr, None, None)
    assert rc == _lib.HX_E_TOO_LARGE
    assert "256" in _lib.last_error()
