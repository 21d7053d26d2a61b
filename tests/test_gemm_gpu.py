"""GPU parity tests: the sm_100a kernels, called through the C ABI, against
the CPU oracle on the same seeded inputs.

Tolerances (stated by the benchmark contract for this path):
  * fp16 / bf16 inputs, fp32 accumulate: max |out - ref| / max |ref| <= 1e-2
    against the fp32 oracle, plus an elementwise bound of 1e-2 * (|ref| + rms(ref));
  * int8 W8A8 with int32 output: bit-exact.
"""

import glob
import os

import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2
GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


def hx():
    import qcom_hexagon_backend as q

    return q


def to_np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def assert_close(out, ref, tol=TOL):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(out).all(), "non-finite output"
    err = O.max_rel_err(out, ref)
    assert err <= tol, f"max rel err {err:.3e} > {tol}"
    rms = np.sqrt(np.mean(ref * ref)) if ref.size else 0.0
    bad = np.abs(out - ref) > tol * (np.abs(ref) + rms) + 1e-6
    assert not bad.any(), f"{bad.sum()} elements outside elementwise bound; first at {np.argwhere(bad)[0]}"


def make_inputs(M, N, K, dtype, *, epilogue="none", b_layout="nk", seed=0, dev="cuda"):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(dtype)
    rows = 2 * N if epilogue == "swiglu" else N
    w = (torch.randn(rows, K, generator=g) * 0.02).to(dtype) if b_layout == "nk" else \
        (torch.randn(K, N, generator=g) * 0.02).to(dtype)
    bias = (torch.randn(N, generator=g) * 0.02).to(dtype)
    res = torch.randn(M, N, generator=g).to(dtype)
    return a.to(dev), w.to(dev), bias.to(dev), res.to(dev)


def run_and_check(M, N, K, dtype, epilogue, b_layout="nk", seed=0, **kw):
    q = hx()
    a, w, bias, res = make_inputs(M, N, K, dtype, epilogue=epilogue, b_layout=b_layout, seed=seed)
    use_bias = epilogue in ("bias", "bias_gelu_tanh", "bias_residual", "bias_silu")
    use_res = epilogue in ("bias_residual", "residual")
    out = q.gemm(a, w, b_layout=b_layout, epilogue=epilogue, bias=bias if use_bias else None,
                 residual=res if use_res else None, **kw)
    torch.cuda.synchronize()
    ref = O.linear_ref(to_np32(a), to_np32(w), b_layout=b_layout, epilogue=epilogue,
                       bias=to_np32(bias), residual=to_np32(res))
    assert_close(to_np32(out), ref)
    return out


# ---------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_fp_" in p], ids=os.path.basename)
def test_golden_fp(cuda_device, path):
    q = hx()
    z = np.load(path)
    dt = str(z["dtype"])
    tdt = torch.float16 if dt == "float16" else torch.bfloat16

    def t(x):
        if dt == "bfloat16":
            return torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(cuda_device)
        return torch.from_numpy(x).to(cuda_device)

    a, w, bias, res = t(z["a"]), t(z["w"]), t(z["bias"]), t(z["residual"])
    assert a.dtype == tdt
    epi = str(z["epilogue"])
    use_bias = epi in ("bias", "bias_gelu_tanh", "bias_residual", "bias_silu")
    use_res = epi in ("bias_residual", "residual")
    out = q.gemm(a, w, b_layout=str(z["b_layout"]), epilogue=epi,
                 bias=bias if use_bias else None, residual=res if use_res else None)
    torch.cuda.synchronize()
    assert_close(to_np32(out), z["out"])


@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_int8_" in p], ids=os.path.basename)
def test_golden_int8_exact(cuda_device, path):
    q = hx()
    z = np.load(path)
    out = q.gemm(torch.from_numpy(z["a"]).to(cuda_device), torch.from_numpy(z["w"]).to(cuda_device))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), z["out"])


@pytest.mark.parametrize("path", [p for p in GOLDEN if "golden_w8a16_" in p], ids=os.path.basename)
def test_golden_w8a16(cuda_device, path):
    q = hx()
    z = np.load(path)
    d = cuda_device
    y = q.gemv_w8a16(torch.from_numpy(z["x"]).to(d), torch.from_numpy(z["w"]).to(d),
                     torch.from_numpy(z["scale"]).to(d))
    torch.cuda.synchronize()
    assert_close(to_np32(y), z["out"])


# ---------------------------------------------------------------- config 1
def test_config1_fp16_1024_cube(cuda_device):
    """C = A.B, M=N=K=1024, A,B ~ N(0,1) fp16, fp32 acc, fp16 out."""
    q = hx()
    g = torch.Generator().manual_seed(1234)
    a = torch.randn(1024, 1024, generator=g).half()
    b = torch.randn(1024, 1024, generator=g).half()
    out = q.matmul(a.cuda(), b.cuda())
    torch.cuda.synchronize()
    ref = O.matmul_f32(a.float().numpy(), b.float().numpy(), "kn")
    assert_close(to_np32(out), ref)


def test_hexkl_dropin(cuda_device):
    """hexkl_matmul_f16f16_f32 shape of the reference's HMX test (1024x64 . 64x512)."""
    q = hx()
    g = torch.Generator().manual_seed(7)
    act = (torch.randn(1024, 64, generator=g) * 0.5).half()
    w = (torch.randn(64, 512, generator=g) * 0.5).half()
    out = q.matmul_f16f16_f32(act.cuda(), w.cuda())
    torch.cuda.synchronize()
    ref = O.matmul_f32(act.numpy(), w.numpy(), "kn")
    assert out.dtype == torch.float32
    # wrapper.cpp:30,57 bound: |diff| <= 1e-2 elementwise
    assert np.abs(out.cpu().numpy() - ref).max() <= 1e-2


# ---------------------------------------------------------------- shapes x epilogues
SHAPES = [(128, 128, 64), (256, 512, 128), (200, 300, 136), (1, 64, 64), (129, 257, 40),
          (1024, 2304, 768), (333, 1000, 520)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gemm_nk_none(cuda_device, dtype, shape):
    run_and_check(*shape, dtype, "none")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("shape", [(128, 128, 64), (200, 320, 136), (64, 1000, 72)],
                         ids=lambda s: "x".join(map(str, s)))
def test_gemm_kn(cuda_device, dtype, shape):
    run_and_check(*shape, dtype, "none", b_layout="kn")


@pytest.mark.parametrize("epilogue", ["bias", "bias_gelu_tanh", "bias_silu", "bias_residual",
                                      "residual", "swiglu"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_epilogues(cuda_device, epilogue, dtype):
    run_and_check(300, 264, 200, dtype, epilogue, seed=3)


@pytest.mark.parametrize("tile_n", [64, 128, 256])
@pytest.mark.parametrize("epilogue", ["none", "bias_residual", "swiglu"])
def test_tile_overrides(cuda_device, tile_n, epilogue):
    run_and_check(384, 520, 256, torch.float16, epilogue, tile_n=tile_n, seed=5)


@pytest.mark.parametrize("tile_n", [96, 192])
@pytest.mark.parametrize("epilogue", ["none", "bias_gelu_tanh", "bias_residual"])
def test_tile_n_not_pow2(cuda_device, tile_n, epilogue):
    """96- and 192-column tiles (TMEM allocation rounded up to a power of two)."""
    run_and_check(384, 520, 256, torch.float16, epilogue, tile_n=tile_n, seed=15)
    run_and_check(1000, 3 * tile_n + 17, 768, torch.bfloat16, epilogue, tile_n=tile_n, seed=16)


def test_tile_n_192_swiglu_and_int8(cuda_device):
    run_and_check(256, 400, 384, torch.bfloat16, "swiglu", tile_n=192, seed=17)
    q = hx()
    g = torch.Generator().manual_seed(18)
    a = torch.randint(-127, 128, (300, 512), generator=g, dtype=torch.int64).to(torch.int8)
    w = torch.randint(-127, 128, (500, 512), generator=g, dtype=torch.int64).to(torch.int8)
    for tn in (96, 192):
        out = q.gemm(a.cuda(), w.cuda(), tile_n=tn)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), O.int8_gemm_exact(a.numpy(), w.numpy()))


def test_tile_n_rejected_combinations(cuda_device):
    q = hx()
    from qcom_hexagon_backend._lib import HexagonB200Error
    a = torch.randn(128, 128, device="cuda").half()
    with pytest.raises((ValueError, HexagonB200Error)):
        q.gemm(a, torch.randn(128, 256, device="cuda").half(), b_layout="kn", tile_n=96)
    with pytest.raises((ValueError, HexagonB200Error)):
        q.gemm(a, torch.randn(128, 128, device="cuda").half(), tile_n=100)


@pytest.mark.parametrize("stages", [2, 3, 4])
def test_stage_overrides(cuda_device, stages):
    run_and_check(512, 512, 1024, torch.bfloat16, "none", tile_n=256, stages=stages, seed=6)


def test_persistent_multi_tile_per_cta(cuda_device):
    """Few CTAs, many tiles: exercises the TMEM double buffer and ring phases."""
    run_and_check(1024, 1024, 512, torch.float16, "bias", max_ctas=3, seed=8)


def test_simt_path_matches(cuda_device):
    run_and_check(200, 300, 136, torch.float16, "bias_gelu_tanh", force_simt=True, seed=9)


def test_unaligned_falls_to_simt(cuda_device):
    """lda*2 not a multiple of 16 bytes: the CUDA-core kernel takes it."""
    run_and_check(100, 90, 37, torch.float16, "bias", seed=10)


# ---------------------------------------------------------------- int8
@pytest.mark.parametrize("shape", [(128, 256, 128), (300, 520, 200), (1024, 1024, 2048), (7, 9, 16)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("b_layout", ["nk", "kn"])
def test_int8_exact(cuda_device, shape, b_layout):
    q = hx()
    M, N, K = shape
    g = torch.Generator().manual_seed(11)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int64).to(torch.int8)
    w = torch.randint(-127, 128, (N, K) if b_layout == "nk" else (K, N), generator=g,
                      dtype=torch.int64).to(torch.int8)
    out = q.gemm(a.cuda(), w.cuda(), b_layout=b_layout)
    torch.cuda.synchronize()
    ref = O.int8_gemm_exact(a.numpy(), w.numpy(), b_layout)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_int8_dequant_epilogue(cuda_device):
    q = hx()
    g = torch.Generator().manual_seed(12)
    a = torch.randint(-127, 128, (256, 512), generator=g, dtype=torch.int64).to(torch.int8)
    w = torch.randint(-127, 128, (384, 512), generator=g, dtype=torch.int64).to(torch.int8)
    scale = torch.rand(384, generator=g) * 1e-4
    out = q.gemm(a.cuda(), w.cuda(), epilogue="dequant_scale", scale=scale.cuda(),
                 out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = O.int8_gemm_exact(a.numpy(), w.numpy()).astype(np.float64) * scale.numpy()[None, :]
    assert_close(out.cpu().numpy(), ref, tol=1e-5)


# ---------------------------------------------------------------- W8A16
@pytest.mark.parametrize("path", ["auto", "auto_const", "cuda_core"])
@pytest.mark.parametrize("M", [1, 2, 3, 8, 32, 64])
@pytest.mark.parametrize("NK", [(2048, 2048), (256, 2048), (5632, 2048), (2048, 5632)],
                         ids=lambda s: f"{s[0]}x{s[1]}")
def test_w8a16(cuda_device, M, NK, path):
    q = hx()
    N, K = NK
    g = torch.Generator().manual_seed(13 + M)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int64).to(torch.int8)
    scale = (torch.rand(N, generator=g) * 0.019 + 0.001).half()
    x = torch.randn(M, K, generator=g).half()
    y = q.gemv_w8a16(x.cuda(), w.cuda(), scale.cuda(), weights_const=(path == "auto_const"),
                     force_cuda_core=(path == "cuda_core"))
    torch.cuda.synchronize()
    assert_close(to_np32(y), O.w8a16_ref(x.numpy(), w.numpy(), scale.numpy()))


@pytest.mark.parametrize("M,N,K", [(128, 300, 1000), (256, 384, 512), (100, 129, 2064), (5, 7, 48)])
def test_w8a16_tc_odd_shapes(cuda_device, M, N, K):
    """Batch up to 256 (MPAD 128/256), N and K tails, bias."""
    q = hx()
    g = torch.Generator().manual_seed(M + N + K)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int64).to(torch.int8)
    scale = (torch.rand(N, generator=g) * 0.019 + 0.001).half()
    bias = (torch.randn(N, generator=g) * 0.02).half()
    x = torch.randn(M, K, generator=g).half()
    y = q.gemv_w8a16(x.cuda(), w.cuda(), scale.cuda(), bias=bias.cuda())
    torch.cuda.synchronize()
    assert_close(to_np32(y), O.w8a16_ref(x.numpy(), w.numpy(), scale.numpy(), bias.numpy()))


def test_w8a16_back_to_back_const(cuda_device):
    """Chained decode projections with the constant-weight prefetch: the
    second call reads the first call's output."""
    q = hx()
    g = torch.Generator().manual_seed(21)
    w1 = torch.randint(-127, 128, (2048, 2048), generator=g, dtype=torch.int64).to(torch.int8)
    w2 = torch.randint(-127, 128, (512, 2048), generator=g, dtype=torch.int64).to(torch.int8)
    s1 = (torch.rand(2048, generator=g) * 0.001 + 0.0005).half()
    s2 = (torch.rand(512, generator=g) * 0.019 + 0.001).half()
    x = torch.randn(8, 2048, generator=g).half()
    d = cuda_device
    for _ in range(3):
        h = q.gemv_w8a16(x.to(d), w1.to(d), s1.to(d), weights_const=True)
        y = q.gemv_w8a16(h, w2.to(d), s2.to(d), weights_const=True)
    torch.cuda.synchronize()
    h_ref = O.w8a16_ref(x.numpy(), w1.numpy(), s1.numpy()).astype(np.float16)
    assert_close(to_np32(y), O.w8a16_ref(h_ref, w2.numpy(), s2.numpy()))


def test_w8a16_unaligned_scalar(cuda_device):
    q = hx()
    g = torch.Generator().manual_seed(14)
    w = torch.randint(-127, 128, (33, 100), generator=g, dtype=torch.int64).to(torch.int8)
    scale = (torch.rand(33, generator=g) * 0.019 + 0.001).half()
    bias = (torch.randn(33, generator=g) * 0.02).half()
    x = torch.randn(3, 100, generator=g).half()
    y = q.gemv_w8a16(x.cuda(), w.cuda(), scale.cuda(), bias=bias.cuda())
    torch.cuda.synchronize()
    assert_close(to_np32(y), O.w8a16_ref(x.numpy(), w.numpy(), scale.numpy(), bias.numpy()))


# ---------------------------------------------------------------- edge cases
def test_empty_dims(cuda_device):
    q = hx()
    a = torch.empty(0, 64, dtype=torch.float16, device="cuda")
    w = torch.randn(32, 64, device="cuda").half()
    assert q.gemm(a, w).shape == (0, 32)


def test_k_zero_gives_epilogue_of_zero(cuda_device):
    q = hx()
    a = torch.empty(16, 0, dtype=torch.float16, device="cuda")
    w = torch.empty(24, 0, dtype=torch.float16, device="cuda")
    bias = torch.randn(24, device="cuda").half()
    out = q.gemm(a, w, epilogue="bias", bias=bias)
    torch.cuda.synchronize()
    assert torch.equal(out, bias.expand(16, 24))


def test_strided_activation_view(cuda_device):
    """A as a column slice of a wider matrix (lda > K), as the stack feeds qkv[:, :768]."""
    q = hx()
    g = torch.Generator().manual_seed(15)
    big = torch.randn(256, 2304, generator=g).half().cuda()
    a = big[:, :768]
    w = (torch.randn(768, 768, generator=g) * 0.02).half().cuda()
    out = q.gemm(a, w)
    torch.cuda.synchronize()
    assert_close(to_np32(out), O.matmul_f32(to_np32(a), to_np32(w)))


def test_repeatable_bitwise(cuda_device):
    q = hx()
    a, w, _, _ = make_inputs(512, 768, 768, torch.float16, seed=16)
    o1 = q.gemm(a, w)
    o2 = q.gemm(a, w)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


def test_cpu_tensor_rejected(cuda_device):
    q = hx()
    with pytest.raises(ValueError):
        q.gemm(torch.randn(4, 4).half(), torch.randn(4, 4).half())


# ---------------------------------------------------------------- grouped W8A16
GROUPED_TC_SHAPES = [(2048, 2048, -1, 0.0015), (256, 2048, -1, 0.02), (5632, 2048, -1, 0.0015),
                     (2048, 2048, 0, 0.02), (2048, 5632, 2, 0.02), (300, 1024, -1, 0.02)]
GROUPED_MIXED_SHAPES = GROUPED_TC_SHAPES[:5] + [(100, 48, -1, 0.02)]  # K=48: CUDA-core kernel


@pytest.mark.parametrize("path,M", [("mma", 1), ("mma", 3), ("mma", 8), ("mma", 9), ("mma", 16),
                                    ("mma_p1", 1), ("mma_p1", 16),
                                    ("tc", 1), ("tc", 3), ("tc", 8), ("tc", 16), ("tc", 17),
                                    ("tc", 32), ("tc", 50), ("tc", 64),
                                    ("mixed", 1), ("mixed", 3), ("mixed", 8),
                                    ("cuda_core", 1), ("cuda_core", 8)])
def test_w8a16_grouped_chain(cuda_device, monkeypatch, path, M):
    """A decode-layer-like list in one launch: independent projections plus a
    dependent chain (q -> o, gate -> down), checked against the oracle.
    "mma": M <= 16 with every K a multiple of 64, the register-fragment MMA
    kernel (the default there; "mma_p1" with 16-byte row pieces per lane);
    "tc": the tcgen05 kernel (the default for M > 16, forced below that
    through HX_GROUPED_PATH); "mixed": one K=48 projection sends the list to
    the CUDA-core kernel; "cuda_core": that kernel forced through
    HX_GROUPED_CUDA_CORE."""
    if path == "cuda_core":
        monkeypatch.setenv("HX_GROUPED_CUDA_CORE", "1")
    elif path == "tc":
        monkeypatch.setenv("HX_GROUPED_PATH", "tc")
    elif path == "mma_p1":
        monkeypatch.setenv("HX_GM_P", "1")
    q = hx()
    d = cuda_device
    g = torch.Generator().manual_seed(30 + M)

    def wq(n, k, s_hi=0.02):
        w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int64).to(torch.int8)
        s = (torch.rand(n, generator=g) * (s_hi - 0.001) + 0.001).half()
        return w, s

    x = torch.randn(M, 2048, generator=g).half()
    shapes = GROUPED_MIXED_SHAPES if path == "mixed" else GROUPED_TC_SHAPES
    grp = q.ops.W8A16Group(M, d)
    ys, ws = [], []
    for i, (n, k, dep, shi) in enumerate(shapes):
        w, s = wq(n, k, shi)
        ws.append((w, s))
        xin = ys[dep] if dep >= 0 else (x.to(d) if k == 2048 else torch.randn(M, k, generator=g).half().to(d))
        y = torch.empty(M, n, dtype=torch.float16, device=d)
        ys.append(y)
        grp.add(xin, w.to(d), s.to(d), y, dep=dep)
        ws[-1] = (w, s, xin)
    for _ in range(2):  # run twice: counters are reset per launch
        grp.run()
    torch.cuda.synchronize()
    assert int(grp.error_flag.item()) == 0
    refs = []
    for i, (n, k, dep, _) in enumerate(shapes):
        w, s, xin = ws[i]
        xr = refs[dep].astype(np.float16) if dep >= 0 else to_np32(xin)
        refs.append(O.w8a16_ref(xr, w.numpy(), s.numpy()))
        assert_close(to_np32(ys[i]), refs[-1])


@pytest.mark.parametrize("path,M", [("mma", 1), ("mma", 8), ("mma", 13), ("mma_p1", 4),
                                    ("tc", 1), ("tc", 24), ("cuda_core", 2)])
def test_w8a16_grouped_bias_strided(cuda_device, monkeypatch, path, M):
    """Bias, strided operands and a ragged last row block: x is a column slice
    of a wider activation (ldx > K), the weight a column slice of a wider
    int8 matrix (ldw > K), y a column slice of a wider output (ldy > N), and
    N = 1000 leaves a partial last item; checked against the oracle."""
    if path == "cuda_core":
        monkeypatch.setenv("HX_GROUPED_CUDA_CORE", "1")
    elif path == "tc":
        monkeypatch.setenv("HX_GROUPED_PATH", "tc")
    elif path == "mma_p1":
        monkeypatch.setenv("HX_GM_P", "1")
    q = hx()
    d = cuda_device
    g = torch.Generator().manual_seed(90 + M)
    N, K = 1000, 1024
    w_full = torch.randint(-127, 128, (N, K + 256), generator=g, dtype=torch.int64).to(torch.int8)
    s = (torch.rand(N, generator=g) * 0.019 + 0.001).half()
    b = (torch.randn(N, generator=g) * 0.1).half()
    x_full = torch.randn(M, K + 128, generator=g).half()
    w_dev, x_dev = w_full.to(d), x_full.to(d)
    y_full = torch.full((M, N + 24), float("nan"), dtype=torch.float16, device=d)
    grp = q.ops.W8A16Group(M, d)
    grp.add(x_dev[:, 64:64 + K], w_dev[:, 128:128 + K], s.to(d), y_full[:, :N], bias=b.to(d))
    grp.run()
    torch.cuda.synchronize()
    assert int(grp.error_flag.item()) == 0
    ref = O.w8a16_ref(x_full[:, 64:64 + K].numpy(), w_full[:, 128:128 + K].numpy(), s.numpy(), b.numpy())
    assert_close(to_np32(y_full[:, :N]), ref)
    assert torch.isnan(y_full[:, N:]).all(), "stores past ldy's N columns"


# ---------------------------------------------------------------- split-K (cluster DSMEM reduction)
@pytest.mark.parametrize("split_k", [2, 3, 4, 8])
@pytest.mark.parametrize("epilogue", ["none", "bias_residual", "bias_gelu_tanh", "swiglu"])
def test_split_k_epilogues(cuda_device, split_k, epilogue):
    run_and_check(256, 384, 2048, torch.float16, epilogue, split_k=split_k, tile_n=128, seed=40 + split_k)


@pytest.mark.parametrize("shape", [(512, 384, 3072), (200, 300, 1000), (130, 520, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("tile_n", [64, 96, 128, 192, 256])
def test_split_k_shapes(cuda_device, shape, tile_n):
    """K tails (2-D maps, one block per load), M/N tails, every tile width."""
    M, N, K = shape
    run_and_check(M, N, K, torch.bfloat16, "bias", split_k=3, tile_n=tile_n, seed=41)


def test_split_k_int8_exact(cuda_device):
    q = hx()
    g = torch.Generator().manual_seed(42)
    a = torch.randint(-127, 128, (256, 4096), generator=g, dtype=torch.int64).to(torch.int8)
    w = torch.randint(-127, 128, (512, 4096), generator=g, dtype=torch.int64).to(torch.int8)
    out = q.gemm(a.cuda(), w.cuda(), split_k=4, tile_n=256)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.int8_gemm_exact(a.numpy(), w.numpy()))


def test_split_k_rejects_oversubscription(cuda_device):
    q = hx()
    a, w, _, _ = make_inputs(4096, 4096, 256, torch.float16)
    with pytest.raises(q._lib.HexagonB200Error):
        q.gemm(a, w, split_k=8)  # 1024 tiles x 8 CTAs cannot be resident


# ---------------------------------------------------------------- CTA pairs (cta_group::2)
@pytest.fixture
def force_pairs():
    os.environ["HX_GEMM_PAIR"] = "1"
    yield
    del os.environ["HX_GEMM_PAIR"]


@pytest.mark.parametrize("epilogue", ["none", "bias", "bias_gelu_tanh", "bias_residual", "swiglu"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_pair_tiles(cuda_device, force_pairs, epilogue, dtype):
    run_and_check(640, 768, 512, dtype, epilogue, seed=50)


@pytest.mark.parametrize("shape", [(256, 256, 64), (300, 520, 192), (1024, 1000, 1024), (129, 2048, 128)],
                         ids=lambda s: "x".join(map(str, s)))
def test_pair_tile_shapes(cuda_device, force_pairs, shape):
    run_and_check(*shape, torch.bfloat16, "bias", seed=51)


def test_pair_int8_exact(cuda_device, force_pairs):
    q = hx()
    g = torch.Generator().manual_seed(52)
    a = torch.randint(-127, 128, (600, 1024), generator=g, dtype=torch.int64).to(torch.int8)
    w = torch.randint(-127, 128, (520, 1024), generator=g, dtype=torch.int64).to(torch.int8)
    out = q.gemm(a.cuda(), w.cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.int8_gemm_exact(a.numpy(), w.numpy()))


def test_pair_default_for_large_gemm(cuda_device):
    """A GEMM with a full wave of 256x256 tiles takes the pair kernel by default."""
    run_and_check(4096, 4096, 1024, torch.bfloat16, "none", seed=53)


# ---------------------------------------------------------------- constant-B prefetch
@pytest.mark.parametrize("tile_n", [64, 128, 192, 256])
def test_b_const_back_to_back(cuda_device, tile_n):
    """HX_GEMM_B_CONST: the weights of a GEMM are fetched before the previous
    kernel in the stream ends; its A (the previous GEMM's output) must still
    be read only after that kernel completes."""
    q = hx()
    g = torch.Generator().manual_seed(60 + tile_n)
    x = torch.randn(512, 768, generator=g).half()
    w1 = (torch.randn(1024, 768, generator=g) * 0.02).half()
    w2 = (torch.randn(768, 1024, generator=g) * 0.02).half()
    b1 = torch.randn(1024, generator=g).half()
    xd, w1d, w2d, b1d = x.cuda(), w1.cuda(), w2.cuda(), b1.cuda()
    for _ in range(3):
        y1 = q.gemm(xd, w1d, epilogue="bias_gelu_tanh", bias=b1d, b_const=True, tile_n=tile_n)
        y2 = q.gemm(y1, w2d, epilogue="residual", residual=xd, b_const=True)
    torch.cuda.synchronize()
    r1 = O.linear_ref(to_np32(x), to_np32(w1), epilogue="bias_gelu_tanh", bias=to_np32(b1))
    assert_close(to_np32(y1), r1)
    r2 = O.linear_ref(to_np32(y1), to_np32(w2), epilogue="residual", residual=to_np32(x))
    assert_close(to_np32(y2), r2)


def test_unknown_flags_rejected(cuda_device):
    import ctypes
    from qcom_hexagon_backend import _lib
    q = hx()
    a = torch.randn(64, 64, device="cuda").half()
    d, out, dev = q.ops.make_desc(a, torch.randn(64, 64, device="cuda").half())
    d.flags = 0x40
    rc = _lib.load().hx_gemm(ctypes.byref(d), None)
    assert rc == _lib.HX_E_INVALID_ARG
