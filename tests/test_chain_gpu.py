"""GPU parity of hx_gemm_chain (a stack of fused linears as one persistent
launch with row-block dependencies) against the CPU oracle and against the
same stack launched GEMM by GEMM."""

import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy()


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def gpt2_oracle(model, x):
    """Layer-by-layer fp32 oracle with fp16 rounding of every stored
    intermediate, as the GPU stores them."""
    h = _np(x)
    for b in model.blocks:
        W = lambda lin: _np(lin.weight)
        B = lambda lin: _np(lin.bias)
        qkv = _f16(O.linear_ref(h, W(b.c_attn), epilogue="bias", bias=B(b.c_attn)))
        a = _f16(O.linear_ref(qkv[:, : b.hidden], W(b.attn_proj), epilogue="bias_residual",
                              bias=B(b.attn_proj), residual=h))
        u = _f16(O.linear_ref(a, W(b.c_fc), epilogue="bias_gelu_tanh", bias=B(b.c_fc)))
        h = _f16(O.linear_ref(u, W(b.mlp_proj), epilogue="bias_residual", bias=B(b.mlp_proj), residual=a))
    return h


@pytest.mark.parametrize("layers,hidden,M", [(2, 256, 384), (3, 768, 1024)])
def test_gpt2_stack_chain_matches_oracle_and_unchained(cuda_device, layers, hidden, M):
    from qcom_hexagon_backend import workloads as WL
    from qcom_hexagon_backend.backend import HexagonOptions, TorchMLIRHexagonLauncher

    model = WL.GPT2LinearStack(layers=layers, hidden=hidden).half()
    x = torch.randn(M, hidden, generator=torch.Generator().manual_seed(3)).half()
    lc = TorchMLIRHexagonLauncher()
    y_chain = lc.run_torch_mlir(model, [x], "stack", options=HexagonOptions(chain_gemms=True))[0]
    y_plain = lc.run_torch_mlir(model, [x], "stack", options=HexagonOptions(chain_gemms=False))[0]
    ref = gpt2_oracle(model, x)
    assert O.max_rel_err(_np(y_chain), ref) <= 1e-2
    assert O.max_rel_err(_np(y_chain), _np(y_plain)) <= 1e-2
    # replay the captured graph again: counters are re-zeroed every launch
    y2 = lc.run_torch_mlir(model, [x], "stack", options=HexagonOptions(chain_gemms=True))[0]
    assert torch.equal(y2, y_chain)


def test_qwen_stack_chain(cuda_device):
    from qcom_hexagon_backend import workloads as WL
    from qcom_hexagon_backend.backend import HexagonOptions, TorchMLIRHexagonLauncher

    model = WL.QwenLinearStack(layers=3, hidden=256, inter=640, kv=64).to(torch.bfloat16)
    x = torch.randn(300, 256, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    lc = TorchMLIRHexagonLauncher()
    y_chain = lc.run_torch_mlir(model, [x], "q", options=HexagonOptions(chain_gemms=True))[0]
    y_plain = lc.run_torch_mlir(model, [x], "q", options=HexagonOptions(chain_gemms=False, use_cuda_graph=False))[0]
    with torch.no_grad():
        ref = model.float()(x.float())
    assert O.max_rel_err(_np(y_chain), _np(ref)) <= 2e-2
    assert O.max_rel_err(_np(y_chain), _np(y_plain)) <= 1e-2


def test_chained_ops_direct(cuda_device):
    """ops.chained(): slice-view dependency, residual dependency, 70 GEMMs
    (more than one launch), an ineligible call in the middle."""
    import qcom_hexagon_backend as q

    g = torch.Generator().manual_seed(5)
    d = cuda_device
    x = torch.randn(256, 128, generator=g).half().to(d)
    ws = [(torch.randn(384, 128, generator=g) * 0.05).half().to(d) for _ in range(35)]
    vs = [(torch.randn(128, 128, generator=g) * 0.05).half().to(d) for _ in range(35)]

    def run():
        h = x
        for w, v in zip(ws, vs):
            t = q.linear(h, w)                       # [256, 384]
            h = q.linear(t[:, 128:256], v, residual=h)
        return h

    ref = run()  # eager, GEMM by GEMM
    with q.ops.chained(d):
        out = run()
    torch.cuda.synchronize()
    assert O.max_rel_err(_np(out), _np(ref)) <= 1e-2
