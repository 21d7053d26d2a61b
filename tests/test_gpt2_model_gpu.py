"""End-to-end model parity: a random-init HF GPT2LMHeadModel (GPT2Config(),
12 layers, fp16) through the reference's compile/run surface
(TorchMLIRHexagonLauncher.run_torch_mlir with HexagonOptions().__dict__),
every linear on the B200 kernels, against the same model run by PyTorch on
the CPU.

The comparison restates compare() of
benchmark_models/run_gpt2lmheadmodel.py:54-68: the top-5 tokens of the last
row's logits must be equal and their values within atol 0.03.  The CPU side
runs in fp32 (the oracle's precision); the reference compares against the
fp16 CPU forward.  No pretrained weights or tokenizer exist offline, so the
weights are random (seeded) and the prompt is 8 seeded token ids.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _top5(logits):
    v, i = torch.topk(logits[0, -1, :].float(), 5)
    return i.tolist(), v


@pytest.mark.parametrize("n_layer", [2, 12])
def test_gpt2lmheadmodel_top5(cuda_device, n_layer):
    transformers = pytest.importorskip("transformers")
    from qcom_hexagon_backend import fx_backend as FX
    from qcom_hexagon_backend.backend import HexagonOptions, TorchMLIRHexagonLauncher

    cfg = transformers.GPT2Config()
    cfg.n_layer = n_layer
    cfg.use_cache = False
    torch.manual_seed(1234)
    model = transformers.GPT2LMHeadModel(cfg).eval()
    ids = torch.randint(0, cfg.vocab_size, (1, 8), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        x86 = model(ids).logits
    model16 = model.half()
    launcher = TorchMLIRHexagonLauncher()
    opts = HexagonOptions().__dict__
    outs = launcher.run_torch_mlir(model16, [ids], "GPT2LMHeadModel", options=opts)
    cg = launcher.compile_torch_mlir(model16, [ids], "GPT2LMHeadModel", opts)
    assert cg.n_hx_calls == 4 * n_layer + 1  # every Conv1D addmm and the LM head
    hexl = outs[0]
    assert hexl.shape == (1, 8, cfg.vocab_size)
    t_hex, c_hex = _top5(hexl)
    t_x86, c_x86 = _top5(x86)
    assert t_hex == t_x86, (t_hex, t_x86)
    assert torch.allclose(c_hex, c_x86, atol=0.03), (c_hex, c_x86)
    # and the whole logits tensor, normwise
    err = (hexl.float() - x86).abs().max() / x86.abs().max()
    assert err <= 2e-2, float(err)
    # the rewritten graph really calls the kernels
    assert FX.count_hx_calls(cg.gm) == 4 * n_layer + 1
