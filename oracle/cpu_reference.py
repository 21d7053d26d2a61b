"""The reference's CPU path for each benchmark workload, timed on the host
cores — TEST / BENCHMARK INFRASTRUCTURE ONLY (bench.py's CPU-baseline and
`--impl reference` legs).

The reference checks every matmul against PyTorch on the host CPU
(test/python/triton/test_matmul.py:90 `torch.matmul`,
test/python/torch-mlir/utils.py:54 the model's PyTorch forward,
benchmark_models/run_gpt2lmheadmodel.py:17-19 x86 logits).  With no
Hexagon SDK/simulator available offline, that CPU golden is the reference's
only runnable implementation of this path, so it is what the CPU legs time:
PyTorch-CPU F.linear + epilogue in the workload's dtype (the same nn.Module
the GPU path compiles), dequantise + fp32 F.linear for W8A16.

Each measurement is a bounded sample (whole layers, or a block of LM-head
rows) scaled to the workload's metric; the sample is described in the
result.
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F

from qcom_hexagon_backend import workloads as WL  # plain nn.Module definitions only


def _timeit(fn, reps):
    fn()  # warm-up
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    ts.sort()
    return ts[len(ts) // 2]


def _gpt2(budget_s):
    model = WL.GPT2LinearStack().half()
    g = torch.Generator().manual_seed(1234)
    x = torch.randn(1024, 768, generator=g).half()
    blk = model.blocks[0]
    with torch.no_grad():
        t1 = _timeit(lambda: blk(x), 2)
        layers = max(1, min(12, int(budget_s / 6 / max(t1, 1e-6))))
        sub = torch.nn.Sequential(*model.blocks[:layers])
        t = _timeit(lambda: sub(x), 5)
    flops = WL.gpt2_stack_flops(layers=layers)
    return dict(metric="GEMM+epilogue TFLOP/s", unit="TFLOP/s", dtype="fp16",
                value=round(flops / t / 1e12, 4), ms_per_step=round(t * 1e3 * 12 / layers, 3),
                sample=f"PyTorch-CPU fp16 forward of {layers} of 12 GPT-2 linear layers "
                       f"(M=1024), median of 5, scaled per layer",
                config={"workload": "gpt2-small linear stack (BASELINE config 2)", "layers_timed": layers})


def _qwen(budget_s):
    model = WL.QwenLinearStack().to(torch.bfloat16)
    g = torch.Generator().manual_seed(1235)
    x = torch.randn(2048, 896, generator=g).to(torch.bfloat16)
    blk = model.blocks[0]
    acc = x.new_zeros(2048, blk.qkv.out_features)
    with torch.no_grad():
        t = _timeit(lambda: blk(x, acc), 5)
    flops = WL.qwen_stack_flops(layers=1)
    return dict(metric="GEMM+epilogue TFLOP/s", unit="TFLOP/s", dtype="bf16",
                value=round(flops / t / 1e12, 4), ms_per_step=round(t * 1e3 * 24, 3),
                sample="PyTorch-CPU bf16 forward of 1 of 24 Qwen2.5-0.5B linear layers (M=2048), median of 5",
                config={"workload": "qwen2.5-0.5b prefill linear stack (BASELINE config 3)", "layers_timed": 1})


def _tinyllama(budget_s, M=1):
    layers = WL.make_tinyllama_w8a16(layers=1)
    g = torch.Generator().manual_seed(1237)
    x = torch.randn(M, 2048, generator=g).half()
    xi = torch.randn(M, 5632, generator=g).half()

    def step():
        for p in WL.TINYLLAMA_PROJ:
            l = layers[0][p]
            wd = l.weight.float() * l.scale.float()[:, None]
            F.linear((xi if p == "down" else x).float(), wd).half()

    t = _timeit(step, 5)
    nbytes = WL.tinyllama_decode_bytes(M, layers=1)
    return dict(metric="W8A16 decode HBM GB/s", unit="GB/s", dtype="int8 x f16 (f32 acc)",
                value=round(nbytes / t / 1e9, 3), ms_per_step=round(t * 1e3 * 22, 3),
                sample=f"PyTorch-CPU dequantise + fp32 F.linear, 1 of 22 TinyLlama layers, M={M}, median of 5",
                config={"workload": f"tinyllama-1.1b decode linears W8A16 M={M} (BASELINE config 4)"})


_LM_CACHE = {}


def _lm_inputs(int8, rows):
    """Seeded LM-head operands (the GPU arm's seed and distributions), built once."""
    key = (int8, rows)
    if key not in _LM_CACHE:
        g = torch.Generator().manual_seed(1238)
        if int8:
            a = torch.randint(-127, 128, (rows, WL.LMHEAD_K), generator=g, dtype=torch.int8)
            w = torch.randint(-127, 128, (WL.LMHEAD_N, WL.LMHEAD_K), generator=g, dtype=torch.int8)
        else:
            a = torch.randn(rows, WL.LMHEAD_K, generator=g).to(torch.bfloat16)
            w = (torch.randn(WL.LMHEAD_N, WL.LMHEAD_K, generator=g) * 0.02).to(torch.bfloat16)
        _LM_CACHE[key] = (a, w)
    return _LM_CACHE[key]


def _lmhead(budget_s, int8=False):
    rows = 256
    a, w = _lm_inputs(int8, rows)
    with torch.no_grad():
        if int8:
            # no int8 GEMM in PyTorch-CPU: exact int32 result through fp64 (|acc| < 2^53)
            wd = w.double()
            t = _timeit(lambda: F.linear(a.double(), wd).to(torch.int32), 3)
        else:
            t = _timeit(lambda: F.linear(a, w), 3)
    flops = 2.0 * rows * WL.LMHEAD_K * WL.LMHEAD_N
    full = t * WL.LMHEAD_M / rows
    dt = "int8 (int32 acc)" if int8 else "bf16"
    return dict(metric="GEMM+epilogue TFLOP/s", unit="TOP/s" if int8 else "TFLOP/s", dtype="int8" if int8 else "bf16",
                value=round(flops / t / 1e12, 4), ms_per_step=round(full * 1e3, 3), scaling="strong",
                sample=f"PyTorch-CPU {dt} F.linear on {rows} of 16384 LM-head rows, median of 3, scaled",
                config={"workload": f"LM head 16384x2048x50304 {dt}, column-sharded (BASELINE config 5)"})


def _attn(budget_s):
    B, H, S, D = 1, 12, 1024, 64  # one of the GPU arm's 8 sequences, scaled
    g = torch.Generator().manual_seed(1240)
    q, k, v = (torch.randn(B, H, S, D, generator=g).half() for _ in range(3))
    with torch.no_grad():
        t = _timeit(lambda: torch.matmul(torch.matmul(q, k.transpose(-1, -2)), v), 3)
    flops = 2 * (2.0 * B * H * S * S * D)
    return dict(metric="batched GEMM TFLOP/s", unit="TFLOP/s", dtype="fp16", value=round(flops / t / 1e12, 4),
                ms_per_step=round(t * 1e3 * 8, 3),
                sample="PyTorch-CPU fp16 q@k^T and p@v for 1 of 8 sequences (12 heads x 1024 x 64), median of 3",
                config={"workload": "GPT-2 attention batched GEMMs (q@k^T, p@v), fp16"})


def _conv(budget_s):
    g = torch.Generator().manual_seed(1240)
    x = torch.randn(1, 256, 64, 64, generator=g).half()  # 1 of the GPU arm's 8 images
    w = (torch.randn(256, 256, 3, 3, generator=g) * 0.02).half()
    with torch.no_grad():
        t = _timeit(lambda: F.conv2d(x, w, padding=1), 3)
    flops = 2.0 * 64 * 64 * 256 * 9 * 256
    return dict(metric="conv TFLOP/s", unit="TFLOP/s", dtype="fp16", value=round(flops / t / 1e12, 4),
                ms_per_step=round(t * 1e3 * 8, 3),
                sample="PyTorch-CPU fp16 F.conv2d 3x3 256->256 on 1 of 8 64x64 images, median of 3",
                config={"workload": "3x3 conv NHWC fp16 as implicit GEMM"})


def _softmax(budget_s):
    rows = 512
    g = torch.Generator().manual_seed(1240)
    x = (torch.randn(rows, WL.LMHEAD_N, generator=g) * 2).to(torch.bfloat16)
    t = _timeit(lambda: torch.softmax(x, -1), 3)
    nbytes = 2.0 * 2 * rows * WL.LMHEAD_N
    return dict(metric="softmax HBM GB/s", unit="GB/s", dtype="bf16", value=round(nbytes / t / 1e9, 3),
                ms_per_step=round(t * 1e3 * WL.LMHEAD_M / rows, 3),
                sample=f"PyTorch-CPU bf16 softmax of {rows} of 16384 vocabulary rows, median of 3, scaled",
                config={"workload": "LM-head vocabulary softmax, bf16 in place"})


def _cube(budget_s):
    g = torch.Generator().manual_seed(1240)
    a = torch.randn(1024, 1024, generator=g).half()
    b = torch.randn(1024, 1024, generator=g).half()
    t = _timeit(lambda: torch.matmul(a, b), 5)
    return dict(metric="GEMM TFLOP/s", unit="TFLOP/s", dtype="fp16", value=round(2.0 * 1024 ** 3 / t / 1e12, 4),
                ms_per_step=round(t * 1e3, 3), sample="PyTorch-CPU fp16 torch.matmul 1024^3, median of 5",
                config={"workload": "fp16 1024^3 matmul (BASELINE config 1)"})


_TABLE = {"cube": _cube, "attn": _attn, "conv": _conv, "softmax": _softmax, "gpt2": _gpt2, "qwen": _qwen, "tinyllama": _tinyllama, "lmhead": _lmhead,
          "lmhead_int8": lambda b: _lmhead(b, int8=True)}


def time_workload(workload, budget_s=15.0, threads=1):
    r = _TABLE[workload](budget_s)
    return r["value"], r["unit"], r["sample"], threads


def run_steps(workload, steps, warmup, threads, budget_s=15.0):
    """`--impl reference`: the bounded CPU sample, measured once per step."""
    vals = []
    last = None
    per = max(2.0, budget_s / max(1, steps + warmup))
    for i in range(steps + warmup):
        last = _TABLE[workload](per)
        if i >= warmup:
            vals.append(last["value"])
    last["value"] = round(sorted(vals)[len(vals) // 2], 4)
    last["sample"] += f"; {steps} steps after {warmup} warm-up, median"
    return last
