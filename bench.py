"""Benchmark of the B200 linear-layer GEMM path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl hx|reference]
                    [--workload lmhead|gpt2|qwen|tinyllama|attn|conv|softmax] [--lm-dtype bf16|int8]

Default workload, at every N (the configuration the headline metric is
quoted on at 1/2/4/8 GPUs): the LM-head GEMM, bf16, M=16384 tokens x
K=2048 x N=50304, weights N(0,0.02), activations N(0,1), column-sharded
over the N ranks.  A "step" is one pass of the sharded GEMM; at N > 1 it
includes the all-gather of the logits onto every rank (by default the GEMM
runs in row chunks and each finished chunk is DMA-copied over NVLink into
every peer's buffer while the next chunk computes; --gather p2p fuses the
transfer into the GEMM's epilogue stores instead, --gather nccl uses NCCL).  value = 2*M*N*K / step
time (max over ranks), strong scaling.  The inputs (1.9 GB) exceed the
126 MB L2, so no flush is needed between steps.

The other workloads are BASELINE's configs 2-4: the GPT-2-small and
Qwen2.5-0.5B linear stacks (CUDA-graph replays of the FX-compiled module,
256 MB L2 flush before each step, replicas at N > 1) and the TinyLlama
W8A16 decode step (one grouped persistent launch).

--impl reference runs the reference's own CPU path for the same workload
(PyTorch-CPU F.linear + epilogue in the config dtype, the golden every
reference test compares against) on rank 0 with all host threads.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hexagon-mlir_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from qcom_hexagon_backend import workloads as WL  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return FALLBACK_PEAKS, "fallback"


def read_traffic(name):
    """Per-launch DRAM bytes recorded from an ncu capture (profiles/<name>), or None."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi during the timed region (SM clock + throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()
        t0 = time.time()
        while not self.lines and time.time() - t0 < 5.0:  # first sample before the timed region
            time.sleep(0.02)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- dist
CHAIN = False  # --chain


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo")
    if world != n_gpus and rank == 0:
        print(f"warning: --gpus {n_gpus} but WORLD_SIZE {world}", file=sys.stderr)
    return world, rank, local


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world, dev):
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize(dev)


# ---------------------------------------------------------------- CPU baseline
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference_time(workload, budget_s=15.0):
    """Reference's CPU golden path, bounded sample.  Returns (value, unit, sample, cores)."""
    from oracle import cpu_reference as CR

    n = cpu_threads()
    torch.set_num_threads(n)
    return CR.time_workload(workload, budget_s=budget_s, threads=n)


# ---------------------------------------------------------------- workloads
def build_gpt2(dev, seed=1234):
    from qcom_hexagon_backend.backend import HexagonOptions, TorchMLIRHexagonLauncher

    model = WL.GPT2LinearStack().half()
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1024, 768, generator=g).half()
    launcher = TorchMLIRHexagonLauncher()
    options = HexagonOptions(device=dev.index, chain_gemms=CHAIN)
    cg = launcher.compile_torch_mlir(model, [x], "gpt2_linear_stack", options)
    flops = WL.gpt2_stack_flops()
    return dict(launcher=launcher, model=model, cg=cg, x=x, options=options, flops=flops, launches=cg.n_hx_calls,
                metric="GEMM+epilogue TFLOP/s", unit="TFLOP/s", dtype="fp16",
                config={"workload": "gpt2-small linear stack (BASELINE config 2)", "model": "gpt2-small-linears",
                        "layers": 12, "global_batch": 1, "seq_len": 1024, "hidden": 768,
                        "gemms_per_step": cg.n_hx_calls, "flops_per_step": flops},
                traffic_file="gemm_gpt2_stack.txt", func="gpt2_linear_stack")


def build_qwen(dev, seed=1235):
    from qcom_hexagon_backend.backend import HexagonOptions, TorchMLIRHexagonLauncher

    model = WL.QwenLinearStack().to(torch.bfloat16)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2048, 896, generator=g).to(torch.bfloat16)
    launcher = TorchMLIRHexagonLauncher()
    options = HexagonOptions(device=dev.index, chain_gemms=CHAIN)
    cg = launcher.compile_torch_mlir(model, [x], "qwen_linear_stack", options)
    flops = WL.qwen_stack_flops()
    return dict(launcher=launcher, model=model, cg=cg, x=x, options=options, flops=flops, launches=cg.n_hx_calls,
                metric="GEMM+epilogue TFLOP/s", unit="TFLOP/s", dtype="bf16",
                config={"workload": "qwen2.5-0.5b prefill linear stack (BASELINE config 3)",
                        "model": "qwen2.5-0.5b-linears", "layers": 24, "global_batch": 1, "seq_len": 2048,
                        "gemms_per_step": cg.n_hx_calls, "flops_per_step": flops},
                traffic_file="gemm_qwen_stack.txt", func="qwen_linear_stack")


def time_graph_steps(cg, steps, flush, dev):
    """Per-step CUDA-event times (ms) of graph replays, L2 flushed before each."""
    stream = torch.cuda.current_stream(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s, e in evs:
        flush.zero_()
        s.record(stream)
        cg.launch()
        e.record(stream)
    torch.cuda.synchronize(dev)
    return [s.elapsed_time(e) for s, e in evs]


def run_hx(args):
    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks, peak_src = load_peaks()
    if args.workload in ("lmhead",):
        return run_lmhead(args, world, rank, dev, peaks, peak_src)
    if args.workload == "tinyllama":
        return run_tinyllama(args, world, rank, dev, peaks, peak_src)
    if args.workload in ("attn", "conv", "softmax", "cube"):
        return run_kernel_bench(args, world, rank, dev, peaks, peak_src)
    W = build_gpt2(dev) if args.workload == "gpt2" else build_qwen(dev)
    cg = W["cg"]
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        flush.zero_()
        cg.launch()
    barrier(world, dev)
    clk = ClockSampler(local)
    clk.start()
    barrier(world, dev)
    step_ms = time_graph_steps(cg, args.steps, flush, dev)
    barrier(world, dev)
    clocks = clk.stop()
    total_ms = max_over_ranks(sum(step_ms), world, dev)
    ms_per_step = total_ms / args.steps
    value = W["flops"] * world / (total_ms / args.steps / 1e3) / 1e12

    # e2e: the reference-facing call with host buffers (pinned), H2D + graph + D2H
    launcher = W["launcher"]
    x_host = W["x"].pin_memory()
    out_host = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in cg.static_out]
    for _ in range(2):
        launcher.run_torch_mlir(W["model"], [x_host], W["func"], options=W["options"], outputs=out_host)
    barrier(world, dev)
    stream = torch.cuda.current_stream(dev)
    e2e_ms = []
    for _ in range(args.steps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        launcher.run_torch_mlir(W["model"], [x_host], W["func"], options=W["options"], outputs=out_host)
        e.record(stream)
        e.synchronize()
        e2e_ms.append(s.elapsed_time(e))
    e2e_total = max_over_ranks(sum(e2e_ms), world, dev)
    e2e_value = W["flops"] * world / (e2e_total / args.steps / 1e3) / 1e12
    h2d = x_host.numel() * x_host.element_size()
    d2h = sum(o.numel() * o.element_size() for o in out_host)

    # The timed region is the captured graph's GEMM launches back to back
    # (the L2 flush sits outside the events), so the kernel's average launch
    # duration is this rank's step time over its launches per step.
    my_ms_per_step = sum(step_ms) / args.steps
    per_launch_ms = my_ms_per_step / W["launches"]
    achieved = W["flops"] / (my_ms_per_step / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    traffic = read_traffic(W["traffic_file"])

    line = {
        "metric": W["metric"], "value": round(value, 2), "unit": W["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": W["dtype"],
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) random-init weights)",
        "config": dict(W["config"], parallelism=f"replicas{world}",
                       l2="flushed (256 MB write) before every timed step"),
        "e2e": {"value": round(e2e_value, 2), "unit": W["unit"], "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "TorchMLIRHexagonLauncher.run_torch_mlir (pinned host in/out)"},
        "gpu_launches": W["launches"] * args.steps,
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "hx_gemm_sm100_kernel", "per_launch_ms": round(per_launch_ms, 5),
                     "peak_source": f"{peak_src} bf16_tflops (burst; fp16 dense peak equals bf16)"},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, unit, sample, cores = cpu_reference_time(args.workload, budget_s=args.cpu_budget)
        line["cpu_baseline"] = {"value": v, "unit": unit, "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_tinyllama(args, world, rank, dev, peaks, peak_src):
    """Config 4: W8A16 decode linears, 22 layers x 7 projections, M in {1,8,32,64}."""
    from qcom_hexagon_backend import ops

    layers = WL.make_tinyllama_w8a16(layers=args.layers)
    dl = [{p: (l[p].weight.to(dev), l[p].scale.to(dev)) for p in l} for l in layers]
    M = args.batch
    g = torch.Generator().manual_seed(1237)
    x = torch.randn(M, 2048, generator=g).half().to(dev)
    xi = torch.randn(M, 5632, generator=g).half().to(dev)
    outs = {p: torch.empty(M, WL.tinyllama_shapes()[p][0], dtype=torch.float16, device=dev)
            for p in WL.TINYLLAMA_PROJ}

    # One persistent grouped launch per decode step (154 projections); each
    # projection writes its own output buffer.
    grp = ops.W8A16Group(M, dev)
    ys = []
    for l in dl:
        for p in WL.TINYLLAMA_PROJ:
            w, s = l[p]
            y = torch.empty(M, w.shape[0], dtype=torch.float16, device=dev)
            ys.append(y)
            grp.add(xi if p == "down" else x, w, s, y)

    def step():
        grp.run()

    step()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        graph.replay()
    barrier(world, dev)
    clk = ClockSampler(dev.index)
    clk.start()
    stream = torch.cuda.current_stream(dev)
    evs = []
    for _ in range(args.steps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        graph.replay()
        e.record(stream)
        evs.append((s, e))
    barrier(world, dev)
    clocks = clk.stop()
    total = max_over_ranks(sum(s.elapsed_time(e) for s, e in evs), world, dev)
    ms = total / args.steps
    nbytes = WL.tinyllama_decode_bytes(M, layers=args.layers)
    gbs = nbytes / (ms / 1e3) / 1e9

    # End to end through the public W8A16Group API: this step's activations
    # from pinned host memory, the launch, and the last projection's output
    # read back to the host.
    x_host, xi_host = x.cpu().pin_memory(), xi.cpu().pin_memory()
    y_host = torch.empty(ys[-1].shape, dtype=ys[-1].dtype).pin_memory()
    e2e_ms = []
    for _ in range(args.steps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        x.copy_(x_host, non_blocking=True)
        xi.copy_(xi_host, non_blocking=True)
        grp.run()
        y_host.copy_(ys[-1], non_blocking=True)
        e.record(stream)
        e.synchronize()
        e2e_ms.append(s.elapsed_time(e))
    e2e_total = max_over_ranks(sum(e2e_ms), world, dev)
    e2e_gbs = nbytes / (e2e_total / args.steps / 1e3) / 1e9
    kernel = ("hx_gemv_w8a16_grouped_mma_kernel" if M <= 16 else "hx_gemv_w8a16_grouped_tc_kernel")
    peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    line = {"metric": "W8A16 decode HBM GB/s", "value": round(gbs * world, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x f16 (f32 acc)", "data": "synthetic",
            "config": {"workload": f"tinyllama-1.1b decode linears W8A16 M={M} (BASELINE config 4)",
                       "layers": args.layers, "M": M, "bytes_per_step": nbytes, "l2": "flushed before every step",
                       "parallelism": f"replicas{world}"},
            "e2e": {"value": round(e2e_gbs * world, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": x_host.numel() * 2 + xi_host.numel() * 2,
                    "d2h_bytes_per_step": y_host.numel() * 2,
                    "api": "ops.W8A16Group.run (pinned host activations in, last output out)"},
            "gpu_launches": args.steps,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4),
                         "traffic": read_traffic("gemv_w8a16_decode.txt") if M <= 16 else None,
                         "kernel": kernel,
                         "peak_source": f"{peak_src} hbm_gbs"},
            "clocks": clocks}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_lmhead(args, world, rank, dev, peaks, peak_src):
    """Config 5: LM head M=16384 x K=2048 x N=50304, bf16 (or int8 W8A8 with int32
    accumulate, --lm-dtype int8), column-sharded over the ranks.  At N > 1 every step
    also all-gathers the logits into [world, M, N/world] on every rank: by default
    (--gather ce) the GEMM runs in row chunks and each finished chunk is copied by the
    copy engines into every peer's buffer (hx_sharded_gemm_gather_ce); --gather p2p is
    one fused launch whose epilogue stores into the peers (hx_sharded_gemm_gather_p2p);
    --gather nccl runs the GEMM in M chunks with chunk c's NCCL all-gather on a side
    stream overlapping chunk c+1.
    gemm_only reports the sharded GEMM alone."""
    from qcom_hexagon_backend import ops
    from qcom_hexagon_backend.sharding import shard_range, shard_width

    M, K, N = WL.LMHEAD_M, WL.LMHEAD_K, WL.LMHEAD_N
    if args.lm_rows:
        M = args.lm_rows
    int8 = args.lm_dtype == "int8"
    ns = shard_width(N, world)
    n0, n1 = shard_range(N, world, rank)
    g = torch.Generator().manual_seed(1238)
    if int8:
        a_cpu = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)[n0:n1]
    else:
        a_cpu = torch.randn(M, K, generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g)[n0:n1] * 0.02).to(torch.bfloat16)
    if w.shape[0] < ns:  # the short last shard: zero rows, equal gather sizes
        w = torch.cat([w, torch.zeros(ns - w.shape[0], K, dtype=w.dtype)], 0)
    a = a_cpu.to(dev)
    w = w.contiguous().to(dev)
    odt = torch.int32 if int8 else torch.bfloat16
    esz = 4 if int8 else 2
    out = torch.empty(M, ns, dtype=odt, device=dev)
    post_softmax = args.lm_post == "softmax"
    p2p = world > 1 and args.gather in ("p2p", "ce") and not post_softmax
    transfer = "copy_engine" if args.gather == "ce" else "epilogue"
    main = torch.cuda.current_stream(dev)

    def gemm_only():
        ops.gemm(a, w, out=out)

    pg = None
    if p2p:
        from qcom_hexagon_backend.sharding import P2PGather
        try:  # all ranks construct it or all raise (collective vote inside)
            pg = P2PGather(M, ns, odt, transfer=transfer, chunks=args.ce_chunks)
        except RuntimeError as ex:
            if rank == 0:
                print(f"{ex}; using NCCL", file=sys.stderr)
            p2p = False
    chunks = 4 if (world > 1 and not p2p and not post_softmax and M % 4 == 0) else 1
    mc = M // chunks
    nccl_gather = world > 1 and not p2p and not post_softmax
    gathered = torch.empty(chunks, world * mc, ns, dtype=odt, device=dev) if nccl_gather else None
    side = torch.cuda.Stream(dev) if nccl_gather else None
    evs_c = [torch.cuda.Event() for _ in range(chunks)]

    def step():
        if post_softmax:  # vocab-parallel softmax of the shards, in place: no logit gather
            from qcom_hexagon_backend.sharding import vocab_parallel_softmax
            gemm_only()
            vocab_parallel_softmax(out, n1 - n0, out=out)
            return
        if world == 1:
            return gemm_only()
        if p2p:  # one fused launch: the GEMM's epilogue writes every rank's buffer over NVLink
            pg.run(a, w)
            return
        for c in range(chunks):
            ops.gemm(a[c * mc:(c + 1) * mc], w, out=out[c * mc:(c + 1) * mc])
            evs_c[c].record(main)
            side.wait_event(evs_c[c])
            with torch.cuda.stream(side):
                dist.all_gather_into_tensor(gathered[c], out[c * mc:(c + 1) * mc])
        main.wait_stream(side)

    def local_shard():
        """This rank's [M, ns] logits after a step (its slot of the gather buffer)."""
        if p2p:
            return pg._local_view[rank]
        return out

    def timed(fn, steps):
        evs = []
        for _ in range(steps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(main)
            fn()
            e.record(main)
            evs.append((s, e))
        barrier(world, dev)
        return sum(s.elapsed_time(e) for s, e in evs)

    for _ in range(args.warmup):
        step()
    barrier(world, dev)
    clk = ClockSampler(dev.index)
    clk.start()
    local_ms = timed(step, args.steps)
    clocks = clk.stop()
    total = max_over_ranks(local_ms, world, dev)
    g_steps = max(3, args.steps // 4)
    gemm_ms = max_over_ranks(timed(gemm_only, g_steps), world, dev) / g_steps
    ms = total / args.steps
    flops = 2.0 * M * N * K
    tflops = flops / (ms / 1e3) / 1e12

    # e2e: host in, host out, every step.  A goes host->device from pinned
    # memory, the step runs (GEMM + gather at N > 1), and this rank's column
    # shard of the logits comes back device->host, so across ranks the full
    # logits are read back once per step.
    a_host = a_cpu.pin_memory()
    out_host = torch.empty(M, ns, dtype=odt, pin_memory=True)

    def e2e_step():
        a.copy_(a_host, non_blocking=True)
        step()
        out_host.copy_(local_shard(), non_blocking=True)

    e2e_step()
    barrier(world, dev)
    e2e_steps = max(3, min(args.steps, 20))
    e2e_ms = []
    for _ in range(e2e_steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(main)
        e2e_step()
        e.record(main)
        e.synchronize()
        e2e_ms.append(s.elapsed_time(e))
    e2e_total = max_over_ranks(sum(e2e_ms), world, dev)
    e2e_value = flops / (e2e_total / e2e_steps / 1e3) / 1e12
    h2d = a_host.numel() * a_host.element_size()
    d2h = out_host.numel() * out_host.element_size()

    # A timed region long enough to run into the 1 kW power cap (seconds of
    # back-to-back GEMMs) is measured against the sustained GEMM peak, a short
    # one against the burst peak.
    sustained = local_ms > 200.0 or "sw_power_cap" in (clocks or {}).get("reasons", [])
    peak_key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])) * (2.0 if int8 else 1.0)
    peak = float(peaks.get(peak_key, FALLBACK_PEAKS[peak_key])) * (2.0 if int8 else 1.0)
    unit = "TOP/s" if int8 else "TFLOP/s"
    dtname = "int8 (int32 acc)" if int8 else "bf16"
    my_flops = 2.0 * M * (n1 - n0) * K
    traffic = read_traffic("gemm_lmhead_int8.txt" if int8 else "gemm_lmhead.txt")
    if traffic is not None and args.lm_rows:
        traffic = None  # the recorded capture is of the full 16384-row launch
    if world == 1 or post_softmax:
        # one GEMM launch per step (plus the softmax kernels with --lm-post
        # softmax): the kernel's average duration is the timed step time
        per_launch = local_ms / args.steps
        achieved = my_flops / (per_launch / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": unit,
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "kernel": "hx_gemm_sm100_2sm_kernel", "per_launch_ms": round(per_launch, 5),
                "frac_of_burst": round(achieved / burst, 4),
                "peak_source": f"{peak_src} {peak_key} "
                               + (f"(sustained: {local_ms:.0f} ms timed, clocks {clocks.get('reasons') if clocks else []})"
                                  if sustained else "(burst)")
                               + (" x2 (int8 dense rate)" if int8 else "")}
    else:
        # A fused compute+collective step: its target time is the slower of the
        # GEMM at the measured tensor peak and the bytes every rank must receive
        # over NVLink at the measured 770 GB/s peer-copy rate.
        recv = (world - 1) * M * ns * esz
        t_tensor = my_flops / (peak * 1e12) * 1e3
        t_link = recv / 770e9 * 1e3
        target = max(t_tensor, t_link)
        roof = {"bound": "nvlink" if t_link >= t_tensor else "tensor",
                "achieved": round(recv / (ms / 1e3) / 1e9, 1) if t_link >= t_tensor else
                round(my_flops / (ms / 1e3) / 1e12, 2),
                "peak": 770.0 if t_link >= t_tensor else peak,
                "unit": "GB/s" if t_link >= t_tensor else unit,
                "frac": round(target / ms, 4), "traffic": traffic if p2p else None,
                "target_ms": round(target, 4), "tensor_ms": round(t_tensor, 4), "nvlink_ms": round(t_link, 4),
                "kernel": ("hx_gemm_sm100_2sm_kernel (fused peer-store epilogue)" if transfer == "epilogue"
                           else "hx_gemm_sm100_2sm_kernel + copy-engine peer copies") if p2p
                else "hx_gemm_sm100_2sm_kernel + NCCL all-gather",
                "peak_source": f"{peak_src} {peak_key} and measured 770 GB/s NVLink peer copy per direction"}
    line = {"metric": "GEMM+epilogue TFLOP/s", "value": round(tflops, 2), "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8" if int8 else "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) random-init weights)",
            "config": {"workload": f"LM head {M}x2048x50304 {dtname}, column-sharded (BASELINE config 5)",
                       "M": M, "K": K, "N": N, "shard_cols": ns,
                       "post": ("vocab-parallel softmax of each rank's logit shard in place (stats all-gathered, "
                                "[M, 2] floats per rank); no logit gather") if post_softmax else "logit gather",
                       "parallelism": f"tp{world} (N-sharded"
                       + ((", logits all-gathered into [world, M, N/world] by the GEMM's own epilogue "
                           "stores over NVLink (fused, hx_sharded_gemm_gather_p2p))" if p2p and transfer == "epilogue" else
                           ", logits all-gathered into [world, M, N/world]: GEMM in row chunks, each chunk "
                           "DMA-copied to every peer over NVLink while the next computes (hx_sharded_gemm_gather_ce))"
                           if p2p else
                           ", logits all-gathered over NCCL into [world, M, N/world], overlapped in "
                           f"{chunks} M-chunks)") if world > 1 else ")"),
                       "l2": "inputs (1.9 GB/step at N=1) larger than L2; no flush"},
            "gemm_only": {"value": round(flops / (gemm_ms / 1e3) / 1e12, 2), "unit": unit,
                          "ms_per_step": round(gemm_ms, 4)},
            "e2e": {"value": round(e2e_value, 2), "unit": unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "api": (f"sharding.P2PGather(transfer={transfer!r}).run" if p2p else "ops.gemm" + (" + NCCL all-gather" if world > 1 else ""))
                    + " with A copied from pinned host memory and this rank's logits shard copied back"},
            "gpu_launches": args.steps * ((3 if transfer == "epilogue" else 2 + pg.last_chunks) if p2p else
                                          (4 if post_softmax else chunks)),
            "roofline": roof,
            "clocks": clocks}
    if world > 1 and not post_softmax:
        recv = (world - 1) * M * ns * esz
        line["gather"] = {"bytes_received_per_rank": recv,
                          "nvlink_gbs_per_rank": round(recv / (ms / 1e3) / 1e9, 1),
                          "gather_only_ms_est": round(max(0.0, ms - gemm_ms), 4),
                          "reference_peer_copy_gbs": 770.0}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, u, sample, cores = cpu_reference_time("lmhead_int8" if int8 else "lmhead", budget_s=args.cpu_budget)
        line["cpu_baseline"] = {"value": v, "unit": u, "cores": cores, "kind": "port", "sample": sample}
    if pg is not None:
        flag = int(pg.error_flag.item())
        if flag != 0:
            line["error"] = f"fused gather error flag {flag}"
        pg.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_kernel_bench(args, world, rank, dev, peaks, peak_src):
    """The rows beside the linear layer, each one step = one call on resident
    inputs, timed with CUDA events (256 MB L2 flush before each step):
      attn     batched GEMMs of GPT-2 attention, batch 8 x 12 heads x S 1024 x
               head 64, fp16: scores q @ k^T (k a transposed view) and context
               p @ v (hx_gemm_batched); HBM-bound on the 201 MB score matrix;
      conv     3x3 convolution, NHWC fp16, batch 8 x 64 x 64 x 256 -> 256,
               padding 1, as an implicit GEMM (hx_conv2d): tensor-bound;
      softmax  softmax over the 50304-wide vocabulary of the LM head's
               16384 rows, bf16 in place (hx_softmax): HBM-bound.
    Independent replicas at N > 1 (weak scaling)."""
    from qcom_hexagon_backend import ops

    g = torch.Generator().manual_seed(1240)
    wl = args.workload
    if wl == "cube":  # C = A.B, 1024^3 fp16, B[K,N], fp32 accumulate
        a_h = torch.randn(1024, 1024, generator=g).half()
        b_h = torch.randn(1024, 1024, generator=g).half()
        host_in = [a_h, b_h]
        a, b = a_h.to(dev), b_h.to(dev)
        c = torch.empty(1024, 1024, dtype=torch.float16, device=dev)

        def step():
            ops.matmul(a, b, out=c)

        outs = [c]
        work = 2.0 * 1024 ** 3
        nbytes = 2.0 * 3 * 1024 * 1024
        launches, bound, kern = 1, "tensor", "hx_gemm_sm100_kernel (B[K,N])"
        cfg = {"workload": "fp16 1024^3 matmul (BASELINE config 1)", "M": 1024, "N": 1024, "K": 1024}
        metric, unit = "GEMM TFLOP/s", "TFLOP/s"
    elif wl == "attn":
        B, Hh, S, D = 8, 12, 1024, 64
        q_h = torch.randn(B, Hh, S, D, generator=g).half()
        k_h = torch.randn(B, Hh, S, D, generator=g).half()
        v_h = torch.randn(B, Hh, S, D, generator=g).half()
        host_in = [q_h, k_h, v_h]
        q, k, v = (t.to(dev) for t in host_in)
        p = torch.empty(B, Hh, S, S, dtype=torch.float16, device=dev)
        ctx = torch.empty(B, Hh, S, D, dtype=torch.float16, device=dev)

        def step():
            ops.bmm(q.view(-1, S, D), k.view(-1, S, D), b_layout="nk", out=p.view(-1, S, S))
            ops.bmm(p.view(-1, S, S), v.view(-1, S, D), b_layout="kn", out=ctx.view(-1, S, D))

        outs = [ctx]
        work = 2 * (2.0 * B * Hh * S * S * D)
        nbytes = 2.0 * (4 * B * Hh * S * D + 2 * B * Hh * S * S)  # q,k,v,ctx + scores written and read
        launches, bound, kern = 2, "hbm", "hx_gemm_sm100_kernel (batched)"
        cfg = {"workload": "GPT-2 attention batched GEMMs (q@k^T, p@v), fp16", "batch": B, "heads": Hh,
               "seq_len": S, "head_dim": D}
        metric, unit = "batched GEMM TFLOP/s", "TFLOP/s"
    elif wl == "conv":
        N_, H, W, C, OC = 8, 64, 64, 256, 256
        x_h = torch.randn(N_, H, W, C, generator=g).half()
        w_h = (torch.randn(OC, 3, 3, C, generator=g) * 0.02).half()
        host_in = [x_h]
        x, w = x_h.to(dev), w_h.to(dev)
        y = torch.empty(N_, H, W, OC, dtype=torch.float16, device=dev)

        def step():
            ops.conv2d_nhwc(x, w, None, padding=1, out=y)

        outs = [y]
        work = 2.0 * N_ * H * W * OC * 9 * C
        nbytes = 2.0 * (x.numel() + w.numel() + y.numel())
        launches, bound, kern = 1, "tensor", "hx_gemm_sm100_kernel (implicit conv)"
        cfg = {"workload": "3x3 conv NHWC fp16 as implicit GEMM", "batch": N_, "H": H, "W": W, "C": C, "OC": OC}
        metric, unit = "conv TFLOP/s", "TFLOP/s"
    else:  # softmax
        M, N = WL.LMHEAD_M, WL.LMHEAD_N
        x_h = (torch.randn(M, N, generator=g) * 2).to(torch.bfloat16)
        host_in = [x_h]
        x = x_h.to(dev)

        def step():
            ops.softmax(x, out=x)

        outs = [x]
        nbytes = 2.0 * 2 * M * N
        work = nbytes
        launches, bound, kern = 1, "hbm", "softmax_rows_kernel"
        cfg = {"workload": "LM-head vocabulary softmax, bf16 in place", "M": M, "N": N}
        metric, unit = "softmax HBM GB/s", "GB/s"
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        step()
    barrier(world, dev)
    stream = torch.cuda.current_stream(dev)
    clk = ClockSampler(dev.index)
    clk.start()
    evs = []
    for _ in range(args.steps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step()
        e.record(stream)
        evs.append((s, e))
    barrier(world, dev)
    clocks = clk.stop()
    local_ms = sum(s.elapsed_time(e) for s, e in evs) / args.steps
    ms = max_over_ranks(local_ms, world, dev)
    if bound == "tensor":
        rate = work / (ms / 1e3) / 1e12
        achieved, peak, runit = work / (local_ms / 1e3) / 1e12, float(peaks.get("bf16_tflops", 1590.0)), "TFLOP/s"
    else:
        achieved, peak, runit = nbytes / (local_ms / 1e3) / 1e9, float(peaks.get("hbm_gbs", 6650.0)), "GB/s"
        rate = (work / (ms / 1e3) / 1e12) if unit == "TFLOP/s" else nbytes / (ms / 1e3) / 1e9
    # e2e: inputs from pinned host memory, the step, outputs back to pinned host memory
    pin_in = [t.pin_memory() for t in host_in]
    dev_in = {"attn": lambda: [q, k, v], "conv": lambda: [x], "softmax": lambda: [x], "cube": lambda: [a, b]}[wl]()
    pin_out = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs]
    e2e_ms = []
    for _ in range(max(3, min(args.steps, 10))):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for d_, h_ in zip(dev_in, pin_in):
            d_.copy_(h_, non_blocking=True)
        step()
        for h_, o_ in zip(pin_out, outs):
            h_.copy_(o_, non_blocking=True)
        e.record(stream)
        e.synchronize()
        e2e_ms.append(s.elapsed_time(e))
    e2e_t = max_over_ranks(sum(e2e_ms) / len(e2e_ms), world, dev)
    e2e_v = (work / (e2e_t / 1e3) / 1e12) if unit == "TFLOP/s" else nbytes / (e2e_t / 1e3) / 1e9
    line = {"metric": metric, "value": round(rate * world, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if wl == "softmax" else "fp16", "data": "synthetic (seeded N(0,1))",
            "config": dict(cfg, parallelism=f"replicas{world}", l2="flushed (256 MB write) before every timed step"),
            "e2e": {"value": round(e2e_v * world, 2), "unit": unit,
                    "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in pin_in),
                    "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in pin_out)},
            "gpu_launches": launches * args.steps,
            "roofline": {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": runit,
                         "frac": round(achieved / peak, 4),
                         "traffic": read_traffic({"attn": "batched_gpt2_attention.txt", "conv": "conv_3x3_implicit.txt",
                                                  "softmax": "softmax_lmhead_vocab.txt"}.get(wl, "")),
                         "kernel": kern, "algorithmic_bytes": nbytes,
                         "peak_source": f"{peak_src} " + ("bf16_tflops (burst)" if bound == "tensor" else "hbm_gbs")},
            "clocks": clocks}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_reference(args):
    """The reference's own CPU path on this box's host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import cpu_reference as CR

    n = cpu_threads()
    torch.set_num_threads(n)
    wl = "lmhead_int8" if (args.workload == "lmhead" and args.lm_dtype == "int8") else args.workload
    vals = CR.run_steps(wl, steps=args.steps, warmup=args.warmup, threads=n,
                        budget_s=args.cpu_budget)
    line = {"impl": "reference", "metric": vals["metric"], "value": vals["value"], "unit": vals["unit"],
            "n_gpus": int(os.environ.get("WORLD_SIZE", args.gpus)), "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": vals["ms_per_step"], "higher_is_better": True, "scaling": vals.get("scaling", "weak"),
            "vs_baseline": None, "dtype": vals["dtype"], "data": "synthetic",
            "config": vals["config"],
            "cpu_baseline": {"value": vals["value"], "unit": vals["unit"], "cores": n, "kind": "port",
                             "sample": vals["sample"]},
            "e2e": {"value": vals["value"], "unit": vals["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["hx", "reference"], default="hx")
    ap.add_argument("--workload", choices=["gpt2", "qwen", "tinyllama", "lmhead", "attn", "conv", "softmax", "cube"],
                    default="lmhead")
    ap.add_argument("--batch", type=int, default=1, help="decode batch M for --workload tinyllama")
    ap.add_argument("--layers", type=int, default=22, help="decoder layers for --workload tinyllama")
    ap.add_argument("--chain", action="store_true",
                    help="stacks: run consecutive linears as one persistent launch (chain_gemms)")
    ap.add_argument("--gather", choices=["p2p", "ce", "nccl"], default="ce",
                    help="LM head at N>1: all-gather by the GEMM's epilogue stores over NVLink (p2p), "
                         "by copy-engine DMA of finished row chunks (ce), or by NCCL")
    ap.add_argument("--ce-chunks", type=int, default=0, help="row chunks of --gather ce (0 = automatic)")
    ap.add_argument("--lm-post", choices=["gather", "softmax"], default="gather",
                    help="LM head step: all-gather the logits (the config's definition) or a vocab-parallel "
                         "softmax of each rank's shard (no gather)")
    ap.add_argument("--lm-dtype", choices=["bf16", "int8"], default="bf16",
                    help="LM head: bf16, or the int8 W8A8 variant (int32 accumulate)")
    ap.add_argument("--lm-rows", type=int, default=0,
                    help="rows M of the LM-head GEMM (default: the config's 16384; smaller for profiling)")
    ap.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of CPU work for the CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    global CHAIN
    CHAIN = args.chain
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_hx(args)


if __name__ == "__main__":
    main()
