#!/usr/bin/env python
"""bench.py — weight-only quantized linear (W4A16 / W8A16) throughput on B200.

Headline (`value`): benchmark config 1, the configuration the metric is quoted
on — W4A16 group-128 GEMV / skinny GEMM, x fp16 [M, K] ~ N(0,1) with M in
{1, 8, 32}, (K, N) in {(1536, 8960), (8960, 1536)}, W ~ N(0, 0.02) quantized
by the reference's RTN quantizer into the reference's packed format.  One
step = every (M, shape) pair over COPIES distinct weight copies per shape (36
x 2 x 7.1 MB = 511 MB, 4.1x the 126 MB L2, cycled so no launch finds its
weights in L2), i.e. 216 kernel launches, recorded once into a CUDA graph.

  value   = algorithmic bytes of all ranks / device time of K steps (GB/s);
            algorithmic bytes per launch = N*K/2 + 2*N*K/128 + 2*M*K + 2*M*N.
  e2e     = the same through the public API with host buffers: each step
            copies its activations from pinned host memory and every output
            back to pinned host memory inside the timed region.
  roofline: achieved GB/s of the step's launches against the measured HBM
            copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline: the reference's CPU path (dequantize to fp32, fp32 linear)
            on the host cores, bounded sample: the reference's own
            w4a16_reference when it is installed under baseline/_ref, else
            its restatement in oracle/.

The rest of the metric rides in the same line (one GPU unless stated):
  config0_w8   W8A16 GEMV [1,1536] x [8960,1536] (fp32 and fp16 row scales);
  prefill      config 3 tensor-core GEMM, TFLOP/s per case and aggregate;
  decode_step  config 2, all 28 layers' projections of a Qwen2.5-1.5B-shaped
               model per step, W4 and W8, M in {1, 4, 16, 64};
  sharded      config 4 at the run's GPU count (every N, all ranks): the
               column-sharded lm_heads and fused gate+up, per case the shard
               compute, NCCL and peer-memory all-gather forwards, the argmax
               head, the same layer unsharded on one GPU in the same run
               (rank 0) and the measured speed-up, plus on-box parity of the
               gathered outputs and the argmax against the unsharded layer.

`--impl reference` times the reference's CPU path alone (rank 0), on the same
metric/config.  Multi-GPU (torchrun): every rank runs the config-1 step on
its own weight copies (replicas: the step has no exchange); the device time
is the max over ranks.  The `sharded` block is the one that shards.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "llm-inference-optimizer_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "W4A16/W8A16 decode GEMV HBM GB/s (% of 8 TB/s); prefill GEMM TFLOPS"
MS = (1, 8, 32)
SHAPES = ((1536, 8960), (8960, 1536))      # (K, N)
COPIES = 36
E2E_CHUNK = 6          # launches whose outputs go back to the host in one copy (e2e leg)
WORKLOAD = ("config1: W4A16 group-128 GEMV, M in {1,8,32}, (K,N) in {(1536,8960),(8960,1536)}, "
            "reference split-half int4 format, fp16 scales [K/128,N], no bias, "
            f"{COPIES} weight copies per shape cycled (511 MB, 4.1x L2)")


def algo_bytes(M: int, K: int, N: int) -> int:
    """Algorithmic bytes of one W4A16 launch: packed weights + fp16 scales +
    fp16 activations in + fp16 outputs out."""
    return N * K // 2 + 2 * N * (K // 128) + 2 * M * K + 2 * M * N


def step_bytes() -> int:
    return sum(algo_bytes(M, K, N) * COPIES for M in MS for K, N in SHAPES)


def _peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def measured_peaks() -> tuple[float, str]:
    d = _peaks()
    if "hbm_gbs" in d:
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tflops() -> tuple[float, str]:
    d = _peaks()
    if "bf16_tflops" in d:
        return float(d["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
    return 1590.0, "fallback"


def profiled_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary
    (profiles/traffic.txt, lines 'name: bytes_per_launch'), else None."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if ":" in line and not line.lstrip().startswith("#"):
            k, v = line.split(":", 1)
            if k.strip() == kernel:
                try:
                    return float(v.split()[0])
                except ValueError:
                    return None
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML during the timed
    regions (read-only; no setting is changed)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, torch_dev: int):
        self.samples = []
        self.active = False
        self.stop_ev = threading.Event()
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            props = torch.cuda.get_device_properties(torch_dev)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.nvml = pynvml
        except Exception:
            self.handle = None
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _reasons(self):
        n = self.nvml
        for fn in ("nvmlDeviceGetCurrentClocksEventReasons", "nvmlDeviceGetCurrentClocksThrottleReasons"):
            if hasattr(n, fn):
                return getattr(n, fn)(self.handle)
        return 0

    def _run(self):
        while not self.stop_ev.is_set():
            if self.active and self.handle is not None:
                try:
                    mhz = self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
                    self.samples.append((mhz, int(self._reasons())))
                except Exception:
                    pass
            time.sleep(0.02)

    def start(self):
        self.thread.start()

    def stop(self):
        self.stop_ev.set()
        self.thread.join(timeout=2)

    def summary(self):
        if self.handle is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples)}


# ------------------------------------------------------------ CPU baseline
def reference_cpu_path():
    """The CPU dequantize-then-fp32-linear path that the CPU legs time:
    (fn(x, packed, scales) on CPU torch tensors, kind, description).  The
    reference's own ``w4a16_reference`` when the reference is installed
    under baseline/_ref (it is plain PyTorch and runs on the host), else the
    oracle's numpy restatement of it."""
    import torch
    ref_dir = ROOT / "baseline" / "_ref"
    if (ref_dir / "src" / "kernels" / "w4a16_matmul_triton.py").exists():
        try:
            sys.dont_write_bytecode = True
            if str(ref_dir) not in sys.path:
                sys.path.append(str(ref_dir))
            from src.kernels.w4a16_matmul_triton import w4a16_reference
            return (w4a16_reference, "reference",
                    "the reference's own w4a16_reference (src/kernels/w4a16_matmul_triton.py:181-187) "
                    "on CPU torch")
        except Exception as e:          # e.g. triton missing on the host
            why = f"reference not importable ({type(e).__name__}); "
    else:
        why = "reference not installed; "
    from oracle import qlinear_oracle as orc

    def port(x, packed, scales):
        return torch.from_numpy(orc.w4a16_reference_f32(x.numpy(), packed.numpy(), scales.numpy()))
    return port, "port", why + "oracle restatement of w4a16_reference (numpy)"


def host_workload(seed=0):
    """Config-1 weights (packed int4 + fp16 scales) and activations as CPU
    torch tensors, quantized by the oracle's restatement of from_linear
    (bit-identical to the reference's, pinned by the golden tests)."""
    import numpy as np
    import torch
    from oracle import qlinear_oracle as orc
    rng = np.random.default_rng(seed)
    layers = {}
    for K, N in SHAPES:
        w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float16)
        packed, scales = orc.quantize_int4_groups(w)
        layers[(K, N)] = (torch.from_numpy(packed), torch.from_numpy(scales))
    xs = {(M, K): torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32).astype(np.float16))
          for M in MS for K, _ in SHAPES}
    return layers, xs


REF_ROUNDS = 6   # rounds of the six config-1 pairs in one CPU step (1/6 of the GPU step's launches)


def cpu_reference_run(fn, layers, xs, *, steps=None, seconds=None, warmup=0):
    """Times `fn` over the config-1 (M, shape) pairs on all host threads.  A
    step is REF_ROUNDS GEMVs of each of the six pairs.  Runs `steps` steps,
    or steps until `seconds` have passed.  Returns (GB/s, seconds, bytes,
    GEMVs, threads)."""
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    pairs = [(M, K, N) for M in MS for K, N in SHAPES] * REF_ROUNDS

    def one_step():
        nb = 0
        for M, K, N in pairs:
            packed, scales = layers[(K, N)]
            fn(xs[(M, K)], packed, scales)
            nb += algo_bytes(M, K, N)
        return nb

    for _ in range(warmup):
        one_step()
    nbytes = n = 0
    t0 = time.perf_counter()
    while True:
        nbytes += one_step()
        n += 1
        el = time.perf_counter() - t0
        if steps is not None and n >= steps:
            break
        if seconds is not None and el >= seconds:
            break
    return nbytes / el / 1e9, el, nbytes, n * len(pairs), threads


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    fn, kind, what = reference_cpu_path()
    layers, xs = host_workload()
    gbs, el, nbytes, n, threads = cpu_reference_run(fn, layers, xs, steps=args.steps, warmup=args.warmup)
    line = {
        "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": WORKLOAD,
                   "step": f"{REF_ROUNDS} GEMVs of each of the six config-1 (M, shape) pairs "
                           f"({6 * REF_ROUNDS} of the GPU step's 216 launches)"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{n} GEMVs in {el:.1f} s ({nbytes / 1e6:.0f} MB algorithmic): {what}"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------- GPU helpers
def _graph_time(torch, g, stream, reps, per):
    """Median of `reps` replays of graph `g` (each holding `per` launches or
    iterations), seconds per launch."""
    ts = []
    for _ in range(reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e-3 / per)
    return statistics.median(ts)


def guarded(name, fn, *a, **kw):
    """Runs one block of the bench line; a Python-level failure is recorded
    in the line instead of losing the headline number."""
    try:
        return fn(*a, **kw)
    except Exception as e:          # recorded, not hidden: the block carries the error
        print(f"[bench] block {name} failed: {type(e).__name__}: {e}", file=sys.stderr, flush=True)
        return {"error": f"{type(e).__name__}: {e}"}


# ---------------------------------------------------------------- config 0
CONFIG0 = (1536, 8960)   # (K, N)


def measure_config0(reps=20):
    """benchmark config 0: W8A16 GEMV, x [1,1536], W [8960,1536] per-row int8.
    Both scale dtypes the format allows (fp32: the reference's buffer; fp16:
    the benchmark's wording).  24 weight copies (330 MB, 2.6x L2) cycled in
    a CUDA graph, so every launch streams its weights from HBM."""
    import torch
    from qlinear.kernels.w8a16_matmul import w8a16_linear, w8a16_quantize_cuda
    dev = torch.device("cuda", torch.cuda.current_device())
    K, N = CONFIG0
    copies = 24
    gen = torch.Generator(device=dev).manual_seed(3)
    layers = []
    for _ in range(copies):
        w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
        layers.append(w8a16_quantize_cuda(w))
        del w
    x = torch.randn(1, K, generator=gen, device=dev).half()
    y = torch.empty(copies, N, dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)
    peak, peak_kind = measured_peaks()
    res = {"shape": "x [1,1536] fp16, W int8 [8960,1536], per-row scale", "copies": copies,
           "reference_rtx4060": {"us": 58.4, "GBps": 235.9, "source": "benchmarks/results/stage7_kernel.json:91-99"}}
    for sdt, tag in ((torch.float32, "f32_scale"), (torch.float16, "f16_scale")):
        sc = [s.to(sdt) for _, s in layers]
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            for c in range(copies):
                w8a16_linear(x, layers[c][0], sc[c], out=y[c:c + 1])
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for c in range(copies):
                    w8a16_linear(x, layers[c][0], sc[c], out=y[c:c + 1])
            for _ in range(3):
                g.replay()
            t = _graph_time(torch, g, stream, reps, copies)
        del g
        nb = N * K + sc[0].element_size() * N + 2 * K + 2 * N
        gbs = nb / t / 1e9
        res[tag] = {"us_per_launch": round(t * 1e6, 3), "GBps": round(gbs, 1), "frac": round(gbs / peak, 4),
                    "bytes_per_launch": nb}
    res["peak"] = peak
    res["peak_kind"] = peak_kind
    return res


# ---------------------------------------------------------------- config 3
PREFILL_MS = (512, 2048, 8192)
PREFILL_SHAPES = ((1536, 8960), (8960, 1536), (4096, 14336), (14336, 4096))   # (K, N)


def prefill_measure(reps=5, wbits_list=(4, 8), ms=PREFILL_MS, shapes=PREFILL_SHAPES):
    """benchmark config 3: dequant-fused GEMM on the tensor cores.  Per
    (wbits, shape, M): best of `reps` CUDA-event timings of one launch, with
    L2 flushed (256 MB write) before every timed launch.  Returns
    {key: {"us": t, "TFLOPS": 2MNK/t}} and the aggregate TFLOPS."""
    import torch
    from qlinear.kernels.w4a16_matmul import w4a16_linear, w4a16_quantize_cuda
    from qlinear.kernels.w8a16_matmul import w8a16_linear, w8a16_quantize_cuda
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(11)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    tot_flop = 0.0
    tot_s = 0.0
    for wbits in wbits_list:
        for K, N in shapes:
            w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
            a, b = w4a16_quantize_cuda(w) if wbits == 4 else w8a16_quantize_cuda(w)
            del w
            fn = w4a16_linear if wbits == 4 else w8a16_linear
            for M in ms:
                x = torch.randn(M, K, generator=gen, device=dev).half()
                y = torch.empty(M, N, dtype=torch.float16, device=dev)
                fn(x, a, b, out=y)
                best = 1e30
                for _ in range(reps):
                    flush.fill_(1)
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    fn(x, a, b, out=y)
                    e1.record()
                    torch.cuda.synchronize(dev)
                    best = min(best, e0.elapsed_time(e1) * 1e-3)
                flop = 2.0 * M * N * K
                out[f"w{wbits}_M{M}_K{K}_N{N}"] = {"us": round(best * 1e6, 2), "TFLOPS": round(flop / best / 1e12, 1)}
                tot_flop += flop
                tot_s += best
                del x, y
            del a, b
    del flush
    return out, tot_flop / tot_s / 1e12


def measure_prefill(reps=3):
    detail, agg = prefill_measure(reps=reps)
    peak, kind = measured_tflops()
    return {"aggregate_TFLOPS": round(agg, 1), "frac": round(agg / peak, 4), "peak": peak, "peak_kind": kind,
            "timing": f"best of {reps} single launches, L2 flushed before each", "cases": detail}


def run_prefill(args):
    """`--workload prefill`: benchmark config 3 as its own JSON line."""
    import torch
    torch.cuda.set_device(0)
    detail, agg = prefill_measure(reps=max(3, args.steps))
    peak = measured_tflops()
    print(json.dumps({
        "metric": METRIC, "value": agg, "unit": "TFLOPS", "n_gpus": 1, "steps": args.steps, "warmup": 1,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "config3: W4A16/W8A16 prefill GEMM, M in {512,2048,8192}, (K,N) in "
                               "{(1536,8960),(8960,1536),(4096,14336),(14336,4096)}, L2 flushed per launch"},
        "roofline": {"bound": "tensor", "achieved": agg, "peak": peak[0], "unit": "TFLOP/s",
                     "frac": agg / peak[0], "peak_kind": peak[1]},
        "detail": detail}), flush=True)
    return 0


# ---------------------------------------------------------------- config 2
DECODE_LAYERS = 28
DECODE_MS = (1, 4, 16, 64)
# Qwen2.5-1.5B projections per layer: (name, K, N, bias)
DECODE_LINEARS = (("q", 1536, 1536, True), ("k", 1536, 256, True), ("v", 1536, 256, True),
                  ("o", 1536, 1536, False), ("gate", 1536, 8960, False), ("up", 1536, 8960, False),
                  ("down", 8960, 1536, False))


def linear_weight_bytes(wbits, K, N, bias):
    """Stored bytes of one quantized projection: int4 packed + fp16 group
    scales, or int8 + fp32 row scales; fp16 bias."""
    w = N * K // 2 + 2 * N * (K // 128) if wbits == 4 else N * K + 4 * N
    return w + (2 * N if bias else 0)


def decode_step_bytes(wbits, M, fused):
    """Algorithmic bytes of one decode step over all layers: every weight
    byte once plus each launch's fp16 activations in and out."""
    per = 0
    for _, K, N, b in DECODE_LINEARS:
        per += linear_weight_bytes(wbits, K, N, b)
    if fused:
        launches = ((1536, 1536 + 2 * 256), (1536, 1536), (1536, 8960), (8960, 1536))   # qkv, o, gate_up_silu, down
    else:
        launches = tuple((K, N) for _, K, N, _ in DECODE_LINEARS)
    per += sum(2 * M * (K + N) for K, N in launches)
    return DECODE_LAYERS * per


def measure_decode_step(reps=20, warmup=3):
    """benchmark config 2.  The seven projections of all 28 layers of a
    random-init Qwen2.5-1.5B (q/k/v with bias), quantized on the device, run
    through the public modules for one decode step at M in {1, 4, 16, 64},
    W4 and W8 — once as seven launches per layer (the reference's module
    structure) and once with the fused kernels (q/k/v stacked in one launch,
    gate+up with the SwiGLU epilogue: four launches per layer).  Each step
    is one CUDA graph; the step's weights (676 MB W4, 1.31 GB W8) exceed L2
    several times over, so no flush is needed.  Projections feed each other
    where the model does (o reads q's output, down reads gate's or the fused
    MLP's output); attention and norms are not part of the path.
    Returns (detail, GB/s over the fused steps, launches timed)."""
    import torch
    from qlinear.kernels.fused_mlp import QuantizedGateUpSiLU
    from qlinear.kernels.fused_qkv import QuantizedQKV
    from qlinear.kernels.w4a16_matmul import w4a16_quantize_cuda
    from qlinear.kernels.w8a16_matmul import w8a16_quantize_cuda
    from qlinear.quantization.int4 import QuantizedLinearInt4
    from qlinear.quantization.int8 import QuantizedLinearInt8

    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(2)
    stream = torch.cuda.Stream(device=dev)
    peak, _ = measured_peaks()
    detail = {}
    tot_bytes = tot_s = 0.0
    launches_total = 0
    for wbits in (4, 8):
        layers = []
        for _ in range(DECODE_LAYERS):
            mods = {}
            for name, K, N, has_bias in DECODE_LINEARS:
                w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
                bias = (torch.randn(N, generator=gen, device=dev) * 0.02).half() if has_bias else None
                if wbits == 4:
                    mods[name] = QuantizedLinearInt4(*w4a16_quantize_cuda(w), bias)
                else:
                    mods[name] = QuantizedLinearInt8(*w8a16_quantize_cuda(w), bias)
                del w
            mods["qkv"] = QuantizedQKV.from_quantized(mods["q"], mods["k"], mods["v"])
            mods["mlp"] = QuantizedGateUpSiLU.from_quantized(mods["gate"], mods["up"])
            layers.append(mods)

        def step_unfused(x):
            for L in layers:
                q = L["q"](x)
                L["k"](x)
                L["v"](x)
                L["o"](q)
                g = L["gate"](x)
                L["up"](x)
                L["down"](g)

        def step_fused(x):
            for L in layers:
                q, _, _ = L["qkv"](x)
                L["o"](q)
                L["down"](L["mlp"](x))

        for M in DECODE_MS:
            x = torch.randn(M, 1536, generator=gen, device=dev).half()
            torch.cuda.synchronize(dev)          # weights and x are made on the default stream
            row = {}
            for fused, fn, nl in ((False, step_unfused, 7), (True, step_fused, 4)):
                with torch.cuda.stream(stream):
                    fn(x)                                  # eager: sizes the workspaces
                    torch.cuda.synchronize(dev)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=stream):
                        fn(x)
                    for _ in range(max(3, warmup)):
                        g.replay()
                    torch.cuda.synchronize(dev)
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for _ in range(reps):
                        g.replay()
                    e1.record(stream)
                    torch.cuda.synchronize(dev)
                t = e0.elapsed_time(e1) * 1e-3 / reps
                del g
                nb = decode_step_bytes(wbits, M, fused)
                key = "fused" if fused else "unfused"
                row[f"{key}_us"] = round(t * 1e6, 1)
                row[f"{key}_GBps"] = round(nb / t / 1e9, 1)
                row[f"{key}_frac"] = round(nb / t / 1e9 / peak, 4)
                row[f"{key}_launches"] = nl * DECODE_LAYERS
                if fused:
                    tot_bytes += nb
                    tot_s += t
                    launches_total += nl * DECODE_LAYERS * reps
            row["speedup_fused"] = round(row["unfused_us"] / row["fused_us"], 3)
            detail[f"w{wbits}_M{M}"] = row
            print(f"[decode_step] w{wbits} M={M}: {row}", file=sys.stderr, flush=True)
            del x
        del layers
        torch.cuda.empty_cache()
    return detail, tot_bytes / tot_s / 1e9, launches_total


def run_decode_step(args):
    """`--workload decode_step`: benchmark config 2 as its own JSON line."""
    import torch
    torch.cuda.set_device(0)
    reps = max(5, min(args.steps, 50))
    detail, value, launches_total = measure_decode_step(reps=reps, warmup=args.warmup)
    from qlinear import _lib
    dev_err = _lib.device_error()
    if dev_err != 0:
        raise RuntimeError(f"device error word {dev_err} after the decode-step workload")
    peak, peak_kind = measured_peaks()
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 1, "steps": reps, "warmup": max(3, args.warmup),
        "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "config2: decode step of a random-init Qwen2.5-1.5B, 28 layers x q/k/v/o/gate/up/"
                               "down (q/k/v biased), W4A16 and W8A16, M in {1,4,16,64}; value over the fused "
                               "path (q/k/v one launch, gate+up with SwiGLU one launch)",
                   "l2": "inputs larger than L2 (one step streams 676 MB / 1.31 GB of distinct weights)"},
        "roofline": {"bound": "hbm", "achieved": value, "peak": peak, "unit": "GB/s", "frac": value / peak,
                     "peak_kind": peak_kind},
        "gpu_launches": launches_total,
        "detail": detail}), flush=True)
    return 0


# ---------------------------------------------------------------- config 4
SHARDED_LAYERS = (("lm_head_1p5b", 1536, 151936, 1), ("lm_head_7b", 4096, 128256, 1),
                  ("gate_up_7b", 4096, 28672, 2))       # (name, K, N, column groups)
SHARDED_MS = (1, 16, 64)


def layer_bytes(wbits, K, N):
    """Algorithmic weight bytes of a full layer (all ranks together)."""
    return N * K // 2 + 2 * N * (K // 128) if wbits == 4 else N * K + 4 * N


def _quantize_module(wbits, w):
    from qlinear.kernels.w4a16_matmul import w4a16_quantize_cuda
    from qlinear.kernels.w8a16_matmul import w8a16_quantize_cuda
    from qlinear.quantization.int4 import QuantizedLinearInt4
    from qlinear.quantization.int8 import QuantizedLinearInt8
    if wbits == 4:
        return QuantizedLinearInt4(*w4a16_quantize_cuda(w), None)
    return QuantizedLinearInt8(*w8a16_quantize_cuda(w), None)


def _dequantized(q):
    """fp32 [N, K] weight of a quantized module, from the device decoder
    (bit-exact with the reference's dequantize_int4 / dequantized_weight)."""
    from qlinear.kernels.w4a16_matmul import dequantize_int4_cuda
    from qlinear.quantization.int4 import QuantizedLinearInt4
    if isinstance(q, QuantizedLinearInt4):
        return dequantize_int4_cuda(q.weight_packed, q.scales, q.layout)
    return q.weight_q.float() * q.scale.float().unsqueeze(1)


def _within_tolerance(y, ref32, xmax, wmax, K):
    """North-star bound on the GPU: max-abs <= 1e-2*|x|inf*|w|inf*sqrt(K)/64
    and rel-L2 <= 2e-3 against the fp32-accumulated result."""
    import torch
    d = y.float() - ref32
    bound = 1e-2 * xmax * wmax * math.sqrt(K) / 64
    max_abs = float(d.abs().max())
    rel = float(torch.linalg.vector_norm(d) / torch.linalg.vector_norm(ref32).clamp_min(1e-30))
    return max_abs <= bound and rel <= 2e-3, max_abs, rel, bound


def solo_arg(solo, q, x, linear):
    """Greedy head of the unsharded layer on one GPU: one launch when the
    decode kernel takes the shape, else the linear then the one-rank
    exchange kernel."""
    ids = solo.linear_argmax(x, q, 0)
    if ids is not None:
        return ids
    return solo.argmax(linear(q, x), 0)


def measure_sharded(world, rank, reps=5, ms=SHARDED_MS, layers=SHARDED_LAYERS):
    """benchmark config 4 at this run's GPU count.  Every rank holds its
    column shard of each layer and runs the local kernel; the fp16 outputs
    are all-gathered by NCCL and by the peer-memory kernel (PeerGather); for
    the lm_heads the greedy head (argmax only) runs with the per-row keys
    exchanged over NVLink (PeerExchange: one launch per rank up to 8 rows,
    else the linear then the exchange kernel).  Per (wbits, layer, M), CUDA
    graphs of back-to-back iterations are timed, each iteration on the next
    of several weight copies (copies x shard bytes > 2 x L2, so no iteration
    finds its weights in L2); time per iteration = median graph time /
    iterations, max over ranks.  Rank 0 also times the same layer unsharded
    on its own GPU (the 1-GPU baseline of the speed-ups).

    Parity on the box: the first copy is the real layer (same seed on every
    rank) cut into shards; every rank checks its gathered [M, N] outputs
    (NCCL and peer path, which must agree bit for bit) and the unsharded
    layer's outputs against an fp32 product of the dequantized weights
    and that each argmax column holds the row's
    maximum of that fp32 product within the same tolerance.  The flags are
    combined over ranks."""
    import torch
    import torch.distributed as dist
    from qlinear.p2p import PeerExchange, PeerGather
    from qlinear.sharded import ShardedQuantizedLinear, local_linear_cuda, shard_bounds

    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.Stream(device=dev)
    gen_rank = torch.Generator(device=dev).manual_seed(100 + rank)
    detail = {}
    agg = {"unsharded_us": 0.0, "e2e_peer_us": 0.0, "e2e_nccl_us": 0.0, "compute_us": 0.0,
           "argmax_unsharded_us": 0.0, "argmax_us": 0.0}
    parity_all = True

    def timed(graph, iters):
        graph.replay()
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            t = _graph_time(torch, graph, stream, reps, iters)
        if world > 1:
            tt = torch.tensor([t], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    def local_time(graph, iters):          # one rank's own time, no collective
        graph.replay()
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            return _graph_time(torch, graph, stream, reps, iters)

    def capture(fn, iters):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(iters):
                fn(i)
        return g

    max_m = max(ms)
    exchange = PeerExchange(rank, world, max_m=max_m)
    solo = PeerExchange(0, 1, max_m=max_m) if (world > 1 and rank == 0) else None
    for li, (name, K, N, groups) in enumerate(layers):
        for wbits in (4, 8):
            n_g = N // groups
            # the real layer, identical on every rank (same seed)
            gen_full = torch.Generator(device=dev).manual_seed(5000 + 10 * li + wbits)
            w = (torch.randn(N, K, generator=gen_full, device=dev) * 0.02).half()
            q_full = _quantize_module(wbits, w)
            del w
            deq = _dequantized(q_full)
            wmax = float(deq.abs().max())
            # shards: copy 0 cut from the real layer, the rest random (L2 cycling)
            lo, hi = shard_bounds(n_g, rank, world)
            rows = groups * (hi - lo)
            shard_bytes = groups * ((n_g + world - 1) // world) * K // (2 if wbits == 4 else 1)
            copies = max(1, min(32, math.ceil(2 * 128e6 / shard_bytes)))
            shs = [ShardedQuantizedLinear.from_quantized(q_full, rank, world, groups=groups)]
            for _ in range(copies - 1):
                wr = (torch.randn(rows, K, generator=gen_rank, device=dev) * 0.02).half()
                shs.append(ShardedQuantizedLinear(_quantize_module(wbits, wr), N, rank, world, groups=groups))
                del wr
            if groups == 1:
                for sh in shs:
                    sh.exchange = exchange
            iters = copies * max(1, math.ceil(16 / copies))
            # unsharded copies (rank 0, when sharded): the 1-GPU baseline
            full = []
            if world > 1 and rank == 0:
                full_copies = max(1, min(8, math.ceil(2 * 128e6 / layer_bytes(wbits, K, N))))
                full = [q_full]
                for _ in range(full_copies - 1):
                    wr = (torch.randn(N, K, generator=gen_rank, device=dev) * 0.02).half()
                    full.append(_quantize_module(wbits, wr))
                    del wr
            gatherer = PeerGather(rank, world, max_m=max_m, n_cols=N) if world > 1 else None
            for M in ms:
                gx = torch.Generator(device=dev).manual_seed(7000 + M)
                x = torch.randn(M, K, generator=gx, device=dev).half()   # same on every rank
                # weights, dequantized copy and x come from the default stream:
                # all done before the side stream reads them
                torch.cuda.synchronize(dev)
                with torch.cuda.stream(stream):
                    # ---- parity (real layer)
                    ref32 = x.float() @ deq.t()
                    xmax = float(x.abs().max())
                    y_one = local_linear_cuda(q_full, x)
                    y_nccl = shs[0](x)
                    if gatherer is not None:
                        shs[0].gatherer = gatherer
                        y_peer = shs[0](x)
                        shs[0].gatherer = None
                    else:
                        y_peer = y_nccl
                    ids = shs[0].argmax(x) if groups == 1 else None
                    torch.cuda.synchronize(dev)
                ok_n, abs_n, rel_n, bound = _within_tolerance(y_nccl, ref32, xmax, wmax, K)
                ok_1, abs_1, rel_1, _ = _within_tolerance(y_one, ref32, xmax, wmax, K)
                same = bool(torch.equal(y_nccl, y_peer))
                ok_a = True
                if ids is not None:
                    picked = ref32.gather(1, ids.view(-1, 1)).squeeze(1)
                    ok_a = bool((picked >= ref32.max(dim=1).values - 2 * bound).all())
                flags = torch.tensor([int(ok_n), int(ok_1), int(same), int(ok_a)], device=dev, dtype=torch.int32)
                if world > 1:
                    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
                fl = [bool(v) for v in flags.tolist()]
                case_ok = all(fl)
                parity_all = parity_all and case_ok
                del ref32, y_one, y_nccl, y_peer

                # ---- timing
                with torch.cuda.stream(stream):
                    y_loc = shs[0].local_forward(x)
                    for sh in shs:                       # warm-up: every path once per copy
                        sh(x)
                        if groups == 1:
                            sh.argmax(x)
                    torch.cuda.synchronize(dev)
                    g_loc = capture(lambda i: shs[i % copies].local_forward(x), iters)
                    g_e2e = capture(lambda i: shs[i % copies](x), iters)
                    g_col = capture(lambda i: shs[0].gather(y_loc), iters) if world > 1 else None
                    g_arg = capture(lambda i: shs[i % copies].argmax(x), iters) if groups == 1 else None
                    g_arg2 = (capture(lambda i: shs[i % copies].argmax(x, fused=False), iters)
                              if groups == 1 else None)
                    g_p2p = None
                    if gatherer is not None:
                        for sh in shs:
                            sh.gatherer = gatherer
                            sh(x)
                        torch.cuda.synchronize(dev)
                        g_p2p = capture(lambda i: shs[i % copies](x), iters)
                        for sh in shs:
                            sh.gatherer = None
                t_loc, t_e2e = timed(g_loc, iters), timed(g_e2e, iters)
                t_p2p = timed(g_p2p, iters) if g_p2p is not None else t_e2e
                t_col = timed(g_col, iters) if g_col is not None else 0.0
                t_arg = timed(g_arg, iters) if g_arg is not None else None
                t_arg2 = timed(g_arg2, iters) if g_arg2 is not None else None
                # graphs holding NCCL calls must be gone before the process group is destroyed
                torch.cuda.synchronize(dev)
                del g_loc, g_col, g_e2e, g_arg, g_arg2, g_p2p, y_loc

                # ---- the same layer unsharded, on rank 0's GPU alone
                t_one, t_one_arg = t_loc, t_arg
                if full:
                    fc = len(full)
                    fit = fc * max(1, math.ceil(8 / fc))
                    with torch.cuda.stream(stream):
                        for q in full:
                            local_linear_cuda(q, x)
                            if groups == 1:
                                solo_arg(solo, q, x, local_linear_cuda)
                        torch.cuda.synchronize(dev)
                        g1 = capture(lambda i: local_linear_cuda(full[i % fc], x), fit)
                        g1a = (capture(lambda i: solo_arg(solo, full[i % fc], x, local_linear_cuda), fit)
                               if groups == 1 else None)
                    t_one = local_time(g1, fit)
                    t_one_arg = local_time(g1a, fit) if g1a is not None else None
                    del g1, g1a

                if rank == 0:
                    print(f"[sharded x{world}] w{wbits} {name} M={M}: local {t_loc * 1e6:.1f} us, all-gather "
                          f"{t_col * 1e6:.1f} us, forward {t_e2e * 1e6:.1f} us (NCCL) / {t_p2p * 1e6:.1f} us "
                          f"(peer), 1 GPU {t_one * 1e6:.1f} us"
                          + (f", argmax head {t_arg * 1e6:.1f} us (1 GPU {t_one_arg * 1e6:.1f} us)"
                             if t_arg is not None else "") + f", parity {fl}",
                          file=sys.stderr, flush=True)
                lb = layer_bytes(wbits, K, N)
                row = {
                    "compute_us": round(t_loc * 1e6, 2), "allgather_nccl_us": round(t_col * 1e6, 2),
                    "e2e_nccl_us": round(t_e2e * 1e6, 2), "e2e_peer_us": round(t_p2p * 1e6, 2),
                    "unsharded_us": round(t_one * 1e6, 2),
                    "speedup_vs_1gpu": {"compute": round(t_one / t_loc, 3), "logits_peer": round(t_one / t_p2p, 3),
                                        "logits_nccl": round(t_one / t_e2e, 3)},
                    "GBps_e2e_peer": round(lb / t_p2p / 1e9, 1),
                    "GBps_compute_per_gpu": round(lb / world / t_loc / 1e9, 1),
                    "parity": {"ok": case_ok, "gathered_vs_fp32": fl[0], "unsharded_vs_fp32": fl[1],
                               "peer_equals_nccl": fl[2], "argmax_is_row_max": fl[3],
                               "max_abs": round(max(abs_n, abs_1), 5), "bound": round(bound, 5),
                               "rel_l2": round(max(rel_n, rel_1), 6)},
                    "copies": copies, "iterations_per_graph": iters}
                if t_arg is not None:
                    row["argmax_us"] = round(t_arg * 1e6, 2)
                    row["argmax_two_launch_us"] = round(t_arg2 * 1e6, 2)
                    row["argmax_unsharded_us"] = round(t_one_arg * 1e6, 2)
                    row["speedup_vs_1gpu"]["argmax"] = round(t_one_arg / t_arg, 3)
                    agg["argmax_us"] += t_arg
                    agg["argmax_unsharded_us"] += t_one_arg
                agg["unsharded_us"] += t_one
                agg["e2e_peer_us"] += t_p2p
                agg["e2e_nccl_us"] += t_e2e
                agg["compute_us"] += t_loc
                detail[f"w{wbits}_{name}_M{M}"] = row
                del x
            del shs, full, q_full, deq
            if gatherer is not None:
                gatherer.close()
            torch.cuda.empty_cache()
    exchange.close()
    if solo is not None:
        solo.close()
    su = {"logits_peer": agg["unsharded_us"] / agg["e2e_peer_us"],
          "logits_nccl": agg["unsharded_us"] / agg["e2e_nccl_us"],
          "compute": agg["unsharded_us"] / agg["compute_us"],
          "argmax": agg["argmax_unsharded_us"] / agg["argmax_us"] if agg["argmax_us"] else None}
    return {"gpus_active": world, "sharded_parity": parity_all,
            "speedup_vs_1gpu_all_cases": {k: (round(v, 3) if v is not None else None) for k, v in su.items()},
            "timing": "CUDA graphs of back-to-back iterations over weight copies past L2; median of "
                      f"{reps} replays; max over ranks; 1-GPU baseline timed on rank 0 in the same run",
            "cases": detail}


def _init_dist(world, local):
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return torch.device("cuda", local)


def run_sharded(args):
    """`--workload sharded`: benchmark config 4 as its own JSON line (strong
    scaling: the same layers at every GPU count)."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    _init_dist(world, local)
    reps = max(3, min(args.steps, 7))
    res = measure_sharded(world, rank, reps=reps)
    from qlinear import _lib
    dev_err = _lib.device_error()
    if dev_err != 0:
        raise RuntimeError(f"device error word {dev_err} after the sharded workload")
    if rank == 0:
        tot_b = tot_s = 0.0
        for name, K, N, _ in SHARDED_LAYERS:
            for wbits in (4, 8):
                for M in SHARDED_MS:
                    tot_b += layer_bytes(wbits, K, N)
                    tot_s += res["cases"][f"w{wbits}_{name}_M{M}"]["e2e_peer_us"] * 1e-6
        print(json.dumps({
            "metric": METRIC, "value": tot_b / tot_s / 1e9, "unit": "GB/s", "n_gpus": world,
            "steps": reps, "warmup": 1, "ms_per_step": tot_s * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "config4: column-sharded lm_head 1536->151936, lm_head 4096->128256, fused "
                                   "gate+up 4096->28672 (2 groups), W4A16 and W8A16, M in {1,16,64}; value "
                                   "over the forward with the fp16 outputs all-gathered by the peer-memory kernel",
                       "parallelism": f"column shards x{world}"},
            "sharded": res}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------ the default line
def run_ours(args):
    import torch
    import torch.distributed as dist

    from qlinear.kernels.w4a16_matmul import w4a16_linear, w4a16_quantize_cuda

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = _init_dist(world, local)

    # weights: COPIES distinct copies per shape, quantized on the device
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    layers = {}
    for K, N in SHAPES:
        copies = []
        for _ in range(COPIES):
            w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
            copies.append(w4a16_quantize_cuda(w))
            del w
        layers[(K, N)] = copies
    xs = {(M, K): torch.randn(M, K, generator=gen, device=dev).half() for M in MS for K, _ in SHAPES}
    # one output buffer; every launch writes its own slice
    slots = []
    off = 0
    for M in MS:
        for K, N in SHAPES:
            for c in range(COPIES):
                slots.append((M, K, N, c, off))
                off += M * N
    ybuf = torch.empty(off, dtype=torch.float16, device=dev)

    def step():
        for M, K, N, c, o in slots:
            packed, scales = layers[(K, N)][c]
            w4a16_linear(xs[(M, K)], packed, scales, out=ybuf[o:o + M * N].view(M, N))

    launches_per_step = len(slots)
    nbytes = step_bytes()

    # eager warm-up (sizes the split-K workspace), then capture
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        step()
        torch.cuda.synchronize(dev)
        g_val = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_val, stream=stream):
            step()
        # e2e: pinned host activations in, every output back to pinned host.
        # The outputs of each run of E2E_CHUNK launches are copied back on a
        # side stream while the next launches compute (a serving loop would
        # do the same); the step ends when the last copy has landed.
        x_host = {k: v.cpu().pin_memory() for k, v in xs.items()}
        y_host = torch.empty(ybuf.shape, dtype=ybuf.dtype, pin_memory=True)
        side = torch.cuda.Stream(device=dev)
        g_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_e2e, stream=stream):
            for k, v in xs.items():
                v.copy_(x_host[k], non_blocking=True)
            for i0 in range(0, len(slots), E2E_CHUNK):
                chunk = slots[i0:i0 + E2E_CHUNK]
                for M, K, N, c, o in chunk:
                    packed, scales = layers[(K, N)][c]
                    w4a16_linear(xs[(M, K)], packed, scales, out=ybuf[o:o + M * N].view(M, N))
                lo = chunk[0][4]
                hi = chunk[-1][4] + chunk[-1][0] * chunk[-1][2]
                side.wait_stream(stream)
                with torch.cuda.stream(side):
                    y_host[lo:hi].copy_(ybuf[lo:hi], non_blocking=True)
            stream.wait_stream(side)
    h2d = sum(v.numel() * 2 for v in xs.values())
    d2h = ybuf.numel() * 2
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(dev.index)
    clocks.start()

    def timed(graph, K, W):
        with torch.cuda.stream(stream):
            for _ in range(W):
                graph.replay()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize(dev)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            clocks.active = True
            e0.record(stream)
            for _ in range(K):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            clocks.active = False
            if world > 1:
                dist.barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    ms_val = timed(g_val, args.steps, args.warmup)
    ms_e2e = timed(g_e2e, args.steps, args.warmup)

    # per-(M, shape) breakdown on this rank (same cycling, graphs of COPIES launches)
    detail = {}
    reps = max(20, args.steps // 4)
    with torch.cuda.stream(stream):
        for M in MS:
            for K, N in SHAPES:
                sub = [s for s in slots if s[0] == M and s[1] == K]
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for _, K_, N_, c, o in sub:
                        packed, scales = layers[(K_, N_)][c]
                        w4a16_linear(xs[(M, K_)], packed, scales, out=ybuf[o:o + M * N_].view(M, N_))
                for _ in range(3):
                    g.replay()
                torch.cuda.synchronize(dev)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                clocks.active = True
                e0.record(stream)
                for _ in range(reps):
                    g.replay()
                e1.record(stream)
                torch.cuda.synchronize(dev)
                clocks.active = False
                us = e0.elapsed_time(e1) * 1e3 / (reps * len(sub))
                gbs = algo_bytes(M, K, N) / (us * 1e-6) / 1e9
                detail[f"M{M}_K{K}_N{N}"] = {"us_per_launch": round(us, 3), "GBps": round(gbs, 1)}
                del g
    clocks.stop()
    from qlinear import _lib
    dev_err = _lib.device_error()
    if dev_err != 0:
        raise RuntimeError(f"device error word {dev_err}: a bounded wait gave up during the bench")

    peak, peak_kind = measured_peaks()
    per_rank_gbs = nbytes / (ms_val / args.steps * 1e-3) / 1e9
    value = world * per_rank_gbs
    e2e_gbs = world * nbytes / (ms_e2e / args.steps * 1e-3) / 1e9
    avg_launch_bytes = nbytes / launches_per_step
    traffic = profiled_traffic("qgemv_w4_config1")
    # the launch with the largest per-launch time (M 32 down projection)
    dom_key = max(detail, key=lambda k: detail[k]["us_per_launch"]) if detail else None
    dominant = None
    if dom_key:
        dm, dk, dn = (int(v[1:]) for v in dom_key.split("_"))
        dbytes = algo_bytes(dm, dk, dn)
        dus = detail[dom_key]["us_per_launch"]
        dominant = {"shape": dom_key, "us_per_launch": dus, "bytes_per_launch": dbytes,
                    "achieved": dbytes / (dus * 1e-6) / 1e9, "frac": dbytes / (dus * 1e-6) / 1e9 / peak,
                    "traffic": profiled_traffic("qgemm_w4_m32_cluster") if dm == 32 else None}

    # free the config-1 weights before the other blocks
    del g_val, g_e2e, layers, ybuf
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()

    blocks = {}
    if not args.no_extra:
        if world == 1:
            blocks["config0_w8"] = guarded("config0_w8", measure_config0)
            blocks["prefill"] = guarded("prefill", measure_prefill, reps=3)

            def _decode():
                d, v, _ = measure_decode_step(reps=20, warmup=3)
                return {"GBps_fused_all_cases": round(v, 1), "frac": round(v / peak, 4), "cases": d}
            blocks["decode_step"] = guarded("decode_step", _decode)
        # every rank, every N: the column-sharded layers (collective)
        blocks["sharded"] = measure_sharded(world, rank, reps=3)
        dev_err = _lib.device_error()
        if dev_err != 0:
            raise RuntimeError(f"device error word {dev_err}: a bounded wait gave up in the extra blocks")

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fn, kind, what = reference_cpu_path()
        hl, hx = host_workload()
        gbs, el, cb, n, threads = cpu_reference_run(fn, hl, hx, seconds=args.cpu_seconds, warmup=1)
        cpu_baseline = {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind,
                        "sample": f"{n} config-1 GEMVs in {el:.1f} s ({cb / 1e6:.0f} MB algorithmic): {what}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_val / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": list(MS), "l2": "inputs larger than L2 "
                       "(weights cycled; each launch's weights last touched 71 launches earlier)",
                       "launches_per_step": launches_per_step, "bytes_per_step": nbytes,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": per_rank_gbs, "peak": peak, "unit": "GB/s",
                         "frac": per_rank_gbs / peak, "peak_kind": peak_kind,
                         "kernel": "qgemv_kernel<4,0,1> (M 1, M 8 gate/up) and qgemm_kernel<4,0,16|32> "
                                   "(M 8 down, M 32): the step's 216 launches averaged",
                         "bytes_per_launch": avg_launch_bytes,
                         "traffic": traffic, "pct_of_8TBs": per_rank_gbs / 8000.0,
                         "dominant_launch": dominant},
            "cpu_baseline": cpu_baseline,
            "e2e": {"value": e2e_gbs, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e / args.steps,
                    "path": "QuantizedLinearInt4 API (w4a16_linear) in a CUDA graph with pinned host I/O; "
                            f"outputs copied back per {E2E_CHUNK} launches on a side stream, overlapping compute"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "detail": detail,
        }
        line.update(blocks)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_profile_one(args):
    """A handful of eager launches of one (wbits, M, K, N) layer with its
    weights cycled over enough copies to exceed L2: the small case that the
    ncu captures in profiles/ are taken on."""
    import torch

    from qlinear.kernels.w4a16_matmul import w4a16_linear, w4a16_quantize_cuda
    from qlinear.kernels.w8a16_matmul import w8a16_linear, w8a16_quantize_cuda
    parts = [int(v) for v in args.profile_one.split(",")]
    wbits, M, K, N = parts
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(7)
    per = N * K // (2 if wbits == 4 else 1)
    copies = max(2, int(300e6 // max(per, 1)) + 1)
    layers = []
    for _ in range(copies):
        w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
        layers.append(w4a16_quantize_cuda(w) if wbits == 4 else w8a16_quantize_cuda(w))
        del w
    x = torch.randn(M, K, generator=gen, device=dev).half()
    if args.path == "auto":
        for i in range(args.steps):
            a, b = layers[i % copies]
            (w4a16_linear if wbits == 4 else w8a16_linear)(x, a, b)
    else:
        # one kernel family forced through the C ABI (its split-K workspace included)
        from qlinear import _lib
        lib = _lib.load()
        flag = {"gemm": _lib.QL_FLAG_FORCE_GEMM, "gemv": _lib.QL_FLAG_FORCE_GEMV,
                "tcdec": _lib.QL_FLAG_FORCE_TCDEC}[args.path] | _lib.QL_FLAG_PDL
        out = torch.empty(M, N, dtype=torch.float16, device=dev)
        ws = torch.zeros(64 << 20, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        for i in range(args.steps):
            a, b = layers[i % copies]
            if wbits == 4:
                st = lib.ql_w4a16_linear(x.data_ptr(), 0, a.data_ptr(), 0, b.data_ptr(), None, 0, out.data_ptr(),
                                         M, N, K, K, K // 2, N, N, ws.data_ptr(), ws.numel(), flag, stream)
            else:
                st = lib.ql_w8a16_linear(x.data_ptr(), 0, a.data_ptr(), b.data_ptr(), 1, None, 0, out.data_ptr(),
                                         M, N, K, K, K, N, ws.data_ptr(), ws.numel(), flag, stream)
            _lib.check(st)
    torch.cuda.synchronize()
    print(json.dumps({"profile_one": args.profile_one, "path": args.path, "launches": args.steps, "copies": copies}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="config-1 step only (no config0/prefill/decode_step/sharded blocks)")
    ap.add_argument("--workload", choices=("config1", "decode_step", "prefill", "sharded"), default="config1")
    ap.add_argument("--profile-one", default=None, metavar="WBITS,M,K,N",
                    help="a few eager launches of one layer shape (small case for ncu)")
    ap.add_argument("--path", choices=("auto", "gemv", "gemm", "tcdec"), default="auto",
                    help="with --profile-one: force the decode, prefill or small-batch tensor-core kernel")
    args = ap.parse_args()
    if args.profile_one:
        return run_profile_one(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "sharded":
        return run_sharded(args)
    if args.workload == "decode_step":
        return run_decode_step(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
