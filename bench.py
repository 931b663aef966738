#!/usr/bin/env python
"""INT4 dequant-GEMV benchmark on B200, and the reference's CPU path beside it.

Workload, one step: every Llama-3.2-1B linear at M=1 in model order -- 16
layers x (q_proj 2048->2048, k_proj / v_proj 2048->512, o_proj 2048->2048,
gate_proj / up_proj 2048->8192, down_proj 8192->2048) + lm_head 2048->128256
= 113 fused INT4 GEMVs (group 128) over distinct weights, seeded per layer
(seed 1000*layer + shape index, lm_head layer 16), W ~ N(0, 0.02), x ~ N(0, 1).
The step streams 658,160,128 algorithmic bytes (sum of K*N/2 + 4*(K/128)*N +
2*M*K + 2*M*N), more than 2x the 126 MB L2, so every step reads its weights
from HBM (no L2 flush needed).

  value      whole-job GB/s with inputs resident in HBM: one CUDA graph of the
             113 int4_linear_out calls replayed `--steps` times, CUDA events on
             the replay stream, max over ranks.
  e2e        the same step through the public API with host buffers: H2D copy
             of the step's x vectors from pinned memory, the 113 calls (graph
             replay), D2H copy of the 113 outputs, all inside the timed region.
  roofline   the GEMV kernel (every launch in the timed region is one): bytes of
             the step / its device time against the measured HBM copy peak.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With --gpus N > 1 (one process per GPU under torchrun) every rank runs its
own replica of the stream (the decode GEMV path needs no data exchange):
weak scaling, value = total bytes of all ranks / max time over ranks.
--impl reference times the reference's CPU implementation (the oracle port
of llama/quantize.py's v1 forward) on the host cores, on bounded samples.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "llama-efficient-inference_b200")
for _p in (REPO, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "INT4 dequant-GEMV HBM GB/s (% of B200 peak) at M=1–16; 1B decode tokens/sec"
LAYER_SHAPES = [("q_proj", 2048, 2048), ("k_proj", 512, 2048), ("v_proj", 512, 2048), ("o_proj", 2048, 2048),
                ("gate_proj", 8192, 2048), ("up_proj", 8192, 2048), ("down_proj", 2048, 8192)]
LM_HEAD = ("lm_head", 128256, 2048)
FUSED_SHAPES = [("qkv_fused", 3072, 2048), ("gate_up_fused", 16384, 2048)]  # the fused decode step's linears
N_LAYERS = 16
GROUP = 128
L2_BYTES = 126 * 2 ** 20


def stream_shapes():
    """(name, N, K, seed) for the 113 GEMVs of one decode step, in model order."""
    out = []
    for layer in range(N_LAYERS):
        for idx, (name, N, K) in enumerate(LAYER_SHAPES):
            out.append((f"layers.{layer}.{name}", N, K, 1000 * layer + idx))
    out.append((LM_HEAD[0], LM_HEAD[1], LM_HEAD[2], 1000 * N_LAYERS))
    return out


def gemv_bytes(N: int, K: int, M: int) -> int:
    return K * N // 2 + 4 * (K // GROUP) * N + 2 * M * K + 2 * M * N


def workload_config(M: int, world: int) -> dict:
    """The `config` of both arms' JSON lines (the same workload, the same keys)."""
    shapes = stream_shapes()
    return {"workload": "llama3.2-1b int4 g128 decode linears, 16 layers x 7 + lm_head, M=%d" % M,
            "M": M, "gemvs_per_step": len(shapes), "bytes_per_step": sum(gemv_bytes(N, K, M) for _, N, K, _ in shapes),
            "group_size": GROUP, "parallelism": f"replicas x{world}" if world > 1 else "single gpu",
            "l2": "no flush: 658 MB of distinct weights per step > 2x the 126 MB L2",
            "timing": "one CUDA graph of the 113 int4_linear_out calls per step, CUDA events"}


def measured_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# Clock sampling during the timed region (NVML, read-only)
# ---------------------------------------------------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device: torch.device, period_s: float = 0.05):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._thread = None
        self.period = period_s
        try:
            import pynvml

            props = torch.cuda.get_device_properties(device)
            ids = (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
            if not all(isinstance(v, int) for v in ids):  # NVML takes the id as a C string only
                raise TypeError(f"unexpected PCI id fields {ids!r}")
            bus_id = "%08x:%02x:%02x.0" % ids
            pynvml.nvmlInit()
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus_id)
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 -- clocks are reported as unavailable, never guessed
            self.nvml, self.err = None, str(e)

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                self.reasons |= reasons(self.h)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "err", "no nvml")}
        reasons = [name for bit, name in _REASONS.items() if self.reasons & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# Distributed plumbing (one process per GPU; replicas, no data-path collective)
# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int, device):
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index])


def max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# The GPU arm
# ---------------------------------------------------------------------------
class Stream:
    """Quantized weights + static x / y buffers of the 113-GEMV step on one GPU."""

    def __init__(self, device: torch.device, M: int):
        from llama.quantize import QuantizedLinear

        self.device, self.M = device, M
        self.shapes = stream_shapes()
        self.weights = []
        for name, N, K, seed in self.shapes:
            gen = torch.Generator(device=device).manual_seed(seed)
            w = (torch.randn(N, K, generator=gen, device=device) * 0.02).half()
            self.weights.append(QuantizedLinear.quantize_tensor(w, GROUP))
            del w
        xk = sum(M * K for _, _, K, _ in self.shapes)
        yn = sum(M * N for _, N, _, _ in self.shapes)
        gen = torch.Generator(device=device).manual_seed(12345)
        self.x_flat = torch.randn(xk, generator=gen, device=device).half()
        self.y_flat = torch.empty(yn, dtype=torch.float16, device=device)
        self.xs, self.ys = [], []
        xo = yo = 0
        for _, N, K, _ in self.shapes:
            self.xs.append(self.x_flat[xo:xo + M * K].view(M, K))
            self.ys.append(self.y_flat[yo:yo + M * N].view(M, N))
            xo += M * K
            yo += M * N
        self.bytes_per_step = sum(gemv_bytes(N, K, M) for _, N, K, _ in self.shapes)
        torch.cuda.synchronize(device)

    def run_eager(self):
        from llama.int4_gemv import int4_linear_out

        for x, (p, s, z), y in zip(self.xs, self.weights, self.ys):
            int4_linear_out(x, p, s, z, y, GROUP)

    def capture(self):
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(2):
                self.run_eager()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.run_eager()
        torch.cuda.synchronize(self.device)


def time_graph(stream: Stream, steps: int, warmup: int, world: int, sampler=None) -> float:
    dev = stream.device
    for _ in range(warmup):
        stream.graph.replay()
    torch.cuda.synchronize(dev)
    barrier(world, dev)
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        start.record()
        for _ in range(steps):
            stream.graph.replay()
        end.record()
        torch.cuda.synchronize(dev)
    barrier(world, dev)
    return start.elapsed_time(end) / steps


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def time_concurrent(stream: Stream, n_streams: int = 4, reps: int = 50) -> dict:
    """The same 113 independent GEMVs issued round-robin on `n_streams` streams, one CUDA graph with
    parallel branches (int4_linear_out, each stream with a split-K workspace of its own): device time per
    step, GB/s, fraction of the measured HBM peak."""
    from llama.int4_gemv import int4_linear_out

    dev = stream.device
    sides = [torch.cuda.Stream(dev) for _ in range(n_streams)]
    wss = [torch.zeros(16 << 20, dtype=torch.uint8, device=dev) for _ in range(n_streams)]
    order = sorted(range(len(stream.shapes)), key=lambda i: -gemv_bytes(*stream.shapes[i][1:3], stream.M))

    def run():
        main = torch.cuda.current_stream(dev)  # the capturing stream inside graph capture: the branches fork from it
        for s_ in sides:
            s_.wait_stream(main)
        for j, i in enumerate(order):  # largest first, dealt round-robin
            with torch.cuda.stream(sides[j % n_streams]):
                p, s, z = stream.weights[i]
                int4_linear_out(stream.xs[i], p, s, z, stream.ys[i], GROUP, workspace=wss[j % n_streams])
        for s_ in sides:
            main.wait_stream(s_)

    us = _graph_us(run, 1, dev, reps=reps)
    gbps = stream.bytes_per_step / (us * 1e-6) / 1e9
    return {"streams": n_streams, "ms_per_step": round(us / 1e3, 4), "GBps": round(gbps, 1),
            "frac": round(gbps / measured_peak()[0], 4),
            "how": "the step's 113 GEMVs are independent (each its own x): issued largest first, round-robin on "
                   f"{n_streams} streams of one CUDA graph"}


def time_grouped(stream: Stream, reps: int = 50) -> dict:
    """The same 113 independent GEMVs as one persistent launch (llama.int4_gemv.GroupedGemv,
    li4_int4_linear_grouped): device time per step, GB/s, fraction of the measured HBM peak, and the
    largest difference from the 113-launch step's outputs (the order of the fp32 sums differs)."""
    from llama.int4_gemv import GroupedGemv

    dev = stream.device
    if any(stream.M * K * 2 > 32768 for _, _, K, _ in stream.shapes):
        return {"unavailable": f"M={stream.M}: x of a problem above the grouped kernel's 32 KB staging"}
    stream.graph.replay()
    torch.cuda.synchronize(dev)
    y_step = stream.y_flat.clone()
    grouped = GroupedGemv([(stream.xs[i], *stream.weights[i], stream.ys[i]) for i in range(len(stream.shapes))])
    us = _graph_us(grouped, 1, dev, reps=reps)
    torch.cuda.synchronize(dev)
    diff = float((stream.y_flat.float() - y_step.float()).abs().max())
    gbps = stream.bytes_per_step / (us * 1e-6) / 1e9
    return {"ms_per_step": round(us / 1e3, 4), "GBps": round(gbps, 1), "frac": round(gbps / measured_peak()[0], 4),
            "ranges": grouped.units, "max_abs_diff_vs_step": diff,
            "how": "the step's 113 GEMVs are independent (each its own x): one persistent launch streams them all, "
                   "their 16-row tiles cut into per-CTA ranges of equal weight bytes, each warp's tiles through one "
                   "register ring"}


def time_e2e(stream: Stream, steps: int, warmup: int, world: int, eager: bool = False):
    """H2D x (pinned) -> 113 calls -> D2H y (pinned), every step inside the timed region."""
    dev = stream.device
    hx = torch.empty(stream.x_flat.shape, dtype=torch.float16, pin_memory=True)
    hx.copy_(stream.x_flat.cpu())
    hy = torch.empty(stream.y_flat.shape, dtype=torch.float16, pin_memory=True)

    def step():
        stream.x_flat.copy_(hx, non_blocking=True)
        if eager:
            stream.run_eager()
        else:
            stream.graph.replay()
        hy.copy_(stream.y_flat, non_blocking=True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world, dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize(dev)
    barrier(world, dev)
    return start.elapsed_time(end) / steps, hx.numel() * 2, hy.numel() * 2


def _graph_us(run, copies: int, dev, reps: int = 7) -> float:
    """Device time per launch of a CUDA graph of `copies` back-to-back launches (run() issues them),
    median of `reps` replays, CUDA events on the replay stream."""
    run()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    g.replay()
    torch.cuda.synchronize(dev)
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize(dev)
        times.append(a.elapsed_time(b) / copies)
    del g
    return statistics.median(times) * 1e3


SWEEP_M = (1, 2, 4, 8, 16)
REFERENCE_M = (1, 8, 16)
PER_SHAPE = LAYER_SHAPES + [LM_HEAD]


def load_reference_int4_gemv():
    """The reference's own llama/int4_gemv.py (Triton), from the unmodified copy that
    baseline/stage_reference.py puts in baseline/_ref, loaded by file path as the reference's
    int4_linear_fn does.  Returns (module, None) or (None, why)."""
    import importlib.util

    path = os.path.join(REPO, "baseline", "_ref", "llama", "int4_gemv.py")
    if not os.path.exists(path):
        return None, "baseline/_ref/llama/int4_gemv.py is absent (run baseline/stage_reference.py)"
    try:
        spec = importlib.util.spec_from_file_location("reference_int4_gemv", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod, None
    except Exception as e:  # noqa: BLE001 -- reported, never substituted
        return None, f"import failed: {type(e).__name__}: {e}"[:200]


def per_shape(stream: Stream, peak: float, reference=None):
    """Configuration 2: every distinct shape of the step (7 layer shapes + lm_head) at M in {1, 2, 4, 8, 16},
    each a CUDA graph of back-to-back int4_linear_out launches over rotating weight copies totalling
    > 3x L2 (weights stream from HBM), device time per launch: us, GB/s of the algorithmic bytes,
    fraction of the measured HBM peak, and the kernel the dispatcher ran.  With the reference's own
    Triton int4_linear (`reference`), the same graphs through it at M in {1, 8, 16}."""
    from llama import _native
    from llama.int4_gemv import int4_linear_out

    dev = stream.device
    out = {}
    for name, N, K in PER_SHAPE:
        idx = next(i for i, sh in enumerate(stream.shapes) if sh[0].split(".")[-1] == name)
        p, s, z = stream.weights[idx]
        copies = max(2, 3 * L2_BYTES // gemv_bytes(N, K, 0) + 1)
        ws = [(p, s, z)] + [(p.clone(), s.clone(), z.clone()) for _ in range(copies - 1)]
        gen = torch.Generator(device=dev).manual_seed(N + K)
        rec = {"N": N, "K": K, "launches_per_graph": copies}
        for M in SWEEP_M:
            x = torch.randn(M, K, generator=gen, device=dev).half()
            y = torch.empty(M, N, dtype=torch.float16, device=dev)

            def run():
                for pi, si, zi in ws:
                    int4_linear_out(x, pi, si, zi, y, GROUP)

            us = _graph_us(run, copies, dev)
            gbps = gemv_bytes(N, K, M) / (us * 1e-6) / 1e9
            plan = _native.plan(M, N, K, GROUP)
            rec[f"M{M}"] = {"us": round(us, 2), "GBps": round(gbps, 1), "frac": round(gbps / peak, 4),
                            "kernel": plan["kernel"], "split": plan["split"]}
            if reference is not None and M in REFERENCE_M:
                def run_ref():
                    for pi, si, zi in ws:
                        reference.int4_linear(x, pi, si, zi, GROUP)

                try:
                    rus = _graph_us(run_ref, copies, dev)
                    rg = gemv_bytes(N, K, M) / (rus * 1e-6) / 1e9
                    rec[f"M{M}"]["reference_gpu"] = {"us": round(rus, 2), "GBps": round(rg, 1),
                                                     "frac": round(rg / peak, 4)}
                except Exception as e:  # noqa: BLE001 -- recorded beside the number it replaces
                    rec[f"M{M}"]["reference_gpu"] = {"error": f"{type(e).__name__}: {e}"[:160]}
        out[name] = rec
        del ws
        torch.cuda.empty_cache()
    return out


def reference_step(stream: Stream, reference, steps: int = 50) -> dict:
    """The 113-GEMV step through the reference's Triton int4_linear (one CUDA graph of the 113 calls in
    model order, as the repo's step): ms per step and GB/s, on the same B200 and the same weights."""
    dev = stream.device

    def run():
        for x, (p, s, z) in zip(stream.xs, stream.weights):
            reference.int4_linear(x, p, s, z, GROUP)

    us = _graph_us(run, 1, dev, reps=steps)
    return {"ms_per_step": round(us / 1e3, 4), "GBps": round(stream.bytes_per_step / (us * 1e-6) / 1e9, 1),
            "impl": "reference llama/int4_gemv.py int4_linear (Triton), unmodified"}


PREFILL_SHAPES = [("q_proj", 2048, 2048), ("k_proj", 512, 2048), ("gate_proj", 8192, 2048), ("down_proj", 2048, 8192),
                  ("lm_head", 128256, 2048)]


def prefill_gemm(stream: Stream) -> dict:
    """The tensor-core INT4 GEMM (li4_int4_gemm) on the prefill linears: M = 512 (a 512-token prompt at batch
    1) and 8192 (batch 16), a CUDA graph of back-to-back launches per shape: us, TFLOP/s, fraction of the
    measured dense bf16 peak, and beside it the path it replaces, the exact dequantize kernel + cuBLAS fp16
    (F.linear), timed the same way."""
    import torch.nn.functional as F

    from llama.int4_gemv import int4_gemm
    from llama.quantize import QuantizedLinear

    dev = stream.device
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            tf_peak = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        tf_peak = 1590.0
    out = {"peak_tflops": tf_peak}
    for M in (512, 8192):
        for name, N, K in PREFILL_SHAPES:
            if name == "lm_head" and M > 512:
                continue
            idx = next(i for i, sh in enumerate(stream.shapes) if sh[0].split(".")[-1] == name)
            p, s, z = stream.weights[idx]
            x = torch.randn(M, K, device=dev).half()
            us = _graph_us(lambda: int4_gemm(x, p, s, z, GROUP), 1, dev, reps=10)
            us_ref = _graph_us(lambda: F.linear(x, QuantizedLinear.dequantize_packed(p, s, z, GROUP)), 1, dev, reps=10)
            tflops = 2 * M * N * K / (us * 1e-6) / 1e12
            out[f"{name}/M{M}"] = {"us": round(us, 1), "TFLOPs": round(tflops, 1), "frac": round(tflops / tf_peak, 4),
                                   "dequant_cublas_us": round(us_ref, 1)}
    return out


def per_kernel_roofline(stream: Stream, peak: float) -> dict:
    """The step split by kernel: a graph of the step's launches of one kernel family (the layer GEMVs on
    the streaming-warp kernel, lm_head on the tile kernel), device time per launch, algorithmic bytes per
    launch, GB/s and fraction of the measured HBM peak."""
    from llama import _native
    from llama.int4_gemv import int4_linear_out

    dev = stream.device
    groups = {}
    for i, (name, N, K, _) in enumerate(stream.shapes):
        groups.setdefault(_native.plan(stream.M, N, K, GROUP)["symbol"], []).append(i)
    out = {}
    for sym, idx in groups.items():
        def run():
            for i in idx:
                p, s, z = stream.weights[i]
                int4_linear_out(stream.xs[i], p, s, z, stream.ys[i], GROUP)

        us = _graph_us(run, len(idx), dev, reps=20)
        nbytes = sum(gemv_bytes(stream.shapes[i][1], stream.shapes[i][2], stream.M) for i in idx) / len(idx)
        gbps = nbytes / (us * 1e-6) / 1e9
        out[sym] = {"launches_per_step": len(idx), "bytes_per_launch": int(nbytes), "us_per_launch": round(us, 3),
                    "GBps": round(gbps, 1), "frac": round(gbps / peak, 4)}
    return out


def profile_shape(a):
    """--profile-shape NAME: `--launches` eager launches of one shape (a small case for ncu captures)."""
    from llama.int4_gemv import int4_linear_out
    from llama.quantize import QuantizedLinear

    shapes = {n: (N, K) for n, N, K in LAYER_SHAPES + FUSED_SHAPES + [LM_HEAD]}
    N, K = shapes[a.profile_shape]
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
    p, s, z = QuantizedLinear.quantize_tensor(w, GROUP)
    del w
    x = torch.randn(a.m, K, generator=gen, device=dev).half()
    y = torch.empty(a.m, N, dtype=torch.float16, device=dev)
    kernel = {"auto": 0, "stream": 3, "tile": 4, "bulk": 5, "slab": 6, "ring": 8}[a.kernel]
    for _ in range(a.launches):
        int4_linear_out(x, p, s, z, y, GROUP, kernel=kernel)
    torch.cuda.synchronize(dev)
    print(json.dumps({"profile_shape": a.profile_shape, "N": N, "K": K, "M": a.m, "launches": a.launches,
                      "kernel": a.kernel, "bytes_per_launch": gemv_bytes(N, K, a.m)}))


def profile_grouped(a):
    """--profile-grouped: `--launches` grouped launches of the 113-GEMV workload (a case for ncu captures of
    gemv_grouped_kernel; 658 MB of weights on the device)."""
    from llama.int4_gemv import GroupedGemv

    dev = torch.device("cuda", 0)
    stream = Stream(dev, a.m)
    grouped = GroupedGemv([(stream.xs[i], *stream.weights[i], stream.ys[i]) for i in range(len(stream.shapes))])
    for _ in range(a.launches):
        grouped()
    torch.cuda.synchronize(dev)
    print(json.dumps({"profile_grouped": len(stream.shapes), "M": a.m, "launches": a.launches, "ranges": grouped.units,
                      "bytes_per_launch": stream.bytes_per_step}))


def profile_gemm(a):
    """--profile-gemm M,N,K: `--launches` launches of the tensor-core INT4 GEMM on one weight set (a small
    case for ncu captures of int4_gemm_kernel)."""
    from llama.int4_gemv import int4_gemm
    from llama.quantize import QuantizedLinear

    M, N, K = (int(v) for v in a.profile_gemm.split(","))
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
    p, s, z = QuantizedLinear.quantize_tensor(w, GROUP)
    del w
    x = torch.randn(M, K, generator=gen, device=dev).half()
    for _ in range(a.launches):
        int4_gemm(x, p, s, z, GROUP)
    torch.cuda.synchronize(dev)
    print(json.dumps({"profile_gemm": [M, N, K], "launches": a.launches, "flops_per_launch": 2 * M * N * K}))


def profile_attention(a):
    """--profile-attention BS: `--launches` decode-attention launches (Llama-3.2-1B heads: 32 query /
    8 KV, head_dim 64) at position 512 of a 640-row fp16 cache of batch BS, an L2 flush (256 MB
    write) before each -- the small case for ncu captures of li4_decode_attention."""
    from llama import fused

    dev = torch.device("cuda", 0)
    bs, S, H, KV, HD = a.profile_attention, 640, 32, 8, 64
    gen = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(bs, H * HD, generator=gen, device=dev).half()
    ck = torch.randn(bs, S, KV, HD, generator=gen, device=dev).half()
    cv = torch.randn(bs, S, KV, HD, generator=gen, device=dev).half()
    out = torch.empty_like(q)
    pos = torch.tensor([512], dtype=torch.long, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(a.launches):
        flush.zero_()
        fused.decode_attention(q, ck, cv, pos, out, H, KV)
    torch.cuda.synchronize(dev)
    print(json.dumps({"profile_attention": bs, "launches": a.launches, "kv_bytes": 2 * bs * 513 * KV * HD * 2}))


def roofline_traffic(stream: "Stream"):
    """DRAM bytes per step: the sum over the step's launches of the per-launch DRAM bytes that ncu measured
    for the same kernel on the same shape (profiles/gemv_dram_per_launch.json, one small capture per shape);
    None when the file does not cover a kernel / shape the dispatcher now picks."""
    from llama import _native

    path = os.path.join(REPO, "profiles", "gemv_dram_per_launch.json")
    try:
        with open(path) as f:
            table = json.load(f)["launches"]
    except (OSError, ValueError, KeyError):
        return None
    total = 0
    for _, N, K, _ in stream.shapes:
        key = f"{_native.plan(stream.M, N, K, GROUP)['symbol']}/M{stream.M}/N{N}/K{K}"
        if key not in table:
            return None
        total += table[key]
    return int(total)


# ---------------------------------------------------------------------------
# The CPU arm: the reference's v1 path as restated by the oracle
# ---------------------------------------------------------------------------
class CpuStream:
    """Host copies of a stream's weights (random INT4 data; CPU cost is data-independent)."""

    def __init__(self, M: int, seed: int = 0):
        rng = np.random.default_rng(seed)
        self.M = M
        self.shapes = stream_shapes()
        self.items = []
        for name, N, K, _ in self.shapes:
            packed = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
            scale = rng.uniform(0.002, 0.004, size=(N, K // GROUP)).astype(np.float16)
            zero = rng.integers(0, 16, size=(N, K // GROUP)).astype(np.float16)
            x = rng.standard_normal((M, K)).astype(np.float16)
            self.items.append((name, N, K, x, packed, scale, zero))

    def run_rows(self, start_row: int, n_rows: int):
        """Process `n_rows` output rows of the stream starting at global row `start_row` (wrapping)."""
        from oracle import oracle

        total = sum(it[1] for it in self.items)
        done_bytes = 0
        row = start_row % total
        remaining = n_rows
        while remaining > 0:
            acc = 0
            for name, N, K, x, packed, scale, zero in self.items:
                if row < acc + N:
                    r0 = row - acc
                    r1 = min(N, r0 + remaining)
                    oracle.linear(x, packed[r0:r1], scale[r0:r1], zero[r0:r1], GROUP)
                    rows = r1 - r0
                    done_bytes += rows * (K // 2 + 4 * (K // GROUP) + 2 * self.M) + \
                        2 * self.M * K * rows // N
                    remaining -= rows
                    row = (row + rows) % total
                    break
                acc += N
        return done_bytes


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_rate(cs: CpuStream, seconds: float):
    """Run the stream on the CPU for about `seconds`; returns (GB/s, rows, bytes, elapsed)."""
    t0 = time.perf_counter()
    nbytes = rows = 0
    chunk = 4096
    while time.perf_counter() - t0 < seconds:
        nbytes += cs.run_rows(rows, chunk)
        rows += chunk
    dt = time.perf_counter() - t0
    return nbytes / dt / 1e9, rows, nbytes, dt


def reference_cpu_child(a):
    """Child process (`--reference-cpu-child`): the reference's own CPU path, imported from the unmodified
    copy in baseline/_ref (its package is also named `llama`, hence a process of its own).
      gemv    QuantizedLinear.forward with the default DEQUANT_IMPL "v1" (dequantize_packed + fp16
              F.linear, llama/quantize.py:128-147) on CPU tensors over the 113-GEMV step in model order,
              on all host threads and on one; GB/s of algorithmic bytes over a bounded sample.
      decode  one Llama-3.2-1B INT4 decode step of the reference model (llama/model.py) at batch 1,
              position 512, with its .cuda() cache allocation (llama/model.py:205-220) stubbed to stay on
              the host; its 113 linears are the reference's QuantizedLinear with zero buffers (the cost
              of the v1 path does not depend on the values)."""
    ref = os.path.join(REPO, "baseline", "_ref")
    sys.path[:] = [ref] + [q for q in sys.path if os.path.abspath(q) not in (PKG_DIR, REPO)]
    out = {}
    try:
        from llama import quantize as Q  # the reference's own module
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"unavailable": f"reference import failed: {type(e).__name__}: {e}"[:200]}), flush=True)
        return
    rng = torch.Generator().manual_seed(0)
    mods = {}
    for name, N, K in PER_SHAPE:
        m = Q.QuantizedLinear(K, N, GROUP)
        m.packed_weight.copy_(torch.randint(0, 256, (N, K // 2), generator=rng, dtype=torch.uint8))
        m.scale.copy_((torch.rand(N, K // GROUP, generator=rng) * 0.002 + 0.002).half())
        m.zero_point.copy_(torch.randint(0, 16, (N, K // GROUP), generator=rng).half())
        mods[name] = m
    xs = {K: torch.randn(1, K, generator=rng).half() for _, _, K in PER_SHAPE}
    order = [sh[0].split(".")[-1] for sh in stream_shapes()]
    Q.set_dequant_impl("v1")
    all_threads = cpu_threads()
    gemv = {}
    for threads in (all_threads, 1):
        torch.set_num_threads(threads)
        with torch.no_grad():
            mods["q_proj"](xs[2048])  # warm-up
            t0, nbytes, calls = time.perf_counter(), 0, 0
            while time.perf_counter() - t0 < a.ref_cpu_seconds:
                name = order[calls % len(order)]
                m = mods[name]
                m(xs[m.in_features])
                nbytes += gemv_bytes(m.out_features, m.in_features, 1)
                calls += 1
            dt = time.perf_counter() - t0
        gemv[f"threads_{threads}"] = {"GBps": round(nbytes / dt / 1e9, 3), "cores": threads,
                                      "sample": f"{calls} GEMV calls ({calls / len(order):.2f} decode steps) in "
                                                f"{dt:.1f} s"}
    out["gemv"] = gemv
    torch.set_num_threads(all_threads)
    try:
        from torch import nn

        from llama.model import Llama, ModelArgs
        saved = (torch.Tensor.cuda, nn.Linear.reset_parameters, nn.Embedding.reset_parameters)
        torch.Tensor.cuda = lambda self, *args, **kw: self
        nn.Linear.reset_parameters = lambda self: None  # allocation only: every nn.Linear is replaced below
        nn.Embedding.reset_parameters = lambda self: None
        try:
            torch.set_default_dtype(torch.float16)
            model = Llama(ModelArgs(max_batch_size=1, max_seq_len=640))
        finally:
            torch.set_default_dtype(torch.float32)
            torch.Tensor.cuda, nn.Linear.reset_parameters, nn.Embedding.reset_parameters = saved
        model.eval()
        nn.init.zeros_(model.tok_embeddings.weight)
        # the 113 nn.Linear -> the reference's QuantizedLinear, as its quantize_model does, with the packed
        # buffers left at zero instead of quantizing 1.2 B weights on the host first
        for name, mod in [(n, m) for n, m in model.named_modules() if isinstance(m, nn.Linear)]:
            parent, child = name.rsplit(".", 1) if "." in name else ("", name)
            setattr(model.get_submodule(parent) if parent else model, child,
                    Q.QuantizedLinear(mod.in_features, mod.out_features, GROUP))
        tok = torch.randint(0, 128256, (1, 1), generator=rng)
        times = []
        with torch.no_grad():
            for i in range(a.ref_cpu_decode_steps + 1):
                t0 = time.perf_counter()
                model(tok, 512 + i)
                times.append(time.perf_counter() - t0)
        ms = statistics.median(times[1:]) * 1e3
        out["decode"] = {"bs": 1, "position": 512, "steps_timed": a.ref_cpu_decode_steps, "ms_per_step": round(ms, 1),
                         "tok_s": round(1e3 / ms, 3), "cores": all_threads,
                         "note": "KV cache rows 0..511 left zero (no prefill); the step's cost does not depend "
                                 "on their values"}
    except Exception as e:  # noqa: BLE001
        out["decode"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    print(json.dumps(out), flush=True)


def reference_cpu(a) -> dict:
    """Run reference_cpu_child in a child process; its JSON, or why it is unavailable."""
    import subprocess

    if not os.path.exists(os.path.join(REPO, "baseline", "_ref", "llama", "quantize.py")):
        return {"unavailable": "baseline/_ref/llama is absent (run baseline/stage_reference.py)"}
    cmd = [sys.executable, os.path.abspath(__file__), "--reference-cpu-child", "--ref-cpu-seconds",
           str(a.ref_cpu_seconds), "--ref-cpu-decode-steps", str(a.ref_cpu_decode_steps)]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
        return json.loads(r.stdout.strip().splitlines()[-1])
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}


def run_reference(a):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle

    threads = cpu_threads()
    oracle.set_threads(threads)
    cs = CpuStream(a.m)
    # calibrate, then size each step's sample so the whole run stays within ~2 minutes
    rate, _, _, _ = cpu_rate(cs, 2.0)
    budget_s = 90.0
    total_rows = sum(it[1] for it in cs.items)
    bytes_per_row = sum(gemv_bytes(N, K, a.m) for _, N, K, *_ in cs.items) / sum(it[1] for it in cs.items)
    rows_per_step = max(64, int(rate * 1e9 * budget_s / (a.steps + a.warmup) / bytes_per_row))
    rows_per_step = min(rows_per_step, total_rows)
    row = 0
    for _ in range(a.warmup):
        cs.run_rows(row, rows_per_step)
        row += rows_per_step
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(a.steps):
        nbytes += cs.run_rows(row, rows_per_step)
        row += rows_per_step
    dt = time.perf_counter() - t0
    gbps = nbytes / dt / 1e9
    sample = (f"{rows_per_step} output rows of the 113-GEMV stream per step (model order, wrapping; "
              f"{total_rows} rows = one full decode step)")
    line = {
        "metric": METRIC, "value": round(gbps, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt / a.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (random INT4 weights, N(0,1) x)",
        "config": workload_config(a.m, world),
        "cpu_baseline": {"value": round(gbps, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbps, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "world_size": world,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Decode: Llama-3.2-1B, all 113 linears INT4, one CUDA graph per step
# ---------------------------------------------------------------------------
def build_decode_model(device, bs: int, max_seq_len: int, seed: int = 0):
    """Random-init Llama-3.2-1B (N(0, 0.02) weights, output tied to the embeddings), quantized INT4 g128."""
    from llama import quantize
    from llama.model import Llama, ModelArgs

    args = ModelArgs(max_batch_size=bs, max_seq_len=max_seq_len)
    torch.manual_seed(seed)
    torch.set_default_dtype(torch.float16)
    try:
        with torch.device(device):
            model = Llama(args)
    finally:
        torch.set_default_dtype(torch.float32)
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if name.endswith("norm.weight"):
                prm.fill_(1.0)
            else:
                prm.normal_(0.0, 0.02)
        model.output.weight = model.tok_embeddings.weight  # tied, as in the released checkpoint
    model.eval()
    quantize.quantize_model(model, GROUP)
    quantize.set_dequant_impl("v4")
    return model


def run_decode(device, bs: int, prompt_len: int, gen: int, reps: int, world: int, fused: bool = True,
               program: bool = False):
    """Prefill + `gen` greedy decode steps replayed from one graph; timings are the max over ranks.
    fused: the step as llama.fused kernels (five launches per block), else the module-by-module step."""
    from llama.generation import DecodeGraph

    gen_t = torch.Generator(device=device).manual_seed(1)
    tokens = torch.randint(0, 128256, (bs, prompt_len), generator=gen_t, device=device)
    check_steps = min(16, gen - 1)
    ref = None
    if world > 1:
        # the same seeded model unsharded (TP = 1) on this rank: its greedy tokens and first-step logits
        # are what the sharded step must reproduce.  toks[0] is the token after the prefill, toks[i + 1]
        # the output of decode step i (and the input of step i + 1).
        model = build_decode_model(device, bs, prompt_len + gen)
        if fused:
            model.enable_fused_decode(program=program)
        g1 = DecodeGraph(model, bs)
        with torch.no_grad():
            g1.start(tokens)
            toks, logits1 = [g1.tok.clone()], None
            for i in range(check_steps):
                g1.replay()
                if i == 0:
                    logits1 = g1.logits.float().clone()
                toks.append(g1.tok.clone())
        torch.cuda.synchronize(device)
        ref = (torch.cat(toks, 1), logits1)
        del g1, model
        torch.cuda.empty_cache()
    model = build_decode_model(device, bs, prompt_len + gen)
    if world > 1:
        from llama.tp import shard_model

        shard_model(model)
    if fused:
        model.enable_fused_decode(program=program)
    torch.cuda.synchronize(device)
    graph = DecodeGraph(model, bs)
    steps, prefills, e2es = [], [], []
    parity = None
    if ref is not None:
        # Teacher-forced: every step of the sharded model gets the TP = 1 run's input token, so each
        # step's greedy token is compared on identical inputs (one near-tie flipped by the rounding of
        # the fp16 partial sums then changes one token, not every token after it).
        with torch.no_grad():
            graph.start(tokens)
            toks, logits1 = [graph.tok.clone()], None
            for i in range(check_steps):
                graph.tok.copy_(ref[0][:, i:i + 1])
                graph.replay()
                if i == 0:
                    logits1 = graph.logits.float().clone()
                toks.append(graph.tok.clone())
        torch.cuda.synchronize(device)
        tp_toks = torch.cat(toks, 1)
        agree = float((tp_toks == ref[0]).float().mean())
        full = ref[1].reshape(bs, -1)
        local = logits1.reshape(bs, -1)
        if local.shape[-1] != full.shape[-1]:  # the fused TP step keeps its vocabulary shard of the logits
            import torch.distributed as dist

            r0 = dist.get_rank() * local.shape[-1]
            full = full[:, r0:r0 + local.shape[-1]]
        rel = float((local - full).abs().max() / full.abs().max())
        import torch.distributed as dist

        t = torch.tensor([agree, -rel], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)  # the worst rank
        parity = {"tokens_match_tp1": bool(t[0].item() == 1.0), "tp1_token_agreement": round(float(t[0].item()), 4),
                  "tp1_first_step_logits_rel_err": float(-t[1].item()), "steps_checked": check_steps,
                  "tp1_check": "teacher-forced: the prefill token and each step's greedy token on the TP=1 run's inputs"}
    for rep in range(reps + 1):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(gen + 1)]
        barrier(world, device)
        ev[0].record()
        with torch.no_grad():
            graph.start(tokens)
        ev[1].record()
        for i in range(gen - 1):
            graph.replay()
            ev[i + 2].record()
        torch.cuda.synchronize(device)
        if rep == 0:
            continue  # warm-up
        prefills.append(ev[0].elapsed_time(ev[1]))
        steps += [ev[i].elapsed_time(ev[i + 1]) for i in range(1, gen)]
        e2es.append(ev[0].elapsed_time(ev[gen]))
    step_ms = max_over_ranks(statistics.median(steps), world, device)
    e2e_ms = max_over_ranks(statistics.median(e2es), world, device)
    prefill_ms = max_over_ranks(statistics.median(prefills), world, device)
    q = statistics.quantiles(steps, n=10)
    path = getattr(getattr(model, "_fused", None), "last_path", None)
    del graph, model
    torch.cuda.empty_cache()
    row = {"bs": bs, "prompt": prompt_len, "generated": gen, "tp": world, "reps": reps,
            "step": ("one-launch program (llama.program)" if path == "program" else "fused launches (llama.fused)")
            if fused else "unfused (module by module)",
            "decode_ms_per_step": round(step_ms, 4), "decode_p10_ms": round(q[0], 4), "decode_p90_ms": round(q[-1], 4),
            "decode_tok_s": round(bs / (step_ms * 1e-3), 1), "prefill_ms": round(prefill_ms, 3),
            "e2e_tok_s": round(bs * gen / (e2e_ms * 1e-3), 1)}
    if parity is not None:
        row.update(parity)
    return row


def log(msg: str) -> None:
    """Phase markers on stderr (the JSON line alone goes to stdout)."""
    print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def run_gpu(a):
    world, rank, local = dist_setup(a.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if a.only_decode:
        rows = []
        for bs in a.decode_bs:
            log(f"decode: Llama-3.2-1B INT4, bs={bs}, {a.decode_prompt}-token prefill, {a.decode_gen} steps, tp={world}")
            rows.append(run_decode(dev, bs, a.decode_prompt, a.decode_gen, a.decode_reps, world,
                                   program=a.decode_program))
            if a.decode_unfused:
                rows.append(run_decode(dev, bs, a.decode_prompt, a.decode_gen, a.decode_reps, world, fused=False))
        if rank == 0:
            print(json.dumps({"metric": "Llama-3.2-1B INT4 decode tokens/s", "n_gpus": world, "decode": rows}),
                  flush=True)
        return
    log("building the quantized weights of the 113-GEMV stream")
    stream = Stream(dev, a.m)
    log("capturing the step graph")
    stream.capture()
    log("clock sampler")
    sampler = ClockSampler(dev)
    log(f"timing {a.steps} graph replays")
    ms = time_graph(stream, a.steps, a.warmup, world, sampler)
    ms_max = max_over_ranks(ms, world, dev)
    log("e2e timing")
    e2e_steps = max(3, min(a.steps, 2000))
    e2e_ms, h2d, d2h = time_e2e(stream, e2e_steps, max(3, a.warmup), world)
    e2e_ms = max_over_ranks(e2e_ms, world, dev)
    eager_steps = max(3, min(a.steps, 200))
    eager_ms, _, _ = time_e2e(stream, eager_steps, 3, world, eager=True)
    eager_ms = max_over_ranks(eager_ms, world, dev)

    decode = []
    if not a.no_decode:
        for bs in a.decode_bs:
            log(f"decode: Llama-3.2-1B INT4, bs={bs}, {a.decode_prompt}-token prefill, {a.decode_gen} steps, tp={world}")
            decode.append(run_decode(dev, bs, a.decode_prompt, a.decode_gen, a.decode_reps, world,
                                     program=a.decode_program))
            if a.decode_unfused:
                decode.append(run_decode(dev, bs, a.decode_prompt, a.decode_gen, a.decode_reps, world, fused=False))
    peak, peak_kind = measured_peak()
    kernels, shapes_cfg2, ref_step, ref_why, concurrent, gemm = None, None, None, None, None, None
    grouped = None
    if rank == 0:
        log("per-kernel timing of the step")
        kernels = per_kernel_roofline(stream, peak)
        log("the step's independent GEMVs on 4 streams")
        concurrent = time_concurrent(stream)
        if a.m <= 8:
            log("the step's independent GEMVs as one grouped launch")
            grouped = time_grouped(stream)
        log("prefill GEMM (tensor cores) against dequantize + cuBLAS")
        gemm = prefill_gemm(stream)
        reference = None
        if not a.no_reference_gpu:
            reference, ref_why = load_reference_int4_gemv()
        if not a.no_per_shape:
            log("configuration 2: every shape at M in 1, 2, 4, 8, 16" + (" (and the reference's Triton kernel)"
                                                                          if reference else ""))
            shapes_cfg2 = per_shape(stream, peak, reference)
        if reference is not None:
            log("the 113-GEMV step through the reference's Triton int4_linear")
            try:
                ref_step = reference_step(stream, reference)
            except Exception as e:  # noqa: BLE001 -- recorded, never substituted
                ref_why = f"{type(e).__name__}: {e}"[:200]
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        from oracle import oracle

        log("CPU baseline (oracle port of the reference path)")
        threads = cpu_threads()
        oracle.set_threads(threads)
        cs = CpuStream(a.m)
        gbps, rows, nbytes, dt = cpu_rate(cs, a.cpu_seconds)
        total_rows = sum(it[1] for it in cs.items)
        cpu = {"value": round(gbps, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{rows} output rows ({rows / total_rows:.2f} decode steps) of the 113-GEMV stream "
                         f"in {dt:.1f} s"}
        if not a.no_reference_cpu:
            log("the reference's own CPU path (torch v1 GEMVs, one reference-model decode step)")
            cpu["reference_torch"] = reference_cpu(a)
    if rank != 0:
        return
    bps = stream.bytes_per_step
    value = world * bps / (ms_max * 1e-3) / 1e9
    achieved = bps / (ms * 1e-3) / 1e9
    counts = {}
    for _, N, K, _ in stream.shapes:
        sym = __import__("llama._native", fromlist=["plan"]).plan(a.m, N, K, GROUP)["symbol"]
        counts[sym] = counts.get(sym, 0) + 1
    kernel_desc = " + ".join(f"{n} {k}" for k, n in sorted(counts.items(), key=lambda kv: -kv[1]))
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_max, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (W ~ N(0,0.02) quantized INT4 g128 by the CUDA quantizer, x ~ N(0,1) fp16)",
        "config": workload_config(a.m, world),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": roofline_traffic(stream),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s",
                     "kernel": f"the step's {len(stream.shapes)} launches ({kernel_desc}, the dispatcher's plans); "
                               "achieved and traffic are per step",
                     "per_kernel": kernels},
        "e2e": {"value": round(world * bps / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 5),
                "path": "pinned H2D x -> graph of 113 int4_linear_out calls -> D2H y"},
        "e2e_eager": {"value": round(world * bps / (eager_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                      "ms_per_step": round(eager_ms, 5),
                      "path": "pinned H2D x -> 113 eager Python int4_linear_out calls -> D2H y"},
        "concurrent": concurrent,
        "grouped": grouped,
        "prefill_gemm": gemm,
        "gpu_launches": len(stream.shapes) * a.steps,
        "clocks": sampler.summary(),
        "cpu_baseline": cpu,
        "per_shape": shapes_cfg2,
        "reference_gpu": ref_step if ref_step is not None else {"unavailable": ref_why or "not run"},
        "decode": decode,
        "gpu": torch.cuda.get_device_name(dev),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--m", type=int, default=1, help="rows of x per GEMV (decode batch), 1..16")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-shape", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's Triton int4_linear (baseline/_ref) on the same GPU")
    ap.add_argument("--no-reference-cpu", action="store_true",
                    help="skip the reference's own torch CPU path (baseline/_ref) in cpu_baseline")
    ap.add_argument("--ref-cpu-seconds", type=float, default=6.0,
                    help="seconds per thread count of the reference's CPU GEMV sample")
    ap.add_argument("--ref-cpu-decode-steps", type=int, default=1,
                    help="timed CPU decode steps of the reference model")
    ap.add_argument("--reference-cpu-child", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--no-decode", action="store_true", help="skip the full-model decode measurement")
    ap.add_argument("--decode-bs", type=int, nargs="+", default=None,
                    help="decode batch sizes (default: 1, 8 and 16 on one GPU, 16 under tensor parallelism)")
    ap.add_argument("--decode-prompt", type=int, default=512)
    ap.add_argument("--decode-gen", type=int, default=128)
    ap.add_argument("--decode-reps", type=int, default=3)
    ap.add_argument("--decode-program", action="store_true",
                    help="run the fused decode step as one persistent launch (llama.program)")
    ap.add_argument("--decode-unfused", action="store_true",
                    help="also time the module-by-module decode step (ATen ops around the INT4 GEMVs)")
    ap.add_argument("--profile-shape", default=None,
                    choices=[n for n, _, _ in LAYER_SHAPES] + [LM_HEAD[0], "qkv_fused", "gate_up_fused"],
                    help="only run --launches launches of one shape (for ncu), no timing")
    ap.add_argument("--profile-attention", type=int, default=0, metavar="BS",
                    help="only run --launches decode-attention launches at batch BS (for ncu), no timing")
    ap.add_argument("--profile-gemm", default=None, metavar="M,N,K",
                    help="only run --launches tensor-core INT4 GEMM launches of one shape (for ncu), no timing")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--profile-grouped", action="store_true",
                    help="run --launches grouped launches of the 113-GEMV workload (for ncu captures)")
    ap.add_argument("--kernel", default="auto", choices=["auto", "stream", "tile", "bulk", "slab", "ring"],
                    help="kernel family for --profile-shape (default: the dispatcher's choice)")
    ap.add_argument("--only-decode", action="store_true",
                    help="only the full-model decode measurement (one JSON line with the decode rows)")
    a = ap.parse_args()
    if a.reference_cpu_child:
        reference_cpu_child(a)
        return
    if a.profile_grouped:
        profile_grouped(a)
        return
    if a.profile_shape:
        profile_shape(a)
        return
    if a.profile_attention:
        profile_attention(a)
        return
    if a.profile_gemm:
        profile_gemm(a)
        return
    if a.warmup < 3:
        a.warmup = 3
    if a.decode_bs is None:
        a.decode_bs = [1, 8, 16] if int(os.environ.get("WORLD_SIZE", "1")) == 1 else [16]
    if a.impl == "reference":
        run_reference(a)
    else:
        run_gpu(a)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 and a.impl != "reference":
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
