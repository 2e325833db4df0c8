#!/usr/bin/env python
"""bench.py -- decode + GEMM throughput of the B200 path.

Default workload (one GPU): the format sweep at M = N = K = 4096.  One step is,
for each stored weight format TF32, BF16, FP8 E4M3 and FP4 E2M1 (A = weights
drawn from N(0, 0.02), per-tensor scale FORMAT_MAX/maxabs for FP8/FP4, B =
FP16 activations from N(0, 1)):
    * the fused decode-in-shared-memory GEMM  D = alpha * decode(A) @ B^T
    * the unfused path: decode kernel to FP16 in HBM, then the tcgen05 GEMM
and the both-quantized case qA @ qB with E4M3 x E4M3 and E2M1 x E2M1 on the
native kind::f8f6f4 tensor-core path; FP32 output, as the reference.  That is
10 GEMMs of 2*4096^3 flops per step.  `value` is whole-job TFLOP/s.

The same JSON line also carries, measured after the timed steps, the
weight-only MLP shapes (W 14336x4096 and 4096x14336, 1-2048 tokens, GB/s
against HBM), the 8192^3 fused FP4 GEMM with FP16 output, and the
16384x53248 E4M3 weight GEMM column-sharded over the N GPUs, every rank ending
with the whole output: the fused kernel's epilogue stores each tile into the
peers' D over NVLink, with the NCCL all-gather variant timed beside it
(strong scaling).

On N GPUs (torchrun) every rank runs the same sweep on its own data (the
sweep has no exchange step): weak scaling, value = all ranks' flops / the
slowest rank's time.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode+GEMM TFLOPS (% tcgen05 peak) and GB/s (% HBM) per format; rel-Frob err"
UNIT = "TFLOP/s"
FORMATS = ["tf32", "bf16", "e4m3", "e2m1"]
FORMAT_MAX = {"e4m3": 448.0, "e2m1": 6.0}


def load_package():
    name = "tensor_bridge_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = os.path.join(ROOT, "tensor-bridge_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---- clocks sampled during the timed region ------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index: int, interval_ms: int = 100):
        # nvidia-smi numbers GPUs physically; map through CUDA_VISIBLE_DEVICES.
        self.interval_ms = interval_ms
        vis = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.gpu = vis[cuda_index].strip() if cuda_index < len(vis) else str(cuda_index)
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", str(self.interval_ms)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, watts, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            try:
                watts.append(float(parts[3]))
            except ValueError:
                pass
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "samples": len(sm),
                "power_w": statistics.median(watts) if watts else None, "reasons": sorted(reasons)}


# ---- distributed plumbing ------------------------------------------------------------------

class Dist:
    def __init__(self, torch, want_gpus: int):
        self.torch = torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist
        else:
            torch.cuda.set_device(0)

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max(self, v: float) -> float:
        if not self.dist:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.dist:
            self.dist.destroy_process_group()


# ---- the format sweep ----------------------------------------------------------------------

class Sweep:
    def __init__(self, torch, tb, M: int, N: int, K: int, seed: int):
        self.torch, self.tb = torch, tb
        self.M, self.N, self.K = M, N, K
        dev = torch.device("cuda")
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        F = tb.Format
        self.fmt = {"tf32": F.TF32, "bf16": F.BF16, "e4m3": F.E4M3, "e2m1": F.E2M1}
        self.a32 = {}
        self.Aq, self.alpha = {}, {}
        amax = torch.zeros(1, dtype=torch.float32, device=dev)
        for i, name in enumerate(FORMATS):
            a = torch.randn(M, K, generator=g, device=dev) * 0.02
            scale = 1.0
            if name in FORMAT_MAX:
                tb.absmax(a, a.numel(), amax)
                m = float(amax.item())
                scale = float(np.float32(FORMAT_MAX[name]) / np.float32(m if m > 0 else 1.0))
            f = self.fmt[name]
            q = torch.empty(tb.stored_bytes(f, M * K), dtype=torch.uint8, device=dev)
            tb.quantize(f, a, q, M * K, scale=scale)
            self.Aq[name] = q
            self.a32[name] = a
            self.alpha[name] = float(np.float32(1.0) / np.float32(scale))
        b = torch.randn(N, K, generator=g, device=dev)
        self.b32 = b
        self.B16 = torch.empty(N * K * 2, dtype=torch.uint8, device=dev)
        tb.quantize(F.F16, b, self.B16, N * K)
        # both-quantized case qA @ qB on kind::f8f6f4: B quantized with its own
        # per-tensor scale; FP4 operands in the tensor core's nibble order
        tb.absmax(b, b.numel(), amax)
        bmax = float(amax.item())
        self.native = {}
        for name, f in (("e4m3", F.E4M3), ("e2m1", F.E2M1_HW)):
            sb = float(np.float32(FORMAT_MAX[name]) / np.float32(bmax))
            sa = float(np.float32(1.0) / np.float32(self.alpha[name]))
            qa = torch.empty(tb.stored_bytes(f, M * K), dtype=torch.uint8, device=dev)
            tb.quantize(f, self.a32[name], qa, M * K, scale=sa)
            qb = torch.empty(tb.stored_bytes(f, N * K), dtype=torch.uint8, device=dev)
            tb.quantize(f, b, qb, N * K, scale=sb)
            self.native[name] = (f, qa, qb, float(np.float32(1.0) / (np.float32(sa) * np.float32(sb))))
        self.A16 = torch.empty(M * K * 2, dtype=torch.uint8, device=dev)
        self.Dfused = {n: torch.empty(M, N, dtype=torch.float32, device=dev) for n in FORMATS}
        self.Dunf = torch.empty(M, N, dtype=torch.float32, device=dev)
        self.Dnat = {n: torch.empty(M, N, dtype=torch.float32, device=dev) for n in self.native}
        self.flops_per_gemm = 2.0 * M * N * K
        self.launches = 0

    # The GEMMs of one step, each as (label, callable).
    def ops(self):
        tb, M, N, K = self.tb, self.M, self.N, self.K
        out = []
        for name in FORMATS:
            f, A, al = self.fmt[name], self.Aq[name], self.alpha[name]
            out.append((f"fused_{name}", lambda f=f, A=A, al=al, name=name: tb.gemm_fused(
                f, A, self.B16, self.Dfused[name], M, N, K, out=tb.Out.F32, alpha=al)))
            out.append((f"decode_{name}", lambda f=f, A=A: tb.decode(f, A, self.A16, M * K)))
            out.append((f"gemm_after_{name}", lambda al=al: tb.gemm_f16(self.A16, self.B16, self.Dunf, M, N, K,
                                                                        out=tb.Out.F32, alpha=al)))
        for name, (f, qa, qb, al) in self.native.items():
            out.append((f"native_{name}", lambda f=f, qa=qa, qb=qb, al=al, name=name: tb.gemm_native(
                f, qa, f, qb, self.Dnat[name], M, N, K, out=tb.Out.F32, alpha=al)))
        return out

    def gemm_flops(self, label: str) -> float:
        return 0.0 if label.startswith("decode_") else self.flops_per_gemm

    def step_flops(self) -> float:
        return sum(self.gemm_flops(l) for l, _ in self.ops())

    def decode_bytes(self, name: str) -> int:
        return self.Aq[name].numel() + self.M * self.K * 2


def flush_l2(torch, buf):
    buf.add_(1)  # read + write 256 MiB, larger than the 126 MB L2


def run_device(torch, tb, sw: Sweep, steps: int, warmup: int, dist: Dist):
    ops = sw.ops()
    stream = torch.cuda.current_stream()
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        flush_l2(torch, flush)
        for _, fn in ops:
            fn()
    torch.cuda.synchronize()
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in ops]
          for _ in range(steps)]
    clocks = ClockSampler(dist.local)
    clocks.start()
    time.sleep(0.3)
    dist.barrier()
    torch.cuda.synchronize()
    launches = 0
    for s in range(steps):
        flush_l2(torch, flush)  # between timed steps, outside the events
        for j, (_, fn) in enumerate(ops):
            ev[s][j][0].record(stream)
            fn()
            ev[s][j][1].record(stream)
            launches += 1
    torch.cuda.synchronize()
    dist.barrier()
    clock = clocks.stop()
    per_op = {}
    total_ms = 0.0
    for s in range(steps):
        for j, (label, _) in enumerate(ops):
            ms = ev[s][j][0].elapsed_time(ev[s][j][1])
            per_op.setdefault(label, []).append(ms)
            total_ms += ms
    return total_ms, per_op, launches, clock


def run_e2e(torch, tb, sw: Sweep, steps: int, warmup: int):
    """The same GEMMs through the C ABI with host inputs and outputs: every
    GEMM copies its operands from pinned host memory, runs, and copies D back.
    Copies and kernels are pipelined over three streams with two buffer sets:
    the host->device copies of GEMM j+1 and the device->host copy of GEMM j-1
    overlap GEMM j (PCIe carries both directions at once); each stream waits
    only on the events of the buffers it reuses."""
    M, N, K = sw.M, sw.N, sw.K
    hA = {n: sw.Aq[n].cpu().pin_memory() for n in FORMATS}
    hB16 = sw.B16.cpu().pin_memory()
    hN = {n: (v[1].cpu().pin_memory(), v[2].cpu().pin_memory()) for n, v in sw.native.items()}
    hD = [torch.empty(M, N, dtype=torch.float32).pin_memory() for _ in range(2)]
    amax = max(max(a.numel() for a in sw.Aq.values()), max(v[1].numel() for v in sw.native.values()))
    bmax = max(sw.B16.numel() * sw.B16.element_size(), max(v[2].numel() for v in sw.native.values()))
    dA = [torch.empty(amax, dtype=torch.uint8, device="cuda") for _ in range(2)]
    dB = [torch.empty(bmax, dtype=torch.uint8, device="cuda") for _ in range(2)]
    dD = [torch.empty(M, N, dtype=torch.float32, device="cuda") for _ in range(2)]
    s_in, s_run, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    hB16b = hB16.view(torch.uint8).reshape(-1)

    # (label, host A, host B (bytes), kernel launcher(dA, dB, dD, stream))
    jobs = []
    for name in FORMATS:
        f, al = sw.fmt[name], sw.alpha[name]
        jobs.append((hA[name], hB16b, lambda a, b, d, st, f=f, al=al: tb.gemm_fused(
            f, a, b, d, M, N, K, out=tb.Out.F32, alpha=al, stream=st)))
        jobs.append((hA[name], hB16b, lambda a, b, d, st, f=f, al=al: (
            tb.decode(f, a, sw.A16, M * K, stream=st),
            tb.gemm_f16(sw.A16, b, d, M, N, K, out=tb.Out.F32, alpha=al, stream=st))))
    for name, (f, _, _, al) in sw.native.items():
        ha, hb = hN[name]
        jobs.append((ha, hb, lambda a, b, d, st, f=f, al=al: tb.gemm_native(
            f, a, f, b, d, M, N, K, out=tb.Out.F32, alpha=al, stream=st)))
    h2d = sum(a.numel() + b.numel() for a, b, _ in jobs)
    d2h = len(jobs) * hD[0].numel() * 4
    ev_in, ev_run, ev_out = [None, None], [None, None], [None, None]

    def step():
        for j, (ha, hb, run) in enumerate(jobs):
            k = j & 1
            with torch.cuda.stream(s_in):
                if ev_run[k] is not None:
                    s_in.wait_event(ev_run[k])  # the kernels that read this input slot are done
                dA[k][:ha.numel()].copy_(ha.view(torch.uint8).reshape(-1), non_blocking=True)
                dB[k][:hb.numel()].copy_(hb.reshape(-1), non_blocking=True)
                ev_in[k] = torch.cuda.Event()
                ev_in[k].record(s_in)
            s_run.wait_event(ev_in[k])
            if ev_out[k] is not None:
                s_run.wait_event(ev_out[k])  # this output slot has been copied out
            run(dA[k], dB[k], dD[k], s_run)
            ev_run[k] = torch.cuda.Event()
            ev_run[k].record(s_run)
            s_out.wait_event(ev_run[k])
            with torch.cuda.stream(s_out):
                hD[k].copy_(dD[k], non_blocking=True)
                ev_out[k] = torch.cuda.Event()
                ev_out[k].record(s_out)

    cur = torch.cuda.current_stream()
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for st in (s_in, s_run, s_out):
        st.wait_event(e0)
    for _ in range(steps):
        step()
    for st in (s_in, s_run, s_out):
        cur.wait_stream(st)
    e1.record(cur)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    return ms, h2d, d2h


def quality(torch, tb, sw: Sweep, rows: int = 256):
    """rel-Frobenius error of the fused result against the unquantized FP32
    product (the reference's err measure, bench/bench_formats.cu:97-103), on
    `rows` sampled rows; and whether fused == unfused bitwise."""
    out = {}
    r = torch.arange(0, sw.M, max(1, sw.M // rows), device="cuda")[:rows]
    ref = sw.a32  # fp32 originals
    for name in FORMATS:
        want = ref[name][r].double() @ sw.b32.double().T
        got = sw.Dfused[name][r].double()
        err = float(torch.linalg.norm(got - want) / torch.linalg.norm(want))
        # unfused result for the same format, recomputed here for the bitwise check
        tb.decode(sw.fmt[name], sw.Aq[name], sw.A16, sw.M * sw.K)
        tb.gemm_f16(sw.A16, sw.B16, sw.Dunf, sw.M, sw.N, sw.K, out=tb.Out.F32, alpha=sw.alpha[name])
        torch.cuda.synchronize()
        same = bool(torch.equal(sw.Dfused[name].view(torch.int32), sw.Dunf.view(torch.int32)))
        out[name] = {"rel_frob_vs_fp32": err, "fused_equals_unfused": same}
    for name in sw.native:
        want = ref[name][r].double() @ sw.b32.double().T
        out[f"native_{name}"] = {"rel_frob_vs_fp32": float(torch.linalg.norm(sw.Dnat[name][r].double() - want) /
                                                           torch.linalg.norm(want))}
    return out


# ---- the other configurations, reported beside the headline ----------------------------

def time_each(torch, fn, iters: int, flush) -> float:
    """Median device time (ms) of `fn`, one launch per CUDA-event pair with an
    L2 flush between launches (outside the events)."""
    stream = torch.cuda.current_stream()
    for _ in range(3):
        fn()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for a, b in ev:
        flush_l2(torch, flush)
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in ev)


def weights_q(torch, tb, fmt, rows: int, cols: int, std: float, seed: int):
    """Seeded N(0, std) weights quantized with scale FORMAT_MAX / maxabs."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    a = torch.randn(rows, cols, generator=g, device="cuda") * std
    amax = torch.zeros(1, dtype=torch.float32, device="cuda")
    tb.absmax(a, a.numel(), amax)
    fmax = 448.0 if fmt == tb.Format.E4M3 else 6.0
    scale = float(np.float32(fmax) / np.float32(float(amax.item())))
    q = torch.empty(tb.stored_bytes(fmt, rows * cols), dtype=torch.uint8, device="cuda")
    tb.quantize(fmt, a, q, rows * cols, scale=scale)
    return q, float(np.float32(1.0) / np.float32(scale))


def time_graph(torch, fns, iters: int = 20) -> float:
    """Median device time (ms) per launch of a back-to-back sequence: every
    callable of `fns` once, in order, captured in one CUDA graph that is
    replayed `iters` times, each replay between a CUDA-event pair, divided by
    len(fns).  The callables work on distinct buffers whose total is larger
    than the 126 MB L2, so every launch reads its inputs from HBM, as
    consecutive layers of a model do."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for fn in fns:  # first calls (kernel attributes) outside the capture
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for fn in fns:
            fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for a, b in ev:
        a.record(stream)
        g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b) for a, b in ev) / len(fns)
    del g
    return ms


ROTATE_BYTES = 400_000_000  # > 3 x L2


def mlp_weight_only(torch, tb, peaks, iters: int = 20):
    """Weight-only inference shapes: W 14336 x 4096 and 4096 x 14336 (output
    features x K) in E4M3 and packed E2M1, activations FP16 [tokens x K],
    FP32 out, tokens 1/16/128/2048.  Fused decode-in-shared-memory GEMM
    against decode kernel + GEMM.  Each figure is per launch of a back-to-back
    sequence over C copies of the weight (C x stored bytes > 400 MB, so every
    launch streams its weight from HBM) inside a CUDA graph, median of 20
    replays; the few-token fused kernels of the sequence overlap their
    successor's start through programmatic dependent launch, as consecutive
    layers would.  Each weight's cases start after one second of idle GPU.
    Algorithmic bytes = stored W + X + D."""
    out = []
    for (M, K) in ((14336, 4096), (4096, 14336)):
        for fname, fmt in (("e4m3", tb.Format.E4M3), ("e2m1", tb.Format.E2M1)):
            A, alpha = weights_q(torch, tb, fmt, M, K, 0.02, seed=M + K + int(fmt))
            copies = max(2, -(-ROTATE_BYTES // A.numel()))
            As = [A] + [A.clone() for _ in range(copies - 1)]
            A16 = [torch.empty(M * K, dtype=torch.float16, device="cuda") for _ in range(2)]
            for N in (1, 16, 128, 2048):
                if N == 1:
                    # The previous weight's 2048-token GEMMs leave the GPU under
                    # its power cap; a decode loop of few-token GEMMs runs
                    # without them, so its cases start from an idle second.
                    torch.cuda.synchronize()
                    time.sleep(1.0)
                g = torch.Generator(device="cuda")
                g.manual_seed(N)
                B = torch.randn(N, K, generator=g, device="cuda").half()
                D = torch.empty(M, N, dtype=torch.float32, device="cuda")
                wsb = tb.fused_workspace_bytes(fmt, M, N, K)
                ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device="cuda")
                fused = time_graph(torch, [lambda Ai=Ai: tb.gemm_fused(fmt, Ai, B, D, M, N, K, alpha=alpha,
                                                                          workspace=ws, workspace_bytes=wsb)
                                              for Ai in As], iters)
                dec = time_graph(torch, [lambda i=i, Ai=Ai: tb.decode(fmt, Ai, A16[i & 1], M * K)
                                            for i, Ai in enumerate(As)], iters)
                gemm = time_graph(torch, [lambda i=i: tb.gemm_f16(A16[i & 1], B, D, M, N, K, alpha=alpha)
                                             for i in range(copies)], iters)
                nbytes = A.numel() + N * K * 2 + M * N * 4
                flops = 2.0 * M * N * K
                out.append({"W": f"{M}x{K}", "fmt": fname, "tokens": N, "weight_copies": copies,
                            "fused_us": fused * 1e3, "unfused_us": (dec + gemm) * 1e3,
                            "fused_gbs": nbytes / fused / 1e6,
                            "fused_pct_hbm": 100 * nbytes / fused / 1e6 / peaks["hbm_gbs"],
                            "fused_tflops": flops / fused / 1e9, "fused_vs_unfused": (dec + gemm) / fused})
            del A16, As
    return out


def decode_streams(torch, tb, peaks, rows: int = 14336, cols: int = 4096, iters: int = 20):
    """The standalone decode streamers on a 14336 x 4096 weight per format
    (N(0, 0.02) quantized per tensor): per launch of a back-to-back sequence
    alternating over two (input, output) pairs, 2 x (stored + FP16) bytes >
    L2, inside a CUDA graph, median of 20 replays.  Algorithmic bytes = stored bytes read + FP16 bytes written."""
    n = rows * cols
    out = {}
    F = tb.Format
    for name, fmt in (("tf32", F.TF32), ("bf16", F.BF16), ("e4m3", F.E4M3), ("e2m1", F.E2M1)):
        if name in FORMAT_MAX:
            A, _ = weights_q(torch, tb, fmt, rows, cols, 0.02, seed=7 + int(fmt))
        else:
            g = torch.Generator(device="cuda")
            g.manual_seed(7 + int(fmt))
            a = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
            A = torch.empty(tb.stored_bytes(fmt, n), dtype=torch.uint8, device="cuda")
            tb.quantize(fmt, a, A, n)
            del a
        pairs = [(A, torch.empty(n, dtype=torch.float16, device="cuda")),
                 (A.clone(), torch.empty(n, dtype=torch.float16, device="cuda"))]
        ms = time_graph(torch, [lambda s=s, d=d: tb.decode(fmt, s, d, n) for s, d in pairs] * 2, iters)
        nbytes = A.numel() + 2 * n
        out[name] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                     "pct_hbm": 100 * nbytes / ms / 1e6 / peaks["hbm_gbs"]}
        del pairs, A
    # Block-scaled FP4: packed codes + one E4M3 scale byte per 16 values.
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    q = torch.randint(0, 256, (n // 2,), generator=g, device="cuda", dtype=torch.uint8)
    sc = torch.randint(0x20, 0x60, (n // 16,), generator=g, device="cuda", dtype=torch.uint8)
    trip = [(q, sc, torch.empty(n, dtype=torch.float16, device="cuda")),
            (q.clone(), sc.clone(), torch.empty(n, dtype=torch.float16, device="cuda"))]
    ms = time_graph(torch, [lambda q=q, s=s, d=d: tb.decode_nvfp4(q, s, d, n) for q, s, d in trip] * 2, iters)
    nbytes = n // 2 + n // 16 + 2 * n
    out["nvfp4"] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                    "pct_hbm": 100 * nbytes / ms / 1e6 / peaks["hbm_gbs"]}
    del trip, q, sc
    return out


def int8_square(torch, tb, n: int = 4096, iters: int = 10):
    """The INT8 path at n^3: INT8 GEMM on tcgen05 kind::i8 (exact INT32), and
    the reference-shaped FP8 -> INT8 fused entry (both operands converted with
    scale 127/448, then the GEMM).  Dense integer peak 4.5 POPS."""
    g = torch.Generator(device="cuda")
    g.manual_seed(8)
    A8 = torch.randint(-128, 128, (n, n), generator=g, device="cuda", dtype=torch.int8)
    B8 = torch.randint(-128, 128, (n, n), generator=g, device="cuda", dtype=torch.int8)
    D = torch.empty(n, n, dtype=torch.int32, device="cuda")
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    ms = time_each(torch, lambda: tb.gemm_i8(A8, B8, D, n, n, n), iters, flush)
    A, _ = weights_q(torch, tb, tb.Format.E4M3, n, n, 1.0, seed=9)
    B, _ = weights_q(torch, tb, tb.Format.E4M3, n, n, 1.0, seed=10)
    wsb = tb.lib().tb_gemm_fp8_fused_int8_workspace(n, n, n)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    scale = float(np.float32(127.0) / np.float32(448.0))
    ms_f = time_each(torch, lambda: tb.gemm_fp8_fused_int8(A, B, D, n, n, n, scale, ws, wsb), iters, flush)
    ops = 2.0 * n ** 3
    return {"M": n, "N": n, "K": n, "gemm_i8_ms": ms, "gemm_i8_tops": ops / ms / 1e9,
            "pct_i8_dense_peak": 100 * ops / ms / 1e9 / 4500.0, "fp8_fused_int8_ms": ms_f,
            "fp8_fused_int8_tops": ops / ms_f / 1e9}


def rested(torch, section, pause_s: float = 2.0):
    """Run `section()` after `pause_s` seconds of idle GPU; returns its result
    and the SM clocks, power and throttle reasons sampled every 10 ms while it
    ran."""
    clocks = ClockSampler(torch.cuda.current_device(), interval_ms=10)
    clocks.start()  # nvidia-smi takes a moment to start sampling
    time.sleep(pause_s)
    clocks.lines.clear()  # keep only the samples taken while the section runs
    res = section()
    return res, clocks.stop()


def native_square(torch, tb, n: int = 8192, iters: int = 20):
    """Both operands quantized at n^3: E4M3 x E4M3 on tcgen05 kind::f8f6f4
    (operands N(0, 1) with scale 448/maxabs each, alpha = 1/(sA sB)) and
    INT8 x INT8 on kind::i8 (uniform over all codes, exact INT32 out); FP16
    and INT32 outputs.  Dense FP8 / INT8 peak 4.5 P nominal."""
    A, sa = weights_q(torch, tb, tb.Format.E4M3, n, n, 1.0, seed=81)
    B, sb = weights_q(torch, tb, tb.Format.E4M3, n, n, 1.0, seed=82)
    D = torch.empty(n, n, dtype=torch.float16, device="cuda")
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    al = float(np.float32(sa) * np.float32(sb))
    ms = time_each(torch, lambda: tb.gemm_native(tb.Format.E4M3, A, tb.Format.E4M3, B, D, n, n, n, out=tb.Out.F16,
                                                 alpha=al), iters, flush)
    del A, B, D
    g = torch.Generator(device="cuda")
    g.manual_seed(83)
    A8 = torch.randint(-128, 128, (n, n), generator=g, device="cuda", dtype=torch.int8)
    B8 = torch.randint(-128, 128, (n, n), generator=g, device="cuda", dtype=torch.int8)
    D32 = torch.empty(n, n, dtype=torch.int32, device="cuda")
    ms_i8 = time_each(torch, lambda: tb.gemm_i8(A8, B8, D32, n, n, n), iters, flush)
    ops = 2.0 * n ** 3
    return {"M": n, "N": n, "K": n, "e4m3_ms": ms, "e4m3_tflops": ops / ms / 1e9,
            "e4m3_pct_fp8_dense_peak": 100 * ops / ms / 1e9 / 4500.0, "i8_ms": ms_i8, "i8_tops": ops / ms_i8 / 1e9,
            "i8_pct_i8_dense_peak": 100 * ops / ms_i8 / 1e9 / 4500.0}


def fused_square(torch, tb, peaks, fmt_name: str = "e2m1", n: int = 8192, iters: int = 40):
    """Large square fused GEMM: A packed E2M1 (or E4M3) from N(0, 1) with scale
    FORMAT_MAX/maxabs, B FP16 N(0, 1), FP32 accumulation, FP16 output.  The SM
    clocks and power are sampled every 10 ms over this section alone
    ("clocks"): a GEMM at this rate runs into the 1 kW power cap, which lowers
    the clock."""
    fmt = tb.Format.E2M1 if fmt_name == "e2m1" else tb.Format.E4M3
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    A, alpha = weights_q(torch, tb, fmt, n, n, 1.0, seed=8192)
    g = torch.Generator(device="cuda")
    g.manual_seed(8193)
    B = torch.randn(n, n, generator=g, device="cuda").half()
    D = torch.empty(n, n, dtype=torch.float16, device="cuda")
    clocks = ClockSampler(torch.cuda.current_device(), interval_ms=10)
    clocks.start()
    ms = time_each(torch, lambda: tb.gemm_fused(fmt, A, B, D, n, n, n, out=tb.Out.F16, alpha=alpha), iters, flush)
    clk = clocks.stop()
    tf = 2.0 * n ** 3 / ms / 1e9
    return {"M": n, "N": n, "K": n, "fmt": "e2m1 packed" if fmt_name == "e2m1" else "e4m3", "out": "f16",
            "ms": ms, "tflops": tf, "pct_f16_dense_peak_nominal": 100 * tf / 2250.0,
            "frac_of_measured_bf16": tf / peaks["bf16_tflops"], "clocks": clk}


def nvfp4_square(torch, tb, n: int = 8192, iters: int = 20):
    """Block-scaled FP4 with both operands quantized (packed E2M1 codes, one
    UE4M3 scale byte per 16 values) at n^3 on tcgen05 kind::mxf4nvf4, FP16
    out; codes uniform over all 16 values, scale bytes uniform in 0x30-0x47.
    Dense FP4 peak 9 PFLOP/s nominal."""
    g = torch.Generator(device="cuda")
    g.manual_seed(94)
    A = torch.randint(0, 256, (n, n // 2), generator=g, device="cuda", dtype=torch.uint8)
    B = torch.randint(0, 256, (n, n // 2), generator=g, device="cuda", dtype=torch.uint8)
    SA = torch.randint(0x30, 0x48, (n, n // 16), generator=g, device="cuda", dtype=torch.uint8)
    SB = torch.randint(0x30, 0x48, (n, n // 16), generator=g, device="cuda", dtype=torch.uint8)
    D = torch.empty(n, n, dtype=torch.float16, device="cuda")
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    ms = time_each(torch, lambda: tb.gemm_nvfp4(A, SA, B, SB, D, n, n, n, out=tb.Out.F16, alpha=1e-4), iters, flush)
    tf = 2.0 * n ** 3 / ms / 1e9
    return {"M": n, "N": n, "K": n, "out": "f16", "ms": ms, "tflops": tf, "pct_fp4_dense_peak_nominal": 100 * tf / 9000.0,
            "pct_fp8_dense_peak_nominal": 100 * tf / 4500.0}


def config_256(torch, tb, iters: int = 50):
    """The 256 x 256 x 256 FP8 E4M3 weight-only GEMM: A from U[-1, 1] (seed 0)
    quantized with scale 448/maxabs, B from U[-1, 1] (seed 1) in FP16; fused
    decode + GEMM, FP32 out.  Reports its device time (median, one launch per
    event pair) and its relative Frobenius error against the unquantized FP32
    product, the measure the reference publishes for this case."""
    n = 256
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    a = torch.rand(n, n, generator=g, device="cuda") * 2 - 1
    g.manual_seed(1)
    b = torch.rand(n, n, generator=g, device="cuda") * 2 - 1
    amax = torch.zeros(1, dtype=torch.float32, device="cuda")
    tb.absmax(a, a.numel(), amax)
    scale = float(np.float32(448.0) / np.float32(float(amax.item())))
    A = torch.empty(n * n, dtype=torch.uint8, device="cuda")
    tb.quantize(tb.Format.E4M3, a, A, n * n, scale=scale)
    B = b.half()
    D = torch.empty(n, n, dtype=torch.float32, device="cuda")
    alpha = float(np.float32(1.0) / np.float32(scale))
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    ms = time_each(torch, lambda: tb.gemm_fused(tb.Format.E4M3, A, B, D, n, n, n, alpha=alpha), iters, flush)
    want = a.double() @ b.double().T
    err = float(torch.linalg.norm(D.double() - want) / torch.linalg.norm(want))
    return {"M": n, "N": n, "K": n, "fmt": "e4m3", "us": ms * 1e3, "tflops": 2.0 * n ** 3 / ms / 1e9,
            "rel_frob_vs_unquantized_fp32": err}


def sharded_weight_gemm(torch, tb, dist, steps: int = 5, warmup: int = 2):
    """The 16384 x 53248 E4M3 weight (N(0, 0.02), per-tensor scale 448/maxabs),
    used as its transpose in the weight role: M = 53248 output rows, K = 16384;
    X = 8192 FP16 tokens from N(0, 1), replicated; FP16 output.  On one GPU it
    is one fused GEMM.  On N GPUs the output rows are split over the ranks and
    every rank ends with all of D, two ways:
      p2p   (the product path) each rank's fused kernel stores every finished
            tile into all ranks' D over NVLink (peer-mapped buffers), one
            launch over the rank's M / N contiguous rows;
      nccl  block-cyclic rows in 4 chunks per rank, the fused kernel per
            chunk, NCCL all-gathers in place on a second stream.
    Each is checked after timing.  Also timed: the rank's GEMM alone (all SMs,
    no exchange) and the NCCL all-gathers alone.  Device time, max over ranks."""
    M, N, K = 53248, 8192, 16384
    world, rank = dist.world, dist.rank
    chunks = 4
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    W = torch.randn(M, K, generator=g, device="cuda") * 0.02
    amax = torch.zeros(1, dtype=torch.float32, device="cuda")
    tb.absmax(W, W.numel(), amax)
    scale = float(np.float32(448.0) / np.float32(float(amax.item())))

    def quantized(rows):
        q = torch.empty(rows.numel(), dtype=torch.uint8, device="cuda")
        tb.quantize(tb.Format.E4M3, rows, q, rows.numel(), scale=scale)
        return q

    A1 = quantized(W if world == 1 else tb.shard_rows(W, M, world, 1, rank))  # contiguous rows
    A4 = quantized(tb.shard_rows(W, M, world, chunks, rank)) if world > 1 else None
    # Rows kept for the check after timing: 8 from each of the world*chunks
    # row blocks (a block straddles 128-row tile boundaries at offsets that
    # differ per block), computed by every rank or gathered from the others.
    nblk = max(world * chunks, 8)
    mc = M // nblk
    sample = torch.tensor(sorted({b * mc + (37 * b + 120 + 3 * i) % mc for b in range(nblk) for i in range(8)}),
                          device="cuda")
    W_s = W[sample].contiguous()
    del W
    g.manual_seed(6)
    X = torch.randn(N, K, generator=g, device="cuda").half()
    D = torch.empty(M, N, dtype=torch.float16, device="cuda")
    alpha = float(np.float32(1.0) / np.float32(scale))
    st, cst = torch.cuda.Stream(), torch.cuda.Stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        return dist.max(e0.elapsed_time(e1) / steps)

    flops = 2.0 * M * N * K
    res = {"M": M, "N": N, "K": K, "fmt": "e4m3", "out": "f16", "world": world, "scaling": "strong",
           "allgather_bytes_per_rank": (world - 1) * (M // world) * N * 2 if world > 1 else 0}
    if world == 1:
        ms = timed(lambda: tb.gemm_fused(tb.Format.E4M3, A1, X, D, M, N, K, out=tb.Out.F16, alpha=alpha,
                                         stream=st.cuda_stream))
        check = sharded_check(torch, tb, dist, W_s, sample, X, D, N, K, scale, alpha)
        res.update({"path": "one fused GEMM", "ms": ms, "gemm_only_ms": ms, "check": check})
    else:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(tb.nccl_unique_id()), dtype=torch.uint8))
        dist.dist.broadcast(uid, 0)
        comm = tb.nccl_comm_init(world, rank, bytes(uid.cpu().numpy()))
        try:
            # p2p: one launch per rank over its contiguous M / world rows
            handle = tb.peer_buffer_register(comm, D, stream=st.cuda_stream)
            try:
                p2p_ms = timed(lambda: tb.gemm_sharded_fused_p2p(tb.Format.E4M3, A1, X, handle, M, N, K, chunks=1,
                                                                 out=tb.Out.F16, alpha=alpha, stream=st.cuda_stream))
                D.fill_(float("nan"))  # the check must see D written by the p2p path alone
                torch.cuda.synchronize()
                tb.gemm_sharded_fused_p2p(tb.Format.E4M3, A1, X, handle, M, N, K, chunks=1, out=tb.Out.F16,
                                          alpha=alpha, stream=st.cuda_stream)
                torch.cuda.synchronize()
                p2p_check = sharded_check(torch, tb, dist, W_s, sample, X, D, N, K, scale, alpha)
            finally:
                tb.peer_buffer_release(handle, stream=st.cuda_stream)
            ml = M // world
            gemm_ms = timed(lambda: tb.gemm_fused(tb.Format.E4M3, A1, X, D[rank * ml:(rank + 1) * ml], ml, N, K,
                                                  out=tb.Out.F16, alpha=alpha, stream=st.cuda_stream))

            # nccl: block-cyclic chunks, in-place all-gathers on a second stream
            def nccl_step():
                tb.gemm_sharded_fused(tb.Format.E4M3, A4, X, D, M, N, K, comm, chunks, out=tb.Out.F16,
                                      alpha=alpha, stream=st.cuda_stream, comm_stream=cst.cuda_stream)

            nccl_ms = timed(nccl_step)
            mcw = M // (world * chunks)

            def ag_only():
                with torch.cuda.stream(st):
                    for c in range(chunks):
                        grp = D[c * world * mcw:(c + 1) * world * mcw]
                        dist.dist.all_gather_into_tensor(grp, grp[rank * mcw:(rank + 1) * mcw])

            ag_ms = timed(ag_only)
            D.fill_(float("nan"))
            torch.cuda.synchronize()
            nccl_step()
            torch.cuda.synchronize()
            nccl_check = sharded_check(torch, tb, dist, W_s, sample, X, D, N, K, scale, alpha)
        finally:
            torch.cuda.synchronize()
            tb.nccl_comm_destroy(comm)
        res.update({"path": "p2p: fused GEMM epilogue stores tiles into peers' D", "ms": p2p_ms,
                    "gemm_only_ms": gemm_ms, "check": p2p_check,
                    "nccl": {"chunks": chunks, "ms": nccl_ms, "allgather_only_ms": ag_ms, "check": nccl_check}})
    res["tflops_total"] = flops / res["ms"] / 1e9
    res["tflops_per_gpu"] = res["tflops_total"] / world
    return res


def sharded_check(torch, tb, dist, W_s, sample, X, D, N: int, K: int, scale: float, alpha: float):
    """Correctness of the sharded GEMM's D on every rank, on the sampled rows
    of every row block (own and all-gathered): (1) bit for bit against the
    single-GPU fused GEMM of the same quantized rows, run unsplit (same
    kernel arithmetic, same K order), and (2) relative Frobenius error against
    an FP64 product of the decoded rows (decode bit-exact to the reference's
    primitives) and the FP16 activations.  Worst case over ranks."""
    S = sample.numel()
    A_s = torch.empty(S * K, dtype=torch.uint8, device="cuda")
    tb.quantize(tb.Format.E4M3, W_s, A_s, S * K, scale=scale)
    D_s = torch.empty(S, N, dtype=torch.float16, device="cuda")
    tb.gemm_fused(tb.Format.E4M3, A_s, X, D_s, S, N, K, out=tb.Out.F16, alpha=alpha)  # no workspace: unsplit
    A16 = torch.empty(S, K, dtype=torch.float16, device="cuda")
    tb.decode(tb.Format.E4M3, A_s, A16, S * K)
    torch.cuda.synchronize()
    got = D[sample]
    bitwise = bool(torch.equal(got.view(torch.int16), D_s.view(torch.int16)))
    want = (A16.double() @ X.double().T) * alpha
    err = float(torch.linalg.norm(got.double() - want) / torch.linalg.norm(want))
    bad = dist.max(0.0 if bitwise else 1.0)
    err = dist.max(err)
    return {"rows_per_rank": S, "blocks": S // 8, "bitwise_vs_1gpu": bad == 0.0, "rel_frob_max_vs_fp64": err,
            "pass": bad == 0.0 and err <= 1e-3}


# ---- CPU baseline: the reference's own host path ---------------------------------------

def cpu_baseline(sw_shape, seconds: float = 12.0):
    """Time tensor-bridge's host decode primitives + its FP32 GEMM loop
    (oracle/_ref, compiled from the reference headers) on a row sample of the
    sweep, on all host threads.  Falls back to the oracle port if _ref is absent."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    M, N, K = sw_shape
    threads = host_threads()
    fmts = {"tf32": O.TF32, "bf16": O.BF16, "e4m3": O.E4M3, "e2m1": O.E2M1}
    rng_rows = 32
    data = {}
    b = O.normal(1, (N, K), 1.0)
    B16 = O.f32_to_f16_bits(b).reshape(N, K)
    for name, f in fmts.items():
        a = O.normal(2, (rng_rows * 64, K), 0.02)
        s = O.per_tensor_scale(a, f)
        data[name] = (f, O.quantize(f, a, s), float(np.float32(1) / np.float32(s)))
    use_ref = O.ref_lib() is not None
    run = (lambda f, A, al, rows: O.ref_cpu_gemm(f, A, B16, A.shape[0], N, K, rows=rows, alpha=al,
                                                 threads=threads)) if use_ref else \
          (lambda f, A, al, rows: O.gemm(f, A, O.F16, B16, A.shape[0], N, K, rows=rows, alpha=al,
                                         threads=threads))
    # calibrate: rows per format so the whole sample takes about `seconds`
    t0 = time.perf_counter()
    for f, A, al in data.values():
        run(f, A, al, (0, threads))
    per_row = (time.perf_counter() - t0) / (threads * len(data))
    rows = max(threads, int(seconds / (per_row * len(data))) // threads * threads)
    rows = min(rows, rng_rows * 64)
    t0 = time.perf_counter()
    for f, A, al in data.values():
        run(f, A, al, (0, rows))
    dt = time.perf_counter() - t0
    flops = 2.0 * rows * N * K * len(data)
    out = {"value": flops / dt / 1e12, "unit": UNIT, "cores": threads,
           "kind": "reference" if use_ref else "port",
           "sample": f"{rows} rows x N={N} x K={K} of each of {len(data)} weight-only GEMMs "
                     f"({', '.join(data)}), decode + FP32 loop, {dt:.1f} s"}
    if use_ref:
        out["naive_single_thread"] = naive_loop_times(O)
    return out


def naive_loop_times(O):
    """The reference's own naive single-thread CPU product (bench/bench_formats.cu:183-186:
    decode, then for every (i, j) an FP32 sum over k with B read [K x N]) on
    the 256^3 and 512^3 E4M3 weight-only cases, one host thread."""
    res = {}
    for n in (256, 512):
        a, b = O.uniform(0, (n, n)), O.uniform(1, (n, n))
        s = O.per_tensor_scale(a, O.E4M3)
        A = O.quantize(O.E4M3, a, s)
        B16 = O.f32_to_f16_bits(b).reshape(n, n)
        reps, t0 = 0, time.perf_counter()
        while True:
            O.ref_naive_gemm(O.E4M3, A, B16, n, n, n, alpha=float(np.float32(1) / np.float32(s)))
            reps += 1
            if time.perf_counter() - t0 > 1.0:
                break
        ms = (time.perf_counter() - t0) / reps * 1e3
        res[f"{n}^3"] = {"ms": ms, "gflops": 2.0 * n ** 3 / ms / 1e6, "cores": 1}
    return res


def sweep_config(M: int, N: int, K: int, world: int) -> dict:
    """The workload's `config` object, shared by both arms of the benchmark."""
    return {"workload": f"format sweep {M}x{N}x{K}: fused + unfused decode+GEMM for TF32/BF16/E4M3/E2M1, "
                        f"native E4M3xE4M3 and E2M1xE2M1; FP32 out", "M": M, "N": N, "K": K,
            "gemms_per_step": 10, "l2": "flushed between steps (256 MiB write)",
            "parallelism": f"replicas x{world}"}


def reference_arm(args):
    """--impl reference: the reference's own CPU implementation of the path
    (its host decode primitives + FP32 GEMM loop, oracle/_ref) on the host
    cores, rank 0 only, one bounded sample of the sweep per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    M = N = K = args.size
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = host_threads()
    b = O.normal(1, (N, K), 1.0)
    B16 = O.f32_to_f16_bits(b).reshape(N, K)
    fmts = {"tf32": O.TF32, "bf16": O.BF16, "e4m3": O.E4M3, "e2m1": O.E2M1}
    # 8 rows per thread: B is widened once per GEMM call (in parallel), so the
    # row loop dominates as it does in cpu_baseline's calibrated sample.
    rows = 8 * threads
    data = []
    for name, f in fmts.items():
        a = O.normal(2, (rows, K), 0.02)
        s = O.per_tensor_scale(a, f)
        data.append((f, O.quantize(f, a, s), float(np.float32(1) / np.float32(s))))
    use_ref = O.ref_lib() is not None

    def step():
        for f, A, al in data:
            if use_ref:
                O.ref_cpu_gemm(f, A, B16, rows, N, K, alpha=al, threads=threads)
            else:
                O.gemm(f, A, O.F16, B16, rows, N, K, alpha=al, threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    flops = 2.0 * rows * N * K * len(data) * args.steps
    value = flops / dt / 1e12
    sample = (f"{rows} rows x N={N} x K={K} per weight-only GEMM, formats {list(fmts)}, reference host decode "
              f"primitives + FP32 loop per step")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (decoded f16 operands)", "data": "synthetic",
            "impl": "reference",
            "config": sweep_config(M, N, K, 1),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads,
                             "kind": "reference" if use_ref else "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def traffic_from_profiles(label: str):
    """DRAM bytes per launch of the dominant kernel, from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic_per_launch.txt")
    try:
        for ln in open(path):
            k, _, v = ln.partition("=")
            if k.strip() == label:
                return float(v.strip())
    except OSError:
        pass
    return None


def profile_case(case: str):
    """Five launches of one fused weight-only GEMM: A = N(0, 0.02) weights of
    the given format (per-tensor scale), B = N(0, 1) FP16 activations."""
    import torch
    tb = load_package()
    fname, shape = case.split(":")
    if fname == "nvfp4":  # the block-scaled FP4 decode streamer on a ROWS x COLS weight
        rows, cols = (int(v) for v in shape.lower().split("x"))
        n = rows * cols
        g = torch.Generator(device="cuda")
        g.manual_seed(11)
        q = torch.randint(0, 256, (n // 2,), generator=g, device="cuda", dtype=torch.uint8)
        sc = torch.randint(0x20, 0x60, (n // 16,), generator=g, device="cuda", dtype=torch.uint8)
        d = torch.empty(n, dtype=torch.float16, device="cuda")
        for _ in range(5):
            tb.decode_nvfp4(q, sc, d, n)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": case, "ok": True}))
        return
    if fname.startswith("decode_"):  # a decode streamer on a ROWS x COLS weight (N(0, 0.02), per-tensor scale)
        rows, cols = (int(v) for v in shape.lower().split("x"))
        fmt = {"e4m3": tb.Format.E4M3, "e2m1": tb.Format.E2M1, "bf16": tb.Format.BF16,
               "tf32": tb.Format.TF32}[fname[len("decode_"):]]
        n = rows * cols
        if fname[len("decode_"):] in FORMAT_MAX:
            A, _ = weights_q(torch, tb, fmt, rows, cols, 0.02, seed=7)
        else:
            a = torch.randn(rows, cols, device="cuda") * 0.02
            A = torch.empty(tb.stored_bytes(fmt, n), dtype=torch.uint8, device="cuda")
            tb.quantize(fmt, a, A, n)
        d = torch.empty(n, dtype=torch.float16, device="cuda")
        for _ in range(5):
            tb.decode(fmt, A, d, n)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": case, "ok": True}))
        return
    M, N, K = (int(v) for v in shape.lower().split("x"))
    if fname == "nvfp4gemm":  # the block-scaled FP4 GEMM (kind::mxf4nvf4)
        g = torch.Generator(device="cuda")
        g.manual_seed(94)
        A = torch.randint(0, 256, (M, K // 2), generator=g, device="cuda", dtype=torch.uint8)
        B = torch.randint(0, 256, (N, K // 2), generator=g, device="cuda", dtype=torch.uint8)
        SA = torch.randint(0x30, 0x48, (M, K // 16), generator=g, device="cuda", dtype=torch.uint8)
        SB = torch.randint(0x30, 0x48, (N, K // 16), generator=g, device="cuda", dtype=torch.uint8)
        D = torch.empty(M, N, dtype=torch.float16, device="cuda")
        for _ in range(5):
            tb.gemm_nvfp4(A, SA, B, SB, D, M, N, K, out=tb.Out.F16, alpha=1e-4)
        torch.cuda.synchronize()
        assert tb.device_error() == 0, "a kernel reported a device-side wait timeout"
        print(json.dumps({"profile_case": case, "ok": True}))
        return
    if fname == "e4m3xe4m3":  # the native FP8 GEMM (both operands E4M3, per-tensor scales)
        A, sa = weights_q(torch, tb, tb.Format.E4M3, M, K, 0.02, seed=1)
        B, sb = weights_q(torch, tb, tb.Format.E4M3, N, K, 1.0, seed=2)
        D = torch.empty(M, N, dtype=torch.float32, device="cuda")
        for _ in range(5):
            tb.gemm_native(tb.Format.E4M3, A, tb.Format.E4M3, B, D, M, N, K, alpha=sa * sb)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": case, "ok": True}))
        return
    if fname == "f16":  # the plain FP16 GEMM
        A = torch.randn(M, K, device="cuda").half()
        B = torch.randn(N, K, device="cuda").half()
        D = torch.empty(M, N, dtype=torch.float32, device="cuda")
        for _ in range(5):
            tb.gemm_f16(A, B, D, M, N, K)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": case, "ok": True}))
        return
    fmt = {"e4m3": tb.Format.E4M3, "e2m1": tb.Format.E2M1, "bf16": tb.Format.BF16, "tf32": tb.Format.TF32}[fname]
    if fname in FORMAT_MAX:
        A, alpha = weights_q(torch, tb, fmt, M, K, 0.02, seed=1)
    else:
        a = torch.randn(M, K, device="cuda") * 0.02
        A = torch.empty(tb.stored_bytes(fmt, M * K), dtype=torch.uint8, device="cuda")
        tb.quantize(fmt, a, A, M * K)
        alpha = 1.0
    B = torch.randn(N, K, device="cuda").half()
    D = torch.empty(M, N, dtype=torch.float32, device="cuda")
    wsb = tb.fused_workspace_bytes(fmt, M, N, K)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device="cuda")
    for _ in range(5):
        tb.gemm_fused(fmt, A, B, D, M, N, K, alpha=alpha, workspace=ws, workspace_bytes=wsb)
    torch.cuda.synchronize()
    assert tb.device_error() == 0, "a kernel reported a device-side wait timeout"
    print(json.dumps({"profile_case": case, "ok": True}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--size", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the MLP-shape and 8192^3 FP4 sub-objects")
    ap.add_argument("--profile-case", metavar="FMT:MxNxK",
                    help="run only 5 fused weight-only GEMMs of this case (e.g. e4m3:14336x16x4096; f16:MxNxK for "
                         "the plain FP16 GEMM, e4m3xe4m3:MxNxK for the native FP8 GEMM, nvfp4gemm:MxNxK for the "
                         "block-scaled FP4 GEMM, nvfp4:ROWSxCOLS for 5 "
                         "block-scaled FP4 decodes, decode_FMT:ROWSxCOLS for 5 decodes of one format) and exit; "
                         "the command profiles/ captures of single kernels use")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        reference_arm(args)
        return

    import torch
    tb = load_package()
    dist = Dist(torch, args.gpus)
    M = N = K = args.size
    sw = Sweep(torch, tb, M, N, K, seed=1234 + dist.rank)
    total_ms, per_op, launches, clock = run_device(torch, tb, sw, args.steps, args.warmup, dist)
    t_max = dist.max(total_ms)
    e2e_ms, h2d, d2h = run_e2e(torch, tb, sw, max(2, args.steps // 2), 1)
    e2e_max = dist.max(e2e_ms)
    e2e_steps = max(2, args.steps // 2)
    q = quality(torch, tb, sw)

    step_flops = sw.step_flops()
    value = dist.world * step_flops * args.steps / (t_max / 1e3) / 1e12
    peaks = measured_peaks()
    # per-format and per-kernel figures (rank-local)
    mean = {k: sum(v) / len(v) for k, v in per_op.items()}
    formats = {}
    for name in FORMATS:
        dec_ms = mean[f"decode_{name}"]
        formats[name] = {
            "fused_tflops": sw.flops_per_gemm / mean[f"fused_{name}"] / 1e9,
            "unfused_tflops": sw.flops_per_gemm / (dec_ms + mean[f"gemm_after_{name}"]) / 1e9,
            "fused_pct_f16_dense_peak": 100 * sw.flops_per_gemm / mean[f"fused_{name}"] / 1e9 / 2250.0,
            "decode_gbs": sw.decode_bytes(name) / dec_ms / 1e6,
            "decode_pct_hbm": 100 * sw.decode_bytes(name) / dec_ms / 1e6 / peaks["hbm_gbs"],
            **q[name],
        }
    for name in sw.native:
        # per-tensor FP4 goes through kind::f8f6f4 and runs at the FP8 rate
        formats[f"native_{name}"] = {"tflops": sw.flops_per_gemm / mean[f"native_{name}"] / 1e9,
                                     "pct_fp8_dense_peak": 100 * sw.flops_per_gemm / mean[f"native_{name}"] / 1e9
                                     / 4500.0, **q[f"native_{name}"]}
    # dominant kernel: the kernel (instantiation) with the largest total time;
    # the four post-decode GEMMs are one kernel, the tcgen05 FP16 GEMM
    groups = {}
    for k, v in per_op.items():
        groups.setdefault("gemm_f16" if k.startswith("gemm_after_") else k, []).extend(v)
    totals = {k: sum(v) for k, v in groups.items()}
    dom = max(totals, key=totals.get)
    dom_ms = sum(groups[dom]) / len(groups[dom])
    if dom.startswith("decode_"):
        nm = dom.split("_", 1)[1]
        achieved = sw.decode_bytes(nm) / dom_ms / 1e6
        roof = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"]}
    else:
        achieved = sw.flops_per_gemm / dom_ms / 1e9
        roof = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"]}
    roof["peak_source"] = f"{peaks['source']} (MEASURED_PEAKS.json burst cuBLAS bf16 / copy)"
    roof["traffic"] = traffic_from_profiles(dom)
    roof["share_of_step"] = totals[dom] / total_ms
    roof["launches_per_step"] = len(groups[dom]) // args.steps

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16xf16->f32 (decoded operands); e4m3xe4m3, e2m1xe2m1->f32 native",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": sweep_config(M, N, K, dist.world),
        "roofline": roof,
        "e2e": {"value": dist.world * step_flops * e2e_steps / (e2e_max / 1e3) / 1e12, "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clock,
        "formats": formats,
    }
    if not args.no_extra:
        extra_clocks = ClockSampler(dist.local)
        extra_clocks.start()
        # Each section starts from an empty allocator cache.  The 8192^3 FP4
        # GEMM runs first: right after the seconds-long MLP section the GPU
        # sits under its power cap (measured 1612 MHz, 770 us a launch,
        # against 1965 MHz and 643 us three seconds later); its own clocks
        # are recorded with it, and it runs once more at the end ("after load").
        torch.cuda.empty_cache()
        line["fp4_8192_fused"] = fused_square(torch, tb, peaks, "e2m1")
        torch.cuda.empty_cache()
        line["e4m3_8192_fused"] = fused_square(torch, tb, peaks, "e4m3")
        torch.cuda.empty_cache()
        line["config_256_e4m3"] = config_256(torch, tb)
        torch.cuda.empty_cache()
        # The next three sections start after a pause of two seconds, in the
        # power state an idle GPU returns to, and record their own clocks:
        # right after the large GEMMs above the GPU sits under its power cap
        # at a lower SM clock.
        for key, section in (("nvfp4_8192", nvfp4_square), ("native_8192", native_square)):
            res, clk = rested(torch, lambda: section(torch, tb))
            res["clocks"] = clk
            line[key] = res
            torch.cuda.empty_cache()
        line["decode_stream_14336x4096"] = decode_streams(torch, tb, peaks)
        torch.cuda.empty_cache()
        line["weight_only_mlp"], line["weight_only_mlp_clocks"] = rested(torch, lambda: mlp_weight_only(torch, tb, peaks))
        torch.cuda.empty_cache()
        line["int8_4096"] = int8_square(torch, tb)
        torch.cuda.empty_cache()
        line["fp4_8192_fused_after_load"] = fused_square(torch, tb, peaks, "e2m1")
        torch.cuda.empty_cache()
        # clocks over the extra sections (the headline's own are in "clocks")
        line["clocks_extras"] = extra_clocks.stop()
        line["sharded_weight_gemm"] = sharded_weight_gemm(torch, tb, dist)
    assert tb.device_error() == 0, "a kernel reported a device-side wait timeout"
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline((M, N, K))
    if not args.no_extra:
        line["targets"] = targets(line)
    dist.close()
    if dist.rank == 0:
        print(json.dumps(line), flush=True)


def targets(line: dict) -> dict:
    """The target figures in one compact object, printed last on the line."""
    r = lambda v, d=1: None if v is None else round(float(v), d)
    t = {}
    f4, f4l, e4 = line["fp4_8192_fused"], line["fp4_8192_fused_after_load"], line["e4m3_8192_fused"]
    t["fused_8192_pct_f16_dense_nominal"] = {"e2m1_rested": r(f4["pct_f16_dense_peak_nominal"]),
                                             "e2m1_after_load": r(f4l["pct_f16_dense_peak_nominal"]),
                                             "e4m3": r(e4["pct_f16_dense_peak_nominal"]), "goal": 70}
    skinny = {}
    for row in line["weight_only_mlp"]:
        if row["tokens"] <= 16:
            key = f"{row['W']}_{row['fmt']}"
            lo, hi = skinny.get(key, (1e9, 0.0))
            skinny[key] = (min(lo, row["fused_pct_hbm"]), max(hi, row["fused_pct_hbm"]))
    t["skinny_pct_hbm_min_max"] = {k: [r(lo), r(hi)] for k, (lo, hi) in skinny.items()}
    t["skinny_goal_pct_hbm"] = 80
    fm = line["formats"]
    t["fused_ge_unfused_4096"] = {k: fm[k]["fused_tflops"] >= fm[k]["unfused_tflops"] for k in FORMATS}
    t["native_pct_fp8_dense"] = {k: r(fm[f"native_{k}"]["pct_fp8_dense_peak"]) for k in ("e4m3", "e2m1")}
    nv = line.get("nvfp4_8192")
    if nv:
        t["nvfp4_8192"] = {"tflops": r(nv["tflops"], 0), "pct_fp4_dense": r(nv["pct_fp4_dense_peak_nominal"])}
    t["int8_pct_i8_dense"] = r(line["int8_4096"]["pct_i8_dense_peak"])
    nat = line.get("native_8192")
    if nat:
        t["native_8192_pct_dense"] = {"e4m3": r(nat["e4m3_pct_fp8_dense_peak"]), "i8": r(nat["i8_pct_i8_dense_peak"])}
    sh = line["sharded_weight_gemm"]
    t["sharded"] = {"world": sh["world"], "ms": r(sh["ms"], 3), "gemm_only_ms": r(sh.get("gemm_only_ms"), 3),
                    "check_pass": sh["check"]["pass"], "rel_frob": float(f"{sh['check']['rel_frob_max_vs_fp64']:.2e}")}
    if "nccl" in sh:
        t["sharded"]["nccl"] = {"ms": r(sh["nccl"]["ms"], 3), "allgather_only_ms": r(sh["nccl"]["allgather_only_ms"], 3),
                                "check_pass": sh["nccl"]["check"]["pass"]}
    c1 = line["config_256_e4m3"]
    t["config_256"] = {"us": r(c1["us"], 2), "rel_frob_vs_fp32_pct": r(100 * c1["rel_frob_vs_unquantized_fp32"], 3)}
    nv = (line.get("cpu_baseline") or {}).get("naive_single_thread")
    if nv:
        t["ref_naive_1thread_ms"] = {k: r(v["ms"], 2) for k, v in nv.items()}
    return t


if __name__ == "__main__":
    main()
