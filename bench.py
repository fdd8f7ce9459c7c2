"""Benchmark of the krsi_b200 hot path on B200 (driver contract: one JSON line from rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W]
                  [--workload block|attn|attn_fwd|rmsnorm|geglu|linear_geglu]
  python bench.py --impl reference ...      # the reference's torch CPU path on the host cores
  torchrun --nproc-per-node N bench.py --gpus N ...
  python bench.py --profile-case KIND N [S] # one small seeded case for a profiler (ncu), no timing

Workloads (all inputs synthetic, seeded, CPU-generated):
  block     config 5: 28 pre-norm layers (RMSNorm -> qkv GEMM -> relpos attention -> out GEMM ->
            +res -> RMSNorm -> wi GEMM -> GEGLU -> wo GEMM -> +res), x [32,1024,1152] bf16,
            fwd+bwd with loss = mean(out.float()^2); batch-sharded over N ranks, NCCL all-reduce of
            the weight gradients.  The whole training step (forward, backward, the bucketed
            all-reduces) is one CUDA graph replay; the wi GEMM and the GEGLU forward are one
            kernel.  Metric: tok/s (whole job).  The default; at N=1 its line also carries an
            `ops` object with configs 1-4 and linear_geglu below.
  attn      config 4: relpos attention fwd+bwd, B=8 H=16 L=2048 D=72 bf16. TFLOP/s (12*B*H*L^2*D).
  attn_fwd  config 3: relpos attention fwd, B=2 H=16 L=1024 D=72 bf16. TFLOP/s (4*B*H*L^2*D).
  rmsnorm   config 1: RMSNorm fwd+bwd fp32 [2048,1152]. GB/s (algorithmic bytes).
  geglu     config 2: GEGLU fwd+bwd bf16 [2048,9216]. GB/s (algorithmic bytes).
  linear_geglu  one config-5 layer's gate|value projection with GEGLU in the GEMM epilogue,
            x [32768,1152] @ wi [9216,1152]^T bf16, forward. TFLOP/s (2*rows*K*2F); the breakdown
            times the unfused cuBLAS GEMM + GEGLU kernel on the same inputs.
For the op workloads a step replays one CUDA graph holding C calls, one per rotating input copy
(C copies > 3x the L2 cache, as the reference's time_calls rotates them); N>1 runs replicas.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "kernel-rsi_b200"
for _p in (str(ROOT), str(PKG), str(PKG / "library")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

L2_BYTES = 126 * 1024 * 1024
MAX_COPIES = 32


# ---------------------------------------------------------------- environment helpers

def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def ncu_traffic(kernel_key: str):
    """DRAM bytes per launch of the dominant kernel from a committed ncu capture summary, or None."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.is_file():
        return None
    return json.loads(p.read_text()).get(kernel_key)


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: str):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        loaded = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def physical_gpu() -> str:
    """nvidia-smi's id of this rank's GPU (CUDA_VISIBLE_DEVICES entry, else the local index)."""
    local = int(os.environ.get("LOCAL_RANK", 0))
    vis = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    return vis[local].strip() if local < len(vis) else str(local)


def cpu_info() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def unit_scale(unit: str) -> float:
    return 1e9 if unit == "GB/s" else (1e12 if unit == "TFLOP/s" else 1.0)


# ---------------------------------------------------------------- op workloads
# Each workload exposes: metric, unit, work (per step), setup(dev), step(timed), e2e_loop(dev, n)
# (host buffers in, results read back), launches_per_step, roofline() of its dominant kernel(s), and
# cpu_sample() for the baseline (the reference's torch path on the host cores).

class OpWorkload:
    """An op's fwd(+bwd) over C rotating device-resident input copies (C x inputs > 3 x L2).  All C
    calls are captured in one CUDA graph, as the reference's time_calls does (tools/common.py:
    238-298): a step replays it, so a step is C calls and the device time per call is the step
    time / C, with no host launch cost in it."""
    higher_is_better = True
    scaling = "weak"
    in_bytes = 0
    work_per_call = 0
    launches_per_call = 1

    def __init__(self, rank: int, world: int):
        self.rank, self.world = rank, world
        self.copies = max(2, min(MAX_COPIES, math.ceil(3 * L2_BYTES / max(self.in_bytes, 1))))

    @property
    def work(self):
        return self.work_per_call * self.copies

    @property
    def launches_per_step(self):
        return self.launches_per_call * self.copies

    def setup(self, dev):
        self.setup_host()
        self.dev_inputs = [tuple(t.to(dev) for t in self.host) for _ in range(self.copies)]
        self.e2e_in = tuple(t.pin_memory() for t in self.host)
        self.capture()
        self.i = 0

    def capture(self):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for inp in self.dev_inputs:
                self.call(*inp)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for inp in self.dev_inputs:
                self.call(*inp)
        torch.cuda.synchronize()

    def step(self, timed=None):
        if timed is not None:
            timed[0].record()
        self.graph.replay()
        if timed is not None:
            timed[1].record()

    def roofline(self, kms, pk):
        t = kms / self.copies                               # ms per call
        ach = self.work_per_call / (t / 1e3) / 1e9
        self._call_ms = t
        return {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": ach / pk["hbm_gbs"], "traffic": ncu_traffic(self.kernel_key), "kernel": self.kernel_key,
                "peak_source": pk["source"] + " (STREAM-style copy)",
                "per_launch_group": f"fwd+bwd launches of one call ({self.launches_per_call}), device time "
                                    "per call from the graph replay"}

    def extra(self):
        return {"breakdown": {"ms_per_call": getattr(self, "_call_ms", None), "calls_per_step": self.copies}}

    def e2e_loop(self, dev, n: int):
        """n end-to-end calls through the public API: each call's inputs are copied from pinned host
        memory, the library functions run forward and backward on them, and every result is copied
        back into pinned host memory.  The copies run on their own streams, so call i+1's
        host->device copy and call i-1's device->host copy overlap call i's kernels (two device
        input sets and two host result sets alternate).  Returns (h2d, d2h) bytes per call."""
        main = torch.cuda.current_stream()
        if not hasattr(self, "e2e_dev"):
            self.h2d_stream, self.d2h_stream = torch.cuda.Stream(), torch.cuda.Stream()
            self.e2e_dev = [[torch.empty_like(t, device=dev) for t in self.e2e_in] for _ in range(2)]
            self.e2e_out = [None, None]
        loaded = [torch.cuda.Event(), torch.cuda.Event()]
        consumed = [torch.cuda.Event(), torch.cuda.Event()]

        def load(i):
            k = i % 2
            with torch.cuda.stream(self.h2d_stream), torch.no_grad():
                if i >= 2:
                    self.h2d_stream.wait_event(consumed[k])
                for d, h in zip(self.e2e_dev[k], self.e2e_in):
                    d.copy_(h, non_blocking=True)
                loaded[k].record()

        self.h2d_stream.wait_stream(main)     # the previous loop's kernels are done with the inputs
        load(0)
        d2h = 0
        for i in range(n):
            k = i % 2
            if i + 1 < n:
                load(i + 1)
            main.wait_event(loaded[k])
            res = self.e2e_compute(self.e2e_dev[k])
            consumed[k].record(main)
            if self.e2e_out[k] is None:
                self.e2e_out[k] = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res]
            with torch.cuda.stream(self.d2h_stream):
                self.d2h_stream.wait_stream(main)
                for h, r in zip(self.e2e_out[k], res):
                    r.record_stream(self.d2h_stream)
                    h.copy_(r.detach(), non_blocking=True)
            d2h = sum(r.numel() * r.element_size() for r in res)
        main.wait_stream(self.d2h_stream)
        return sum(t.numel() * t.element_size() for t in self.e2e_in), d2h

    e2e_work = property(lambda self: self.work_per_call)   # e2e steps are single calls

    def close(self):
        self.graph = None


class RMSNormWorkload(OpWorkload):
    name, metric, unit, dtype = "rmsnorm", "RMSNorm fwd+bwd throughput", "GB/s", "f32"
    ROWS, N = 2048, 1152
    # algorithmic bytes: fwd reads x, w, writes y, rstd; bwd reads g, x, w, rstd, writes dx, dw
    FWD_B = ROWS * N * 4 * 2 + N * 4 + ROWS * 4
    BWD_B = ROWS * N * 4 * 3 + N * 4 * 2 + ROWS * 4
    work_per_call = FWD_B + BWD_B
    launches_per_call = 3   # fwd, bwd rows, bwd dw reduction
    kernel_key = "rmsnorm_fwd_bwd"
    in_bytes = 3 * ROWS * N * 4

    def config(self):
        return {"workload": "rmsnorm fwd+bwd fp32 x[2,1024,1152] (config 1)", "rows": self.ROWS, "n": self.N,
                "eps": 1e-6, "l2": "rotating input copies > 3x L2",
                "timing": f"one CUDA graph of {self.copies} calls per step"}

    def setup_host(self):
        from harness.inputs import rmsnorm_inputs

        self.host = rmsnorm_inputs(self.ROWS, self.N, torch.float32, seed=0)

    def call(self, x, w, g):
        y, rstd = torch.ops.krsi.rmsnorm_fwd(x, w, 1e-6)
        return torch.ops.krsi.rmsnorm_bwd(g, x, w, rstd)

    def e2e_compute(self, inputs):
        import rmsnorm

        x, w, g = inputs
        xr, wr = x.requires_grad_(True), w.requires_grad_(True)
        y = rmsnorm.rmsnorm(xr, wr, 1e-6)
        dx, dw = torch.autograd.grad(y, [xr, wr], g)
        return [y.detach(), dx, dw]

    def cpu_sample(self):
        from oracle import ops as O

        x, w, g = self.host
        xr, wr = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
        y = O.rmsnorm_reference(xr, wr, 1e-6)
        torch.autograd.grad(y, [xr, wr], g)
        return self.work_per_call, "one full fwd+bwd of config 1 (reference torch fp32 path)"


class GegluWorkload(RMSNormWorkload):
    name, metric, unit, dtype = "geglu", "GEGLU fwd+bwd throughput", "GB/s", "bf16"
    ROWS, F = 2048, 4608
    FWD_B = ROWS * 2 * F * 2 + ROWS * F * 2
    BWD_B = ROWS * F * 2 + ROWS * 2 * F * 2 * 2
    work_per_call = FWD_B + BWD_B
    launches_per_call = 2
    kernel_key = "geglu_fwd_bwd"
    in_bytes = 3 * ROWS * F * 2

    def config(self):
        return {"workload": "geglu fwd+bwd bf16 u[2,1024,9216] (config 2)", "rows": self.ROWS, "F": self.F,
                "l2": "rotating input copies > 3x L2", "timing": f"one CUDA graph of {self.copies} calls per step"}

    def setup_host(self):
        from harness.inputs import geglu_inputs

        self.host = geglu_inputs(self.ROWS, self.F, torch.bfloat16, seed=0)

    def call(self, u, g):
        torch.ops.krsi.geglu_fwd(u)
        return torch.ops.krsi.geglu_bwd(g, u)

    def e2e_compute(self, inputs):
        import geglu

        u, g = inputs
        ur = u.requires_grad_(True)
        out = geglu.geglu(ur)
        (du,) = torch.autograd.grad(out, [ur], g)
        return [out.detach(), du]

    def cpu_sample(self):
        from oracle import ops as O

        u, g = (t.float() for t in self.host)
        ur = u.clone().requires_grad_(True)
        out = O.geglu_reference(ur)
        torch.autograd.grad(out, [ur], g)
        return self.work_per_call, "one full fwd+bwd of config 2 (reference torch path, fp32 on CPU)"


class LinearGegluWorkload(OpWorkload):
    """The block's feed-forward input at one layer's shape: x [32768, 1152] @ wi [9216, 1152]^T with
    GEGLU in the GEMM's epilogue (krsi::linear_geglu_fwd, one tcgen05 kernel), forward.  Tensor-bound:
    the roofline is the GEMM's FLOPs against the measured bf16 peak.  The breakdown times the unfused
    pair it replaces (cuBLAS GEMM, then the GEGLU kernel) on the same inputs."""
    name, metric, unit, dtype = "linear_geglu", "gate|value projection + GEGLU forward throughput", "TFLOP/s", "bf16"
    ROWS, K, F = 32768, 1152, 4608
    work_per_call = 2 * ROWS * K * 2 * F
    launches_per_call = 1
    kernel_key = "linear_geglu_pair_kernel"
    in_bytes = (ROWS * K + 2 * F * K) * 2

    def config(self):
        return {"workload": "gate|value projection + GEGLU fwd, x[32768,1152] @ wi[9216,1152]^T bf16 (one config-5 "
                            "layer's feed-forward input)", "rows": self.ROWS, "K": self.K, "F": self.F,
                "l2": "rotating input copies > 3x L2 (u and out, 906 MB per call, are written fresh)",
                "timing": f"one CUDA graph of {self.copies} calls per step"}

    def setup_host(self):
        from harness.inputs import gen

        self.host = (gen((self.ROWS, self.K), 21, torch.bfloat16),
                     gen((2 * self.F, self.K), 22, torch.bfloat16, std=0.02))

    def call(self, x, w):
        return torch.ops.krsi.linear_geglu_fwd(x, w)

    def roofline(self, kms, pk):
        t = kms / self.copies
        ach = self.work_per_call / (t / 1e3) / 1e12
        self._call_ms = t
        return {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": ach / pk["bf16_tflops"], "traffic": ncu_traffic(self.kernel_key), "kernel": self.kernel_key,
                "peak_source": pk["source"] + " (cuBLAS bf16 GEMM, burst: the kernel is timed alone)",
                "per_launch_group": "one launch per call, device time per call from the graph replay"}

    def breakdown(self, dev, kms):
        """Device time per call of the unfused pair (cuBLAS GEMM + GEGLU kernel) and of the cuBLAS GEMM
        alone, each as one CUDA graph over the same input copies."""
        res = {}
        for key, fn in (("unfused_ms_per_call", lambda x, w: torch.ops.krsi.geglu_fwd(x @ w.t())),
                        ("cublas_gemm_ms_per_call", lambda x, w: x @ w.t())):
            for inp in self.dev_inputs:
                fn(*inp)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for inp in self.dev_inputs:
                    fn(*inp)
            g.replay()
            torch.cuda.synchronize()
            times = []
            for _ in range(5):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1) / self.copies)
            res[key] = statistics.median(times)
            del g
        return res

    def extra(self):
        b = {"ms_per_call": getattr(self, "_call_ms", None), "calls_per_step": self.copies}
        b.update(getattr(self, "_breakdown", {}))
        return {"breakdown": b}

    def e2e_compute(self, inputs):
        import linear_geglu

        x, w = inputs
        return [linear_geglu.linear_geglu(x, w)]

    def cpu_sample(self):
        x, w = self.host
        rows = 256
        gate, value = (x[:rows].float() @ w.float().t()).chunk(2, dim=-1)
        torch.nn.functional.gelu(gate, approximate="tanh") * value
        return 2 * rows * self.K * 2 * self.F, f"{rows} rows of the projection + GEGLU (reference torch path, fp32)"


class AttnWorkload(OpWorkload):
    """Config 4: relpos attention fwd+bwd, B=8 H=16 L=2048 D=72 bf16 (training mode).  The C forward
    calls and the C backward calls are captured as two CUDA graphs, so the backward (the dominant
    kernels) is timed on its own with CUDA events between them."""
    name, metric, unit, dtype = "attn", "relpos attention fwd+bwd throughput", "TFLOP/s", "bf16"
    B, S, H, D = 8, 2048, 16, 72
    fwd_only = False
    kernel_key = "relpos_bwd_main_kernel"

    @property
    def work_per_call(self):
        return (4 if self.fwd_only else 12) * self.B * self.H * self.S ** 2 * self.D

    @property
    def in_bytes(self):
        return self.B * self.S * self.H * self.D * 2 * (3 if self.fwd_only else 4)

    @property
    def launches_per_call(self):
        return 1 if self.fwd_only else 6   # fwd; bwd prep, main, dq, dpd_diag, dpd

    def config(self):
        return {"workload": f"relpos attention {'fwd' if self.fwd_only else 'fwd+bwd'} bf16 "
                            f"B={self.B} H={self.H} L={self.S} D={self.D}", "flop_convention":
                "4*B*H*L^2*D fwd, 8*B*H*L^2*D bwd (D=72 counted, not the padded 80; bwd recompute not counted)",
                "l2": "rotating input copies > 3x L2",
                "timing": f"CUDA graphs of {self.copies} forward and {self.copies} backward calls per step"}

    def setup_host(self):
        from harness.inputs import attn_inputs

        self.host = attn_inputs(self.B, self.S, self.H, self.D, torch.bfloat16, seed=0)
        self.scale = self.D ** -0.5
        if self.fwd_only:
            self.host = self.host[:2]

    def run_fwd(self, qkv, pd, *rest):
        return torch.ops.krsi.relpos_attn_fwd(qkv, pd, self.B, self.S, self.H, self.D, self.scale)

    def run_bwd(self, saved, qkv, pd, dout):
        _, out32, lse = saved
        return torch.ops.krsi.relpos_attn_bwd(dout, qkv, pd, out32, lse, self.B, self.S, self.H, self.D, self.scale)

    def capture(self):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for inp in self.dev_inputs:
                saved = self.run_fwd(*inp)
                if not self.fwd_only:
                    self.run_bwd(saved, *inp)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.fwd_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.fwd_graph):
            self.saved = [self.run_fwd(*inp) for inp in self.dev_inputs]
        self.bwd_graph = None
        if not self.fwd_only:
            self.bwd_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.bwd_graph):
                for sv, inp in zip(self.saved, self.dev_inputs):
                    self.run_bwd(sv, *inp)
        torch.cuda.synchronize()
        self.events = []

    def step(self, timed=None):
        if timed is None:
            self.fwd_graph.replay()
            if self.bwd_graph is not None:
                self.bwd_graph.replay()
            return
        mid = torch.cuda.Event(enable_timing=True)
        timed[0].record()
        self.fwd_graph.replay()
        mid.record()
        if self.bwd_graph is not None:
            self.bwd_graph.replay()
        timed[1].record()
        self.events.append((timed[0], mid, timed[1]))

    def roofline(self, kms, pk):
        fwd = [a.elapsed_time(m) / self.copies for a, m, _ in self.events]
        bwd = [m.elapsed_time(b) / self.copies for _, m, b in self.events]
        self.fwd_ms, self.bwd_ms = statistics.median(fwd), statistics.median(bwd)
        if self.fwd_only:
            t, flop, key = self.fwd_ms, self.work_per_call, "relpos_fwd_kernel"
        else:
            t, flop, key = self.bwd_ms, 8 * self.B * self.H * self.S ** 2 * self.D, "relpos_bwd (5 kernels)"
        ach = flop / (t / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": ach / pk["bf16_tflops"], "traffic": ncu_traffic(key), "kernel": key,
                "peak_source": pk["source"] + " (burst bf16 cuBLAS)"}

    def extra(self):
        f, b = self.fwd_ms, self.bwd_ms
        d = {"fwd_ms_per_call": f, "calls_per_step": self.copies,
             "fwd_tflops": 4 * self.B * self.H * self.S ** 2 * self.D / (f / 1e3) / 1e12}
        if not self.fwd_only:
            d.update(bwd_ms_per_call=b, bwd_tflops=8 * self.B * self.H * self.S ** 2 * self.D / (b / 1e3) / 1e12,
                     fwd_bwd_tflops_14bhl2d=14 * self.B * self.H * self.S ** 2 * self.D / ((f + b) / 1e3) / 1e12)
        return {"breakdown": d}

    def e2e_compute(self, inputs):
        import relpos_attention as ra

        q, p = inputs[0].requires_grad_(True), inputs[1].requires_grad_(True)
        out = ra.relpos_attention(q, p, self.B, self.S, self.H, self.D, self.scale)
        if self.fwd_only:
            return [out.detach()]
        dq, dp = torch.autograd.grad(out, [q, p], inputs[2])
        return [out.detach(), dq, dp]

    def cpu_sample(self):
        """One batch element (B=1) of the config on the reference's torch path in fp32 (the math
        backend SDPA); work is counted for that batch element only."""
        from harness.inputs import attn_inputs
        from oracle import ops as O

        B1 = 1
        qkv, pd, dout = attn_inputs(B1, self.S, self.H, self.D, torch.bfloat16, seed=0)
        q = qkv.float().requires_grad_(True)
        p = pd.clone().requires_grad_(True)
        out = O.relpos_reference(q, p, B1, self.S, self.H, self.D, self.scale)
        if not self.fwd_only:
            torch.autograd.grad(out, [q, p], dout.float())
        flop = (4 if self.fwd_only else 12) * B1 * self.H * self.S ** 2 * self.D
        return flop, (f"B=1 of the config ({'fwd' if self.fwd_only else 'fwd+bwd'}), reference torch "
                      "fp32 math-SDPA path")

    def close(self):
        self.fwd_graph = self.bwd_graph = None
        self.saved = None


class AttnFwdWorkload(AttnWorkload):
    """Config 3: relpos attention forward, B=2 H=16 L=1024 D=72 bf16."""
    name, metric = "attn_fwd", "relpos attention fwd throughput"
    B, S, H, D = 2, 1024, 16, 72
    fwd_only = True
    kernel_key = "relpos_fwd_kernel"


# ---------------------------------------------------------------- block workload

class BlockWorkload:
    """Config 5: 28-layer pre-norm block stack, x [32,1024,1152] bf16, fwd+bwd, loss =
    mean(out.float()^2); the global batch is sharded over the ranks (strong scaling) and the only
    collective is the layer-bucketed weight-gradient all-reduce (NCCL).  The step runs as one CUDA
    graph replay (harness/graphed.py) of the model built on the library ops."""
    name, metric, unit, dtype = "block", "block stack fwd+bwd training throughput", "tok/s", "bf16"
    higher_is_better = True
    scaling = "strong"
    GLOBAL_B = 32
    kernel_key = "relpos_attention fwd+bwd (in block step)"
    # our kernels per layer per step: rmsnorm 2 x (fwd 1 + bwd 2), attention fwd 1 + bwd 5, geglu 2
    LAUNCHES_PER_LAYER = 14
    # gradient all-reduce buckets: the bf16 weights of this many layers, the last TAIL layers one each
    # (tunable: KRSI_BUCKET_LAYERS, KRSI_BUCKET_TAIL)
    LAYERS_PER_BUCKET = int(os.environ.get("KRSI_BUCKET_LAYERS", "4"))
    TAIL_LAYERS = int(os.environ.get("KRSI_BUCKET_TAIL", "2"))

    def __init__(self, rank, world):
        import harness.block as hb

        self.rank, self.world = rank, world
        self.cfg = hb.BlockConfig()
        self.tokens_per_step = self.GLOBAL_B * self.cfg.seq // world      # this rank's tokens
        self.work = self.cfg.flops_per_token() * self.GLOBAL_B * self.cfg.seq
        self.launches_per_step = self.cfg.layers * self.LAUNCHES_PER_LAYER

    def config(self):
        c = self.cfg
        return {"workload": "block stack (config 5) fwd+bwd", "layers": c.layers, "global_batch": self.GLOBAL_B,
                "seq_len": c.seq, "d_model": c.d, "heads": c.heads, "head_dim": c.head_dim, "ffn": c.ffn,
                "parallelism": f"dp{self.world} (batch-sharded, NCCL grad all-reduce)",
                "allreduce_bucket_layers": self.LAYERS_PER_BUCKET, "allreduce_tail_layers": self.TAIL_LAYERS,
                "flop_per_step": self.work, "l2": "inputs and activations >> L2",
                "timing": "one CUDA graph replay per step (forward, backward, bucketed all-reduce), CUDA events"}

    def setup_host(self):
        g = torch.Generator().manual_seed(0)
        self.x_global = torch.randn(self.GLOBAL_B, self.cfg.seq, self.cfg.d, generator=g).to(torch.bfloat16)

    def setup(self, dev):
        import harness.block as hb
        from harness.graphed import GraphedTrainStep
        from harness.grad_sync import LayerBucketAllReduce, shard_batch

        self.setup_host()
        self.model = hb.BlockStack(self.cfg, hb.LibraryOps(), dev, seed=0)
        self.timer = hb.AttentionTimer(self.model)
        self.reducer = LayerBucketAllReduce(self.model.layers, layers_per_bucket=self.LAYERS_PER_BUCKET,
                                            tail_layers=self.TAIL_LAYERS)
        x = shard_batch(self.x_global, self.rank, self.world)
        self.x = x.to(dev)
        self.x_pinned = x.contiguous().pin_memory()
        self.loss_fn = hb.loss_fn
        self.graphed = GraphedTrainStep(self.model, self.reducer, self.world, self.loss_fn, self.x)

    def step(self, timed=None):
        if timed is not None:
            timed[0].record()
        loss = self.graphed()
        if timed is not None:
            timed[1].record()
        return loss

    def roofline(self, kms, pk):
        # the attention events of the last replay in the timed region
        fwd, bwd = self.timer.fwd_ms(), self.timer.bwd_ms()
        t = fwd + bwd
        c = self.cfg
        B_local = self.GLOBAL_B // self.world
        flop = 12 * B_local * c.heads * c.seq ** 2 * c.head_dim * c.layers
        ach = flop / (t / 1e3) / 1e12
        self._attn = {"attn_ms_per_step": t, "attn_fwd_ms_per_step": fwd, "attn_bwd_ms_per_step": bwd,
                      "attn_share_of_step": t / kms if kms else None}
        return {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": ach / pk["bf16_tflops_sustained"], "traffic": ncu_traffic(self.kernel_key),
                "kernel": self.kernel_key,
                "peak_source": pk["source"] + " (sustained bf16 cuBLAS: timed inside a long step)"}

    def breakdown(self, dev, kms):
        """Where a step's time goes on this rank, beyond the attention share: the same step without
        the gradient all-reduce (a second graph, same shapes), hence the exposed communication; and
        the eager (non-graph) step with the host time it takes to issue it."""
        from harness.graphed import GraphedTrainStep
        from harness.grad_sync import train_step

        out = dict(self._attn)
        out["step_ms"] = kms
        if self.world > 1:
            nocomm = GraphedTrainStep(self.model, self.reducer, self.world, self.loss_fn, self.x,
                                      pool=self.graphed.pool(), allreduce=False)
            ms = []
            for i in range(6):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                nocomm()
                b.record()
                b.synchronize()
                if i:
                    ms.append(a.elapsed_time(b))
            nocomm.close()
            out["compute_only_ms"] = statistics.median(ms)
            out["exposed_allreduce_ms"] = kms - out["compute_only_ms"]
            out["allreduce_bytes"] = self.reducer.bytes
        # eager steps through the same model (the host issues every launch)
        eager, host = [], []
        for i in range(4):
            torch.cuda.synchronize()
            if dist.is_initialized():
                dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            a.record()
            train_step(self.model, self.x, self.reducer, self.world, self.loss_fn)
            b.record()
            t1 = time.perf_counter()
            b.synchronize()
            if i:
                eager.append(a.elapsed_time(b))
                host.append((t1 - t0) * 1e3)
        out["eager_step_ms"] = statistics.median(eager)
        out["eager_host_issue_ms"] = statistics.median(host)
        return out

    def extra(self):
        return {"breakdown": getattr(self, "_breakdown", getattr(self, "_attn", {})),
                "model_tflops": self.work / (self._step_ms / 1e3) / 1e12 if getattr(self, "_step_ms", None) else None}

    def e2e_loop(self, dev, n: int):
        """n training steps through the harness's public step API, each copying its batch shard
        from pinned host memory into the step's input buffer and reading the loss back to the host
        (which also ends the step).  Returns (h2d, d2h) bytes per step."""
        for _ in range(n):
            self.graphed.static_x.copy_(self.x_pinned, non_blocking=True)   # host -> device, pinned
            loss = self.graphed()
            loss.item()                   # device -> host read of the step's result
        return self.x_pinned.numel() * 2, 4

    def cpu_sample(self):
        """One layer at B=1 (1024 tokens) fwd+bwd on the reference's torch path in fp32; reported
        as tokens through the full 28-layer stack per second (time x 28 layers)."""
        import harness.block as hb
        from oracle import ops as O

        class RefOps:
            rmsnorm = staticmethod(O.rmsnorm_reference)
            geglu = staticmethod(O.geglu_reference)
            relpos_attention = staticmethod(O.relpos_reference)

        if not hasattr(self, "_cpu_layer"):
            cfg1 = hb.BlockConfig(layers=1)
            self._cpu_layer = hb.BlockStack(cfg1, RefOps(), torch.device("cpu"), seed=0, dtype=torch.float32)
        x = self.x_global[:1].float().clone().requires_grad_(True)
        loss = hb.loss_fn(self._cpu_layer(x))
        loss.backward()
        return self.cfg.seq / self.cfg.layers, "1 layer, B=1 (1024 tokens) fwd+bwd fp32 reference torch path, counted as 1024/28 full-stack tokens"

    def close(self):
        if getattr(self, "graphed", None) is not None:
            self.graphed.close()
            self.graphed = None


WORKLOADS = {"rmsnorm": RMSNormWorkload, "geglu": GegluWorkload, "attn": AttnWorkload,
             "attn_fwd": AttnFwdWorkload, "linear_geglu": LinearGegluWorkload, "block": BlockWorkload}
OPS_IN_DEFAULT_LINE = ("rmsnorm", "geglu", "attn_fwd", "attn", "linear_geglu")


# ---------------------------------------------------------------- timing

def time_steps(wl, steps, warmup):
    for _ in range(warmup):
        wl.step()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu()) as clk:
        start.record()
        for i in range(steps):
            wl.step(timed=ev[i])
        end.record()
        torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    total_ms = start.elapsed_time(end)
    kernel_ms = [a.elapsed_time(b) for a, b in ev]
    return total_ms, kernel_ms, clk.summary()


def max_over_ranks(v: float) -> float:
    if not dist.is_initialized():
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_baseline(wl, budget_s=15.0, max_samples=50):
    """The reference's torch CPU path on the host cores, bounded to about budget_s seconds."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    work, desc = wl.cpu_sample()             # warm-up call
    t0 = time.perf_counter()
    n, done = 0, 0.0
    while True:
        w, desc = wl.cpu_sample()
        n += 1
        done += w
        if time.perf_counter() - t0 > budget_s or n >= max_samples:
            break
    dt = time.perf_counter() - t0
    return {"value": done / dt / unit_scale(wl.unit), "unit": wl.unit, "cores": threads, "kind": "port",
            "sample": f"{n} x {desc}; {dt:.1f} s on {cpu_info()}"}


def measure_e2e(wl, dev, min_ms=100.0):
    """End to end through the public API with host buffers: three timed runs of >= min_ms each (at
    least 3 steps); the median run is reported, so one host-side stall does not decide it."""
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    wl.e2e_loop(dev, 2)                   # allocates the pinned and device buffers
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    wl.e2e_loop(dev, 2)
    torch.cuda.synchronize()
    est_ms = (time.perf_counter() - t0) * 1e3 / 2
    n = max(3, min(1000, math.ceil(min_ms / max(est_ms, 1e-3))))
    runs = []
    for _ in range(3):
        torch.cuda.synchronize()
        if dist.is_initialized():
            dist.barrier()
        t0 = time.perf_counter()
        h2d, d2h = wl.e2e_loop(dev, n)
        torch.cuda.synchronize()
        runs.append((time.perf_counter() - t0) * 1e3 / n)
    return max_over_ranks(statistics.median(runs)), h2d, d2h, n


# ---------------------------------------------------------------- arms

def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU path (torch eager, as restated in oracle/) on the host
    cores, rank 0 only; other ranks exit without work."""
    if rank != 0:
        return
    wl = WORKLOADS[args.workload](rank, world)
    wl.setup_host()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for _ in range(args.warmup):
        wl.cpu_sample()
    t0 = time.perf_counter()
    done, desc = 0.0, ""
    for _ in range(args.steps):
        w, desc = wl.cpu_sample()
        done += w
    dt = time.perf_counter() - t0
    value = done / dt / unit_scale(wl.unit)
    line = {"impl": "reference", "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / max(args.steps, 1),
            "higher_is_better": wl.higher_is_better, "scaling": wl.scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": wl.config(),
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": f"{args.steps} x {desc} on {cpu_info()}"},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def measure_workload(wl, args, dev, rank, world, steps, warmup, cpu_budget_s):
    """Timed steps, e2e, roofline, (N=1) CPU baseline of one workload; returns the JSON dict."""
    wl.setup(dev)
    total_ms, kernel_ms, clocks = time_steps(wl, steps, warmup)
    ms = max_over_ranks(total_ms / steps)
    scale = unit_scale(wl.unit)
    if wl.unit == "tok/s":
        value = wl.tokens_per_step * world / (ms / 1e3)
    else:
        value = wl.work * world / (ms / 1e3) / scale
    wl._step_ms = ms
    pk = peaks()
    kms = statistics.median(kernel_ms) if kernel_ms else None
    roof = wl.roofline(kms, pk)         # reads the events of the timed region: before anything else
    if hasattr(wl, "breakdown"):
        wl._breakdown = wl.breakdown(dev, kms)
    e2e_ms, h2d, d2h, e2e_n = measure_e2e(wl, dev)
    if wl.unit == "tok/s":
        e2e_val = wl.tokens_per_step * world / (e2e_ms / 1e3)
    else:
        e2e_val = wl.e2e_work * world / (e2e_ms / 1e3) / scale
    line = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms, "higher_is_better": wl.higher_is_better,
            "scaling": wl.scaling, "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded, CPU-generated)",
            "config": wl.config(), "clocks": clocks,
            "e2e": {"value": e2e_val, "unit": wl.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "timing": f"median of 3 host-timed runs of {e2e_n} steps"},
            "gpu_launches": wl.launches_per_step * steps, "roofline": roof}
    if world == 1 and cpu_budget_s > 0 and rank == 0:
        line["cpu_baseline"] = cpu_baseline(wl, budget_s=cpu_budget_s)
    if hasattr(wl, "extra"):
        line.update(wl.extra())
    return line


def release(wl):
    wl.close()
    del wl
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def run_krsi_arm(args, rank, world):
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    import rmsnorm  # noqa: F401  (loads the native extension; fails loudly without it)

    wl = WORKLOADS[args.workload](rank, world)
    try:
        line = measure_workload(wl, args, dev, rank, world, args.steps, args.warmup,
                                0.0 if args.no_cpu_baseline else 15.0)
    finally:
        release(wl)
    if args.workload == "block" and world == 1 and not args.no_ops:
        # configs 1-4 and the fused projection on the same GPU, each graph-timed with its roofline
        # and CPU baseline
        ops = {}
        for name in OPS_IN_DEFAULT_LINE:
            owl = WORKLOADS[name](rank, world)
            try:
                d = measure_workload(owl, args, dev, rank, world, 20, 5, 0.0 if args.no_cpu_baseline else 4.0)
            finally:
                release(owl)
            ops[name] = {k: d[k] for k in ("metric", "value", "unit", "dtype", "steps", "warmup", "ms_per_step",
                                          "config", "roofline", "e2e", "clocks", "gpu_launches",
                                          "cpu_baseline", "breakdown") if k in d}
        line["ops"] = ops
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_profile_case(which: str, n: int, S: int | None):
    """Three warm-up calls and one more of one small seeded case (for ncu: pair with -s/-c)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    import _ext
    from harness.inputs import attn_inputs, geglu_inputs, rmsnorm_inputs

    ops = torch.ops.krsi
    for _ in range(4):
        if which in ("rmsnorm", "rmsnorm_bf16"):
            dt = torch.float32 if which == "rmsnorm" else torch.bfloat16
            x, w, g = (t.to(dev) for t in rmsnorm_inputs(n, 1152, dt, seed=0))
            y, r = ops.rmsnorm_fwd(x, w, 1e-6)
            ops.rmsnorm_bwd(g, x, w, r)
        elif which == "geglu":
            u, g = (t.to(dev) for t in geglu_inputs(n, 4608, torch.bfloat16, seed=0))
            ops.geglu_fwd(u)
            ops.geglu_bwd(g, u)
        elif which == "linear_geglu":
            from harness.inputs import gen

            x = gen((n, 1152), 21, torch.bfloat16).to(dev)
            w = gen((2 * 4608, 1152), 22, torch.bfloat16, std=0.02).to(dev)
            ops.linear_geglu_fwd(x, w)
        elif which == "linear_geglu_bwd":
            from harness.inputs import gen

            dy = gen((n, 1152), 23, torch.bfloat16).to(dev)
            w = gen((1152, 4608), 24, torch.bfloat16, std=0.02).to(dev)
            u = gen((n, 2 * 4608), 25, torch.bfloat16).to(dev)
            ops.linear_geglu_bwd(dy, w, u)
        elif which == "t5_bias":
            H, nb = 16, 32
            g = torch.Generator().manual_seed(0)
            table = (0.5 * torch.randn(nb, H, generator=g)).to(dev)
            pd = ops.t5_bias_fwd(table, n, nb, 128, True)
            ops.t5_bias_bwd(torch.randn_like(pd), table, n, nb, 128, True)
        elif which in ("attn", "attn_fwd"):
            H, D = 16, 72
            qkv, pd, dout = (t.to(dev) for t in attn_inputs(n, S, H, D, torch.bfloat16, seed=0))
            out, out32, lse = ops.relpos_attn_fwd(qkv, pd, n, S, H, D, D ** -0.5)
            if which == "attn":
                ops.relpos_attn_bwd(dout, qkv, pd, out32, lse, n, S, H, D, D ** -0.5)
        else:
            raise SystemExit(f"unknown profile case {which!r}")
    torch.cuda.synchronize()
    assert _ext.device_status(clear=True) == 0
    print("ok", which, flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="krsi", choices=["krsi", "reference"])
    ap.add_argument("--workload", default=os.environ.get("KRSI_BENCH_WORKLOAD", "block"), choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ops", action="store_true", help="block at N=1: skip the `ops` object (configs 1-4, linear_geglu)")
    ap.add_argument("--profile-case", nargs="+", metavar="ARG",
                    help="KIND N [S]: rmsnorm|rmsnorm_bf16 ROWS, geglu ROWS, attn|attn_fwd B S, t5_bias S")
    args = ap.parse_args()
    if args.profile_case:
        pc = args.profile_case
        run_profile_case(pc[0], int(pc[1]), int(pc[2]) if len(pc) > 2 else None)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and args.impl != "reference":
        from datetime import timedelta

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        # NCCL's kernels run on a high-priority stream: the compute kernels are chained by dependent
        # launches (the next grid is always pending), so at equal priority the block scheduler hands
        # freed SMs to compute first and the gradient all-reduces wait for SMs
        # (KRSI_NCCL_HIGH_PRIORITY=0 restores the default priority)
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = os.environ.get("KRSI_NCCL_HIGH_PRIORITY", "1") != "0"
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), pg_options=opts,
                                device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
    try:
        if args.impl == "reference":
            run_reference_arm(args, rank, world)
        else:
            run_krsi_arm(args, rank, world)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
