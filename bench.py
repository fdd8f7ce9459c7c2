"""Benchmark of the krsi_b200 hot path on B200 (driver contract: one JSON line from rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload block|attn|attn_fwd|rmsnorm|geglu]
  python bench.py --impl reference ...      # the reference's torch CPU path on the host cores
  torchrun --nproc-per-node N bench.py --gpus N ...

Workloads (all inputs synthetic, seeded, CPU-generated):
  block     config 5: 28 pre-norm layers (RMSNorm -> qkv GEMM -> relpos attention -> out GEMM ->
            +res -> RMSNorm -> wi GEMM -> GEGLU -> wo GEMM -> +res), x [32,1024,1152] bf16,
            fwd+bwd with loss = mean(out.float()^2); batch-sharded over N ranks, NCCL all-reduce of
            the weight gradients. Metric: tok/s (whole job). The default.
  attn      config 4: relpos attention fwd+bwd, B=8 H=16 L=2048 D=72 bf16. TFLOP/s (12*B*H*L^2*D).
  attn_fwd  config 3: relpos attention fwd, B=2 H=16 L=1024 D=72 bf16. TFLOP/s (4*B*H*L^2*D).
  rmsnorm   config 1: RMSNorm fwd+bwd fp32 [2048,1152]. GB/s (algorithmic bytes).
  geglu     config 2: GEGLU fwd+bwd bf16 [2048,9216]. GB/s (algorithmic bytes).
For the op workloads a "step" is one fwd+bwd (or fwd) of the op; N>1 runs replicas (weak scaling).
"""
from __future__ import annotations

import argparse
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

    def __init__(self, gpu_index: int):
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


# ---------------------------------------------------------------- workloads
# Each workload exposes: metric, unit, work_per_step (bytes or FLOP), setup(dev), step(),
# e2e_loop(dev, n) (host buffers in, results read back), launches_per_step, dominant kernel timing,
# and a CPU sample for the baseline.

class OpWorkload:
    """An op fwd(+bwd) on rotating device-resident input copies (working set > L2).  Each copy's
    call is captured once in a CUDA graph, so the timed region measures device time, not the
    host's op dispatch; a step replays one copy's graph."""
    higher_is_better = True
    scaling = "weak"
    in_bytes = 0

    def __init__(self, rank: int, world: int):
        self.rank, self.world = rank, world

    def setup(self, dev):
        self.setup_host()
        self.copies = max(2, math.ceil(3 * L2_BYTES / max(self.in_bytes, 1)))
        self.dev_inputs = [tuple(t.to(dev) for t in self.host) for _ in range(self.copies)]
        self.e2e_in = tuple(t.pin_memory() for t in self.host)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for inp in self.dev_inputs:
                self.call(*inp)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graphs = []
        for inp in self.dev_inputs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.call(*inp)
            self.graphs.append(g)
        self.i = 0

    def e2e_loop(self, dev, n: int):
        """n end-to-end steps through the public API: each step's inputs are copied from pinned host
        memory, the library functions run forward and backward on them, and every result is copied
        back into pinned host memory.  The copies run on their own streams, so step i+1's
        host->device copy and step i-1's device->host copy overlap step i's kernels (two device
        input sets and two host result sets alternate).  Returns (h2d, d2h) bytes per step."""
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

    def step(self, timed=None):
        g = self.graphs[self.i % self.copies]
        self.i += 1
        if timed is not None:
            timed[0].record()
        g.replay()
        if timed is not None:
            timed[1].record()


class RMSNormWorkload(OpWorkload):
    name, metric, unit, dtype = "rmsnorm", "RMSNorm fwd+bwd throughput", "GB/s", "f32"
    ROWS, N = 2048, 1152
    # algorithmic bytes: fwd reads x, w, writes y, rstd; bwd reads g, x, w, rstd, writes dx, dw
    FWD_B = ROWS * N * 4 * 2 + N * 4 + ROWS * 4
    BWD_B = ROWS * N * 4 * 3 + N * 4 * 2 + ROWS * 4
    work = FWD_B + BWD_B
    launches_per_step = 3   # fwd, bwd rows, bwd dw reduction
    kernel_key = "rmsnorm_fwd_bwd"

    def config(self):
        return {"workload": "rmsnorm fwd+bwd fp32 x[2,1024,1152] (config 1)", "rows": self.ROWS, "n": self.N,
                "eps": 1e-6, "l2": "rotating input copies > L2", "timing": "CUDA graph per call"}

    def setup_host(self):
        from oracle import ops as O  # seeded input generator only

        self.host = O.rmsnorm_inputs(self.ROWS, self.N, torch.float32, seed=0)

    in_bytes = 3 * ROWS * N * 4

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
        return self.work, "one full fwd+bwd of config 1 (reference torch fp32 path)"


class GegluWorkload(RMSNormWorkload):
    name, metric, unit, dtype = "geglu", "GEGLU fwd+bwd throughput", "GB/s", "bf16"
    ROWS, F = 2048, 4608
    FWD_B = ROWS * 2 * F * 2 + ROWS * F * 2
    BWD_B = ROWS * F * 2 + ROWS * 2 * F * 2 * 2
    work = FWD_B + BWD_B
    launches_per_step = 2
    kernel_key = "geglu_fwd_bwd"

    def config(self):
        return {"workload": "geglu fwd+bwd bf16 u[2,1024,9216] (config 2)", "rows": self.ROWS, "F": self.F,
                "l2": "rotating input copies > L2", "timing": "CUDA graph per call"}

    def setup_host(self):
        from oracle import ops as O

        self.host = O.geglu_inputs(self.ROWS, self.F, torch.bfloat16, seed=0)

    in_bytes = 3 * ROWS * F * 2

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
        return self.work, "one full fwd+bwd of config 2 (reference torch path, fp32 on CPU)"


class AttnWorkload(OpWorkload):
    """Config 4: relpos attention fwd+bwd, B=8 H=16 L=2048 D=72 bf16 (training mode).  Forward and
    backward are captured as separate CUDA graphs so the backward (the dominant kernel) is timed on
    its own with CUDA events."""
    name, metric, unit, dtype = "attn", "relpos attention fwd+bwd throughput", "TFLOP/s", "bf16"
    B, S, H, D = 8, 2048, 16, 72
    fwd_only = False

    @property
    def work(self):
        return (4 if self.fwd_only else 12) * self.B * self.H * self.S ** 2 * self.D

    @property
    def in_bytes(self):
        return self.B * self.S * self.H * self.D * 2 * (3 if self.fwd_only else 4)

    launches_per_step = 6   # fwd; bwd prep, main, dq, dpd_diag, dpd
    kernel_key = "relpos_bwd_main_kernel"

    def config(self):
        return {"workload": f"relpos attention {'fwd' if self.fwd_only else 'fwd+bwd'} bf16 "
                            f"B={self.B} H={self.H} L={self.S} D={self.D}", "flop_convention":
                "4*B*H*L^2*D fwd, 8*B*H*L^2*D bwd (D=72 counted, not the padded 80; bwd recompute not counted)",
                "l2": "rotating input copies > L2", "timing": "CUDA graphs (fwd, bwd)"}

    def setup_host(self):
        from oracle import ops as O

        self.host = O.attn_inputs(self.B, self.S, self.H, self.D, torch.bfloat16, seed=0)
        self.scale = self.D ** -0.5

    def setup(self, dev):
        self.setup_host()
        self.copies = max(2, math.ceil(3 * L2_BYTES / max(self.in_bytes, 1)))
        self.dev_inputs = [tuple(t.to(dev) for t in self.host) for _ in range(self.copies)]
        self.e2e_in = tuple(t.pin_memory() for t in (self.host[:2] if self.fwd_only else self.host))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for inp in self.dev_inputs:
                self.run_fwd(*inp)
                if not self.fwd_only:
                    self.run_bwd(*inp)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.fwd_graphs, self.bwd_graphs = [], []
        for inp in self.dev_inputs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.run_fwd(*inp)
            self.fwd_graphs.append(g)
            if not self.fwd_only:
                g2 = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g2):
                    self.run_bwd(*inp)
                self.bwd_graphs.append(g2)
        self.i = 0
        self.bwd_ms, self.fwd_ms = [], []

    def run_fwd(self, qkv, pd, dout):
        self.saved = torch.ops.krsi.relpos_attn_fwd(qkv, pd, self.B, self.S, self.H, self.D, self.scale)
        return self.saved

    def run_bwd(self, qkv, pd, dout):
        _, out32, lse = self.saved
        return torch.ops.krsi.relpos_attn_bwd(dout, qkv, pd, out32, lse, self.B, self.S, self.H, self.D, self.scale)

    def step(self, timed=None):
        k = self.i % self.copies
        self.i += 1
        if timed is None:
            self.fwd_graphs[k].replay()
            if not self.fwd_only:
                self.bwd_graphs[k].replay()
            return
        mid = torch.cuda.Event(enable_timing=True)
        timed[0].record()
        self.fwd_graphs[k].replay()
        mid.record()
        if not self.fwd_only:
            self.bwd_graphs[k].replay()
        timed[1].record()
        self._pending = (timed[0], mid, timed[1])
        self.events = getattr(self, "events", []) + [self._pending]

    def roofline(self, kms, pk):
        fwd = [a.elapsed_time(m) for a, m, _ in self.events]
        bwd = [m.elapsed_time(b) for _, m, b in self.events]
        self.fwd_ms, self.bwd_ms = fwd, bwd
        if self.fwd_only:
            t, flop, key = statistics.median(fwd), self.work, "relpos_fwd_kernel"
        else:
            t, flop, key = statistics.median(bwd), 8 * self.B * self.H * self.S ** 2 * self.D, "relpos_bwd (5 kernels)"
        ach = flop / (t / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": ach / pk["bf16_tflops"], "traffic": ncu_traffic(key), "kernel": key,
                "peak_source": pk["source"] + " (burst bf16 cuBLAS)"}

    def extra(self):
        f = statistics.median(self.fwd_ms) if self.fwd_ms else None
        b = statistics.median(self.bwd_ms) if self.bwd_ms else None
        d = {"fwd_ms": f}
        if not self.fwd_only:
            d.update(bwd_ms=b, fwd_tflops=4 * self.B * self.H * self.S ** 2 * self.D / (f / 1e3) / 1e12,
                     bwd_tflops=8 * self.B * self.H * self.S ** 2 * self.D / (b / 1e3) / 1e12,
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
        from oracle import ops as O

        B1 = 1
        qkv, pd, dout = (t[: B1 * self.S] if t.dim() == 2 and t.shape[0] == self.B * self.S else t for t in self.host)
        q = qkv.float().clone().requires_grad_(True)
        p = pd.clone().requires_grad_(True)
        out = O.relpos_reference(q, p, B1, self.S, self.H, self.D, self.scale)
        if not self.fwd_only:
            torch.autograd.grad(out, [q, p], dout.float())
        flop = (4 if self.fwd_only else 12) * B1 * self.H * self.S ** 2 * self.D
        return flop, (f"B=1 slice of the config ({'fwd' if self.fwd_only else 'fwd+bwd'}), reference torch "
                      "fp32 math-SDPA path")


class AttnFwdWorkload(AttnWorkload):
    """Config 3: relpos attention forward, B=2 H=16 L=1024 D=72 bf16."""
    name, metric = "attn_fwd", "relpos attention fwd throughput"
    B, S, H, D = 2, 1024, 16, 72
    fwd_only = True
    launches_per_step = 1
    kernel_key = "relpos_fwd_kernel"


class TimedAttention(torch.autograd.Function):
    """relpos_attention with CUDA events around its forward and backward kernels (same ops as the
    library's RelPosAttention), so the block step can report the attention roofline live."""
    log = None

    @staticmethod
    def forward(ctx, qkv, pd, B, S, H, D, scale):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out, out32, lse = torch.ops.krsi.relpos_attn_fwd(qkv, pd, B, S, H, D, scale)
        e1.record()
        if TimedAttention.log is not None:
            TimedAttention.log.append(("fwd", e0, e1))
        ctx.save_for_backward(qkv, pd, out32, lse)
        ctx.dims = (B, S, H, D, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dqkv, dpd = torch.ops.krsi.relpos_attn_bwd(dout.contiguous(), *ctx.saved_tensors, *ctx.dims)
        e1.record()
        if TimedAttention.log is not None:
            TimedAttention.log.append(("bwd", e0, e1))
        return dqkv, dpd, None, None, None, None, None


class BlockWorkload:
    """Config 5: 28-layer pre-norm block stack, x [32,1024,1152] bf16, fwd+bwd, loss =
    mean(out.float()^2); the global batch is sharded over the ranks (strong scaling) and the only
    collective is the layer-bucketed weight-gradient all-reduce (NCCL)."""
    name, metric, unit, dtype = "block", "block stack fwd+bwd training throughput", "tok/s", "bf16"
    higher_is_better = True
    scaling = "strong"
    GLOBAL_B = 32
    kernel_key = "relpos_attention fwd+bwd (in block step)"

    def __init__(self, rank, world):
        import harness.block as hb

        self.rank, self.world = rank, world
        self.cfg = hb.BlockConfig()
        self.tokens_per_step = self.GLOBAL_B * self.cfg.seq // world      # this rank's tokens
        self.work = self.cfg.flops_per_token() * self.GLOBAL_B * self.cfg.seq
        self.launches_per_step = self.cfg.layers * 14   # rmsnorm 2x(1+2), attn 1+5, geglu 1+1

    def config(self):
        c = self.cfg
        return {"workload": "block stack (config 5) fwd+bwd", "layers": c.layers, "global_batch": self.GLOBAL_B,
                "seq_len": c.seq, "d_model": c.d, "heads": c.heads, "head_dim": c.head_dim, "ffn": c.ffn,
                "parallelism": f"dp{self.world} (batch-sharded, NCCL grad all-reduce)",
                "flop_per_step": self.work, "l2": "inputs and activations >> L2",
                "timing": "eager autograd (CUDA events)"}

    def setup_host(self):
        g = torch.Generator().manual_seed(0)
        self.x_global = torch.randn(self.GLOBAL_B, self.cfg.seq, self.cfg.d, generator=g).to(torch.bfloat16)

    def setup(self, dev):
        import harness.block as hb
        from harness.grad_sync import LayerBucketAllReduce, shard_batch

        self.setup_host()
        ops = hb.LibraryOps()
        ops.relpos_attention = TimedAttention.apply
        self.model = hb.BlockStack(self.cfg, ops, dev, seed=0)
        self.reducer = LayerBucketAllReduce(self.model.layers)
        x = shard_batch(self.x_global, self.rank, self.world)
        self.x = x.to(dev)
        self.x_pinned = x.contiguous().pin_memory()
        self.events = []
        self.loss_fn = hb.loss_fn

    def step(self, timed=None):
        from harness.grad_sync import train_step

        TimedAttention.log = [] if timed is not None else None
        if timed is not None:
            timed[0].record()
        loss = train_step(self.model, self.x, self.reducer, self.world, self.loss_fn)
        if timed is not None:
            timed[1].record()
            self.events.append(TimedAttention.log)
        TimedAttention.log = None
        return loss

    def roofline(self, kms, pk):
        per_step = [sum(a.elapsed_time(b) for _, a, b in log) for log in self.events]
        fwd = [sum(a.elapsed_time(b) for k, a, b in log if k == "fwd") for log in self.events]
        t = statistics.median(per_step)
        c = self.cfg
        B_local = self.GLOBAL_B // self.world
        flop = 12 * B_local * c.heads * c.seq ** 2 * c.head_dim * c.layers
        ach = flop / (t / 1e3) / 1e12
        self._attn = {"attn_ms_per_step": t, "attn_fwd_ms_per_step": statistics.median(fwd),
                      "attn_share_of_step": t / kms if kms else None}
        return {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": ach / pk["bf16_tflops_sustained"], "traffic": ncu_traffic(self.kernel_key),
                "kernel": self.kernel_key, "peak_source": pk["source"] + " (sustained bf16 cuBLAS: timed inside a long step)"}

    def extra(self):
        return {"breakdown": getattr(self, "_attn", {}),
                "model_tflops": self.work / (self._step_ms / 1e3) / 1e12 if getattr(self, "_step_ms", None) else None}

    def e2e_loop(self, dev, n: int):
        """n training steps through the public API, each copying its batch shard from pinned host
        memory and reading the loss back to the host (which also ends the step).  Returns (h2d,
        d2h) bytes per step."""
        from harness.grad_sync import train_step

        for _ in range(n):
            x = self.x_pinned.to(dev, non_blocking=True)
            loss = train_step(self.model, x, self.reducer, self.world, self.loss_fn)
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


WORKLOADS = {"rmsnorm": RMSNormWorkload, "geglu": GegluWorkload, "attn": AttnWorkload,
             "attn_fwd": AttnFwdWorkload, "block": BlockWorkload}


def load_workloads():
    try:
        import bench_attn  # noqa: F401  (registers attn / attn_fwd / block when present)
    except ImportError:
        pass


# ---------------------------------------------------------------- timing

def time_steps(wl, steps, warmup, dev):
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


def cpu_baseline(wl, budget_s=15.0):
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
        if time.perf_counter() - t0 > budget_s or n >= 50:
            break
    dt = time.perf_counter() - t0
    scale = 1e9 if wl.unit == "GB/s" else (1e12 if wl.unit == "TFLOP/s" else 1.0)
    return {"value": done / dt / scale, "unit": wl.unit, "cores": threads, "kind": "port",
            "sample": f"{n} x {desc}; {dt:.1f} s on {cpu_info()}"}


# ---------------------------------------------------------------- arms

def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU path (torch eager, as restated in oracle/) on the host
    cores, rank 0 only; other ranks exit without work."""
    if rank != 0:
        return
    load_workloads()
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
    scale = 1e9 if wl.unit == "GB/s" else (1e12 if wl.unit == "TFLOP/s" else 1.0)
    value = done / dt / scale
    line = {"impl": "reference", "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / max(args.steps, 1),
            "higher_is_better": wl.higher_is_better, "scaling": wl.scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": wl.config(),
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": f"{args.steps} x {desc} on {cpu_info()}"},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_krsi_arm(args, rank, world):
    load_workloads()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    import rmsnorm  # noqa: F401  (loads the native extension; fails loudly without it)

    wl = WORKLOADS[args.workload](rank, world)
    wl.setup(dev)
    total_ms, kernel_ms, clocks = time_steps(wl, args.steps, args.warmup, dev)
    ms = max_over_ranks(total_ms / args.steps)
    scale = 1e9 if wl.unit == "GB/s" else (1e12 if wl.unit == "TFLOP/s" else 1.0)
    per_step_work = wl.work * (world if wl.scaling == "weak" and wl.unit != "tok/s" else 1)
    value = per_step_work / (ms / 1e3) / scale if wl.unit != "tok/s" else wl.tokens_per_step * world / (ms / 1e3)
    wl._step_ms = ms

    # end to end through the public API, host buffers in and results out, every step
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    wl.e2e_loop(dev, 2)                   # allocates the pinned and device buffers
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    wl.e2e_loop(dev, 2)
    torch.cuda.synchronize()
    est_ms = (time.perf_counter() - t0) * 1e3 / 2
    # three timed runs of >= 100 ms each (at least 3 steps); the median run is reported, so one
    # host-side stall in a sub-millisecond step does not decide the number
    e2e_steps = max(3, min(1000, math.ceil(100.0 / max(est_ms, 1e-3))))
    runs = []
    for _ in range(3):
        torch.cuda.synchronize()
        if dist.is_initialized():
            dist.barrier()
        t0 = time.perf_counter()
        h2d, d2h = wl.e2e_loop(dev, e2e_steps)
        torch.cuda.synchronize()
        runs.append((time.perf_counter() - t0) * 1e3 / e2e_steps)
    e2e_ms = max_over_ranks(statistics.median(runs))
    e2e_val = (per_step_work / (e2e_ms / 1e3) / scale if wl.unit != "tok/s"
               else wl.tokens_per_step * world / (e2e_ms / 1e3))

    # roofline of the dominant kernel (its own CUDA-event time inside the timed region)
    pk = peaks()
    kms = statistics.median(kernel_ms) if kernel_ms else None
    roof = wl.roofline(kms, pk) if hasattr(wl, "roofline") else {
        "bound": "hbm", "achieved": wl.work / (kms / 1e3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
        "frac": wl.work / (kms / 1e3) / 1e9 / pk["hbm_gbs"], "traffic": ncu_traffic(wl.kernel_key),
        "kernel": wl.kernel_key, "peak_source": pk["source"]}

    if rank != 0:
        return
    line = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": wl.higher_is_better,
            "scaling": wl.scaling, "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded, CPU-generated)",
            "config": wl.config(), "clocks": clocks,
            "e2e": {"value": e2e_val, "unit": wl.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "timing": f"median of 3 host-timed runs of {e2e_steps} steps"},
            "gpu_launches": wl.launches_per_step * args.steps, "roofline": roof}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl)
    if hasattr(wl, "extra"):
        line.update(wl.extra())
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="krsi", choices=["krsi", "reference"])
    ap.add_argument("--workload", default=os.environ.get("KRSI_BENCH_WORKLOAD", "block"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and args.impl != "reference":
        from datetime import timedelta

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
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
