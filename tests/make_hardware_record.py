"""Measure this GPU's ceilings and write them in the reference's hardware-record format.

The reference's tools/hw.py measures, once per machine, the figures its tools divide by (dense GEMM
TFLOP/s per dtype as cuBLAS reaches them; HBM copy, read and write bandwidth) and writes
hardware/<slug of the device name>.json (tools/hw.py:90-183, file name from tools/common.py:31-37);
its H20 record is hardware/nvidia_h20_3e.json.  The consumers read few keys: tools/common.py:55-64
(peaks) takes `tflops` fp16 / bf16 / fp32 / tf32 and the larger of `bw_copy_gbs` and `bw_read_gbs`;
tools/region.py:140-180 and tools/bench.py:302-322 name `device`.  Those tools are not present on the
GPU hosts this repository runs on, so this script makes the same measurements with its own code (the
same operand sizes, best of 5 rounds of timed calls after 3 warm-up calls, so that the figures
compare with the reference's record) and writes the same keys:

  python tests/make_hardware_record.py --out kernel-rsi_b200/hardware/nvidia_b200.json [--probe-ncu]

Where it differs, on purpose:
- No Triton probe: this build has no Triton kernels.  Launch overhead is measured for a torch
  elementwise op, for one of this library's ops (`krsi::geglu_fwd`, eager) and for a CUDA graph
  holding that op (`launch_us_torch`, `launch_us_krsi`, `launch_us_graph_replay`).
- The ncu probe is opt-in (`--probe-ncu`).  It runs a tiny program once without ncu and, only if that
  exits 0, once under ncu for one kernel's duration (one pass) with the GPU's clocks left alone
  (`--clock-control none`).
- `features` adds `tcgen05_tmem` (sm_100 tensor cores with TMEM accumulators) and `wgmma` (Hopper
  only); `hopper_wgmma_tma` keeps the reference's rule, compute capability >= 9.0.
- Device facts come from torch's device properties rather than Triton's driver utilities, and the SM
  clock just after the bf16 GEMMs is added (`sm_clock_mhz_after_bf16_gemm`: the B200's dense GEMMs
  run under its power cap).
"""
from __future__ import annotations

import argparse
import json
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
DEFAULT_DIR = ROOT / "kernel-rsi_b200" / "hardware"


def device_slug(name: str) -> str:
    """File stem of a device's record: non-alphanumerics become '_', trimmed, lower case
    ("NVIDIA H20-3e" -> "nvidia_h20_3e", the reference's naming)."""
    return "".join(ch if ch.isalnum() else "_" for ch in name).strip("_").lower()


def best_call_ms(fn, calls: int = 10, rounds: int = 5, warmup: int = 3) -> float:
    """Shortest mean device time of one call over `rounds` rounds of `calls` back-to-back calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(rounds):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(calls):
            fn()
        t1.record()
        torch.cuda.synchronize()
        times.append(t0.elapsed_time(t1) / calls)
    return min(times)


def ridge(tflops: dict, bw_gbs: float) -> dict:
    """FLOP per byte at which each numeric peak meets the bandwidth ceiling."""
    return {k: round(v * 1e12 / (bw_gbs * 1e9), 1) for k, v in tflops.items() if isinstance(v, (int, float))}


def square_gemm_tflops(n: int, dtype: torch.dtype, calls: int = 10) -> float:
    a = torch.randn(n, n, device="cuda", dtype=dtype)
    b = torch.randn(n, n, device="cuda", dtype=dtype)
    ms = best_call_ms(lambda: torch.mm(a, b), calls=calls)
    return round(2 * n ** 3 / ms / 1e9, 1)


def gemm_peaks(cap: tuple[int, int], n: int) -> tuple[dict, float | None]:
    """Dense GEMM TFLOP/s per dtype (cuBLAS through torch), the skinny bf16 shapes, and the SM clock
    read right after the bf16 GEMMs (None where it cannot be read)."""
    out = {"fp16": square_gemm_tflops(n, torch.float16)}
    clock = None
    if cap >= (8, 0):
        out["bf16"] = square_gemm_tflops(n, torch.bfloat16)
        try:
            clock = int(torch.cuda.clock_rate())
        except Exception:  # noqa: BLE001 - NVML may be unavailable; the clock is context only
            clock = None
    tf32_before = torch.backends.cuda.matmul.allow_tf32
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        out["fp32"] = square_gemm_tflops(n, torch.float32, calls=3)
        if cap >= (8, 0):
            torch.backends.cuda.matmul.allow_tf32 = True
            out["tf32"] = square_gemm_tflops(n, torch.float32, calls=3)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32_before
    if cap >= (8, 9):
        try:
            a = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn)
            b = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn).t().contiguous().t()   # column-major
            unit = torch.ones((), device="cuda")
            ms = best_call_ms(lambda: torch._scaled_mm(a, b, unit, unit, out_dtype=torch.bfloat16))
            out["fp8"] = round(2 * n ** 3 / ms / 1e9, 1)
            del a, b
        except Exception:  # noqa: BLE001 - the fp8 GEMM entry point differs between torch versions
            pass
    half = torch.bfloat16 if cap >= (8, 0) else torch.float16
    skinny = {}
    for m in (16, 64, 256, 1024):
        a = torch.randn(m, 4096, device="cuda", dtype=half)
        b = torch.randn(4096, 4096, device="cuda", dtype=half)
        ms = best_call_ms(lambda: torch.mm(a, b), calls=50)
        skinny[f"M{m}xN4096xK4096"] = round(2 * m * 4096 * 4096 / ms / 1e9, 1)
    out["skinny_" + ("bf16" if cap >= (8, 0) else "fp16")] = skinny
    torch.cuda.empty_cache()
    return out, clock


def hbm_bandwidth(total_memory: int) -> dict:
    """Copy (read + write), read (a sum) and write (a fill) GB/s over fp16 buffers of up to 1 GiB."""
    numel = min(512 << 20, total_memory // 16)
    src = torch.randn(numel, device="cuda", dtype=torch.float16)
    dst = torch.empty_like(src)
    gbs = {
        "bw_copy_gbs": round(4 * numel / best_call_ms(lambda: dst.copy_(src)) / 1e6),
        "bw_read_gbs": round(2 * numel / best_call_ms(lambda: src.sum(dtype=torch.float32)) / 1e6),
        "bw_write_gbs": round(2 * numel / best_call_ms(lambda: dst.fill_(1.0)) / 1e6),
    }
    del src, dst
    torch.cuda.empty_cache()
    return gbs


def per_call_us(fn, calls: int = 2000) -> float:
    """Mean time of one call over `calls` back-to-back calls (launch-bound for tiny work)."""
    for _ in range(50):
        fn()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(calls):
        fn()
    t1.record()
    torch.cuda.synchronize()
    return round(t0.elapsed_time(t1) / calls * 1000, 1)


def launch_overheads() -> dict:
    """A torch elementwise op, one of this library's ops (eager) and a CUDA graph holding that op."""
    for p in (ROOT, ROOT / "kernel-rsi_b200", ROOT / "kernel-rsi_b200" / "library"):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))
    import _ext  # noqa: F401, PLC0415 - loads the krsi:: ops; raises when the extension is missing

    y = torch.empty(1024, device="cuda")
    u = torch.randn(1, 2048, device="cuda", dtype=torch.bfloat16)
    op = torch.ops.krsi.geglu_fwd
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            op(u)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        op(u)
    res = {"launch_us_krsi": per_call_us(lambda: op(u)), "launch_us_torch": per_call_us(lambda: y.add_(1)),
           "launch_us_graph_replay": per_call_us(graph.replay)}
    del graph
    return res


NCU_PROBE = "import torch\nx = torch.randn(1 << 20, device='cuda')\ny = x * 2\ntorch.cuda.synchronize()\n"


def ncu_probe() -> str:
    """Whether ncu can read this GPU's counters: one kernel, one metric (one pass), clocks untouched,
    and only after the same program has exited 0 without ncu."""
    ncu = shutil.which("ncu") or ("/usr/local/cuda/bin/ncu" if Path("/usr/local/cuda/bin/ncu").is_file() else None)
    if not ncu:
        return "unavailable: ncu not found"
    with tempfile.TemporaryDirectory(prefix="krsi-hw-") as tmp:
        prog = Path(tmp) / "probe.py"
        prog.write_text(NCU_PROBE)
        plain = subprocess.run([sys.executable, "-I", str(prog)], text=True, capture_output=True, timeout=300)
        if plain.returncode != 0:
            return f"not probed: the probe program failed without ncu: {(plain.stdout + plain.stderr)[-200:]}"
        p = subprocess.run([ncu, "--clock-control", "none", "--metrics", "gpu__time_duration.sum", "-c", "1",
                            sys.executable, "-I", str(prog)], text=True, capture_output=True, timeout=600)
    out = p.stdout + p.stderr
    if "ERR_NVGPUCTRPERM" in out:
        return f"unavailable: {ncu} has no counter permission (ERR_NVGPUCTRPERM)"
    if p.returncode != 0 or "gpu__time_duration.sum" not in out:
        return f"unavailable: {out[-300:]}"
    return f"available: {ncu} (probed with --clock-control none)"


def measure(probe_ncu: bool) -> dict:
    if not torch.cuda.is_available():
        raise SystemExit("no CUDA device")
    props = torch.cuda.get_device_properties(0)
    cap = torch.cuda.get_device_capability(0)
    n = 4096 if props.total_memory < (12 << 30) else 8192
    tflops, clock = gemm_peaks(cap, n)
    bw = hbm_bandwidth(props.total_memory)
    info = {
        "device": props.name,
        "sm": f"sm_{cap[0]}{cap[1]}",
        "sms": props.multi_processor_count,
        "l2_mb": round(props.L2_cache_size / 2 ** 20, 1),
        "memory_gb": round(props.total_memory / 2 ** 30, 1),
        "tflops": tflops,
        **bw,
        "ridge_flop_per_byte": ridge(tflops, max(bw["bw_copy_gbs"], bw["bw_read_gbs"])),
        "default_half_dtype": "bf16" if "bf16" in tflops else "fp16",
        "features": {"bf16_tensor_cores": cap >= (8, 0), "tf32": cap >= (8, 0), "fp8": cap >= (8, 9),
                     "hopper_wgmma_tma": cap >= (9, 0), "wgmma": cap == (9, 0), "tcgen05_tmem": cap[0] == 10},
        "smem_per_block_kb": props.shared_memory_per_block_optin // 1024,
        "regs_per_sm": props.regs_per_multiprocessor,
        "sm_clock_mhz": props.clock_rate // 1000,
    }
    if clock is not None:
        info["sm_clock_mhz_after_bf16_gemm"] = clock
    info.update(launch_overheads())
    try:
        import triton  # noqa: PLC0415

        info["triton"] = f"{triton.__version__} (installed; this build has no Triton kernels)"
    except ImportError:
        info["triton"] = "not installed (this build has no Triton kernels)"
    info["ncu"] = ncu_probe() if probe_ncu else "not probed (run with --probe-ncu)"
    info["torch"] = torch.__version__
    info["recorded_by"] = "tests/make_hardware_record.py"
    return info


def main() -> None:
    ap = argparse.ArgumentParser(description="Measure this GPU and write its hardware record.")
    ap.add_argument("--out", type=Path, default=None,
                    help="output file (default: kernel-rsi_b200/hardware/<device slug>.json)")
    ap.add_argument("--probe-ncu", action="store_true", help="also check that ncu can read the counters")
    args = ap.parse_args()
    info = measure(args.probe_ncu)
    out = args.out or DEFAULT_DIR / f"{device_slug(info['device'])}.json"
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(info, indent=2) + "\n")
    for k, v in info.items():
        print(f"{k:>30}: {v}")
    print(f"wrote {out}")


if __name__ == "__main__":
    main()
