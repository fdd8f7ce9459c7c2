"""Record the library's self-tests on this GPU in the reference's replay format.

The reference's tools/replay.py runs every library/*.py selftest() and writes
library/replay/<gpu>.json (tools/replay.py:24-59; its H20 record is library/replay/nvidia_h20_3e.json).
Its tools are not present on the GPU hosts this repository runs on, so this script restates the
procedure of one selftest (tools/common.py:476-518, selftest_autograd) with this repository's
restatement of the reference's compare() (oracle/compare.py) and writes the same JSON layout:

  python tests/make_replay_record.py --out kernel-rsi_b200/library/replay/nvidia_b200.json

Per library op, at the shapes of its selftest(): the fp32 reference run (TF32 off), the bf16 original
and the kernel with one random cotangent (x 1e-2) are compared (slack 2), eager and under
torch.compile(fullgraph=True); then kernel and reference forward+backward are timed in interleaved
rounds, each a CUDA graph of repeated calls, and reported with the replay's significance rule
(faster / slower only when the rounds' ranges do not overlap).  Test infrastructure: it imports the
oracle's compare() and is not part of the product.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "kernel-rsi_b200", ROOT / "kernel-rsi_b200" / "library"):
    sys.path.insert(0, str(p))

from oracle.compare import compare  # noqa: E402


def run(f, xs, dtype=None, cot=None):
    xs = [x.detach().to(dtype or x.dtype).requires_grad_(x.is_floating_point()) for x in xs]
    out = f(*xs)
    cot = torch.randn_like(out.float()).mul_(1e-2) if cot is None else cot
    grads = torch.autograd.grad(out, [x for x in xs if x.requires_grad], cot.to(out.dtype))
    return [out.detach()] + [g.detach() for g in grads], cot


def check(fn, ref, inputs):
    prev = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    try:
        ref32, cot = run(ref, inputs, torch.float32)
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev
    orig, _ = run(ref, inputs, cot=cot)
    cand, _ = run(fn, inputs, cot=cot)
    return compare(ref32, orig, cand)["pass"], ref32, orig, cot


def graph_time_us(step, reps=10):
    """Device time of one call: a CUDA graph of `reps` calls, replayed once."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            step()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) * 1e3 / reps


def timed_rounds(variants, rounds=5):
    per = {k: [] for k in variants}
    for r in range(rounds):
        for name in (list(variants) if r % 2 == 0 else list(reversed(variants))):
            per[name].append(graph_time_us(variants[name]))
    return per


def significance(base, cand):
    if max(cand) < min(base):
        return "faster"
    if min(cand) > max(base):
        return "slower"
    return "within noise"


def record(fn, ref, inputs):
    ok, _, _, cot = check(fn, ref, inputs)
    leaves = [x.detach().requires_grad_(x.is_floating_point()) for x in inputs]
    g = cot.to(inputs[0].dtype)

    def step(f):
        return lambda: torch.autograd.grad(f(*leaves), [x for x in leaves if x.requires_grad], g)

    variants = {"reference": step(ref), "kernel": step(fn)}
    torch._dynamo.reset()
    cfn, cref = torch.compile(fn, fullgraph=True), torch.compile(ref)
    c_ok, ref32, orig, _ = check(cfn, ref, inputs)
    variants.update(compiled_reference=step(cref), compiled_kernel=step(cfn))
    t = timed_rounds(variants)
    med = {k: round(statistics.median(v), 1) for k, v in t.items()}
    return {"pass": bool(ok and c_ok), "reference_us": med["reference"], "kernel_us": med["kernel"],
            "speedup": round(med["reference"] / med["kernel"], 2),
            "significance": significance(t["reference"], t["kernel"]),
            "compiled": {"pass": bool(c_ok), "kernel_us": med["compiled_kernel"],
                         "reference_us": med["compiled_reference"],
                         "speedup": round(med["compiled_reference"] / med["compiled_kernel"], 2),
                         "significance": significance(t["compiled_reference"], t["compiled_kernel"])}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    import geglu
    import linear_geglu
    import relpos_attention as ra
    import rmsnorm
    import t5_bias

    torch.manual_seed(0)
    dev = "cuda"
    info = {"device": torch.cuda.get_device_name(0), "torch": torch.__version__, "cuda": torch.version.cuda,
            "triton": None}
    cases = {}
    # the shapes and scales of each module's selftest()
    x = torch.randn(4096, 1024, device=dev, dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(1024, device=dev)).to(torch.bfloat16)
    cases["rmsnorm"] = (lambda x, w: rmsnorm.rmsnorm(x, w, 1e-6), lambda x, w: rmsnorm.reference(x, w, 1e-6), [x, w])
    u = torch.randn(2048, 2 * 2816, device=dev, dtype=torch.bfloat16)
    cases["geglu"] = (geglu.geglu, geglu.reference, [u])
    B, S, H, D = 4, 512, 16, 64
    qkv = (0.6 * torch.randn(B * S, 3 * H * D, device=dev)).to(torch.bfloat16)
    pd = torch.randn(H, 2 * S - 1, device=dev)
    cases["relpos_attention"] = (lambda q, p: ra.relpos_attention(q, p, B, S, H, D, 1.0),
                                 lambda q, p: ra.reference(q, p, B, S, H, D, 1.0), [qkv, pd])
    xl = torch.randn(2048, 768, device=dev, dtype=torch.bfloat16)
    wl = (torch.randn(2 * 2048, 768, device=dev) * 768 ** -0.5).to(torch.bfloat16)
    cases["linear_geglu"] = (linear_geglu.linear_geglu, linear_geglu.reference, [xl, wl])
    table = 0.1 * torch.randn(32, 12, device=dev)
    cases["t5_bias"] = (lambda t: t5_bias.t5_relpos_bias(t, 512), lambda t: t5_bias.reference(t, 512), [table])
    out = {"versions": info, "library": {}, "regions": {},
           "note": "recorded by tests/make_replay_record.py (this repository's restatement of tools/replay.py "
                   "and selftest_autograd; the reference's tools are not present on this host)"}
    for name, (fn, ref, inputs) in cases.items():
        r = record(fn, ref, inputs)
        out["library"][name] = {"pass": r["pass"], **info, **{k: v for k, v in r.items() if k != "pass"}}
        c = r["compiled"]
        print(f"{name:<18} {'PASS' if r['pass'] else 'FAIL'}  eager: {r['kernel_us']:.1f} us vs "
              f"{r['reference_us']:.1f} us {r['speedup']:.2f}x ({r['significance']}) | compile(fullgraph): "
              f"{'ok' if c['pass'] else 'FAIL'} {c['kernel_us']:.1f} us vs compiled ref {c['reference_us']:.1f} us "
              f"{c['speedup']:.2f}x ({c['significance']})", flush=True)
    Path(a.out).parent.mkdir(parents=True, exist_ok=True)
    Path(a.out).write_text(json.dumps(out, indent=2) + "\n")
    bad = [k for k, v in out["library"].items() if not v["pass"]]
    print(f"saved {a.out}" + (f"\nFAILED: {bad}" if bad else ""))
    raise SystemExit(1 if bad else 0)


if __name__ == "__main__":
    main()
