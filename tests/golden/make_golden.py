"""Generate the golden fixtures in tests/golden/ from the reference implementation itself.

Run in a container that has the kernel-rsi reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/kernel-rsi

It imports the reference's library modules and records, on seeded CPU inputs in fp32:
  * the reference's Triton kernels, executed by Triton's CPU interpreter (TRITON_INTERPRET=1):
      rmsnorm _fwd/_bwd (library/rmsnorm.py:22-68), geglu _fwd/_bwd (library/geglu.py:20-68),
      relpos_attention _forward/_backward_impl (library/relpos_attention.py:132-157; D must be a
      power of two there, so D = 32 and 64);
  * the reference's eager reference() functions and their autograd gradients (fp32), including
    D = 72, which the reference kernels cannot run.
The fixtures pin the oracle (oracle/ops.py) in tests/test_oracle_golden.py; nothing at run time
needs the reference checkout.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"   # must precede the first triton import

import torch  # noqa: E402

OUT = Path(__file__).resolve().parent


def seeded(shape, seed, std=1.0, mean=0.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32) * std + mean


def load_reference_module(ref: Path, name: str):
    lib = ref / "library"
    sys.path.insert(0, str(lib))
    sys.path.insert(0, str(ref / "tools"))
    # rmsnorm.py reads the SM count of CUDA device 0 at import (rmsnorm.py:19); give it a CPU stand-in.
    real = torch.cuda.get_device_properties

    class _Props:
        multi_processor_count = 8

    torch.cuda.get_device_properties = lambda *_a, **_k: _Props()
    try:
        spec = importlib.util.spec_from_file_location(f"krsi_ref_{name}", lib / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        torch.cuda.get_device_properties = real
    return mod


def grads_of(fn, inputs, cot):
    xs = [x.detach().clone().requires_grad_(True) for x in inputs]
    out = fn(*xs)
    gs = torch.autograd.grad(out, xs, cot)
    return out.detach(), [g.detach() for g in gs]


def make_rmsnorm(ref: Path):
    m = load_reference_module(ref, "rmsnorm")
    cases = {}
    for tag, rows, n, seed in (("small", 37, 96, 10), ("wide", 6, 1152, 20)):
        x = seeded((rows, n), seed)
        w = seeded((n,), seed + 1, std=0.02, mean=1.0)
        g = seeded((rows, n), seed + 2)
        eps = 1e-6
        y, rstd = m._fwd(x, w, eps, launch=m._raw)
        case = dict(x=x, w=w, g=g, eps=torch.tensor(eps), kernel_y=y, kernel_rstd=rstd)
        try:
            dx, dw = m._bwd(g, x, w, rstd, launch=m._raw)
            case.update(kernel_dx=dx, kernel_dw=dw)
        except Exception as e:  # noqa: BLE001
            # _rms_bwd calls .to() on a Python loop index (rmsnorm.py:42), which Triton's CPU
            # interpreter does not support; its gradients are pinned by reference() autograd below.
            print(f"rmsnorm[{tag}]: reference _rms_bwd not runnable in the interpreter: {type(e).__name__}")
        y_ref, (dx_ref, dw_ref) = grads_of(lambda a, b: m.reference(a, b, eps), [x, w], g)
        case.update(ref_y=y_ref, ref_dx=dx_ref, ref_dw=dw_ref)
        cases[tag] = case
    torch.save(cases, OUT / "rmsnorm_golden.pt")


def make_geglu(ref: Path):
    m = load_reference_module(ref, "geglu")
    cases = {}
    for tag, rows, F, seed in (("small", 19, 40, 30), ("odd", 5, 13, 40), ("wide", 2, 4608, 50)):
        u = seeded((rows, 2 * F), seed)
        g = seeded((rows, F), seed + 1)
        out = m._fwd(u, launch=m._raw)
        du = m._bwd(g, u, launch=m._raw)
        out_ref, (du_ref,) = grads_of(m.reference, [u], g)
        cases[tag] = dict(u=u, g=g, kernel_out=out, kernel_du=du, ref_out=out_ref, ref_du=du_ref)
    torch.save(cases, OUT / "geglu_golden.pt")


def make_relpos(ref: Path):
    m = load_reference_module(ref, "relpos_attention")
    cases = {}
    # (B, S, H, D): the kernel cases need a power-of-two D; S is not a multiple of the 64 tile.
    for tag, (B, S, H, D), seed, kernel in (("d32", (2, 70, 2, 32), 60, True),
                                            ("d64", (1, 80, 2, 64), 70, True),
                                            ("d72", (2, 37, 2, 72), 80, False)):
        scale = D ** -0.5
        qkv = seeded((B * S, 3 * H * D), seed, std=D ** -0.5)
        pd = seeded((H, 2 * S - 1), seed + 1, std=0.02)
        dout = seeded((B * S, H * D), seed + 2)
        case = dict(qkv=qkv, pd=pd, dout=dout, dims=torch.tensor([B, S, H, D]), scale=torch.tensor(scale))
        if kernel:
            out, out32, lse = m._forward(qkv, pd, B, S, H, D, scale, launch=m._raw)
            dqkv, dpd = m._backward_impl(dout, qkv, pd, out32, lse, B, S, H, D, scale, launch=m._raw)
            case.update(kernel_out=out, kernel_out32=out32, kernel_lse=lse, kernel_dqkv=dqkv, kernel_dpd=dpd)
        out_ref, (dqkv_ref, dpd_ref) = grads_of(lambda q, p: m.reference(q, p, B, S, H, D, scale), [qkv, pd], dout)
        case.update(ref_out=out_ref, ref_dqkv=dqkv_ref, ref_dpd=dpd_ref)
        cases[tag] = case
    torch.save(cases, OUT / "relpos_golden.pt")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the kernel-rsi checkout to run")
    a = ap.parse_args()
    ref = Path(a.reference)
    torch.backends.cuda.matmul.allow_tf32 = False
    make_rmsnorm(ref)
    make_geglu(ref)
    make_relpos(ref)
    for p in sorted(OUT.glob("*.pt")):
        print(p.name, p.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
