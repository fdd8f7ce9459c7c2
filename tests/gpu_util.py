"""Helpers shared by the GPU parity tests (checker side only)."""
import ctypes

import torch

import _ext  # noqa: F401  (loads the native libraries: registers the krsi::* operators)
from conftest import PKG

DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_lib = None


def capi():
    """The C ABI library itself, for tests that call the boundary directly (no torch binding)."""
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(PKG / "lib" / "libkrsi_b200.so"))
    return _lib


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def run_reference_path(fn, inputs, cot, dtype=None):
    """Output and input gradients of fn (the reference's eager expression) for cotangent cot."""
    xs = [x.detach().to(dtype or x.dtype).requires_grad_(x.is_floating_point()) for x in inputs]
    out = fn(*xs)
    grads = torch.autograd.grad(out, [x for x in xs if x.requires_grad], cot.to(out.dtype))
    return [out.detach()] + [g.detach() for g in grads]


def reference_compare(kernel_fn, ref_fn, inputs, cot):
    """The reference's selftest criterion (tools/common.py:476-490): ref32 = reference in fp32 with
    TF32 off, orig = reference in the inputs' dtype, cand = kernel; compare() with slack 2."""
    from oracle.compare import compare

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref32 = run_reference_path(ref_fn, inputs, cot, torch.float32)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    orig = run_reference_path(ref_fn, inputs, cot)
    cand = run_reference_path(kernel_fn, inputs, cot)
    return compare(ref32, orig, cand), ref32, cand
