"""Loader for the krsi_b200 native libraries, plus the compile-path glue of the krsi::* ops.

The CUDA kernels live in lib/libkrsi_b200.so (C ABI, include/krsi_b200.h); lib/_krsi_torch.so
registers the operators krsi::rmsnorm_fwd/bwd, krsi::geglu_fwd/bwd and krsi::relpos_attn_fwd/bwd
with the schemas of the reference's triton_ops (library/rmsnorm.py:86-103, library/geglu.py:85-101,
library/relpos_attention.py:175-195), plus krsi::linear_geglu_fwd (the gate|value projection with
the GEGLU forward in its epilogue) and the T5 bias ops, which have no reference operator.
This module adds what torch.compile needs on top: fake (meta) implementations and
register_autograd for each forward op.

There is no fallback: if the native libraries are missing this import fails with the command
that builds them.  Search order for the libraries: $KRSI_B200_LIB, then ../lib and ./lib
relative to this file.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
_CANDIDATES = [Path(p) for p in [os.environ.get("KRSI_B200_LIB", "")] if p] + [_HERE.parent / "lib", _HERE / "lib"]


def _find(name: str) -> Path:
    for d in _CANDIDATES:
        if (d / name).is_file():
            return d / name
    raise ImportError(
        f"krsi_b200: native library {name} not found in {[str(d) for d in _CANDIDATES]}; "
        "build it with `python kernel-rsi_b200/build.py` (nvcc, sm_100a). There is no CPU or Triton fallback."
    )


LIB_PATH = _find("libkrsi_b200.so")
TORCH_EXT_PATH = _find("_krsi_torch.so")
capi = ctypes.CDLL(str(LIB_PATH))
capi.krsi_error_string.restype = ctypes.c_char_p
capi.krsi_error_string.argtypes = [ctypes.c_int]
capi.krsi_abi_version.restype = ctypes.c_int
capi.krsi_device_status.restype = ctypes.c_int
capi.krsi_device_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_int]

if not hasattr(torch.ops, "krsi") or not hasattr(torch.ops.krsi, "rmsnorm_fwd"):
    torch.ops.load_library(str(TORCH_EXT_PATH))
ops = torch.ops.krsi


def device_status(clear: bool = False) -> int:
    """Device watchdog word of the current device: 0, or the code a bounded wait recorded when it
    gave up.  Synchronises the device (a test/diagnostic call, not for hot paths)."""
    st = ctypes.c_int(0)
    rc = capi.krsi_device_status(ctypes.byref(st), int(clear))
    if rc:
        raise RuntimeError(f"krsi_device_status failed: {capi.krsi_error_string(rc).decode()}")
    return st.value


def check_device_status() -> None:
    """Raise if a bounded device-side wait gave up since the last check (clears the word)."""
    st = device_status(clear=True)
    if st:
        raise RuntimeError(f"krsi device watchdog fired: status {st:#x} "
                           f"({capi.krsi_error_string(st & 0xff).decode()}), role {st >> 8}")


# ---------------------------------------------------------------- torch.compile glue
_registered = False


def _register_compile_support() -> None:
    global _registered
    if _registered:
        return
    _registered = True
    reg_fake = torch.library.register_fake

    @reg_fake("krsi::rmsnorm_fwd")
    def _(x2d, w, eps):
        return torch.empty_like(x2d), x2d.new_empty((x2d.shape[0],), dtype=torch.float32)

    @reg_fake("krsi::rmsnorm_bwd")
    def _(g, x2d, w, rstd):
        return torch.empty_like(x2d), torch.empty_like(w)

    @reg_fake("krsi::rmsnorm_bwd_add")
    def _(g, x2d, w, rstd, gadd):
        return torch.empty_like(x2d), torch.empty_like(w)

    @reg_fake("krsi::geglu_fwd")
    def _(u):
        return u.new_empty((u.shape[0], u.shape[1] // 2))

    @reg_fake("krsi::geglu_bwd")
    def _(g, u):
        return torch.empty_like(u)

    @reg_fake("krsi::linear_geglu_fwd")
    def _(x2d, w):
        return x2d.new_empty((x2d.shape[0], w.shape[0])), x2d.new_empty((x2d.shape[0], w.shape[0] // 2))

    @reg_fake("krsi::linear_geglu_bwd")
    def _(dy, w, u):
        return torch.empty_like(u)

    @reg_fake("krsi::relpos_attn_fwd")
    def _(qkv, pd, B, S, H, D, scale):
        return (qkv.new_empty((B * S, H * D)), qkv.new_empty((B * S, H * D), dtype=torch.float32),
                qkv.new_empty((B * H, S), dtype=torch.float32))

    @reg_fake("krsi::relpos_attn_bwd")
    def _(dout, qkv, pd, out32, lse, B, S, H, D, scale):
        return qkv.new_empty((B * S, 3 * H * D)), pd.new_empty((H, max(2 * S - 1, 0)), dtype=torch.float32)

    @reg_fake("krsi::t5_bias_fwd")
    def _(table, S, num_buckets, max_distance, bidirectional):
        return table.new_empty((table.shape[1], max(2 * S - 1, 0)), dtype=torch.float32)

    @reg_fake("krsi::t5_bias_bwd")
    def _(dpd, table, S, num_buckets, max_distance, bidirectional):
        return torch.empty_like(table)

    # Autograd of the forward ops, used when a compiled graph contains them (the eager path
    # uses the autograd.Function classes of each module instead).
    def rms_setup(ctx, inputs, output):
        ctx.save_for_backward(inputs[0], inputs[1], output[1])

    def rms_backward(ctx, gy, _grstd):
        x2d, w, rstd = ctx.saved_tensors
        dx, dw = ops.rmsnorm_bwd(gy.contiguous(), x2d, w, rstd)
        return dx, dw, None

    torch.library.register_autograd("krsi::rmsnorm_fwd", rms_backward, setup_context=rms_setup)

    def geglu_setup(ctx, inputs, output):
        ctx.save_for_backward(inputs[0])

    def geglu_backward(ctx, g):
        (u,) = ctx.saved_tensors
        return ops.geglu_bwd(g.contiguous(), u)

    torch.library.register_autograd("krsi::geglu_fwd", geglu_backward, setup_context=geglu_setup)

    def lg_setup(ctx, inputs, output):
        ctx.save_for_backward(inputs[0], inputs[1], output[0])

    def lg_backward(ctx, gu, gout):
        x2d, w, u = ctx.saved_tensors
        du = ops.geglu_bwd(gout.contiguous(), u)
        if gu is not None:
            du = du + gu
        return du @ w, du.t() @ x2d

    torch.library.register_autograd("krsi::linear_geglu_fwd", lg_backward, setup_context=lg_setup)

    def attn_setup(ctx, inputs, output):
        qkv, pd, B, S, H, D, scale = inputs
        ctx.save_for_backward(qkv, pd, output[1], output[2])
        ctx.dims = (B, S, H, D, scale)

    def attn_backward(ctx, dout, _d32, _dlse):
        dqkv, dpd = ops.relpos_attn_bwd(dout.contiguous(), *ctx.saved_tensors, *ctx.dims)
        return dqkv, dpd, None, None, None, None, None

    torch.library.register_autograd("krsi::relpos_attn_fwd", attn_backward, setup_context=attn_setup)

    def t5_setup(ctx, inputs, output):
        table, S, nb, md, bi = inputs
        ctx.save_for_backward(table)
        ctx.args = (S, nb, md, bi)

    def t5_backward(ctx, dpd):
        (table,) = ctx.saved_tensors
        return ops.t5_bias_bwd(dpd.contiguous(), table, *ctx.args), None, None, None, None

    torch.library.register_autograd("krsi::t5_bias_fwd", t5_backward, setup_context=t5_setup)


_register_compile_support()
