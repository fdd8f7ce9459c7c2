"""The T5 feed-forward's gate|value projection with the GEGLU forward in the GEMM's epilogue, on
B200 (a hand-written tcgen05 GEMM). Use linear_geglu(x2d, w).

linear_geglu(x2d, w) == geglu(x2d @ w.t()) of this library (geglu.py:104-108 of the reference),
computed in one kernel: the GEMM accumulates in fp32, rounds u = x2d @ w.t() to the input dtype as
the separate GEMM would, and applies GEGLU's arithmetic to the rounded u before anything leaves the
SM, so the GEGLU forward's read of u is gone. The result equals geglu() applied to the kernel's own
u bit for bit; u itself differs from cuBLAS's only in the fp32 summation order.

x2d: [rows, K]; w: [2F, K] (nn.Linear's weight: rows [0, F) gate, [F, 2F) value), one dtype (bf16
or f16); returns [rows, F]. The backward is GEGLU's backward kernel on the saved u followed by the
two GEMMs of the projection (dx = du @ w, dw = du^T @ x2d).

feed_forward(x2d, wi, wo, res) is the whole gated-GELU feed-forward, res + geglu(x2d @ wi.t()) @
wo.t(): its backward also fuses GEGLU's backward into the down projection's input-gradient GEMM
(krsi::linear_geglu_bwd: du = geglu_bwd(dy @ wo, u), the GEMM's output never written).
Kernels: kernel-rsi_b200/csrc/linear_geglu.cu; C ABI: include/krsi_b200.h (krsi_linear_geglu_fwd,
krsi_linear_geglu_bwd).
"""
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "tools"))   # the skill's tools (selftest)
sys.path.insert(0, str(Path(__file__).resolve().parent))
from _compat import compiling  # noqa: E402
from _ext import ops  # noqa: E402


class LinearGEGLU(torch.autograd.Function):
    """Eager path: saves (x2d, w, u); returns (dx, dw)."""

    @staticmethod
    def forward(ctx, x2d, w):
        u, out = ops.linear_geglu_fwd(x2d, w)
        ctx.save_for_backward(x2d, w, u)
        return out

    @staticmethod
    def backward(ctx, g):
        x2d, w, u = ctx.saved_tensors
        du = ops.geglu_bwd(g.contiguous(), u)
        dx = du @ w if ctx.needs_input_grad[0] else None
        dw = du.t() @ x2d if ctx.needs_input_grad[1] else None
        return dx, dw


def linear_geglu(x2d, w):
    """gelu_tanh(h[:, :F]) * h[:, F:] with h = x2d @ w.t(), for x2d [rows, K] and w [2F, K]."""
    if compiling():
        return ops.linear_geglu_fwd(x2d, w)[1]
    return LinearGEGLU.apply(x2d, w)


class FeedForwardGEGLU(torch.autograd.Function):
    """res + geglu(x2d @ wi^T) @ wo^T with both fused kernels: the forward's gate|value projection
    with GEGLU in its epilogue, and the backward's down-projection input gradient with GEGLU's
    backward in its epilogue (krsi::linear_geglu_bwd), so neither u's read by GEGLU's forward nor
    GEGLU's input gradient ever reaches memory.  Saves (x2d, wi, wo, u, g); returns
    (dx, dwi, dwo, dres)."""

    @staticmethod
    def forward(ctx, x2d, wi, wo, res):
        u, g = ops.linear_geglu_fwd(x2d, wi)
        ctx.save_for_backward(x2d, wi, wo, u, g)
        ctx.has_res = res is not None
        return torch.addmm(res, g, wo.t()) if res is not None else g @ wo.t()

    @staticmethod
    def backward(ctx, gy):
        x2d, wi, wo, u, g = ctx.saved_tensors
        gy = gy.contiguous()
        dwo = gy.t() @ g if ctx.needs_input_grad[2] else None
        du = ops.linear_geglu_bwd(gy, wo, u)
        dx = du @ wi if ctx.needs_input_grad[0] else None
        dwi = du.t() @ x2d if ctx.needs_input_grad[1] else None
        return dx, dwi, dwo, (gy if ctx.has_res else None)


def feed_forward(x2d, wi, wo, res=None):
    """res + geglu(x2d @ wi.t()) @ wo.t(): the T5 gated-GELU feed-forward on the fused kernels, for
    x2d [rows, d], wi [2F, d], wo [d, F] (and res [rows, d])."""
    if compiling():
        y = ops.linear_geglu_fwd(x2d, wi)[1] @ wo.t()
        return y if res is None else y + res
    return FeedForwardGEGLU.apply(x2d, wi, wo, res)


def feed_forward_reference(x2d, wi, wo, res=None):
    """The eager torch expression feed_forward replaces."""
    y = reference(x2d, wi) @ wo.t()
    return y if res is None else y + res


def reference(x2d, w):
    """The eager torch expression this op replaces: the projection, then the reference GEGLU."""
    gate, value = (x2d @ w.t()).chunk(2, dim=-1)
    return torch.nn.functional.gelu(gate, approximate="tanh") * value


def selftest():
    """The reference's autograd self-test criterion on the T5 v1.1 base feed-forward shape
    (d_model 768, d_ff 2048) at 2048 tokens."""
    from common import selftest_autograd  # noqa: PLC0415

    x = torch.randn(2048, 768, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(2 * 2048, 768, device="cuda") * 768 ** -0.5).to(torch.bfloat16)
    return selftest_autograd(linear_geglu, reference, [x, w])


def selftest_feed_forward():
    """The same criterion for the whole feed-forward (both fused kernels) on the T5 v1.1 base shape."""
    from common import selftest_autograd  # noqa: PLC0415

    x = torch.randn(2048, 768, device="cuda", dtype=torch.bfloat16)
    wi = (torch.randn(2 * 2048, 768, device="cuda") * 768 ** -0.5).to(torch.bfloat16)
    wo = (torch.randn(768, 2048, device="cuda") * 2048 ** -0.5).to(torch.bfloat16)
    return selftest_autograd(feed_forward, feed_forward_reference, [x, wi, wo])


if __name__ == "__main__":
    print(selftest())
