"""RMSNorm forward + backward on B200 (hand-written sm_100a CUDA). Use rmsnorm(x2d, weight, eps).

Drop-in for kernel-rsi's library/rmsnorm.py: same public function (rmsnorm.py:106-110), same
autograd.Function contract (RMSNorm, rmsnorm.py:71-83: saves (x2d, w, rstd), returns (dx, dw, None)),
same operator names under torch.compile (krsi::rmsnorm_fwd / krsi::rmsnorm_bwd, rmsnorm.py:86-103),
plus reference() and selftest().

y = weight * (x * rsqrt(mean(x^2) + eps)).to(weight.dtype), rounding as in HF T5LayerNorm / LlamaRMSNorm.
The forward saves an fp32 rstd per row; the backward computes dx in one pass over each row and dw as
fixed-order per-block partial sums plus a second reduction kernel (deterministic, no atomics).
Rows up to 16384 elements (fp32; 32768 for 16-bit types with aligned rows).
Kernels: kernel-rsi_b200/csrc/rmsnorm.cu; C ABI: include/krsi_b200.h.
"""
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "tools"))   # the skill's tools (selftest)
sys.path.insert(0, str(Path(__file__).resolve().parent))
from _compat import compiling  # noqa: E402
from _ext import ops  # noqa: E402


class RMSNorm(torch.autograd.Function):
    """Eager path: calls the krsi ops directly (no registered-op autograd overhead)."""

    @staticmethod
    def forward(ctx, x2d, w, eps):
        y, rstd = ops.rmsnorm_fwd(x2d, w, eps)
        ctx.save_for_backward(x2d, w, rstd)
        return y

    @staticmethod
    def backward(ctx, g):
        x2d, w, rstd = ctx.saved_tensors
        dx, dw = ops.rmsnorm_bwd(g.contiguous(), x2d, w, rstd)
        return dx, dw, None


def rmsnorm(x2d, w, eps):
    """y = w * (x * rsqrt(mean(x^2) + eps)).to(w.dtype), over the rows of a 2-D tensor."""
    if compiling():
        return ops.rmsnorm_fwd(x2d, w, eps)[0]
    return RMSNorm.apply(x2d, w, eps)


def reference(x2d, w, eps):
    """The torch expression this op reproduces (rmsnorm.py:113-115): fp32 statistics, the normalised
    row cast back to the input dtype, then scaled by the weight."""
    xf = x2d.float()
    inv = torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + eps)
    return w * (xf * inv).to(x2d.dtype)


def selftest():
    """Same check as the reference's selftest (rmsnorm.py:118-123): kernel vs torch, output and
    gradients, eager and compiled, via the skill's tools/common.py."""
    from common import selftest_autograd  # noqa: PLC0415

    x = torch.randn(4096, 1024, device="cuda", dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(1024, device="cuda")).to(torch.bfloat16)
    return selftest_autograd(lambda x, w: rmsnorm(x, w, 1e-6), lambda x, w: reference(x, w, 1e-6), [x, w])


if __name__ == "__main__":
    print(selftest())
