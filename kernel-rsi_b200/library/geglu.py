"""GEGLU forward + backward on B200 (hand-written sm_100a CUDA) over a merged [gate | value] GEMM
output. Use geglu(u).

Drop-in for kernel-rsi's library/geglu.py: same public function (geglu.py:104-108), same
autograd.Function contract (GEGLU, geglu.py:71-82: saves u, returns du), same operator names under
torch.compile (krsi::geglu_fwd / krsi::geglu_bwd, geglu.py:85-101), plus reference() and selftest().

u: [rows, 2F]; returns gelu_tanh(u[:, :F]) * u[:, F:] with the eager bf16 rounding points. The backward
writes d[gate | value] into one [rows, 2F] tensor, so the merged GEMM's backward reads one gradient.
Kernels: kernel-rsi_b200/csrc/geglu.cu; C ABI: include/krsi_b200.h.
"""
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "tools"))   # the skill's tools (selftest)
sys.path.insert(0, str(Path(__file__).resolve().parent))
from _compat import compiling  # noqa: E402
from _ext import ops  # noqa: E402


class GEGLU(torch.autograd.Function):
    """Eager path: calls the krsi ops directly."""

    @staticmethod
    def forward(ctx, u):
        ctx.save_for_backward(u)
        return ops.geglu_fwd(u)

    @staticmethod
    def backward(ctx, g):
        (u,) = ctx.saved_tensors
        return ops.geglu_bwd(g.contiguous(), u)


def geglu(u):
    """gelu_tanh(u[:, :F]) * u[:, F:] for a [rows, 2F] tensor."""
    if compiling():
        return ops.geglu_fwd(u)
    return GEGLU.apply(u)


def reference(u):
    """The torch expression this op reproduces (geglu.py:111-113)."""
    gate, value = u.chunk(2, dim=-1)
    return torch.nn.functional.gelu(gate, approximate="tanh") * value


def selftest():
    """Same check as the reference's selftest (geglu.py:116-120)."""
    from common import selftest_autograd  # noqa: PLC0415

    u = torch.randn(2048, 2 * 2816, device="cuda", dtype=torch.bfloat16)
    return selftest_autograd(geglu, reference, [u])


if __name__ == "__main__":
    print(selftest())
