"""T5 bucketed relative position on B200: the learned bias table -> the per-distance bias row the
relpos attention op takes, and the gradient back to the table (hand-written sm_100a CUDA).

t5_relpos_bias(table, S, bidirectional=True, num_buckets=32, max_distance=128) -> pd [H, 2S-1] fp32
  table: [num_buckets, H] (T5's relative_attention_bias.weight), any float dtype
  pd[h, t] = table[bucket(t - (S - 1)), h], so relpos_attention(qkv, pd, B, S, H, D, scale) adds
  T5's position bias (bias[h, i, j] = pd[h, j - i + S - 1]).

T5's bucket of a distance rel = key - query (HF transformers T5Attention._relative_position_bucket):
with n = num_buckets / 2 if bidirectional (rel > 0 adds n) else num_buckets, e = n / 2 and
a = |rel| (bidirectional) or max(-rel, 0): a itself for a < e, else
e + trunc(log(a / e) / log(max_distance / e) * (n - e)), capped at n - 1.  The backward sums the
bias row's gradient over each bucket's run of distances (a fixed-order segmented sum: no scatter
over S x S positions), the step the kernel-rsi lessons describe for a T5 training region
(LESSONS.md:35).  Kernels: kernel-rsi_b200/csrc/t5_bias.cu; C ABI: include/krsi_b200.h.
"""
import math
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "tools"))   # the skill's tools (selftest)
sys.path.insert(0, str(Path(__file__).resolve().parent))
from _compat import compiling  # noqa: E402
from _ext import ops  # noqa: E402


class T5RelPosBias(torch.autograd.Function):
    """Eager path: calls the krsi ops directly."""

    @staticmethod
    def forward(ctx, table, S, num_buckets, max_distance, bidirectional):
        ctx.save_for_backward(table)
        ctx.args = (S, num_buckets, max_distance, bidirectional)
        return ops.t5_bias_fwd(table, S, num_buckets, max_distance, bidirectional)

    @staticmethod
    def backward(ctx, dpd):
        (table,) = ctx.saved_tensors
        return ops.t5_bias_bwd(dpd.contiguous(), table, *ctx.args), None, None, None, None


def t5_relpos_bias(table, S, bidirectional=True, num_buckets=32, max_distance=128):
    """The per-distance bias row [H, 2S-1] (fp32) of T5's bucketed relative position table."""
    if compiling():
        return ops.t5_bias_fwd(table, S, num_buckets, max_distance, bidirectional)
    return T5RelPosBias.apply(table, S, num_buckets, max_distance, bidirectional)


def buckets(S, bidirectional=True, num_buckets=32, max_distance=128, device=None):
    """T5's bucket of every distance rel = -(S-1) .. S-1, in torch ops (as T5 computes it)."""
    rel = torch.arange(-(S - 1), S, device=device)
    n = num_buckets // 2 if bidirectional else num_buckets
    base = (rel > 0).long() * n if bidirectional else torch.zeros_like(rel)
    a = rel.abs() if bidirectional else (-rel).clamp(min=0)
    e = n // 2
    large = e + (torch.log(a.float() / e) / math.log(max_distance / e) * (n - e)).long()
    large = large.clamp(max=n - 1)
    return base + torch.where(a < e, a, large)


def reference(table, S, bidirectional=True, num_buckets=32, max_distance=128):
    """The torch expression this op reproduces: T5's bucket per distance, then a table lookup
    (differentiable: its backward is torch's index scatter-add)."""
    idx = buckets(S, bidirectional, num_buckets, max_distance, device=table.device)
    return table[idx].t().float()


def selftest():
    """The library's self-test contract: kernel vs the torch expression, output and gradient, eager and
    compiled, at a T5-base shape (32 buckets, max distance 128, 12 heads, S = 512)."""
    from common import selftest_autograd  # noqa: PLC0415

    table = 0.1 * torch.randn(32, 12, device="cuda")
    return selftest_autograd(lambda t: t5_relpos_bias(t, 512), lambda t: reference(t, 512), [table])


if __name__ == "__main__":
    print(selftest())
