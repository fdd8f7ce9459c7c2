"""Flash attention forward + backward with an additive bias that depends only on (j - i), on B200
tensor cores (tcgen05 MMA, TMEM accumulators, TMA-fed shared-memory tiles; hand-written sm_100a CUDA).

relpos_attention(qkv, pd, B, S, H, D, scale) -> [B*S, H*D]   (differentiable, torch.compile-friendly)
  qkv: [B*S, 3*H*D] (the fused q|k|v GEMM output, read in place through its row stride)
  pd:  [H, 2S-1] fp32 per-distance bias, bias[h, i, j] = pd[h, j - i + S - 1]; its gradient is the
       batch sum of the diagonal sums of dS.

Drop-in for kernel-rsi's library/relpos_attention.py: same public function (relpos_attention.py:198-201),
same autograd.Function contract (RelPosAttention, :160-172: saves (qkv, pd, out32, lse), returns
(dqkv, dpd, None x 5)), same operator names and outputs under torch.compile (krsi::relpos_attn_fwd ->
(out, out32, lse), krsi::relpos_attn_bwd -> (dqkv, dpd), :175-195), plus reference() and selftest().
The forward keeps an fp32 copy of O so the backward's delta = rowsum(dO * O) is taken in fp32, and lse
is in the log2 domain, as in the reference. No causal mask; D a multiple of 8 up to 128 (D = 72
included), qkv in bf16 or fp16.
Kernels: kernel-rsi_b200/csrc/relpos_attn_fwd.cu and relpos_attn_bwd.cu; C ABI: include/krsi_b200.h.
"""
import sys
from pathlib import Path

import torch
import torch.nn.functional as F

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "tools"))   # the skill's tools (selftest)
sys.path.insert(0, str(Path(__file__).resolve().parent))
from _compat import compiling  # noqa: E402
from _ext import ops  # noqa: E402

LOG2E = 1.4426950408889634


class RelPosAttention(torch.autograd.Function):
    """Eager path: calls the krsi ops directly."""

    @staticmethod
    def forward(ctx, qkv, pd, B, S, H, D, scale):
        out, out32, lse = ops.relpos_attn_fwd(qkv, pd, B, S, H, D, scale)
        ctx.save_for_backward(qkv, pd, out32, lse)
        ctx.dims = (B, S, H, D, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        dqkv, dpd = ops.relpos_attn_bwd(dout.contiguous(), *ctx.saved_tensors, *ctx.dims)
        return dqkv, dpd, None, None, None, None, None


def relpos_attention(qkv, pd, B, S, H, D, scale):
    if compiling():
        return ops.relpos_attn_fwd(qkv, pd, B, S, H, D, scale)[0]
    return RelPosAttention.apply(qkv, pd, B, S, H, D, scale)


def reference(qkv, pd, B, S, H, D, scale):
    """The torch expression this op reproduces (relpos_attention.py:204-212): SDPA on the math backend
    with the Toeplitz bias materialised in qkv's dtype."""
    q, k, v = qkv.view(B, S, 3, H, D).unbind(2)                    # each [B, S, H, D]
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))               # [B, H, S, D]
    idx = torch.arange(S, device=qkv.device)
    bias = pd[:, idx[None, :] - idx[:, None] + (S - 1)].unsqueeze(0).to(qkv.dtype)
    from torch.nn.attention import SDPBackend, sdpa_kernel  # noqa: PLC0415

    with sdpa_kernel(SDPBackend.MATH):
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=bias, scale=scale)
    return o.transpose(1, 2).reshape(B * S, H * D)


def selftest():
    """Same check as the reference's selftest (relpos_attention.py:215-222)."""
    from common import selftest_autograd  # noqa: PLC0415

    B, S, H, D = 4, 512, 16, 64
    qkv = (0.6 * torch.randn(B * S, 3 * H * D, device="cuda")).to(torch.bfloat16)
    pd = torch.randn(H, 2 * S - 1, device="cuda")
    return selftest_autograd(lambda q, p: relpos_attention(q, p, B, S, H, D, 1.0),
                             lambda q, p: reference(q, p, B, S, H, D, 1.0), [qkv, pd])


if __name__ == "__main__":
    print(selftest())
