"""Replacement for T5Block (model_entry.py) on the kernel-rsi library ops, as the tools' impl.py
template asks (tools/region.py IMPL_TEMPLATE: compute the same function as the original forward,
called as forward(mod, ...) with the original module's parameters).

  RMSNorm           library rmsnorm()           (T5LayerNorm's rounding: the row cast to the weight dtype)
  q | k | v GEMM    one GEMM over the concatenated weights (re-concatenated every call: training-safe)
  position bias     library t5_bias.t5_relpos_bias(): the bucket table -> per-distance bias row
  attention         library relpos_attention() with scale 1 (T5 folds the scale into its weights)
  o + residual      addmm (the residual rides in the GEMM)
  wi_0 | wi_1 GEMM  one tcgen05 GEMM with GEGLU (gelu_tanh(gate) * value) in its epilogue:
                    library linear_geglu() (geglu() of the GEMM's output, bit for bit)
  wo + residual     addmm
"""
import sys
from pathlib import Path

import torch

_LIB = Path(__file__).resolve().parent.parent / "library"
if str(_LIB) not in sys.path:
    sys.path.insert(0, str(_LIB))
import linear_geglu  # noqa: E402
import relpos_attention  # noqa: E402
import rmsnorm  # noqa: E402
import t5_bias  # noqa: E402


def forward(mod, x):
    B, S, d = x.shape
    H = mod.relative_attention_bias.weight.shape[1]
    D = mod.q.weight.shape[0] // H
    x2 = x.reshape(B * S, d)
    h = rmsnorm.rmsnorm(x2, mod.ln1.weight, mod.ln1.eps)
    qkv = h @ torch.cat([mod.q.weight, mod.k.weight, mod.v.weight]).t()
    pd = t5_bias.t5_relpos_bias(mod.relative_attention_bias.weight, S, True, mod.relative_attention_bias.num_embeddings,
                                128)
    a = relpos_attention.relpos_attention(qkv, pd, B, S, H, D, 1.0)
    x2 = torch.addmm(x2, a, mod.o.weight.t())
    h = rmsnorm.rmsnorm(x2, mod.ln2.weight, mod.ln2.eps)
    g = linear_geglu.linear_geglu(h, torch.cat([mod.wi_0.weight, mod.wi_1.weight]))
    x2 = torch.addmm(x2, g, mod.wo.weight.t())
    return x2.view(B, S, d)
