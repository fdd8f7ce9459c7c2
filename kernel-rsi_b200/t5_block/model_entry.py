"""A T5 v1.1 encoder layer stack as a user of the kernel-rsi tools would hand it over: the model entry
point of the tools' contract (build / run / shapes / MODE / loss; the reference's README "Use" section
and tools/common.py:81-127).  Plain torch, written the way HF transformers writes T5 (T5LayerNorm,
T5Attention with a bucketed relative position bias, T5DenseGatedActDense with gelu_new), so that the
tools' region -> bench -> swap -> report flow, and the `impl.py` beside this file, have a real target:

  tools/region.py --entry model_entry.py --module layers.0 --out work/r0      (captures a block)
  cp impl.py work/r0/impl.py && tools/bench.py work/r0                          (checks and times it)
  tools/swap.py --entry model_entry.py --impl work/r0 --all-instances           (the whole model)
  tools/report.py work                                                          (krsi_patch.apply(model))

Each layer: x + o(attn(ln1(x))), then + wo(gelu_tanh(wi_0(h)) * wi_1(h)) with h = ln2(x); attention
without the 1/sqrt(d) scale (T5 folds it into the weights), bias = table[bucket(j - i)] per head.
Dims of the kernel-rsi block (d 1152, 16 heads of 72, FFN 4608), bf16 weights.
"""
import math

import torch
import torch.nn.functional as F
from torch import nn

D_MODEL, HEADS, D_KV, D_FF = 1152, 16, 72, 4608
NUM_BUCKETS, MAX_DISTANCE = 32, 128


class T5LayerNorm(nn.Module):
    """RMSNorm as T5 computes it: fp32 statistics, the normalised row cast to the weight's dtype."""

    def __init__(self, d, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        var = x.float().pow(2).mean(-1, keepdim=True)
        x = x * torch.rsqrt(var + self.eps)
        if self.weight.dtype in (torch.float16, torch.bfloat16):
            x = x.to(self.weight.dtype)
        return self.weight * x


def relative_position_bucket(rel, bidirectional=True, num_buckets=NUM_BUCKETS, max_distance=MAX_DISTANCE):
    """T5's bucket of a key - query distance."""
    buckets = 0
    if bidirectional:
        num_buckets //= 2
        buckets = buckets + (rel > 0).long() * num_buckets
        rel = rel.abs()
    else:
        rel = -torch.min(rel, torch.zeros_like(rel))
    max_exact = num_buckets // 2
    large = max_exact + (torch.log(rel.float() / max_exact) / math.log(max_distance / max_exact)
                         * (num_buckets - max_exact)).long()
    large = torch.min(large, torch.full_like(large, num_buckets - 1))
    return buckets + torch.where(rel < max_exact, rel, large)


class T5Block(nn.Module):
    def __init__(self):
        super().__init__()
        inner = HEADS * D_KV
        self.ln1 = T5LayerNorm(D_MODEL)
        self.q = nn.Linear(D_MODEL, inner, bias=False)
        self.k = nn.Linear(D_MODEL, inner, bias=False)
        self.v = nn.Linear(D_MODEL, inner, bias=False)
        self.o = nn.Linear(inner, D_MODEL, bias=False)
        self.relative_attention_bias = nn.Embedding(NUM_BUCKETS, HEADS)
        self.ln2 = T5LayerNorm(D_MODEL)
        self.wi_0 = nn.Linear(D_MODEL, D_FF, bias=False)
        self.wi_1 = nn.Linear(D_MODEL, D_FF, bias=False)
        self.wo = nn.Linear(D_FF, D_MODEL, bias=False)

    def position_bias(self, S, device):
        pos = torch.arange(S, device=device)
        buckets = relative_position_bucket(pos[None, :] - pos[:, None])
        return self.relative_attention_bias(buckets).permute(2, 0, 1).unsqueeze(0)   # [1, H, S, S]

    def forward(self, x):
        B, S, _ = x.shape
        h = self.ln1(x)
        q, k, v = (lin(h).view(B, S, HEADS, D_KV).transpose(1, 2) for lin in (self.q, self.k, self.v))
        scores = q @ k.transpose(-1, -2) + self.position_bias(S, x.device)
        attn = F.softmax(scores.float(), dim=-1).type_as(scores)
        a = (attn @ v).transpose(1, 2).reshape(B, S, HEADS * D_KV)
        x = x + self.o(a)
        h = self.ln2(x)
        x = x + self.wo(F.gelu(self.wi_0(h), approximate="tanh") * self.wi_1(h))
        return x


class T5Stack(nn.Module):
    def __init__(self, layers=2):
        super().__init__()
        self.layers = nn.ModuleList(T5Block() for _ in range(layers))

    def forward(self, x):
        for layer in self.layers:
            x = layer(x)
        return x


def init_(model, seed=0):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("relative_attention_bias.weight"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.5)
            elif p.dim() == 1:
                p.copy_(1 + 0.02 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    return model


def build():
    model = init_(T5Stack()).cuda().to(torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 1024, D_MODEL, generator=g).to("cuda", torch.bfloat16)
    return model, (x,)


def shapes():
    g = torch.Generator().manual_seed(2)
    return [(torch.randn(1, 300, D_MODEL, generator=g).to("cuda", torch.bfloat16),)]


MODE = "train"


def loss(out, inputs):
    return out.float().pow(2).mean()
