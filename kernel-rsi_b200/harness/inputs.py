"""Seeded synthetic inputs of the BASELINE configs, generated on the CPU so every device (and the
CPU oracle) sees the same values.  Used by bench.py, the block harness tests and the GPU tests.

  rmsnorm_inputs  config 1: x [2,1024,1152] -> x2d [2048,1152] ~ N(0,1); w = 1 + N(0, 0.02); g ~ N(0,1)
  geglu_inputs    config 2: u [rows, 2F] ~ N(0,1); g [rows, F] ~ N(0,1)
  attn_inputs     configs 3/4: q, k, v ~ N(0,1)/sqrt(D) packed into qkv [B*S, 3*H*D];
                  pd ~ N(0, 0.02) fp32; dO ~ N(0,1)
"""
from __future__ import annotations

import math

import torch


def gen(shape, seed, dtype=torch.float32, std=1.0, mean=0.0):
    """N(mean, std^2) on the CPU from a seeded generator, then cast."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g, dtype=torch.float32) * std + mean).to(dtype)


def rmsnorm_inputs(rows=2048, n=1152, dtype=torch.float32, seed=0):
    return gen((rows, n), seed, dtype), gen((n,), seed + 1, dtype, std=0.02, mean=1.0), gen((rows, n), seed + 2, dtype)


def geglu_inputs(rows=2048, F=4608, dtype=torch.bfloat16, seed=0):
    return gen((rows, 2 * F), seed, dtype), gen((rows, F), seed + 1, dtype)


def attn_inputs(B=2, S=1024, H=16, D=72, dtype=torch.bfloat16, seed=0):
    qkv = gen((B * S, 3 * H * D), seed, dtype, std=1.0 / math.sqrt(D))
    pd = gen((H, 2 * S - 1), seed + 1, torch.float32, std=0.02)
    dout = gen((B * S, H * D), seed + 2, dtype)
    return qkv, pd, dout
