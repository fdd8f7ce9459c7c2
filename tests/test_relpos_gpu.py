"""Relpos flash attention CUDA kernels (tcgen05 / TMEM / TMA) vs the oracle and the reference's
criterion (B200).  Ordered from the smallest case up so a first failure is the most telling."""
import ctypes
import math

import pytest
import torch

from gpu_util import DT, capi, ptr, reference_compare, stream
from oracle import ops as O
from oracle.compare import norm_max_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def attn_fwd_check(B, S, H, D, dtype=torch.bfloat16, seed=0, tol=1e-2):
    qkv, pd, _ = O.attn_inputs(B, S, H, D, dtype, seed=seed)
    scale = 1.0 / math.sqrt(D)
    out, out32, lse = torch.ops.krsi.relpos_attn_fwd(qkv.to(dev), pd.to(dev), B, S, H, D, scale)
    torch.cuda.synchronize()
    import _ext
    assert _ext.device_status(clear=True) == 0
    o_ref, o32_ref, lse_ref = O.relpos_attn_fwd(qkv.to(dev), pd.to(dev), B, S, H, D, scale)
    e_out = norm_max_err(out.float(), o32_ref)
    e_32 = norm_max_err(out32, o32_ref)
    e_lse = (lse - lse_ref).abs().max().item()
    assert torch.isfinite(out32).all()
    assert e_32 <= tol and e_out <= tol, (e_32, e_out)
    assert e_lse <= 1e-3, e_lse
    return out, out32, lse


@pytest.mark.parametrize("B,S,H,D", [
    (1, 128, 1, 64),     # one key block, one CTA
    (1, 256, 1, 64),     # two key blocks: the online-softmax path
    (1, 128, 1, 72),     # D = 72: zero-padded to 80 by TMA
    (1, 300, 2, 72),     # ragged: partial key block and partial query tile
    (2, 17, 3, 72),      # tiny S
    (1, 1, 1, 72),       # S = 1
    (2, 520, 2, 32),
    (1, 384, 2, 128),
    (1, 200, 1, 96),
])
def test_fwd_small_shapes(B, S, H, D):
    attn_fwd_check(B, S, H, D, seed=B * 1000 + S + D)


def test_fwd_f16():
    attn_fwd_check(1, 300, 2, 72, dtype=torch.float16)


@pytest.mark.parametrize("S", [1024, 300])
def test_fwd_baseline_config(S):
    """Config 3: B=2, H=16, L=1024 (and L=300), D=72, scale 1/sqrt(72)."""
    attn_fwd_check(2, S, 16, 72, seed=S)


def test_fwd_large_logits_rescale():
    """Logits spread over a wide range: exercises the conditional rescale of O."""
    B, S, H, D = 1, 640, 2, 72
    qkv, pd, _ = O.attn_inputs(B, S, H, D, torch.bfloat16, seed=11)
    qkv = (qkv.float() * 6).to(torch.bfloat16)
    pd = pd * 200                    # bias up to ~+-15 nats, varying along the diagonal
    scale = 1.0 / math.sqrt(D)
    out, out32, lse = torch.ops.krsi.relpos_attn_fwd(qkv.to(dev), pd.to(dev), B, S, H, D, scale)
    o_ref, o32_ref, lse_ref = O.relpos_attn_fwd(qkv.to(dev), pd.to(dev), B, S, H, D, scale)
    assert norm_max_err(out32, o32_ref) <= 1e-2
    assert (lse - lse_ref).abs().max().item() <= 1e-3


def test_fwd_strided_qkv_view():
    """qkv as a row-strided view of a wider buffer (read in place through its row stride)."""
    B, S, H, D = 1, 256, 2, 72
    qkv, pd, _ = O.attn_inputs(B, S, H, D, torch.bfloat16, seed=12)
    wide = torch.zeros(B * S, 3 * H * D + 64, dtype=torch.bfloat16, device=dev)
    wide[:, :3 * H * D] = qkv.to(dev)
    view = wide[:, :3 * H * D]
    out, out32, _ = torch.ops.krsi.relpos_attn_fwd(view, pd.to(dev), B, S, H, D, 0.1)
    _, o32_ref, _ = O.relpos_attn_fwd(qkv.to(dev), pd.to(dev), B, S, H, D, 0.1)
    assert norm_max_err(out32, o32_ref) <= 1e-2


def test_fwd_c_abi_direct():
    B, S, H, D = 1, 256, 2, 72
    qkv, pd, _ = (t.to(dev) for t in O.attn_inputs(B, S, H, D, torch.bfloat16, seed=13))
    out = torch.empty(B * S, H * D, dtype=torch.bfloat16, device=dev)
    out32 = torch.empty(B * S, H * D, device=dev)
    lse = torch.empty(B * H, S, device=dev)
    i64 = ctypes.c_int64
    rc = capi().krsi_relpos_attn_fwd(ptr(qkv), i64(3 * H * D), ptr(pd), ptr(out), ptr(out32), ptr(lse), i64(B), i64(S),
                                     i64(H), i64(D), ctypes.c_float(0.1), DT[torch.bfloat16], stream())
    assert rc == 0
    torch.cuda.synchronize()
    o2, o32b, l2 = torch.ops.krsi.relpos_attn_fwd(qkv, pd, B, S, H, D, 0.1)
    assert torch.equal(out, o2) and torch.equal(out32, o32b) and torch.equal(lse, l2)
    # unsupported: D not a multiple of 8, fp32 qkv
    rc = capi().krsi_relpos_attn_fwd(ptr(qkv), i64(3 * H * 70), ptr(pd), ptr(out), ptr(out32), ptr(lse), i64(B),
                                     i64(S), i64(H), i64(70), ctypes.c_float(0.1), DT[torch.bfloat16], stream())
    assert rc == 2
