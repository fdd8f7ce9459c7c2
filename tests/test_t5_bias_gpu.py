"""T5 bucketed relative position kernels (B200) against the oracle (T5's own bucket map from HF
transformers, a table lookup and its float64 gradient) and against T5's own compute_bias."""
import ctypes
import math

import pytest
import torch

from gpu_util import DT, capi, ptr, reference_compare, stream
from oracle import ops as O
from oracle.compare import norm_max_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def table_of(nb, H, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return (0.5 * torch.randn(nb, H, generator=g)).to(dtype)


@pytest.mark.parametrize("S", [1, 2, 17, 300, 1024, 4096])
@pytest.mark.parametrize("bi", [True, False])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fwd_is_the_table_lookup(S, bi, dtype):
    H, nb, md = 16, 32, 128
    table = table_of(nb, H, dtype, S)
    pd = torch.ops.krsi.t5_bias_fwd(table.to(dev), S, nb, md, bi)
    assert torch.equal(pd.cpu(), O.t5_bias_fwd(table, S, bi, nb, md))   # a gather: bit-exact


@pytest.mark.parametrize("S,nb,md,bi", [(1, 32, 128, True), (300, 32, 128, True), (300, 32, 128, False),
                                        (2048, 32, 128, True), (5000, 64, 256, True), (777, 16, 100, False)])
def test_bwd_is_the_bucket_sum(S, nb, md, bi):
    H = 12
    g = torch.Generator().manual_seed(S + nb)
    dpd = torch.randn(H, 2 * S - 1, generator=g)
    table = table_of(nb, H, torch.float32, 1)
    dt = torch.ops.krsi.t5_bias_bwd(dpd.to(dev), table.to(dev), S, nb, md, bi)
    ref = O.t5_bias_bwd(dpd, S, H, bi, nb, md)
    assert (dt.cpu().double() - ref).abs().max().item() <= 1e-5 * max(1.0, ref.abs().max().item())
    # bf16 table: the same sums rounded to bf16
    dtb = torch.ops.krsi.t5_bias_bwd(dpd.to(dev), table.to(dev, torch.bfloat16), S, nb, md, bi)
    assert dtb.dtype == torch.bfloat16 and norm_max_err(dtb.float().cpu(), ref) <= 1e-2


def test_bwd_deterministic():
    S, H, nb = 4096, 16, 32
    dpd = torch.randn(H, 2 * S - 1, device=dev)
    table = torch.zeros(nb, H, device=dev)
    a = torch.ops.krsi.t5_bias_bwd(dpd, table, S, nb, 128, True)
    b = torch.ops.krsi.t5_bias_bwd(dpd, table, S, nb, 128, True)
    assert torch.equal(a, b)


def test_matches_t5_compute_bias():
    """The row the kernel produces, expanded as the attention op does (bias[h, i, j] = pd[h, j - i + S - 1]),
    is T5's own position bias (T5Attention.compute_bias) for the same table."""
    from transformers import T5Config
    from transformers.models.t5.modeling_t5 import T5Attention

    S, H = 300, 8
    for bi in (True, False):
        cfg = T5Config(d_model=64, d_kv=8, num_heads=H, relative_attention_num_buckets=32,
                       relative_attention_max_distance=128, is_decoder=not bi)
        att = T5Attention(cfg, has_relative_attention_bias=True)          # on the CPU, as the oracle
        with torch.no_grad():
            att.relative_attention_bias.weight.copy_(table_of(32, H, torch.float32, 5))
            t5 = att.compute_bias(S, S)[0]                                # [H, S, S]
        pd = torch.ops.krsi.t5_bias_fwd(att.relative_attention_bias.weight.detach().to(dev), S, 32, 128, bi)
        assert torch.equal(O.toeplitz_bias(pd.cpu(), S), t5)


def test_autograd_compile_and_reference_criterion():
    import t5_bias

    S, H = 512, 12
    table = (0.1 * torch.randn(32, H)).to(dev)
    t1 = table.clone().requires_grad_(True)
    pd = t5_bias.t5_relpos_bias(t1, S)
    dpd = torch.randn_like(pd)
    (g1,) = torch.autograd.grad(pd, [t1], dpd)
    fn = torch.compile(lambda t: t5_bias.t5_relpos_bias(t, S), fullgraph=True)
    t2 = table.clone().requires_grad_(True)
    (g2,) = torch.autograd.grad(fn(t2), [t2], dpd)
    assert torch.equal(g1, g2)
    res, _, _ = reference_compare(lambda t: t5_bias.t5_relpos_bias(t, S), lambda t: t5_bias.reference(t, S),
                                  [table], dpd)
    assert res["pass"], res


def test_t5_bias_into_attention_end_to_end():
    """table -> pd -> relpos attention, gradients back to qkv and the table, against the reference path
    (T5's bucket lookup + SDPA with the bias) in fp32."""
    import relpos_attention as ra
    import t5_bias

    B, S, H, D = 2, 256, 4, 64
    qkv, _, dout = (t.to(dev) for t in O.attn_inputs(B, S, H, D, torch.bfloat16, seed=9))
    table = (0.3 * torch.randn(32, H)).to(dev)

    def ours(q, t):
        return ra.relpos_attention(q, t5_bias.t5_relpos_bias(t, S), B, S, H, D, D ** -0.5)

    def ref(q, t):
        return O.relpos_reference(q, O.t5_bias_fwd(t, S), B, S, H, D, D ** -0.5)

    res, ref32, cand = reference_compare(ours, ref, [qkv, table], dout)
    assert res["pass"], res
    for r, c in zip(ref32, cand):
        assert norm_max_err(c, r) <= 1e-2


def test_c_abi_direct():
    S, H, nb = 100, 4, 32
    table = table_of(nb, H, torch.float32, 3).to(dev)
    pd = torch.empty(H, 2 * S - 1, device=dev)
    rc = capi().krsi_t5_bias_fwd(ptr(table), ptr(pd), ctypes.c_int64(S), ctypes.c_int64(H), nb, 128, 1,
                                 DT[torch.float32], stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(pd.cpu(), O.t5_bias_fwd(table.cpu(), S))
