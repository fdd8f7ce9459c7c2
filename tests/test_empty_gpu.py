"""Empty inputs through the public API (B200): zero rows, an empty batch or no positions give outputs
of the right shapes, zero parameter gradients and no device error, and the next real call still
works.  The C-ABI calls behind them return before any launch (tests/test_capi.py checks those
returns on the CPU)."""
import pytest
import torch

import _ext

pytestmark = pytest.mark.gpu
dev = "cuda"


def _leaf(*shape, dtype=torch.bfloat16):
    return torch.randn(*shape, device=dev, dtype=dtype).requires_grad_(True)


def _settled():
    torch.cuda.synchronize()
    assert _ext.device_status() == 0


def test_rmsnorm_zero_rows():
    from rmsnorm import rmsnorm

    x, w = _leaf(0, 1152), _leaf(1152)
    y = rmsnorm(x, w, 1e-6)
    assert y.shape == (0, 1152) and y.dtype == torch.bfloat16
    y.backward(torch.empty_like(y))
    assert x.grad.shape == (0, 1152)
    assert torch.equal(w.grad, torch.zeros_like(w))
    _settled()


def test_geglu_zero_rows():
    from geglu import geglu

    u = _leaf(0, 9216)
    out = geglu(u)
    assert out.shape == (0, 4608)
    out.backward(torch.empty_like(out))
    assert u.grad.shape == (0, 9216)
    _settled()


def test_relpos_attention_empty_batch():
    from relpos_attention import relpos_attention

    H, D, S = 16, 72, 128
    qkv, pd = _leaf(0, 3 * H * D), _leaf(H, 2 * S - 1, dtype=torch.float32)
    out = relpos_attention(qkv, pd, 0, S, H, D, D ** -0.5)
    assert out.shape == (0, H * D)
    out.backward(torch.empty_like(out))
    assert qkv.grad.shape == (0, 3 * H * D)
    assert torch.equal(pd.grad, torch.zeros_like(pd))   # no query attends: the bias gradient is zero
    _settled()


def test_linear_geglu_and_feed_forward_zero_rows():
    from linear_geglu import feed_forward, linear_geglu

    x, wi, wo = _leaf(0, 1152), _leaf(2 * 4608, 1152), _leaf(1152, 4608)
    out = linear_geglu(x, wi)
    assert out.shape == (0, 4608)
    out.backward(torch.empty_like(out))
    assert x.grad.shape == (0, 1152) and torch.equal(wi.grad, torch.zeros_like(wi))
    wi.grad = None
    y = feed_forward(x, wi, wo)
    assert y.shape == (0, 1152)
    y.backward(torch.empty_like(y))
    assert torch.equal(wi.grad, torch.zeros_like(wi)) and torch.equal(wo.grad, torch.zeros_like(wo))
    _settled()


def test_t5_bias_no_positions():
    from t5_bias import t5_relpos_bias

    table = _leaf(32, 12, dtype=torch.float32)
    pd = t5_relpos_bias(table, 0)
    assert pd.shape == (12, 0)
    pd.backward(torch.empty_like(pd))
    assert torch.equal(table.grad, torch.zeros_like(table))
    _settled()


def test_a_real_call_after_the_empty_ones():
    from geglu import geglu, reference

    u = torch.randn(64, 512, device=dev, dtype=torch.bfloat16)
    assert torch.allclose(geglu(u).float(), reference(u.float()), atol=2e-2, rtol=2e-2)
    _settled()
