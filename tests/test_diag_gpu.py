"""Diagnostics on the GPU: the bounded-wait watchdog and the FMA-pipe exp2 of the attention kernels.

- The watchdog self-test waits on an mbarrier that nothing completes, with a short spin limit: the
  kernel must return (no hang, no trap), record the self-test role in the device status word, free
  its TMEM, and leave the context usable for the next real call.
- The FMA-pipe exp2 (Cody-Waite reduction + a degree-3 polynomial, used for a quarter of the
  attention forward's exponentials) must stay within its stated relative error of 7.5e-5 against
  float64 exp2 over [-125, 128), agree with CUDA's exp2f to the same bound, and match a bit-exact
  CPU restatement of its arithmetic."""
import ctypes
import math

import numpy as np
import pytest
import torch

import _ext
from gpu_util import capi, ptr, stream
from oracle import ops as O
from oracle.compare import norm_max_err

pytestmark = pytest.mark.gpu
dev = "cuda"
KRSI_ERR_DEVICE_TIMEOUT = 6
ROLE_SELFTEST = 0x7F


def test_watchdog_wait_gives_up_and_reports():
    _ext.device_status(clear=True)
    flags = torch.full((2,), -1, dtype=torch.int32, device=dev)
    rc = capi().krsi_diag_watchdog_selftest(ctypes.c_uint32(64), ptr(flags), stream())
    assert rc == 0
    torch.cuda.synchronize()                       # the kernel returned
    assert flags.tolist() == [1, 1]                # warp 0 gave up; warp 1 left through the abort flag
    st = _ext.device_status(clear=True)
    assert st & 0xFF == KRSI_ERR_DEVICE_TIMEOUT and st >> 8 == ROLE_SELFTEST, hex(st)
    assert _ext.device_status() == 0               # cleared
    with pytest.raises(RuntimeError, match="watchdog"):
        capi().krsi_diag_watchdog_selftest(ctypes.c_uint32(16), ptr(flags), stream())
        _ext.check_device_status()
    # the context is still usable: a real attention call runs and matches the oracle
    B, S, H, D = 1, 256, 2, 72
    qkv, pd, _ = O.attn_inputs(B, S, H, D, torch.bfloat16, seed=5)
    out, out32, lse = torch.ops.krsi.relpos_attn_fwd(qkv.to(dev), pd.to(dev), B, S, H, D, D ** -0.5)
    torch.cuda.synchronize()
    assert _ext.device_status() == 0
    _, o32_ref, _ = O.relpos_attn_fwd(qkv, pd, B, S, H, D, D ** -0.5)
    assert norm_max_err(out32.cpu(), o32_ref) <= 1e-2


def test_watchdog_selftest_rejects_bad_arguments():
    assert capi().krsi_diag_watchdog_selftest(ctypes.c_uint32(0), ctypes.c_void_p(1), stream()) == 1
    assert capi().krsi_diag_watchdog_selftest(ctypes.c_uint32(8), ctypes.c_void_p(0), stream()) == 1


def exp2_poly_cpu(x: np.ndarray) -> np.ndarray:
    """Bit-exact restatement of the kernel's arithmetic in float32 (round-to-nearest adds, fused
    multiply-adds evaluated exactly in float64 and rounded once)."""
    c3, c2, c1, c0 = (np.float32(v) for v in (0.05517162382602692, 0.2426111251115799,
                                               0.6932609677314758, 0.9999280571937561))

    def fma(a, b, c):
        return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)

    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    magic = np.float32(12582912.0)
    j = (x + magic).astype(np.float32)
    f = (x - (j - magic).astype(np.float32)).astype(np.float32)
    p = fma(fma(fma(np.full_like(f, c3), f, np.full_like(f, c2)), f, np.full_like(f, c1)), f, np.full_like(f, c0))
    return (p.view(np.int32) + (j.view(np.int32) << 23)).astype(np.int32).view(np.float32)


def run_exp2_poly(x: torch.Tensor) -> torch.Tensor:
    y = torch.empty_like(x)
    assert capi().krsi_diag_exp2_poly(ptr(x), ptr(y), ctypes.c_int64(x.numel()), stream()) == 0
    torch.cuda.synchronize()
    return y


def test_exp2_poly_error_bound():
    x = torch.linspace(-125.0, 127.99, (1 << 22) + 1, dtype=torch.float64).float()
    x = torch.cat([x, torch.tensor([-0.5, 0.5, -1e-7, 0.0, 1e-7, 127.5, -124.999])])
    xd = x.to(dev)
    y = run_exp2_poly(xd)
    exact = torch.exp2(x.double())
    rel = ((y.cpu().double() - exact) / exact).abs()
    assert rel.max().item() <= 7.5e-5, (rel.max().item(), x[rel.argmax()].item())
    # CUDA's own exp2f on the same inputs, to the same bound (plus exp2f's own ~2 ulp)
    cuda_ref = torch.exp2(xd).double()
    rel_cuda = ((y.double() - cuda_ref) / cuda_ref).abs().max().item()
    assert rel_cuda <= 7.5e-5 + 4 * 2.0 ** -23, rel_cuda
    # bit-exact against the CPU restatement of the arithmetic
    assert np.array_equal(y.cpu().numpy().view(np.int32), exp2_poly_cpu(x.numpy()).view(np.int32))


def test_exp2_poly_masked_inputs_give_a_tiny_positive():
    x = torch.tensor([-math.inf, -1e30, -300.0, -126.0, -125.0], device=dev)
    y = run_exp2_poly(x).cpu()
    assert torch.isfinite(y).all() and (y > 0).all() and (y <= 2.0 ** -124).all()


def test_exp2_poly_odd_length_and_empty():
    x = torch.tensor([1.0, 2.0, -3.0], device=dev)
    assert torch.allclose(run_exp2_poly(x).cpu(), torch.tensor([2.0, 4.0, 0.125]), rtol=1e-4)
    assert capi().krsi_diag_exp2_poly(ctypes.c_void_p(0), ctypes.c_void_p(0), ctypes.c_int64(0), stream()) == 0
