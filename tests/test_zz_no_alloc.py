"""The allocation-free RMSNorm backward (krsi_rmsnorm_bwd_noalloc) against the workspace entry point.

Callers that cannot allocate device memory (a host that owns every allocation, a loop that must not
stall on cudaMalloc) use this entry point: its scratch is a fixed array inside the library.  This
test first fills that array with NaN partial sums, then calls the entry point through the C ABI
twice in a row, on different inputs, and checks that each result is bitwise equal to
krsi_rmsnorm_bwd with a caller workspace (same kernels, same partial-row count) and within
tolerance of the oracle.  It lives in its own file, collected last, so a failure here never hides
the other GPU tests."""
import ctypes

import pytest
import torch

from gpu_util import DT, capi, ptr, stream
from oracle import ops as O
from oracle.compare import norm_max_err

pytestmark = pytest.mark.gpu
dev = "cuda"
i64 = ctypes.c_int64


def bwd_with_workspace(g, x, w, rstd):
    lib = capi()
    dx, dw = torch.empty_like(x), torch.empty_like(w)
    ws = ctypes.c_size_t(0)
    assert lib.krsi_rmsnorm_bwd_workspace_size(i64(x.shape[0]), i64(x.shape[1]), ctypes.byref(ws)) == 0
    workspace = torch.empty(max(ws.value, 16), dtype=torch.uint8, device=dev)
    rc = lib.krsi_rmsnorm_bwd(ptr(g), ptr(x), ptr(w), ptr(rstd), ptr(dx), ptr(dw), ptr(workspace),
                              ctypes.c_size_t(workspace.numel()), i64(x.shape[0]), i64(x.shape[1]),
                              DT[x.dtype], DT[w.dtype], stream())
    assert rc == 0
    return dx, dw


def bwd_no_alloc(g, x, w, rstd):
    dx, dw = torch.empty_like(x), torch.empty_like(w)
    rc = capi().krsi_rmsnorm_bwd_noalloc(ptr(g), ptr(x), ptr(w), ptr(rstd), ptr(dx), ptr(dw), i64(x.shape[0]),
                                         i64(x.shape[1]), DT[x.dtype], DT[w.dtype], stream())
    assert rc == 0
    return dx, dw


def poison_scratch():
    """One call on non-finite inputs over a larger problem than the calls under test, so every
    partial row they use starts out holding NaN: a row a later launch failed to write would show."""
    x = torch.full((4096, 2048), float("nan"), device=dev)
    w = torch.ones(2048, device=dev)
    rstd = torch.ones(4096, device=dev)
    dx, dw = bwd_no_alloc(x, x, w, rstd)       # 296 partial rows x 2048 columns of NaN
    torch.cuda.synchronize()
    assert torch.isnan(dw).all()


@pytest.mark.parametrize("calls", [[(2048, 1152, torch.float32, 0), (300, 4096, torch.bfloat16, 1)]])
def test_no_alloc_backward_matches_workspace_backward(calls):
    poison_scratch()
    for rows, n, dt, seed in calls:   # two calls in a row, the second on new data and shapes
        x, w, g = (t.to(dev, dt) for t in O.rmsnorm_inputs(rows, n, torch.float32, seed=seed))
        _, rstd = torch.ops.krsi.rmsnorm_fwd(x, w, 1e-6)
        dx_ref, dw_ref = bwd_with_workspace(g, x, w, rstd)
        dx, dw = bwd_no_alloc(g, x, w, rstd)
        torch.cuda.synchronize()
        # the same kernels with the same partial-row count: bitwise equal, not just close
        assert torch.equal(dx, dx_ref)
        assert torch.equal(dw, dw_ref)
        # and both within the tolerance the other RMSNorm tests use against the oracle
        dx_o, dw_o = O.rmsnorm_bwd(g.cpu(), x.cpu(), w.cpu(), rstd.cpu())
        tol = 1e-5 if dt == torch.float32 else 1e-2
        assert norm_max_err(dx.float().cpu(), dx_o.float()) <= tol
        assert norm_max_err(dw.float().cpu(), dw_o.float()) <= tol


def test_no_alloc_rejects_problems_beyond_its_scratch():
    x = torch.empty(8, 2, device=dev)
    rc = capi().krsi_rmsnorm_bwd_noalloc(ptr(x), ptr(x), ptr(x), ptr(x), ptr(x), ptr(x), i64(1 << 20), i64(4096),
                                         DT[torch.float32], DT[torch.float32], stream())
    assert rc == 2   # KRSI_ERR_UNSUPPORTED: 296 partial rows x 4096 > 1,048,576 floats; nothing launched
