"""The gate|value projection with GEGLU in its epilogue (tcgen05 GEMM) vs the oracle, the standalone
GEGLU kernel and the reference's criterion (B200)."""
import ctypes

import pytest
import torch

from gpu_util import DT, capi, ptr, reference_compare, stream
from oracle import ops as O
from oracle.compare import norm_max_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def krsi():
    import linear_geglu
    return linear_geglu


def inputs(rows, K, F, dt, seed):
    """x ~ N(0, 1) [rows, K], w ~ N(0, 1/K) [2F, K] (unit-variance u), g ~ N(0, 1) [rows, F]."""
    x = O.gen((rows, K), seed)
    w = O.gen((2 * F, K), seed + 1, std=K ** -0.5)
    g = O.gen((rows, F), seed + 2)
    return x.to(dt), w.to(dt), g.to(dt)


@pytest.mark.parametrize("rows,K,F,dt", [
    (2048, 1152, 4608, torch.bfloat16),   # the block's feed-forward: d 1152 -> 2 x 4608
    (300, 1152, 4608, torch.bfloat16),    # ragged last row tile
    (128, 1152, 4608, torch.bfloat16),    # the largest size on the one-CTA kernel
    (1, 64, 8, torch.bfloat16),           # one row, one partial F tile
    (129, 72, 200, torch.bfloat16),       # K not a multiple of 64, F not a multiple of 128
    (257, 1000, 136, torch.bfloat16),
    (512, 768, 2048, torch.float16),      # T5 v1.1 base feed-forward, f16
])
def test_fused_vs_oracle_and_standalone_geglu(rows, K, F, dt):
    x, w, _ = inputs(rows, K, F, dt, seed=rows + K + F)
    u, out = torch.ops.krsi.linear_geglu_fwd(x.to(dev), w.to(dev))
    u_o, out_o = O.linear_geglu_fwd(x, w)
    # u: the fp32-accumulated product rounded once; the fp64 product rounded once differs by at most
    # a rounding step where the two sums straddle a rounding boundary
    assert norm_max_err(u.cpu(), u_o) <= 4e-3
    assert (u.cpu() == u_o).float().mean().item() >= 0.99
    # out: the GEGLU arithmetic on the kernel's own u, bit for bit the standalone GEGLU kernel
    assert torch.equal(out, torch.ops.krsi.geglu_fwd(u))
    assert norm_max_err(out.cpu(), out_o) <= 1e-2


def test_autograd_vs_oracle():
    rows, K, F = 512, 1152, 4608
    x, w, g = inputs(rows, K, F, torch.bfloat16, seed=5)
    xr = x.to(dev).requires_grad_(True)
    wr = w.to(dev).requires_grad_(True)
    out = krsi().linear_geglu(xr, wr)
    dx, dw = torch.autograd.grad(out, [xr, wr], g.to(dev))
    u, _ = torch.ops.krsi.linear_geglu_fwd(x.to(dev), w.to(dev))
    dx_o, dw_o = O.linear_geglu_bwd(g, x, w, u.cpu())
    assert norm_max_err(dx.cpu(), dx_o) <= 1e-2
    assert norm_max_err(dw.cpu(), dw_o) <= 1e-2


def test_reference_criterion_bf16():
    """The reference's selftest criterion (compare() with slack 2 against the bf16 original) on the
    T5 v1.1 base feed-forward shape, as linear_geglu.selftest() runs it."""
    x, w, g = inputs(2048, 768, 2048, torch.float32, seed=9)
    res, _, _ = reference_compare(krsi().linear_geglu, krsi().reference,
                                  [x.to(dev, torch.bfloat16), w.to(dev, torch.bfloat16)], g.to(dev) * 1e-2)
    assert res["pass"], res


def test_deterministic_and_graph_capturable():
    x, w, _ = inputs(1024, 1152, 4608, torch.bfloat16, seed=3)
    x, w = x.to(dev), w.to(dev)
    u1, o1 = torch.ops.krsi.linear_geglu_fwd(x, w)
    u2, o2 = torch.ops.krsi.linear_geglu_fwd(x, w)
    assert torch.equal(u1, u2) and torch.equal(o1, o2)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.krsi.linear_geglu_fwd(x, w)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(graph):
        u3, o3 = torch.ops.krsi.linear_geglu_fwd(x, w)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(u3, u1) and torch.equal(o3, o1)
    import _ext
    assert _ext.device_status() == 0


def test_compile_fullgraph():
    x, w, g = (t.to(dev) for t in inputs(256, 512, 512, torch.bfloat16, seed=4))
    fn = torch.compile(krsi().linear_geglu, fullgraph=True)
    xr = x.clone().requires_grad_(True)
    out = fn(xr, w)
    (gx,) = torch.autograd.grad(out, [xr], g)
    xe = x.clone().requires_grad_(True)
    oe = krsi().linear_geglu(xe, w)
    (ge,) = torch.autograd.grad(oe, [xe], g)
    assert torch.equal(out, oe) and torch.equal(gx, ge)


def test_c_abi_direct_call_and_errors():
    lib = capi()
    x, w, _ = (t.to(dev) for t in inputs(64, 256, 128, torch.bfloat16, seed=2))
    u = torch.empty(64, 256, device=dev, dtype=torch.bfloat16)
    out = torch.empty(64, 128, device=dev, dtype=torch.bfloat16)
    args = (ctypes.c_int64(64), ctypes.c_int64(256), ctypes.c_int64(128), DT[torch.bfloat16], stream())
    assert lib.krsi_linear_geglu_fwd(ptr(x), ptr(w), ptr(u), ptr(out), *args) == 0
    torch.cuda.synchronize()
    u2, o2 = torch.ops.krsi.linear_geglu_fwd(x, w)
    assert torch.equal(u, u2) and torch.equal(out, o2)
    # K not a multiple of 8 (TMA row stride), fp32 and a misaligned pointer are refused before launch
    assert lib.krsi_linear_geglu_fwd(ptr(x), ptr(w), ptr(u), ptr(out), ctypes.c_int64(64), ctypes.c_int64(12),
                                     ctypes.c_int64(128), DT[torch.bfloat16], stream()) == 2
    assert lib.krsi_linear_geglu_fwd(ptr(x), ptr(w), ptr(u), ptr(out), ctypes.c_int64(64), ctypes.c_int64(256),
                                     ctypes.c_int64(128), DT[torch.float32], stream()) == 2
    assert lib.krsi_linear_geglu_fwd(ctypes.c_void_p(x.data_ptr() + 2), ptr(w), ptr(u), ptr(out), *args) == 3


# ---------------------------------------------------------------- backward: du = geglu_bwd(dy @ w, u)

@pytest.mark.parametrize("rows,K,F,dt", [
    (2048, 1152, 4608, torch.bfloat16),   # the block's down projection: dy [rows, 1152], wo [1152, 4608]
    (300, 1152, 4608, torch.bfloat16),    # ragged last row tile
    (128, 1152, 4608, torch.bfloat16),    # the largest size on the one-CTA kernel
    (1, 64, 8, torch.bfloat16),
    (129, 72, 200, torch.bfloat16),       # K not a multiple of 64, F not a multiple of 256
    (257, 1000, 136, torch.bfloat16),
    (512, 768, 2048, torch.float16),      # T5 v1.1 base, f16
])
def test_bwd_fused_vs_oracle_and_standalone_geglu(rows, K, F, dt):
    seed = rows + K + F
    dy = O.gen((rows, K), seed).to(dt)
    w = O.gen((K, F), seed + 1, std=K ** -0.5).to(dt)
    u = O.gen((rows, 2 * F), seed + 2).to(dt)
    du = torch.ops.krsi.linear_geglu_bwd(dy.to(dev), w.to(dev), u.to(dev))
    # the unfused pair: cuBLAS's dy @ w (rounded once from fp32, as the fused kernel rounds g), then the
    # GEGLU backward kernel: identical wherever the two GEMMs round g alike
    du_pair = torch.ops.krsi.geglu_bwd(dy.to(dev) @ w.to(dev), u.to(dev))
    assert (du == du_pair).float().mean().item() >= 0.999
    g64 = (dy.double() @ w.double()).to(dt)
    assert norm_max_err(du.cpu(), O.geglu_bwd(g64, u)) <= 1e-2
    import _ext
    assert _ext.device_status() == 0


def ffn_inputs(rows, d, F, seed):
    x = O.gen((rows, d), seed).to(torch.bfloat16)
    wi = O.gen((2 * F, d), seed + 1, std=d ** -0.5).to(torch.bfloat16)
    wo = O.gen((d, F), seed + 2, std=F ** -0.5).to(torch.bfloat16)
    res = O.gen((rows, d), seed + 3).to(torch.bfloat16)
    gy = O.gen((rows, d), seed + 4).to(torch.bfloat16)
    return x, wi, wo, res, gy


def test_feed_forward_autograd_vs_oracle_and_unfused():
    """feed_forward (both fused kernels) against the fp64 oracle chain and against the library's
    unfused composition (linear_geglu forward, GEGLU's backward kernel, cuBLAS GEMMs)."""
    rows, d, F = 512, 1152, 4608
    x, wi, wo, res, gy = ffn_inputs(rows, d, F, seed=6)
    args = [t.to(dev).requires_grad_(True) for t in (x, wi, wo, res)]
    y = krsi().feed_forward(*args)
    grads = torch.autograd.grad(y, args, gy.to(dev))
    args2 = [t.to(dev).requires_grad_(True) for t in (x, wi, wo, res)]
    y2 = torch.addmm(args2[3], krsi().linear_geglu(args2[0], args2[1]), args2[2].t())
    grads2 = torch.autograd.grad(y2, args2, gy.to(dev))
    assert torch.equal(y, y2)
    for a_, b_ in zip(grads, grads2):
        assert norm_max_err(a_.float(), b_.float()) <= 1e-2
    # fp64 oracle chain on the kernel's own u
    u, g = torch.ops.krsi.linear_geglu_fwd(x.to(dev), wi.to(dev))
    u, g = u.cpu(), g.cpu()
    dg = (gy.double() @ wo.double()).to(torch.bfloat16)
    dx_o, dwi_o = O.linear_geglu_bwd(dg, x, wi, u)
    dwo_o = gy.double().t() @ g.double()
    assert norm_max_err(grads[0].cpu(), dx_o) <= 1e-2
    assert norm_max_err(grads[1].cpu(), dwi_o) <= 1e-2
    assert norm_max_err(grads[2].cpu(), dwo_o) <= 1e-2
    assert torch.equal(grads[3], gy.to(dev))


def test_feed_forward_reference_criterion_bf16():
    """The reference's selftest criterion on the whole feed-forward (T5 v1.1 base shape)."""
    rows, d, F = 2048, 768, 2048
    x, wi, wo, _, _ = ffn_inputs(rows, d, F, seed=8)
    cot = O.gen((rows, d), 13).to(dev) * 1e-2
    res, _, _ = reference_compare(krsi().feed_forward, krsi().feed_forward_reference,
                                  [x.to(dev), wi.to(dev), wo.to(dev)], cot)
    assert res["pass"], res


def test_bwd_c_abi_and_errors():
    lib = capi()
    dy = O.gen((64, 256), 1).to(dev, torch.bfloat16)
    w = O.gen((256, 128), 2).to(dev, torch.bfloat16)
    u = O.gen((64, 256), 3).to(dev, torch.bfloat16)
    du = torch.empty_like(u)
    args = (ctypes.c_int64(64), ctypes.c_int64(256), ctypes.c_int64(128), DT[torch.bfloat16], stream())
    assert lib.krsi_linear_geglu_bwd(ptr(dy), ptr(w), ptr(u), ptr(du), *args) == 0
    torch.cuda.synchronize()
    assert torch.equal(du, torch.ops.krsi.linear_geglu_bwd(dy, w, u))
    assert lib.krsi_linear_geglu_bwd(ptr(dy), ptr(w), ptr(u), ptr(du), ctypes.c_int64(64), ctypes.c_int64(250),
                                     ctypes.c_int64(128), DT[torch.bfloat16], stream()) == 2
    assert lib.krsi_linear_geglu_bwd(ptr(dy), ctypes.c_void_p(w.data_ptr() + 8), ptr(u), ptr(du), *args) == 3


@pytest.mark.parametrize("rows,K,F", [(129, 72, 200), (256, 1152, 4608), (300, 1152, 4608), (2048, 768, 2048)])
def test_cta_pairs_match_one_cta_kernels_bitwise(rows, K, F, monkeypatch):
    """Above 128 rows the fused kernels run on CTA pairs (M = 256 tiles split over two CTAs); each CTA
    runs the same K loop as the one-CTA kernel, so both paths give the same bits (KRSI_GEMM_PAIRS=0
    forces the one-CTA kernels)."""
    x, w, _ = inputs(rows, K, F, torch.bfloat16, seed=rows + 7)
    x, w = x.to(dev), w.to(dev)
    dy = O.gen((rows, K), rows + 8).to(dev, torch.bfloat16)
    wo = O.gen((K, F), rows + 9, std=K ** -0.5).to(dev, torch.bfloat16)
    monkeypatch.setenv("KRSI_GEMM_PAIRS", "1")
    u_p, o_p = torch.ops.krsi.linear_geglu_fwd(x, w)
    du_p = torch.ops.krsi.linear_geglu_bwd(dy, wo, u_p)
    monkeypatch.setenv("KRSI_GEMM_PAIRS", "0")
    u_1, o_1 = torch.ops.krsi.linear_geglu_fwd(x, w)
    du_1 = torch.ops.krsi.linear_geglu_bwd(dy, wo, u_p)
    assert torch.equal(u_p, u_1) and torch.equal(o_p, o_1)
    assert torch.equal(du_p, du_1)
    import _ext
    assert _ext.device_status() == 0
