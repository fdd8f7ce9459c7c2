"""GEGLU CUDA kernels vs the oracle and the reference's criterion (B200)."""
import ctypes

import pytest
import torch

from gpu_util import DT, capi, ptr, reference_compare, stream
from oracle import ops as O
from oracle.compare import norm_max_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def krsi():
    import geglu
    return geglu


@pytest.mark.parametrize("rows,F,dt", [
    (2048, 4608, torch.bfloat16),   # config 2: u [2,1024,9216]
    (300, 4608, torch.bfloat16),    # config 2 odd case: u [1,300,9216]
    (1, 8, torch.bfloat16),
    (5, 13, torch.bfloat16),        # F not a multiple of 8: scalar path
    (64, 4608, torch.float16),
    (64, 1000, torch.float32),
])
def test_kernel_semantics_vs_oracle(rows, F, dt):
    u, g = O.geglu_inputs(rows, F, dt, seed=rows + F)
    out = torch.ops.krsi.geglu_fwd(u.to(dev))
    du = torch.ops.krsi.geglu_bwd(g.to(dev), u.to(dev))
    tol = 1e-5 if dt == torch.float32 else 1e-2
    assert norm_max_err(out.cpu(), O.geglu_fwd(u)) <= tol
    assert norm_max_err(du.cpu(), O.geglu_bwd(g, u)) <= tol
    # bf16/f16: identical to the fp64 oracle's rounded result on >= 99.9% of elements
    if dt != torch.float32:
        same = (out.cpu() == O.geglu_fwd(u)).float().mean().item()
        assert same >= 0.999, same


def test_block_shape_vs_oracle():
    """The block harness's shape: u [32768, 9216] bf16.  out and du on 512 sampled rows against the
    oracle (the op is elementwise within a row)."""
    rows, F = 32768, 4608
    u, g = O.geglu_inputs(rows, F, torch.bfloat16, seed=12)
    u, g = u.to(dev), g.to(dev)
    out = torch.ops.krsi.geglu_fwd(u)
    du = torch.ops.krsi.geglu_bwd(g, u)
    sel = torch.cat([torch.arange(0, 256), torch.arange(rows - 256, rows)]).to(dev)
    assert norm_max_err(out[sel].float(), O.geglu_fwd(u[sel]).float()) <= 1e-2
    assert norm_max_err(du[sel].float(), O.geglu_bwd(g[sel], u[sel]).float()) <= 1e-2


@pytest.mark.parametrize("rows", [2048, 300])
def test_reference_criterion_vs_fp32(rows):
    """Outputs and du against the reference's eager expression: compare() slack 2 and the
    BASELINE normalised max error <= 1e-2 against fp32."""
    u, g = O.geglu_inputs(rows, 4608, torch.bfloat16, seed=7)
    res, ref32, cand = reference_compare(krsi().geglu, O.geglu_reference, [u.to(dev)], g.to(dev))
    assert res["pass"], res
    for r, c in zip(ref32, cand):
        assert norm_max_err(c, r) <= 1e-2


def test_deterministic_graph_and_c_abi():
    u, g = (t.to(dev) for t in O.geglu_inputs(256, 4608, torch.bfloat16, seed=8))
    o1 = torch.ops.krsi.geglu_fwd(u)
    out = torch.empty_like(o1)
    rc = capi().krsi_geglu_fwd(ptr(u), ptr(out), ctypes.c_int64(256), ctypes.c_int64(4608), DT[torch.bfloat16], stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(out, o1)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.krsi.geglu_bwd(g, u)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(graph):
        du = torch.ops.krsi.geglu_bwd(g, u)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(du, torch.ops.krsi.geglu_bwd(g, u))


def test_compile_fullgraph():
    u, g = (t.to(dev) for t in O.geglu_inputs(128, 4608, torch.bfloat16, seed=9))
    fn = torch.compile(krsi().geglu, fullgraph=True)
    ur = u.clone().requires_grad_(True)
    out = fn(ur)
    (gu,) = torch.autograd.grad(out, [ur], g)
    assert torch.equal(out, torch.ops.krsi.geglu_fwd(u))
    assert torch.equal(gu, torch.ops.krsi.geglu_bwd(g, u))
