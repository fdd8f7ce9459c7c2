"""The oracle (oracle/ops.py) against the golden fixtures made by the reference's own code
(tests/golden/make_golden.py): its Triton kernels under the CPU interpreter and its eager
reference() functions with autograd, all fp32.  CPU only."""
import pytest
import torch

from oracle import ops


def close(a, b, tol):
    a, b = a.double(), b.double()
    scale = b.abs().max().item() or 1.0
    err = (a - b).abs().max().item() / scale
    assert err <= tol, f"normalised max error {err:.3e} > {tol:.1e}"


@pytest.mark.parametrize("tag", ["small", "wide"])
def test_rmsnorm_oracle_matches_reference(golden, tag):
    c = golden("rmsnorm")[tag]
    y, rstd = ops.rmsnorm_fwd(c["x"], c["w"], float(c["eps"]))
    close(y, c["kernel_y"], 1e-6)
    close(rstd, c["kernel_rstd"], 1e-6)
    close(y, c["ref_y"], 1e-6)
    dx, dw = ops.rmsnorm_bwd(c["g"], c["x"], c["w"], rstd)
    close(dx, c["ref_dx"], 1e-5)
    close(dw, c["ref_dw"], 1e-5)
    if "kernel_dx" in c:
        close(dx, c["kernel_dx"], 1e-5)
        close(dw, c["kernel_dw"], 1e-5)


@pytest.mark.parametrize("tag", ["small", "odd", "wide"])
def test_geglu_oracle_matches_reference(golden, tag):
    c = golden("geglu")[tag]
    out = ops.geglu_fwd(c["u"])
    close(out, c["kernel_out"], 1e-6)
    close(out, c["ref_out"], 1e-6)
    du = ops.geglu_bwd(c["g"], c["u"])
    close(du, c["kernel_du"], 1e-5)
    close(du, c["ref_du"], 1e-5)


@pytest.mark.parametrize("tag", ["d32", "d64", "d72"])
def test_relpos_oracle_matches_reference(golden, tag):
    c = golden("relpos")[tag]
    B, S, H, D = (int(v) for v in c["dims"])
    scale = float(c["scale"])
    out, out32, lse = ops.relpos_attn_fwd(c["qkv"], c["pd"], B, S, H, D, scale)
    close(out32, c["ref_out"], 1e-5)
    dqkv, dpd = ops.relpos_attn_bwd(c["dout"], c["qkv"], c["pd"], out32, lse, B, S, H, D, scale)
    close(dqkv, c["ref_dqkv"], 1e-5)
    close(dpd, c["ref_dpd"], 1e-5)
    if "kernel_out" in c:   # the reference's own Triton kernels (power-of-two D only)
        close(out32, c["kernel_out32"], 1e-5)
        close(lse, c["kernel_lse"], 1e-5)
        dq2, dpd2 = ops.relpos_attn_bwd(c["dout"], c["qkv"], c["pd"], c["kernel_out32"], c["kernel_lse"],
                                        B, S, H, D, scale)
        close(dq2, c["kernel_dqkv"], 1e-5)
        close(dpd2, c["kernel_dpd"], 1e-5)


def test_relpos_oracle_bwd_equals_autograd_fp64():
    """The explicit backward (delta from O32, dS, diagonal sums) equals autograd of the fp64 forward."""
    B, S, H, D = 2, 9, 3, 8
    qkv, pd, dout = ops.attn_inputs(B, S, H, D, torch.float64, seed=5)
    pd = pd.double()
    dout = dout.double()
    q = qkv.clone().requires_grad_(True)
    p = pd.clone().requires_grad_(True)
    out, out32, lse = ops.relpos_attn_fwd(q, p, B, S, H, D, 0.3)
    gq, gp = torch.autograd.grad(out, [q, p], dout)
    dqkv, dpd = ops.relpos_attn_bwd(dout, qkv, pd, out32.double(), lse.double(), B, S, H, D, 0.3)
    close(dqkv, gq, 1e-6)
    close(dpd, gp, 1e-6)


def test_compare_criterion_planted_bugs():
    """The restated compare() passes same-level noise and fails a one-row 5% error and NaNs
    (mirrors the reference's tests/test_tools.py:38-56 on CPU)."""
    from oracle.compare import compare

    g = torch.Generator().manual_seed(0)
    r = torch.randn(64, 1024, generator=g)

    def noisy(seed):
        gg = torch.Generator().manual_seed(seed)
        return r + 1e-2 * r.abs().mean() * torch.randn(r.shape, generator=gg)

    assert compare([r], [noisy(1)], [noisy(2)])["pass"]
    bad = noisy(2)
    bad[5] *= 1.05
    res = compare([r], [noisy(1)], [bad])
    assert not res["pass"] and res["outputs"][0]["bad_rows"] == 1
    nan = noisy(2)
    nan[0, 0] = float("nan")
    assert not compare([r], [noisy(1)], [nan])["pass"]
