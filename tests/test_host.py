"""Host-side contract of the drop-in library: module API and signatures as the reference's,
operator schemas, fake (meta) implementations for torch.compile, and the product path's isolation
from the oracle.  CPU only."""
import ast
import inspect

import pytest
import torch

from conftest import LIBRARY


def test_public_signatures_match_the_reference():
    import geglu
    import relpos_attention
    import rmsnorm

    assert list(inspect.signature(rmsnorm.rmsnorm).parameters) == ["x2d", "w", "eps"]
    assert list(inspect.signature(geglu.geglu).parameters) == ["u"]
    assert list(inspect.signature(relpos_attention.relpos_attention).parameters) == \
        ["qkv", "pd", "B", "S", "H", "D", "scale"]
    for mod, fn_name, cls in ((rmsnorm, "reference", "RMSNorm"), (geglu, "reference", "GEGLU"),
                              (relpos_attention, "reference", "RelPosAttention")):
        assert callable(getattr(mod, fn_name)) and callable(mod.selftest)
        assert issubclass(getattr(mod, cls), torch.autograd.Function)


def test_operator_schemas():
    ops = torch.ops.krsi
    expect = {
        "rmsnorm_fwd": "(Tensor x2d, Tensor w, float eps) -> (Tensor, Tensor)",
        "rmsnorm_bwd": "(Tensor g, Tensor x2d, Tensor w, Tensor rstd) -> (Tensor, Tensor)",
        "geglu_fwd": "(Tensor u) -> Tensor",
        "geglu_bwd": "(Tensor g, Tensor u) -> Tensor",
        "relpos_attn_fwd": "(Tensor qkv, Tensor pd, int B, int S, int H, int D, float scale) -> (Tensor, Tensor, Tensor)",
        "relpos_attn_bwd": "(Tensor dout, Tensor qkv, Tensor pd, Tensor out32, Tensor lse, int B, int S, int H, "
                           "int D, float scale) -> (Tensor, Tensor)",
    }
    import rmsnorm  # noqa: F401  (loads the extension)

    for name, sig in expect.items():
        schema = str(getattr(ops, name).default._schema)
        assert schema == f"krsi::{name}{sig}", schema


def test_fake_impls_give_reference_shapes():
    import rmsnorm  # noqa: F401

    ops = torch.ops.krsi
    x = torch.empty(6, 40, device="meta", dtype=torch.bfloat16)
    y, r = ops.rmsnorm_fwd(x, torch.empty(40, device="meta", dtype=torch.bfloat16), 1e-6)
    assert y.shape == x.shape and r.shape == (6,) and r.dtype == torch.float32
    u = torch.empty(6, 80, device="meta", dtype=torch.bfloat16)
    assert ops.geglu_fwd(u).shape == (6, 40)
    B, S, H, D = 2, 5, 3, 72
    qkv = torch.empty(B * S, 3 * H * D, device="meta", dtype=torch.bfloat16)
    pd = torch.empty(H, 2 * S - 1, device="meta")
    out, out32, lse = ops.relpos_attn_fwd(qkv, pd, B, S, H, D, 0.1)
    assert out.shape == (B * S, H * D) and out32.dtype == torch.float32 and lse.shape == (B * H, S)
    dqkv, dpd = ops.relpos_attn_bwd(out, qkv, pd, out32, lse, B, S, H, D, 0.1)
    assert dqkv.shape == qkv.shape and dpd.shape == (H, 2 * S - 1)


def test_cpu_tensors_are_rejected_loudly():
    """No CPU fallback: the ops exist only for CUDA tensors."""
    import geglu

    with pytest.raises((NotImplementedError, RuntimeError)):
        geglu.geglu(torch.randn(4, 16))


def test_product_never_imports_the_oracle():
    pkg = LIBRARY.parent
    files = (list(LIBRARY.glob("*.py")) + list((pkg / "harness").glob("*.py")) + list((pkg / "t5_block").glob("*.py"))
             + [pkg / "build.py"])
    assert len(files) >= 12
    for py in files:
        tree = ast.parse(py.read_text())
        for node in ast.walk(tree):
            names = []
            if isinstance(node, ast.Import):
                names = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom):
                names = [node.module or ""]
            assert not any(n.split(".")[0] == "oracle" for n in names), f"{py} imports the oracle"
