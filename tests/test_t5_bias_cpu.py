"""T5 bucketed relative position, host side: the bucket map of the C ABI (the one its kernels use)
and of the library's torch expression against T5's own (HF transformers
T5Attention._relative_position_bucket) over T5's configurations and many others, every distance up to
+-20000; argument checks that return before any device work."""
import ctypes
import itertools

import pytest
import torch

from conftest import PKG

transformers = pytest.importorskip("transformers")
from transformers.models.t5.modeling_t5 import T5Attention  # noqa: E402

CONFIGS = [(nb, md, bi) for nb, md, bi in itertools.product([8, 16, 32, 64, 128], [16, 64, 100, 128, 256, 1000, 4096],
                                                            [True, False])
           if md > (nb // 2 if bi else nb) // 2]


@pytest.fixture(scope="module")
def bucket_fn():
    lib = ctypes.CDLL(str(PKG / "lib" / "libkrsi_b200.so"))
    f = lib.krsi_t5_bucket
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.POINTER(ctypes.c_int)]
    return f


@pytest.mark.parametrize("nb,md,bi", CONFIGS)
def test_c_abi_bucket_map_equals_t5(bucket_fn, nb, md, bi):
    R = 20000
    rel = torch.arange(-R, R + 1)
    ref = T5Attention._relative_position_bucket(rel, bidirectional=bi, num_buckets=nb, max_distance=md).tolist()
    out = ctypes.c_int()
    got = []
    for r in range(-R, R + 1):
        assert bucket_fn(nb, md, int(bi), r, ctypes.byref(out)) == 0
        got.append(out.value)
    assert got == ref


@pytest.mark.parametrize("nb,md,bi", [(32, 128, True), (32, 128, False), (64, 256, True), (16, 100, False)])
def test_library_torch_expression_equals_t5(nb, md, bi):
    import t5_bias

    S = 6000
    rel = torch.arange(-(S - 1), S)
    ref = T5Attention._relative_position_bucket(rel, bidirectional=bi, num_buckets=nb, max_distance=md)
    assert torch.equal(t5_bias.buckets(S, bi, nb, md), ref)


def test_argument_checks(bucket_fn):
    out = ctypes.c_int()
    assert bucket_fn(1, 128, 1, 0, ctypes.byref(out)) == 1          # too few buckets
    assert bucket_fn(32, 4, 1, 0, ctypes.byref(out)) == 1           # max_distance within the exact range
    assert bucket_fn(512, 1024, 1, 0, ctypes.byref(out)) == 1       # more buckets than supported
    lib = ctypes.CDLL(str(PKG / "lib" / "libkrsi_b200.so"))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    assert lib.krsi_t5_bias_fwd(vp(0), vp(0), i64(0), i64(4), 32, 128, 1, 0, vp(0)) == 0   # S = 0: no-op
    assert lib.krsi_t5_bias_fwd(vp(0), vp(0), i64(8), i64(4), 32, 128, 1, 0, vp(0)) == 1   # null pointers
    assert lib.krsi_t5_bias_fwd(vp(1), vp(1), i64(8), i64(4), 32, 128, 1, 9, vp(0)) == 1   # bad dtype


def test_oracle_matches_the_torch_expression():
    import t5_bias
    from oracle import ops as O

    table = torch.randn(32, 6, dtype=torch.float64)
    for bi in (True, False):
        assert torch.equal(O.t5_bias_fwd(table, 300, bi), t5_bias.reference(table, 300, bi))
        dpd = torch.randn(6, 599, dtype=torch.float64)
        t = table.clone().requires_grad_(True)
        (g,) = torch.autograd.grad(t5_bias.reference(t, 300, bi), [t], dpd.float())
        torch.testing.assert_close(O.t5_bias_bwd(dpd, 300, 6, bi), g.double(), rtol=1e-6, atol=1e-6)

