"""The C ABI library: it loads without a GPU, exports every function include/krsi_b200.h declares,
and rejects bad arguments with the documented status codes before touching the device."""
import ctypes
import re

import pytest

from conftest import PKG, ROOT

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = set()
    for header in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(krsi_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    return ctypes.CDLL(str(PKG / "lib" / "libkrsi_b200.so"))


def test_header_declares_the_hot_path():
    assert [h.name for h in HEADERS] == ["krsi_b200.h", "krsi_b200_diag.h"]
    names = declared_functions()
    for op in ("rmsnorm_fwd", "rmsnorm_bwd", "geglu_fwd", "geglu_bwd", "relpos_attn_fwd", "relpos_attn_bwd"):
        assert f"krsi_{op}" in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_error_strings_and_version(lib):
    lib.krsi_error_string.restype = ctypes.c_char_p
    for code in range(0, 7):
        assert lib.krsi_error_string(code)
    assert b"unknown" in lib.krsi_error_string(99)
    assert lib.krsi_abi_version() >= 10000


def test_argument_checks_return_codes(lib):
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    # null pointers with real sizes -> INVALID_ARGUMENT (1), before any CUDA call
    rc = lib.krsi_rmsnorm_fwd(vp(0), vp(0), vp(0), vp(0), i64(4), i64(8), ctypes.c_float(1e-6), 0, 0, vp(0))
    assert rc == 1
    rc = lib.krsi_geglu_fwd(vp(0), vp(0), i64(4), i64(8), 1, vp(0))
    assert rc == 1
    # bad dtype code
    rc = lib.krsi_geglu_bwd(vp(1), vp(1), vp(1), i64(4), i64(8), 7, vp(0))
    assert rc == 1
    # empty inputs are a successful no-op
    assert lib.krsi_rmsnorm_fwd(vp(0), vp(0), vp(0), vp(0), i64(0), i64(8), ctypes.c_float(1e-6), 0, 0, vp(0)) == 0
    assert lib.krsi_geglu_fwd(vp(0), vp(0), i64(0), i64(8), 1, vp(0)) == 0


def test_empty_inputs_launch_nothing(lib):
    """Zero rows, batch or sequence length return success before any pointer check or CUDA call
    (the cases with an output to zero, an RMSNorm dw or a T5 table gradient, need a device)."""
    i64, vp, f32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_float
    assert lib.krsi_geglu_bwd(vp(0), vp(0), vp(0), i64(0), i64(8), 1, vp(0)) == 0
    assert lib.krsi_geglu_bwd(vp(0), vp(0), vp(0), i64(4), i64(0), 1, vp(0)) == 0
    for B, S in ((0, 128), (2, 0), (0, 0)):
        assert lib.krsi_relpos_attn_fwd(vp(0), i64(3 * 16 * 72), vp(0), vp(0), vp(0), vp(0), i64(B), i64(S),
                                        i64(16), i64(72), f32(72 ** -0.5), 1, vp(0)) == 0, (B, S)
    assert lib.krsi_relpos_attn_bwd(vp(0), vp(0), i64(3 * 16 * 72), vp(0), vp(0), vp(0), vp(0), i64(3 * 16 * 72),
                                    vp(0), vp(0), ctypes.c_size_t(0), i64(2), i64(0), i64(16), i64(72),
                                    f32(72 ** -0.5), 1, vp(0)) == 0
    assert lib.krsi_t5_bias_fwd(vp(0), vp(0), i64(0), i64(12), 32, 128, 1, 0, vp(0)) == 0
    # a negative size is an argument error, not an empty input
    assert lib.krsi_relpos_attn_fwd(vp(0), i64(3 * 16 * 72), vp(0), vp(0), vp(0), vp(0), i64(-1), i64(128),
                                    i64(16), i64(72), f32(72 ** -0.5), 1, vp(0)) == 1
    assert lib.krsi_geglu_bwd(vp(0), vp(0), vp(0), i64(-1), i64(8), 1, vp(0)) == 1


def test_workspace_queries(lib):
    sz = ctypes.c_size_t(0)
    assert lib.krsi_rmsnorm_bwd_workspace_size(ctypes.c_int64(2048), ctypes.c_int64(1152), ctypes.byref(sz)) == 0
    assert sz.value == 296 * 1152 * 4
    assert lib.krsi_rmsnorm_bwd_workspace_size(ctypes.c_int64(3), ctypes.c_int64(10), ctypes.byref(sz)) == 0
    assert sz.value == 3 * 10 * 4


def test_rmsnorm_bwd_add_argument_checks():
    """The fused residual-gradient RMSNorm backward rejects a missing added gradient before any
    device work (the other checks are the plain backward's)."""
    lib = ctypes.CDLL(str(PKG / "lib" / "libkrsi_b200.so"))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    rc = lib.krsi_rmsnorm_bwd_add(vp(1), vp(1), vp(1), vp(1), vp(0), vp(1), vp(1), vp(1), ctypes.c_size_t(1 << 20),
                                  i64(4), i64(8), 0, 0, vp(0))
    assert rc == 1


def test_linear_geglu_argument_checks(lib):
    """The fused projection + GEGLU refuses, before any device work: null pointers, fp32, a K or F
    that is not a multiple of 8 (TMA row stride, 16-byte epilogue packets) and misaligned buffers;
    zero rows is a no-op."""
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    call = lib.krsi_linear_geglu_fwd
    assert call(vp(0), vp(16), vp(16), vp(16), i64(4), i64(64), i64(64), 1, vp(0)) == 1
    assert call(vp(16), vp(16), vp(16), vp(16), i64(4), i64(64), i64(64), 0, vp(0)) == 2
    assert call(vp(16), vp(16), vp(16), vp(16), i64(4), i64(60), i64(64), 1, vp(0)) == 2
    assert call(vp(16), vp(16), vp(16), vp(16), i64(4), i64(64), i64(20), 1, vp(0)) == 2
    assert call(vp(18), vp(16), vp(16), vp(16), i64(4), i64(64), i64(64), 1, vp(0)) == 3
    assert call(vp(0), vp(0), vp(0), vp(0), i64(0), i64(64), i64(64), 1, vp(0)) == 0


def test_linear_geglu_bwd_argument_checks(lib):
    """The fused down-projection input gradient + GEGLU backward refuses bad arguments before any
    device work, like the forward."""
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    call = lib.krsi_linear_geglu_bwd
    assert call(vp(16), vp(0), vp(16), vp(16), i64(4), i64(64), i64(64), 1, vp(0)) == 1
    assert call(vp(16), vp(16), vp(16), vp(16), i64(4), i64(64), i64(64), 0, vp(0)) == 2
    assert call(vp(16), vp(16), vp(16), vp(16), i64(4), i64(12), i64(64), 1, vp(0)) == 2
    assert call(vp(16), vp(16), vp(24), vp(16), i64(4), i64(64), i64(64), 1, vp(0)) == 3
    assert call(vp(0), vp(0), vp(0), vp(0), i64(0), i64(64), i64(64), 1, vp(0)) == 0
