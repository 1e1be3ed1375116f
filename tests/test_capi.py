"""C ABI checks that need no GPU: the library loads, exports every entry point
declared in include/dc_attn.h, its struct layout matches the ctypes mirror, and
argument validation reports errors (codes + messages) before touching a device."""

import ctypes
import os
import re

import pytest

from dc_triton_opt_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dc_attn.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"DC_API\s+[\w\s\*]*?\b(dc_\w+)\s*\(", src)))


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_abi_and_struct_layout():
    lib = _lib.load()
    assert lib.dc_attn_abi_version() == _lib.ABI_VERSION
    assert lib.dc_attn_params_size() == ctypes.sizeof(_lib.DcAttnParams)


def _params(**kw):
    p = _lib.DcAttnParams()
    p.abi_version = _lib.ABI_VERSION
    p.B, p.T, p.H, p.D, p.G, p.R = 2, 64, 8, 128, 2, 1
    p.window, p.scale, p.dtype, p.kernel = 16, 0.088, _lib.DC_DTYPE_BF16, _lib.DC_KERNEL_AUTO
    p.q = p.k = p.v = p.out = 256
    p.out_sb, p.out_st, p.out_sh = 64 * 8 * 128, 8 * 128, 128
    p.pre.identity = p.post.identity = 1
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("field,value,code,needle", [
    ("abi_version", 99, -2, "abi_version"),
    ("q", None, -1, "non-NULL"),
    ("dtype", 7, -3, "dtype"),
    ("H", 9, -2, "divisible"),
    ("D", 136, -2, "D=136"),
    ("R", 9, -2, "R=9"),
    ("out_sh", 64, -2, "strides"),
    ("kernel", 5, -2, "kernel selector"),
])
def test_validation_errors(field, value, code, needle):
    lib = _lib.load()
    p = _params(**{field: value})
    rc = lib.dc_attn_fwd(ctypes.byref(p), None)
    assert rc == code
    assert needle in lib.dc_attn_last_error().decode()


def test_half_given_rank_factors_rejected():
    lib = _lib.load()
    p = _params()
    p.pre.qw1 = 256
    assert lib.dc_attn_select_kernel(ctypes.byref(p)) == -1
    assert "qw1 and qw2" in lib.dc_attn_last_error().decode()


def test_selection_needs_no_device():
    lib = _lib.load()
    p = _params()
    assert lib.dc_attn_select_kernel(ctypes.byref(p)) in (_lib.DC_KERNEL_SIMT, _lib.DC_KERNEL_TC)
    p.kernel = _lib.DC_KERNEL_SIMT
    assert lib.dc_attn_select_kernel(ctypes.byref(p)) == _lib.DC_KERNEL_SIMT


def test_residual_entry_null_weights():
    lib = _lib.load()
    vp = ctypes.c_void_p
    rc = lib.dc_attn_fwd_residual(vp(256), vp(256), vp(256), None, vp(256), vp(256), vp(256), vp(256),
                                  vp(256), vp(256), 1, 1, 128, None, 1, 8, 8, 128, 2,
                                  ctypes.c_float(0.1), 4, 16, 0, None)
    assert rc == -1
    assert "six DC weights" in lib.dc_attn_last_error().decode()


@pytest.mark.parametrize("cu,B,needle", [
    ([0, 10, 20], 2, "B must be 1"),
    ([1, 10, 64], 1, "start at 0"),
    ([0, 40, 30, 64], 1, "non-decreasing"),
    ([0, 10, 63], 1, "end at T"),
])
def test_varlen_validation_needs_no_device(cu, B, needle):
    """dc_attn_fwd_varlen checks its packed-batch description before any launch."""
    lib = _lib.load()
    p = _params(B=B)
    arr = (ctypes.c_int32 * len(cu))(*cu)
    rc = lib.dc_attn_fwd_varlen(ctypes.byref(p), arr, len(cu) - 1, None)
    assert rc == -2  # DC_ERR_SHAPE
    assert needle in lib.dc_attn_last_error().decode()
