"""ctypes binding of ``libdcattn.so`` (the C ABI in ``include/dc_attn.h``).

The product path is this CUDA library; there is no CPU fallback.  If the
library is missing or cannot be loaded, every call raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libdcattn.so")
ABI_VERSION = 2

DC_DTYPE_BF16, DC_DTYPE_FP16 = 0, 1
DC_KERNEL_AUTO, DC_KERNEL_SIMT, DC_KERNEL_TC, DC_KERNEL_TCS, DC_KERNEL_TCM = 0, 1, 2, 3, 4
KERNELS = {"auto": DC_KERNEL_AUTO, "simt": DC_KERNEL_SIMT, "tc": DC_KERNEL_TC, "tcs": DC_KERNEL_TCS, "tcm": DC_KERNEL_TCM}
STATUS = {0: "DC_OK", -1: "DC_ERR_NULL", -2: "DC_ERR_SHAPE", -3: "DC_ERR_DTYPE",
          -4: "DC_ERR_UNSUPPORTED", -5: "DC_ERR_ALIGN", -6: "DC_ERR_LAUNCH", -7: "DC_ERR_DEVICE"}
DC_TEST_SKIP_LOADS = 1
DEV_ERRORS = {0: "DC_DEV_OK", 1: "DC_DEV_ERR_TIMEOUT_Q", 2: "DC_DEV_ERR_TIMEOUT_FULL",
              3: "DC_DEV_ERR_TIMEOUT_FREE", 4: "DC_DEV_ERR_TIMEOUT_S", 5: "DC_DEV_ERR_TIMEOUT_P",
              6: "DC_DEV_ERR_TIMEOUT_O"}
EXPORTS = ("dc_attn_fwd", "dc_attn_fwd_residual", "dc_attn_select_kernel", "dc_attn_read_error",
           "dc_attn_last_kernel", "dc_attn_last_error", "dc_attn_abi_version", "dc_attn_params_size",
           "dc_attn_bwd", "dc_attn_bwd_params_size", "dc_attn_fwd_varlen", "dc_proj_weights", "dc_proj_weights_noalloc", "dc_attn_fwd_fp8qk")


class DcTerms(ctypes.Structure):
    _fields_ = [("identity", ctypes.c_int32), ("w", ctypes.c_void_p),
                ("qw1", ctypes.c_void_p), ("qw2", ctypes.c_void_p),
                ("kw1", ctypes.c_void_p), ("kw2", ctypes.c_void_p),
                ("qdd", ctypes.c_void_p), ("kdd", ctypes.c_void_p),
                ("qmat", ctypes.c_void_p)]


class DcAttnParams(ctypes.Structure):
    _fields_ = [("abi_version", ctypes.c_int32), ("B", ctypes.c_int32), ("T", ctypes.c_int32),
                ("H", ctypes.c_int32), ("D", ctypes.c_int32), ("G", ctypes.c_int32),
                ("R", ctypes.c_int32), ("window", ctypes.c_int32), ("scale", ctypes.c_float),
                ("dtype", ctypes.c_int32), ("kernel", ctypes.c_int32),
                ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("out_sb", ctypes.c_int64), ("out_st", ctypes.c_int64),
                ("out_sh", ctypes.c_int64), ("seq_lens", ctypes.c_void_p),
                ("err_flag", ctypes.c_void_p), ("pre", DcTerms), ("post", DcTerms),
                ("wait_us", ctypes.c_uint32), ("test_flags", ctypes.c_int32)]


class DcTermGrads(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("qw1", ctypes.c_void_p), ("qw2", ctypes.c_void_p),
                ("qdd", ctypes.c_void_p), ("qmat", ctypes.c_void_p)]


class DcAttnBwdParams(ctypes.Structure):
    _fields_ = [("fwd", DcAttnParams), ("dout", ctypes.c_void_p), ("dq", ctypes.c_void_p),
                ("dk", ctypes.c_void_p), ("dv", ctypes.c_void_p), ("dpre", DcTermGrads),
                ("dpost", DcTermGrads)]


class DcProjParams(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int32), ("Dm", ctypes.c_int32), ("I", ctypes.c_int32), ("H", ctypes.c_int32),
                ("R", ctypes.c_int32), ("dtype", ctypes.c_int32), ("x", ctypes.c_void_p), ("w1", ctypes.c_void_p),
                ("w2", ctypes.c_void_p), ("wdd", ctypes.c_void_p), ("hidden", ctypes.c_void_p),
                ("dw", ctypes.c_void_p * 8), ("dd", ctypes.c_void_p * 4)]


_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and type the CUDA library; raise RuntimeError if it is unusable."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"DC-attention CUDA library not found at {path}; build it with "
                "`python -m dc_triton_opt_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        lib.dc_attn_fwd.argtypes = [ctypes.POINTER(DcAttnParams), ctypes.c_void_p]
        lib.dc_attn_fwd.restype = ctypes.c_int
        lib.dc_attn_select_kernel.argtypes = [ctypes.POINTER(DcAttnParams)]
        lib.dc_attn_select_kernel.restype = ctypes.c_int
        lib.dc_attn_last_error.argtypes = []
        lib.dc_attn_last_error.restype = ctypes.c_char_p
        lib.dc_attn_read_error.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        lib.dc_attn_read_error.restype = ctypes.c_int
        lib.dc_attn_last_kernel.argtypes = []
        lib.dc_attn_last_kernel.restype = ctypes.c_int
        lib.dc_attn_abi_version.restype = ctypes.c_int
        lib.dc_attn_params_size.restype = ctypes.c_int
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        lib.dc_attn_fwd_residual.argtypes = [vp] * 9 + [vp, i64, i64, i64, vp] + [i32] * 5 + \
            [ctypes.c_float, i32, i32, i32, vp]
        lib.dc_attn_fwd_residual.restype = ctypes.c_int
        lib.dc_attn_fwd_varlen.argtypes = [ctypes.POINTER(DcAttnParams), ctypes.c_void_p, ctypes.c_int32,
                                           ctypes.c_void_p]
        lib.dc_attn_fwd_varlen.restype = ctypes.c_int
        lib.dc_attn_fwd_fp8qk.argtypes = [ctypes.POINTER(DcAttnParams), ctypes.c_float, ctypes.c_float,
                                          ctypes.c_void_p]
        lib.dc_attn_fwd_fp8qk.restype = ctypes.c_int
        lib.dc_proj_weights.argtypes = [ctypes.POINTER(DcProjParams), ctypes.c_void_p]
        lib.dc_proj_weights.restype = ctypes.c_int
        lib.dc_proj_weights_noalloc.argtypes = [ctypes.POINTER(DcProjParams), ctypes.c_void_p]
        lib.dc_proj_weights_noalloc.restype = ctypes.c_int
        lib.dc_attn_bwd.argtypes = [ctypes.POINTER(DcAttnBwdParams), ctypes.c_void_p]
        lib.dc_attn_bwd.restype = ctypes.c_int
        lib.dc_attn_bwd_params_size.restype = ctypes.c_int
        if lib.dc_attn_abi_version() != ABI_VERSION:
            raise RuntimeError(f"libdcattn ABI {lib.dc_attn_abi_version()} != binding {ABI_VERSION}")
        if lib.dc_attn_params_size() != ctypes.sizeof(DcAttnParams):
            raise RuntimeError("dc_attn_params layout mismatch between library and binding")
        if lib.dc_attn_bwd_params_size() != ctypes.sizeof(DcAttnBwdParams):
            raise RuntimeError("dc_attn_bwd_params layout mismatch between library and binding")
        _lib = lib
        return lib


def check(rc: int, what: str = "dc_attn_fwd"):
    if rc != 0:
        msg = load().dc_attn_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({STATUS.get(rc, rc)}): {msg}")
