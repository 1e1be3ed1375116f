"""The allocation-free composition-weight producer, ``dc_proj_weights_noalloc``.

Some callers cannot allocate device memory at the point where they need the
weights: code running inside a custom allocator's callbacks, under a framework
whose memory pool owns the whole device, or in a serving process that allows
no allocation after start-up.  This entry point takes inputs and outputs from
the caller and keeps its intermediate activations in a fixed device array of
the library.  The test calls it through the C ABI twice in a row, on
different inputs, and compares each result with the regular entry point
(``dc_proj_weights``, whose workspace the caller provides), under the
tolerance the other tests use.  It also checks that a call beyond the fixed
size is refused.  This file is collected last on purpose, so that a run that
stops at the first failure has run every other test before it.
"""

import ctypes

import numpy as np
import pytest
import torch

import dc_triton_opt_b200 as dc
from dc_triton_opt_b200 import _lib
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _inputs(M, Dm, I, H, R, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    rn = lambda *s, std: (std * torch.randn(*s, generator=g, device=DEV)).to(torch.bfloat16)
    return rn(M, Dm, std=1.0), rn(Dm, I, std=Dm ** -0.5), rn(I, 8 * H * R, std=0.05), rn(Dm, 4 * H, std=0.05)


def _noalloc(x, w1, w2, wdd, H, R):
    """Call the C entry point directly; the caller owns only inputs and outputs."""
    M, Dm = x.shape
    I = w1.shape[1]
    dw = [torch.empty(M, H * R, device=DEV, dtype=x.dtype) for _ in range(8)]
    dd = [torch.empty(M, H, device=DEV, dtype=x.dtype) for _ in range(4)]
    p = _lib.DcProjParams()
    p.M, p.Dm, p.I, p.H, p.R, p.dtype = M, Dm, I, H, R, _lib.DC_DTYPE_BF16
    p.x, p.w1, p.w2, p.wdd = x.data_ptr(), w1.data_ptr(), w2.data_ptr(), wdd.data_ptr()
    p.hidden = None
    for i, t in enumerate(dw):
        p.dw[i] = t.data_ptr()
    for i, t in enumerate(dd):
        p.dd[i] = t.data_ptr()
    lib = _lib.load()
    rc = lib.dc_proj_weights_noalloc(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, dw, dd


def test_noalloc_matches_the_regular_entry_point_twice():
    H, R, Dm, I = 32, 1, 512, 128
    for call, (M, seed) in enumerate(((3000, 1), (1000, 2))):  # second call: fewer tokens, other inputs
        x, w1, w2, wdd = _inputs(M, Dm, I, H, R, seed)
        rc, dw, dd = _noalloc(x, w1, w2, wdd, H, R)
        assert rc == 0, _lib.load().dc_attn_last_error().decode()
        pre, post = dc.dc_proj_weights(x, w1, w2, wdd, H, R)
        torch.cuda.synchronize()
        want = [pre.qw1, pre.qw2, pre.kw1, pre.kw2, post.qw1, post.qw2, post.kw1, post.kw2]
        for i, (g, w) in enumerate(zip(dw, want)):
            assert_close(g.float().cpu().numpy(), w.reshape(M, -1).float().cpu().numpy(), f"call {call} dw[{i}]")
        for i, (g, w) in enumerate(zip(dd, [pre.qdd, pre.kdd, post.qdd, post.kdd])):
            assert_close(g.float().cpu().numpy(), w.reshape(M, -1).float().cpu().numpy(), f"call {call} dd[{i}]")


def test_noalloc_rejects_sizes_beyond_its_workspace():
    I = 128
    M = _lib_max() // I + 1
    x = torch.empty(16, 32, device=DEV, dtype=torch.bfloat16)  # never read: the size check comes first
    p = _lib.DcProjParams()
    p.M, p.Dm, p.I, p.H, p.R, p.dtype = M, 32, I, 2, 1, _lib.DC_DTYPE_BF16
    p.x = p.w1 = p.w2 = p.wdd = x.data_ptr()
    for i in range(8):
        p.dw[i] = x.data_ptr()
    for i in range(4):
        p.dd[i] = x.data_ptr()
    lib = _lib.load()
    assert lib.dc_proj_weights_noalloc(ctypes.byref(p), None) == -2
    assert "exceeds the fixed workspace" in lib.dc_attn_last_error().decode()


def _lib_max():
    return 4 * 1024 * 1024  # DC_PROJ_NOALLOC_MAX_HIDDEN in include/dc_attn.h
