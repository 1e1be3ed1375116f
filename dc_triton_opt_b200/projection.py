"""Producer of the per-token composition weights (``dc_proj_weights`` in
``libdcattn.so``): DCFormer's dynamic weight projection from the hidden states,
the step before the DC-attention forward.  The reference project receives
these weights precomputed and has no code for it.

    hidden = gelu(x @ w1);  dw = hidden @ w2;  dd = tanh(x @ wdd)

``w2`` columns: per set (pre, post) qw1 (H*R) | qw2 (R*H) | kw1 (H*R) | kw2 (R*H);
``wdd`` columns: pre qdd | pre kdd | post qdd | post kdd (H each).
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .api import _DTYPES, DCTerms, _check


def dc_proj_weights(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, wdd: torch.Tensor, H: int, R: int,
                    hidden: Optional[torch.Tensor] = None):
    """x [..., Dm] -> (pre, post) DCTerms with identity and the query- and
    key-wise weights of rank R and both gates, shaped for :func:`dc_attn_fwd`
    (x's leading dims + [H, R] / [R, H] / [H]).  ``hidden`` ([M, I], x's
    dtype) is the workspace; it is allocated when not given."""
    _check(x.dtype in _DTYPES and w1.dtype == x.dtype and w2.dtype == x.dtype and wdd.dtype == x.dtype,
           "x, w1, w2, wdd must share one dtype, bfloat16 or float16")
    _check(x.is_cuda, "x must be a CUDA tensor")
    Dm = x.shape[-1]
    lead = x.shape[:-1]
    x2 = x.reshape(-1, Dm).contiguous()
    M, I = x2.shape[0], w1.shape[1]
    _check(tuple(w1.shape) == (Dm, I), f"w1 must be [Dm={Dm}, I]")
    _check(tuple(w2.shape) == (I, 8 * H * R), f"w2 must be [I={I}, 8*H*R={8 * H * R}]")
    _check(tuple(wdd.shape) == (Dm, 4 * H), f"wdd must be [Dm={Dm}, 4*H={4 * H}]")
    w1, w2, wdd = w1.contiguous(), w2.contiguous(), wdd.contiguous()
    if hidden is None:
        hidden = torch.empty((M, I), device=x.device, dtype=x.dtype)
    _check(tuple(hidden.shape) == (M, I) and hidden.dtype == x.dtype and hidden.is_contiguous(),
           f"hidden must be a contiguous [{M}, {I}] tensor of x's dtype")
    kw = dict(device=x.device, dtype=x.dtype)
    dw = [torch.empty((M, H * R), **kw) for _ in range(8)]
    dd = [torch.empty((M, H), **kw) for _ in range(4)]
    p = _lib.DcProjParams()
    p.M, p.Dm, p.I, p.H, p.R, p.dtype = M, Dm, I, H, R, _DTYPES[x.dtype]
    p.x, p.w1, p.w2, p.wdd, p.hidden = x2.data_ptr(), w1.data_ptr(), w2.data_ptr(), wdd.data_ptr(), hidden.data_ptr()
    for i, t in enumerate(dw):
        p.dw[i] = t.data_ptr()
    for i, t in enumerate(dd):
        p.dd[i] = t.data_ptr()
    lib = _lib.load()
    with torch.cuda.device(x.device):
        _lib.check(lib.dc_proj_weights(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)),
                   "dc_proj_weights")
    hr, rh, hh = (*lead, H, R), (*lead, R, H), (*lead, H)
    sets = []
    for s in range(2):
        a, b, c, d = dw[4 * s: 4 * s + 4]
        sets.append(DCTerms(identity=True, qw1=a.view(hr), qw2=b.view(rh), kw1=c.view(hr), kw2=d.view(rh),
                            qdd=dd[2 * s].view(hh), kdd=dd[2 * s + 1].view(hh)))
    return sets[0], sets[1]
