"""Backward of the DC-attention forward, backed by ``dc_attn_bwd`` in ``libdcattn.so``.

* :func:`dc_attn_bwd` — gradients of q, k, v and of the query-side terms
  (w, qw1, qw2, qdd, qmat) of both sets for an output gradient ``dout``.
* :func:`dc_attn` — the forward as a differentiable torch op
  (``torch.autograd.Function``) over q, k, v and those terms.
* :class:`DCResidual` — the reference's ``TritonDCResidual`` interface
  (``triton_dc_residual.py:1432-1892``): ``alloc_buffers`` / ``forward`` /
  ``backward`` with the residual rank-1 weights; ``backward`` returns dq in the
  input dtype and dk, dv and the six weight gradients in fp32, as the
  reference does.  The saved-state buffers of the reference are accepted and
  not needed: the CUDA backward recomputes everything from q, k, v.

Key-wise terms (kw1, kw2, kdd) have no backward here; a call with them raises.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .api import DCTerms, _check, _params, dc_attn_fwd

_GRAD_TERMS = ("w", "qw1", "qw2", "qdd", "qmat")


def dc_attn_bwd(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                pre: Optional[DCTerms] = None, post: Optional[DCTerms] = None,
                scaling: Optional[float] = None, window: Optional[int] = None, G: int = 1,
                seq_lens: Optional[torch.Tensor] = None):
    """Gradients of ``sum(dc_attn_fwd(q, k, v, pre, post, ...) * dout)``.

    Returns ``(dq, dk, dv, dpre, dpost)``: dq in q's dtype, dk and dv in fp32,
    and per set a dict term name -> fp32 gradient for every query-side term the
    set has.  Runs on q's device and current stream, asynchronously."""
    for tm in (pre, post):
        _check(tm is None or (tm.kw1 is None and tm.kw2 is None and tm.kdd is None),
               "dc_attn_bwd: key-wise terms (kw1, kw2, kdd) have no backward")
    p, _, keep = _params(q, k, v, pre, post, scaling, window, G, seq_lens, None, "auto")
    _check(dout.shape == q.shape and dout.dtype == q.dtype and dout.device == q.device,
           "dout must match q's shape, dtype and device")
    dout = dout.contiguous()
    keep.append(dout)
    B, T, H, D = q.shape
    f32 = dict(device=q.device, dtype=torch.float32)
    dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    dk, dv = torch.empty(q.shape, **f32), torch.empty(q.shape, **f32)
    bp = _lib.DcAttnBwdParams()
    bp.fwd = p
    bp.dout, bp.dq, bp.dk, bp.dv = dout.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    grads = []
    for tm, gs in ((pre, bp.dpre), (post, bp.dpost)):
        gd = {}
        if tm is not None:
            for n in _GRAD_TERMS:
                t = getattr(tm, n)
                if t is not None:
                    gd[n] = torch.empty(t.shape, **f32)
                    setattr(gs, n, gd[n].data_ptr())
        grads.append(gd)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(lib.dc_attn_bwd(ctypes.byref(bp), ctypes.c_void_p(stream)), "dc_attn_bwd")
    return dq, dk, dv, grads[0], grads[1]


def _unflatten(flat, identity):
    return DCTerms(identity=identity, **dict(zip(_GRAD_TERMS, flat)))


class _DCAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, meta, q, k, v, *flat):
        scaling, window, G, seq_lens, id_pre, id_post = meta
        pre = _unflatten(flat[:5], id_pre)
        post = _unflatten(flat[5:], id_post)
        ctx.meta = meta
        ctx.save_for_backward(q, k, v, *[t if t is not None else torch.empty(0) for t in flat])
        ctx.present = [t is not None for t in flat]
        return dc_attn_fwd(q, k, v, pre, post, scaling, window, G, seq_lens)

    @staticmethod
    def backward(ctx, dout):
        scaling, window, G, seq_lens, id_pre, id_post = ctx.meta
        q, k, v, *saved = ctx.saved_tensors
        flat = [t if ok else None for t, ok in zip(saved, ctx.present)]
        pre, post = _unflatten(flat[:5], id_pre), _unflatten(flat[5:], id_post)
        dq, dk, dv, gpre, gpost = dc_attn_bwd(dout.to(q.dtype), q, k, v, pre, post, scaling, window, G, seq_lens)
        out = []
        for gd, tm in ((gpre, pre), (gpost, post)):
            for n in _GRAD_TERMS:
                t = getattr(tm, n)
                out.append(None if t is None else gd[n].to(t.dtype))
        return (None, dq, dk.to(k.dtype), dv.to(v.dtype), *out)


def dc_attn(q, k, v, pre: Optional[DCTerms] = None, post: Optional[DCTerms] = None,
            scaling: Optional[float] = None, window: Optional[int] = None, G: int = 1,
            seq_lens: Optional[torch.Tensor] = None) -> torch.Tensor:
    """:func:`dc_attn_fwd` as a differentiable op: gradients flow to q, k, v and
    to the query-side term tensors (w, qw1, qw2, qdd, qmat) of both sets."""
    for tm in (pre, post):
        _check(tm is None or (tm.kw1 is None and tm.kw2 is None and tm.kdd is None),
               "dc_attn: key-wise terms (kw1, kw2, kdd) have no backward; use dc_attn_fwd")
    flat = []
    for tm in (pre, post):
        flat += [None if tm is None else getattr(tm, n) for n in _GRAD_TERMS]
    meta = (scaling, window, G, seq_lens, pre is None or pre.identity, post is None or post.identity)
    return _DCAttnFn.apply(meta, q, k, v, *flat)


class DCResidual:
    """The reference's ``TritonDCResidual`` (``triton_dc_residual.py:1432``):
    residual rank-1 DC attention over [B,T,N,D] tensors, all heads in one group
    (the reference class has no G)."""

    @staticmethod
    def alloc_buffers(q, window, store_qk=False, store_post_probs=False):
        """Only ``out`` is used; the reference's saved-state buffers are not
        needed by this backward (``triton_dc_residual.py:1436-1458``)."""
        return {"out": torch.empty_like(q)}

    @staticmethod
    def forward(q, k, v, dc_weights, scaling, window, seq_lens=None, *args, buffers=None, **kwargs):
        pw1, pw2, pdd, qw1, qw2, qdd = dc_weights
        out = buffers["out"] if buffers is not None and "out" in buffers else None
        return dc_attn_fwd(q, k, v, DCTerms.residual(pw1, pw2, pdd), DCTerms.residual(qw1, qw2, qdd),
                           scaling, min(int(window), q.shape[1]), 1, seq_lens, out)

    @staticmethod
    def backward(dout, q, k, v, dc_weights, scaling, window, s_buf=None, m_buf=None, l_buf=None,
                 a_buf=None, o_buf=None, seq_lens=None, *args, **kwargs):
        """Returns (dq, dk, dv, d_pre_w1, d_pre_w2, d_pre_dd, d_post_w1,
        d_post_w2, d_post_dd) like ``triton_dc_residual.py:1892``."""
        pw1, pw2, pdd, qw1, qw2, qdd = dc_weights
        dq, dk, dv, gp, gq = dc_attn_bwd(dout, q, k, v, DCTerms.residual(pw1, pw2, pdd),
                                         DCTerms.residual(qw1, qw2, qdd), scaling,
                                         min(int(window), q.shape[1]), 1, seq_lens)
        return (dq, dk, dv, gp["qw1"][..., 0], gp["qw2"][:, :, 0], gp["qdd"],
                gq["qw1"][..., 0], gq["qw2"][:, :, 0], gq["qdd"])


TritonDCResidual = DCResidual
