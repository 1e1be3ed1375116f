"""Drop-in for the reference's ``dc_hopper_cuda`` module
(``dc_hopper_cuda/__init__.py:22-141``, C++ ``dc_hopper_api.cpp:3-81``).

Same function names, positional arguments and return layout ([B,T,N,D]).  The
reference validates its inputs with ``TORCH_CHECK`` (``dc_hopper_kernel.cu:579-635``);
the same conditions raise ``RuntimeError`` here, with two deliberate
widenings: bf16 is accepted next to fp16, and any (chunk_size, window) pair is
accepted (the reference's scaffold only ran BM=32/W=224 and BM=16/W=240,
because its kernel had KL=256 compiled in; ``chunk_size`` never changes the
result).  The ``_ref``, ``_opt`` and ``_cluster`` variants were three kernel
experiments of the same function; here all three run the library's fastest
kernel for the call.
"""

from __future__ import annotations

import torch

from .api import DCTerms, dc_attn_fwd

N_HEADS, HEAD_DIM, GROUPS = 32, 128, 8  # fixed by the reference scaffold (dc_hopper_kernel.cu:16-25)


def _check_fixed_inputs(q, k, v, ws):
    names = ("q", "k", "v", "pre_w1", "pre_w2", "pre_dd", "post_w1", "post_w2", "post_dd")
    for n, t in zip(names, (q, k, v) + tuple(ws)):
        if not t.is_cuda:
            raise RuntimeError(f"{n} must be a CUDA tensor")
        if not t.is_contiguous():
            raise RuntimeError(f"{n} must be contiguous")
        if t.dtype not in (torch.float16, torch.bfloat16) or t.dtype != q.dtype:
            raise RuntimeError(f"{n} must be float16 (or bfloat16), matching q")
    if q.dim() != 4:
        raise RuntimeError("q must have shape [B, T, 32, 128]")
    if k.shape != q.shape:
        raise RuntimeError("k must match q shape")
    if v.shape != q.shape:
        raise RuntimeError("v must match q shape")
    if q.shape[2] != N_HEADS or q.shape[3] != HEAD_DIM:
        raise RuntimeError("only N=32,D=128 is supported")
    if ws[0].dim() != 3 or tuple(ws[0].shape) != tuple(q.shape[:3]):
        raise RuntimeError("pre_w1 must be [B,T,N]")
    for n, t in zip(names[4:], ws[1:]):
        if t.shape != ws[0].shape:
            raise RuntimeError(f"{n} must match pre_w1")


def _forward(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window):
    ws = (pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd)
    _check_fixed_inputs(q, k, v, ws)
    return dc_attn_fwd(q, k, v, DCTerms.residual(pre_w1, pre_w2, pre_dd),
                       DCTerms.residual(post_w1, post_w2, post_dd), float(scaling), int(window), GROUPS)


def forward_hpg4_bm32_ref(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window):
    """HPG=4 (G=8) residual DC forward, output [B,T,N,D] (``dc_hopper_cuda/__init__.py:22``)."""
    return _forward(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window)


def forward_hpg4_wide_ref(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window,
                          chunk_size):
    """HPG=4 (G=8) residual DC forward, output [B,T,N,D] (``dc_hopper_cuda/__init__.py:51``)."""
    return _forward(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window)


def forward_hpg4_wide_opt(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window,
                          chunk_size):
    """Same result as :func:`forward_hpg4_wide_ref` (``dc_hopper_cuda/__init__.py:81``)."""
    return _forward(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window)


def forward_hpg4_wide_cluster(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window,
                              chunk_size):
    """Same result as :func:`forward_hpg4_wide_ref` (``dc_hopper_cuda/__init__.py:111``)."""
    return _forward(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window)
