"""Torch-CPU restatement of the DC-attention forward (TEST/BASELINE INFRASTRUCTURE ONLY).

Same algorithm and term set as :mod:`oracle.dc_oracle` (numpy, float64), written
the way the reference writes it — chunked einsum in fp32 on torch CPU
(``dc_attention_torch.py:159-258``) — so that it runs on all host cores.  It is
the timed CPU baseline of ``bench.py`` (``cpu_baseline`` and ``--impl
reference``); the reference's own module cannot be imported on the GPU host.
Tests check it against the numpy oracle, which is itself pinned to the
reference's golden vectors.
"""

from __future__ import annotations

from typing import Optional

import torch

from .dc_oracle import Terms


def _t(x):
    if x is None:
        return None
    return x if isinstance(x, torch.Tensor) else torch.from_numpy(x)


def _compose(a, tm: Terms, b, hs, g, tq, sk):
    out = a.clone() if tm.identity else torch.zeros_like(a)
    if tm.w is not None:
        out += torch.einsum("hts,hk->kts", a, _t(tm.w)[g].float())
    if tm.qw1 is not None:
        agg = torch.einsum("hts,thr->rts", a, _t(tm.qw1)[b, tq, hs, :].float())
        out += torch.einsum("rts,trh->hts", agg, _t(tm.qw2)[b, tq, :, hs].float())
    if tm.kw1 is not None:
        agg = torch.einsum("hts,shr->rts", a, _t(tm.kw1)[b, sk, hs, :].float())
        out += torch.einsum("rts,srh->hts", agg, _t(tm.kw2)[b, sk, :, hs].float())
    if tm.qdd is not None:
        out += a * _t(tm.qdd)[b, tq, hs].float().T[:, :, None]
    if tm.kdd is not None:
        out += a * _t(tm.kdd)[b, sk, hs].float().T[:, None, :]
    if tm.qmat is not None:
        out += torch.einsum("tij,jts->its", _t(tm.qmat)[b, tq, hs, :].float(), a)
    return out


@torch.no_grad()
def dc_attn_torch_cpu(q, k, v, pre: Terms, post: Terms, scale: float, window: Optional[int],
                      G: int = 1, seq_lens=None, chunk: int = 256, t_range=None) -> torch.Tensor:
    """fp32 torch-CPU forward; returns [B,T,H,D] (rows outside ``t_range`` are 0)."""
    q, k, v = (_t(x).float() for x in (q, k, v))
    B, T, H, D = q.shape
    hpg = H // G
    out = torch.zeros(B, T, H, D)
    ta, tb = (0, T) if t_range is None else t_range
    for b in range(B):
        slen = T if seq_lens is None else int(seq_lens[b])
        for g in range(G):
            hs = slice(g * hpg, (g + 1) * hpg)
            for t0 in range(ta, tb, chunk):
                t1 = min(t0 + chunk, tb)
                k0 = 0 if window is None else max(0, t0 - int(window) + 1)
                tq, sk = slice(t0, t1), slice(k0, t1)
                L = torch.einsum("thd,shd->hts", q[b, tq, hs], k[b, sk, hs]) * scale
                S = _compose(L, pre, b, hs, g, tq, sk)
                ti = torch.arange(t0, t1)[:, None]
                si = torch.arange(k0, t1)[None, :]
                valid = (si <= ti) & (si < slen)
                if window is not None:
                    valid &= (ti - si) < int(window)
                S = S.masked_fill(~valid[None], float("-inf"))
                P = torch.nan_to_num(torch.softmax(S, dim=-1), nan=0.0)
                Pp = _compose(P, post, b, hs, g, tq, sk)
                out[b, tq, hs] = torch.einsum("hts,shd->thd", Pp, v[b, sk, hs])
    return out
