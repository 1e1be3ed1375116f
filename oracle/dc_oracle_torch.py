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
    f = lambda x: _t(x).to(a.dtype)
    out = a.clone() if tm.identity else torch.zeros_like(a)
    if tm.w is not None:
        out = out + torch.einsum("hts,hk->kts", a, f(tm.w)[g])
    if tm.qw1 is not None:
        agg = torch.einsum("hts,thr->rts", a, f(tm.qw1)[b, tq, hs, :])
        out = out + torch.einsum("rts,trh->hts", agg, f(tm.qw2)[b, tq, :, hs])
    if tm.kw1 is not None:
        agg = torch.einsum("hts,shr->rts", a, f(tm.kw1)[b, sk, hs, :])
        out = out + torch.einsum("rts,srh->hts", agg, f(tm.kw2)[b, sk, :, hs])
    if tm.qdd is not None:
        out = out + a * f(tm.qdd)[b, tq, hs].T[:, :, None]
    if tm.kdd is not None:
        out = out + a * f(tm.kdd)[b, sk, hs].T[:, None, :]
    if tm.qmat is not None:
        out = out + torch.einsum("tij,jts->its", f(tm.qmat)[b, tq, hs, :], a)
    return out


@torch.no_grad()
def dc_attn_torch_cpu(q, k, v, pre: Terms, post: Terms, scale: float, window: Optional[int],
                      G: int = 1, seq_lens=None, chunk: int = 256, t_range=None) -> torch.Tensor:
    """fp32 torch-CPU forward; returns [B,T,H,D] (rows outside ``t_range`` are 0)."""
    return _forward(q, k, v, pre, post, scale, window, G, seq_lens, chunk, t_range, torch.float32)


GRAD_TERMS = ("w", "qw1", "qw2", "qdd", "qmat")


def dc_attn_torch_grads(q, k, v, pre: Terms, post: Terms, scale: float, window: Optional[int], G: int,
                        seq_lens, dout, chunk: int = 256):
    """Gradients of sum(out * dout) by torch autograd through the float64
    forward (the backward's checker): a dict with dq, dk, dv and, per set
    ("pre", "post"), the gradient of each query-side term present
    (``GRAD_TERMS``), as numpy arrays."""
    leaf = lambda x: torch.tensor(x, dtype=torch.float64, requires_grad=True)
    qt, kt, vt = leaf(q), leaf(k), leaf(v)
    sets, leaves = [], {}
    for name, tm in (("pre", pre), ("post", post)):
        r = Terms(identity=tm.identity, kw1=tm.kw1, kw2=tm.kw2, kdd=tm.kdd)
        for n in GRAD_TERMS:
            if getattr(tm, n) is not None:
                leaves[(name, n)] = leaf(getattr(tm, n))
                setattr(r, n, leaves[(name, n)])
        sets.append(r)
    with torch.enable_grad():
        out = _forward(qt, kt, vt, sets[0], sets[1], scale, window, G, seq_lens, chunk, None, torch.float64)
        (out * torch.as_tensor(dout, dtype=torch.float64)).sum().backward()
    res = {"dq": qt.grad.numpy(), "dk": kt.grad.numpy(), "dv": vt.grad.numpy()}
    for (name, n), t in leaves.items():
        res[f"{name}_{n}"] = t.grad.numpy()
    return res


def _forward(q, k, v, pre: Terms, post: Terms, scale, window, G, seq_lens, chunk, t_range, dtype):
    q, k, v = (_t(x).to(dtype) for x in (q, k, v))
    B, T, H, D = q.shape
    hpg = H // G
    out = torch.zeros(B, T, H, D, dtype=dtype)
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
