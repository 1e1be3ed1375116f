"""CPU oracle for the DC-attention forward (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The CUDA path in ``dc_triton_opt_b200``
never calls into it and fails loudly when its extension is missing.

It restates, in numpy (float64 accumulation), the algorithm of the reference
project Lisennlp/dc_triton_opt:

* ``dc_attention_torch.py:159-258`` (``dc_attention_window_chunked_residual_grouped``):
  per head group, per query chunk, logits = scale * Q K^T (``:214``), residual
  rank-1 pre-composition (``:217-225``), causal & window & seq_len mask after
  composition (``:228-235``), softmax with NaN -> 0 for empty rows (``:236-237``),
  residual rank-1 post-composition on the probabilities (``:240-248``), P'V (``:251``).
* ``dc_attention_torch.py:88-156`` (the G=1 special case of the above).
* ``dc_attention_torch.py:22-84`` (``dc_attention_decomposed_window_chunked``):
  a per-query N x N mixing matrix applied to logits and probabilities
  (``mixed[i] = sum_j pre_w[b,t,i,j] * L[j]``, ``:59-61`` / ``:76-78``).

and generalises them to the composition family of DCFormer (Xiao et al.,
"Improving Transformers with Dynamically Composable Multi-Head Attention",
ICML 2024), which is the superset the build targets.  For one (b, t, s) pair
and the HPG heads of one group, with ``a`` the vector of per-head logits (pre)
or probabilities (post), the composed vector is

    a'[h] =  [identity] a[h]
           + sum_h' a[h'] * w[g, h', h]                       (static mix)
           + sum_r qw2[b,t,r,h] * sum_h' qw1[b,t,h',r] a[h']  (query-wise rank R)
           + sum_r kw2[b,s,r,h] * sum_h' kw1[b,s,h',r] a[h']  (key-wise rank R)
           + (qdd[b,t,h] + kdd[b,s,h]) * a[h]                 (diagonal gates)
           + sum_j qmat[b,t,h,j] * a[j]                       (per-query matrix)

With identity=True, w=None, R=1 (qw1=pre_w1[...,None], qw2=pre_w2[:,:,None,:]),
qdd=pre_dd and no key-wise terms this is exactly the reference's residual
form; with identity=False and qmat=pre_w it is the reference's decomposed form.

Window convention (``dc_attention_torch.py:230-234``): key s is visible from
query t iff s <= t, t - s < window and s < seq_lens[b].  ``window=None`` in
:func:`dc_attn_oracle` means full causal.  Queries t >= seq_lens[b] are still
computed (the reference only masks keys), exactly as the torch reference does.

Parity status: the residual rank-1 subset and the per-query-matrix form are
pinned by golden vectors produced by the reference's own torch functions
(``tests/golden/make_golden.py``).  The static mix and query-wise rank-R
terms are pinned through the decomposed form (a per-query matrix
``blockdiag(w^T + qw2 (x) qw1 + diag(qdd))``).  The key-wise terms have no
counterpart in the reference ("parity unpinned"); they are checked by
algebraic reduction tests instead.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

TERM_NAMES = ("w", "qw1", "qw2", "kw1", "kw2", "qdd", "kdd", "qmat")


@dataclass
class Terms:
    """One composition term set (pre or post).  Arrays are numpy, any float dtype.

    Shapes: w [G,HPG,HPG]; qw1/kw1 [B,T,H,R]; qw2/kw2 [B,T,R,H];
    qdd/kdd [B,T,H]; qmat [B,T,H,HPG] (row h mixes the HPG heads of h's group).
    """

    identity: bool = True
    w: Optional[np.ndarray] = None
    qw1: Optional[np.ndarray] = None
    qw2: Optional[np.ndarray] = None
    kw1: Optional[np.ndarray] = None
    kw2: Optional[np.ndarray] = None
    qdd: Optional[np.ndarray] = None
    kdd: Optional[np.ndarray] = None
    qmat: Optional[np.ndarray] = None
    extra: dict = field(default_factory=dict)


def _f(x):
    return None if x is None else np.asarray(x, dtype=np.float64)


def compose(a, t: Terms, b: int, g: int, hpg: int, tq: slice, sk: slice):
    """Apply one term set to a[h, t, s] (heads of group g, query range tq, key range sk).

    Restates the composition of ``dc_attention_torch.py:217-225`` (pre) and
    ``:240-248`` (post), generalised as described in the module docstring.
    """
    hs = slice(g * hpg, (g + 1) * hpg)
    out = a.copy() if t.identity else np.zeros_like(a)
    if t.w is not None:
        out += np.einsum("hts,hk->kts", a, _f(t.w)[g])
    if t.qw1 is not None:
        agg = np.einsum("hts,thr->rts", a, _f(t.qw1)[b, tq, hs, :])
        out += np.einsum("rts,trh->hts", agg, _f(t.qw2)[b, tq, :, hs])
    if t.kw1 is not None:
        agg = np.einsum("hts,shr->rts", a, _f(t.kw1)[b, sk, hs, :])
        out += np.einsum("rts,srh->hts", agg, _f(t.kw2)[b, sk, :, hs])
    if t.qdd is not None:
        out += a * _f(t.qdd)[b, tq, hs].T[:, :, None]
    if t.kdd is not None:
        out += a * _f(t.kdd)[b, sk, hs].T[:, None, :]
    if t.qmat is not None:
        out += np.einsum("tij,jts->its", _f(t.qmat)[b, tq, hs, :], a)
    return out


def dc_attn_oracle(q, k, v, pre: Terms, post: Terms, scale: float,
                   window: Optional[int], G: int = 1, seq_lens=None,
                   chunk: int = 64) -> np.ndarray:
    """General DC-attention forward.  q,k,v [B,T,H,D] -> out [B,T,H,D] (float64).

    ``window=None`` means full causal.  ``chunk`` only bounds memory; the mask
    is exact so the result does not depend on it (as in the reference,
    ``dc_attention_torch.py:204-206``).
    """
    q = _f(q); k = _f(k); v = _f(v)
    B, T, H, D = q.shape
    assert H % G == 0, "H must be divisible by G"
    hpg = H // G
    out = np.zeros((B, T, H, D), dtype=np.float64)
    for b in range(B):
        slen = T if seq_lens is None else int(seq_lens[b])
        for g in range(G):
            hs = slice(g * hpg, (g + 1) * hpg)
            for t0 in range(0, T, chunk):
                t1 = min(t0 + chunk, T)
                k0 = 0 if window is None else max(0, t0 - int(window) + 1)
                tq, sk = slice(t0, t1), slice(k0, t1)
                L = np.einsum("thd,shd->hts", q[b, tq, hs], k[b, sk, hs]) * scale
                S = compose(L, pre, b, g, hpg, tq, sk)
                ti = np.arange(t0, t1)[:, None]
                si = np.arange(k0, t1)[None, :]
                valid = (si <= ti) & (si < slen)
                if window is not None:
                    valid &= (ti - si) < int(window)
                S = np.where(valid[None], S, -np.inf)
                m = S.max(axis=-1, keepdims=True)
                m = np.where(np.isfinite(m), m, 0.0)
                e = np.where(valid[None], np.exp(S - m), 0.0)
                l = e.sum(axis=-1, keepdims=True)
                P = e / np.where(l > 0, l, 1.0)
                Pp = compose(P, post, b, g, hpg, tq, sk)
                out[b, tq, hs] = np.einsum("hts,shd->thd", Pp, v[b, sk, hs])
    return out


def residual_terms(w1, w2, dd) -> Terms:
    """The reference's residual rank-1 term set from three [B,T,N] tensors."""
    w1 = _f(w1); w2 = _f(w2); dd = _f(dd)
    return Terms(identity=True, qw1=w1[..., None], qw2=w2[:, :, None, :], qdd=dd)


def grouped_residual(q, k, v, dc_weights, scaling, window=None, seq_lens=None,
                     chunk_size=None, G=1):
    """Oracle twin of ``dc_attention_window_chunked_residual_grouped``
    (``dc_attention_torch.py:159-186``): same defaults (window 256), same output
    layout [B,N,T,D]."""
    pw1, pw2, pdd, qw1, qw2, qdd = dc_weights
    if window is None:
        window = 256
    out = dc_attn_oracle(q, k, v, residual_terms(pw1, pw2, pdd),
                         residual_terms(qw1, qw2, qdd), scaling, window, G, seq_lens)
    return out.transpose(0, 2, 1, 3)


def decomposed(q, k, v, pre_w, post_w, scaling, window, seq_lens):
    """Oracle twin of ``dc_attention_decomposed_window_chunked``
    (``dc_attention_torch.py:22-84``): per-query N x N mix, output [B,T,N,D]."""
    return dc_attn_oracle(q, k, v, Terms(identity=False, qmat=pre_w),
                          Terms(identity=False, qmat=post_w), scaling,
                          max(1, int(window)), 1, seq_lens)


def make_inputs(B, T, H, D, G, R, seed=0, wstd=0.1, mix_std=0.02,
                terms=("w", "qw", "kw", "qdd", "kdd"), dtype=np.float32):
    """Seeded synthetic inputs with the BASELINE distributions:
    q,k,v ~ N(0,1); w = I + N(0, mix_std); qw*, kw*, qdd, kdd ~ N(0, wstd);
    separate pre and post sets."""
    rng = np.random.default_rng(seed)
    hpg = H // G
    q = rng.standard_normal((B, T, H, D)).astype(dtype)
    k = rng.standard_normal((B, T, H, D)).astype(dtype)
    v = rng.standard_normal((B, T, H, D)).astype(dtype)
    sets = []
    for _ in range(2):
        t = Terms(identity=False)
        if "w" in terms:
            t.w = (np.eye(hpg)[None] + mix_std * rng.standard_normal((G, hpg, hpg))).astype(np.float32)
        else:
            t.identity = True
        if "qw" in terms and R > 0:
            t.qw1 = (wstd * rng.standard_normal((B, T, H, R))).astype(dtype)
            t.qw2 = (wstd * rng.standard_normal((B, T, R, H))).astype(dtype)
        if "kw" in terms and R > 0:
            t.kw1 = (wstd * rng.standard_normal((B, T, H, R))).astype(dtype)
            t.kw2 = (wstd * rng.standard_normal((B, T, R, H))).astype(dtype)
        if "qdd" in terms:
            t.qdd = (wstd * rng.standard_normal((B, T, H))).astype(dtype)
        if "kdd" in terms:
            t.kdd = (wstd * rng.standard_normal((B, T, H))).astype(dtype)
        sets.append(t)
    return q, k, v, sets[0], sets[1]


def pairs(T: int, window: Optional[int]) -> int:
    """Number of visible (t, s) pairs per (b, h): T*W - W(W-1)/2, or T(T+1)/2."""
    if window is None or window >= T:
        return T * (T + 1) // 2
    return T * window - window * (window - 1) // 2


def project_weights(x, w1, w2, wdd, H: int, R: int):
    """Composition-weight producer (TEST INFRASTRUCTURE; parity unpinned: the
    reference project has no code for this step).  Restates the DCFormer
    dynamic weight projection (Xiao et al., ICML 2024) as built here:
    hidden = gelu(x W1) (erf form), dw = hidden W2, dd = tanh(x Wdd), with the
    column order of include/dc_attn.h (dc_proj_params).  x [..., Dm]; returns
    (pre, post) Terms with qw1/kw1 [..., H, R], qw2/kw2 [..., R, H], qdd/kdd
    [..., H], plus the float64 hidden activations."""
    from math import erf, sqrt
    x = _f(x)
    h = x @ _f(w1)
    verf = np.vectorize(erf)
    hidden = 0.5 * h * (1.0 + verf(h / sqrt(2.0)))
    dw = hidden @ _f(w2)
    dd = np.tanh(x @ _f(wdd))
    lead = x.shape[:-1]
    HR = H * R
    sets = []
    for s in range(2):
        c = dw[..., s * 4 * HR:(s + 1) * 4 * HR]
        t = Terms(identity=True,
                  qw1=c[..., 0:HR].reshape(*lead, H, R), qw2=c[..., HR:2 * HR].reshape(*lead, R, H),
                  kw1=c[..., 2 * HR:3 * HR].reshape(*lead, H, R), kw2=c[..., 3 * HR:4 * HR].reshape(*lead, R, H),
                  qdd=dd[..., (2 * s) * H:(2 * s + 1) * H], kdd=dd[..., (2 * s + 1) * H:(2 * s + 2) * H])
        sets.append(t)
    return sets[0], sets[1], hidden
