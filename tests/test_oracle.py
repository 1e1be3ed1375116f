"""Pin the CPU oracle against the reference's own golden vectors, and check the
algebraic reductions that cover the terms the reference has no code for."""

import numpy as np
import pytest

from oracle import dc_oracle as O
from tests.golden_cases import load_cases

CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_oracle_matches_reference_golden(case):
    got = O.dc_attn_oracle(case.q, case.k, case.v, case.pre, case.post, case.scale,
                           case.eff_window, case.G, case.seq_lens)
    ref = case.out_btnd
    assert got.shape == ref.shape
    # reference ran in fp32, the oracle in fp64 on the same inputs
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-5)


def test_grouped_wrapper_layout_and_defaults():
    c = next(c for c in CASES if c.name == "residual_defaults")
    got = O.grouped_residual(c.q, c.k, c.v, c.ws, c.scale, None, None, None, 1)
    np.testing.assert_allclose(got, c.out, atol=2e-5, rtol=0)


def test_oracle_independent_of_chunk():
    q, k, v, pre, post = O.make_inputs(1, 70, 8, 16, 2, 2, seed=3)
    a = O.dc_attn_oracle(q, k, v, pre, post, 0.25, 17, 2, None, chunk=64)
    b = O.dc_attn_oracle(q, k, v, pre, post, 0.25, 17, 2, None, chunk=7)
    np.testing.assert_allclose(a, b, atol=1e-12)


def test_keywise_terms_reduce_to_querywise_when_constant_over_keys():
    """kw1/kw2/kdd that do not depend on the key equal the same query-wise terms."""
    B, T, H, D, G, R = 1, 24, 4, 8, 1, 2
    q, k, v, _, _ = O.make_inputs(B, T, H, D, G, R, seed=4)
    rng = np.random.default_rng(5)
    c1 = rng.standard_normal((H, R)) * 0.2
    c2 = rng.standard_normal((R, H)) * 0.2
    cd = rng.standard_normal(H) * 0.2
    kw1 = np.broadcast_to(c1, (B, T, H, R)).copy()
    kw2 = np.broadcast_to(c2, (B, T, R, H)).copy()
    kdd = np.broadcast_to(cd, (B, T, H)).copy()
    kset = O.Terms(identity=True, kw1=kw1, kw2=kw2, kdd=kdd)
    qset = O.Terms(identity=True, qw1=kw1, qw2=kw2, qdd=kdd)
    a = O.dc_attn_oracle(q, k, v, kset, kset, 0.3, 9, G, None)
    b = O.dc_attn_oracle(q, k, v, qset, qset, 0.3, 9, G, None)
    np.testing.assert_allclose(a, b, atol=1e-12)


def test_keywise_terms_match_bruteforce_dense():
    """Dense T x T evaluation of the key-wise composition, pair by pair."""
    B, T, H, D, G, R = 1, 12, 4, 8, 2, 1
    q, k, v, pre, post = O.make_inputs(B, T, H, D, G, R, seed=6)
    W = 5
    got = O.dc_attn_oracle(q, k, v, pre, post, 0.3, W, G, None)
    hpg = H // G
    want = np.zeros_like(got)
    q64, k64, v64 = (x.astype(np.float64) for x in (q, k, v))

    def comp(tset, a, g, t, s):
        hs = slice(g * hpg, (g + 1) * hpg)
        o = np.zeros(hpg)
        for h in range(hpg):
            o[h] = sum(a[j] * tset.w[g, j, h] for j in range(hpg))
            for r in range(R):
                o[h] += tset.qw2[0, t, r, g * hpg + h] * sum(tset.qw1[0, t, g * hpg + j, r] * a[j] for j in range(hpg))
                o[h] += tset.kw2[0, s, r, g * hpg + h] * sum(tset.kw1[0, s, g * hpg + j, r] * a[j] for j in range(hpg))
            o[h] += (tset.qdd[0, t, g * hpg + h] + tset.kdd[0, s, g * hpg + h]) * a[h]
        return o

    for g in range(G):
        hs = range(g * hpg, (g + 1) * hpg)
        for t in range(T):
            keys = [s for s in range(T) if s <= t and t - s < W]
            S = np.array([comp(pre, np.array([0.3 * q64[0, t, h] @ k64[0, s, h] for h in hs]), g, t, s)
                          for s in keys])  # [nk, hpg]
            P = np.exp(S - S.max(0))
            P /= P.sum(0)
            Pp = np.array([comp(post, P[i], g, t, s) for i, s in enumerate(keys)])
            for j, h in enumerate(hs):
                want[0, t, h] = sum(Pp[i, j] * v64[0, s, h] for i, s in enumerate(keys))
    np.testing.assert_allclose(got, want, atol=1e-7)


def test_fully_masked_rows_are_zero():
    q, k, v, pre, post = O.make_inputs(1, 16, 4, 8, 1, 1, seed=7)
    got = O.dc_attn_oracle(q, k, v, pre, post, 0.3, 4, 1, np.array([3], np.int32))
    # queries t >= 3 + 4 - 1 see no key < seq_len=3
    assert np.all(got[0, 6:] == 0)
    assert np.all(np.isfinite(got))


def test_torch_cpu_port_matches_numpy_oracle():
    from oracle.dc_oracle_torch import dc_attn_torch_cpu
    q, k, v, pre, post = O.make_inputs(2, 90, 8, 32, 2, 2, seed=9)
    for window in (17, None):
        a = O.dc_attn_oracle(q, k, v, pre, post, 0.2, window, 2, [90, 50])
        b = dc_attn_torch_cpu(q, k, v, pre, post, 0.2, window, 2, [90, 50], chunk=32).numpy()
        np.testing.assert_allclose(a, b, atol=2e-5, rtol=0)


# ---------------------------------------------------------------- backward oracle

from oracle.dc_oracle_torch import dc_attn_torch_grads  # noqa: E402
from tests.golden_cases import load_grad_cases  # noqa: E402


def _oracle_grads(c):
    pre, post = O.residual_terms(*c.ws[:3]), O.residual_terms(*c.ws[3:])
    g = dc_attn_torch_grads(c.q, c.k, c.v, pre, post, c.scale, c.window, c.G, c.seq_lens, c.dout_btnd)
    # the residual weights are [B,T,N] views of the rank-1 factors [B,T,N,1] / [B,T,1,N]
    return {"dq": g["dq"], "dk": g["dk"], "dv": g["dv"],
            "d_pre_w1": g["pre_qw1"][..., 0], "d_pre_w2": g["pre_qw2"][:, :, 0], "d_pre_dd": g["pre_qdd"],
            "d_post_w1": g["post_qw1"][..., 0], "d_post_w2": g["post_qw2"][:, :, 0], "d_post_dd": g["post_qdd"]}


@pytest.mark.parametrize("case", load_grad_cases(), ids=lambda c: c.name)
def test_backward_oracle_matches_reference_autograd(case):
    """The float64 autograd oracle against autograd through the reference's own
    torch function (fp32) on the same inputs and output gradient."""
    got = _oracle_grads(case)
    for k, ref in case.grads.items():
        scale = max(float(np.abs(ref).max()), 1e-6)
        np.testing.assert_allclose(got[k], ref, rtol=0, atol=2e-5 * max(1.0, scale), err_msg=k)


def _tiny_grad_case(seed=0):
    B, T, H, D, G, R = 1, 12, 4, 8, 2, 2
    q, k, v, pre, post = O.make_inputs(B, T, H, D, G, R, seed=seed, terms=("w", "qw", "qdd"))
    rng = np.random.default_rng(seed + 1)
    for t in (pre, post):
        t.qmat = (0.1 * rng.standard_normal((B, T, H, H // G))).astype(np.float64)
    dout = rng.standard_normal(q.shape)
    return q, k, v, pre, post, dout, G


def test_backward_oracle_matches_finite_differences():
    """The float64 autograd gradients of the terms the reference cannot pin
    (static mix w, rank-2 factors, qmat) against central finite differences."""
    from oracle.dc_oracle_torch import _forward
    import torch
    q, k, v, pre, post, dout, G = _tiny_grad_case()
    scale, W = 8 ** -0.5, 5
    g = dc_attn_torch_grads(q, k, v, pre, post, scale, W, G, None, dout)

    def loss():
        out = _forward(q, k, v, pre, post, scale, W, G, None, 256, None, torch.float64)
        return float((out.numpy() * dout).sum())

    rng = np.random.default_rng(3)
    for name, tm in (("pre", pre), ("post", post)):
        for n in ("w", "qw1", "qw2", "qdd", "qmat"):
            a = getattr(tm, n).astype(np.float64)
            setattr(tm, n, a)
            for _ in range(3):
                idx = tuple(rng.integers(0, s) for s in a.shape)
                old = a[idx]
                a[idx] = old + 1e-5
                lp = loss()
                a[idx] = old - 1e-5
                lm = loss()
                a[idx] = old
                fd = (lp - lm) / 2e-5
                assert abs(fd - g[f"{name}_{n}"][idx]) <= 1e-6 + 1e-5 * abs(fd), (name, n, idx, fd)


def test_backward_oracle_static_mix_grad_is_sum_of_qmat_grads():
    """M_t = w + qmat_t^T inside a group, so dL/dw[g, h', h] equals the sum over
    tokens of dL/dqmat[b, t, g*HPG + h, h']."""
    q, k, v, pre, post, dout, G = _tiny_grad_case(seed=5)
    g = dc_attn_torch_grads(q, k, v, pre, post, 8 ** -0.5, 5, G, None, dout)
    hpg = q.shape[2] // G
    for name in ("pre", "post"):
        dq = g[f"{name}_qmat"].sum(axis=(0, 1))            # [H, HPG]: (h, h')
        want = dq.reshape(G, hpg, hpg).transpose(0, 2, 1)   # [G, h', h]
        np.testing.assert_allclose(g[f"{name}_w"], want, atol=1e-10, rtol=1e-8)
