"""Backward kernel (``dc_attn_bwd``) against the reference's autograd gradients
(golden vectors from ``tests/golden/make_golden_grad.py``) and against the
float64 autograd oracle (``oracle/dc_oracle_torch.dc_attn_torch_grads``) on the
general query-side term family.  Calls go through the C ABI (ctypes)."""

import numpy as np
import pytest
import torch

import dc_triton_opt_b200 as dc
from oracle import dc_oracle as O
from oracle.dc_oracle_torch import dc_attn_torch_grads
from tests.golden_cases import WNAMES, load_grad_cases
from tests.tolerances import assert_grad_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _d(x, dt=torch.bfloat16):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to(DEV).to(dt)


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("case", load_grad_cases(), ids=lambda c: c.name)
def test_backward_matches_reference_autograd(case):
    q, k, v = _d(case.q), _d(case.k), _d(case.v)
    ws = [_d(w) for w in case.ws]
    dout = _d(case.dout_btnd)
    sl = None if case.seq_lens is None else torch.tensor(case.seq_lens, device=DEV)
    dq, dk, dv, gp, gq = dc.dc_attn_bwd(dout, q, k, v, dc.DCTerms.residual(*ws[:3]), dc.DCTerms.residual(*ws[3:]),
                                        case.scale, case.window, case.G, sl)
    torch.cuda.synchronize()
    got = {"dq": _np(dq), "dk": _np(dk), "dv": _np(dv),
           "d_pre_w1": _np(gp["qw1"][..., 0]), "d_pre_w2": _np(gp["qw2"][:, :, 0]), "d_pre_dd": _np(gp["qdd"]),
           "d_post_w1": _np(gq["qw1"][..., 0]), "d_post_w2": _np(gq["qw2"][:, :, 0]), "d_post_dd": _np(gq["qdd"])}
    for key, ref in case.grads.items():
        assert_grad_close(got[key], ref, f"{case.name} {key}")


def _inputs(B, T, H, G, R, seed, qmat=False, identity=False):
    q, k, v, pre, post = O.make_inputs(B, T, H, 128, G, R, seed=seed, terms=("w", "qw", "qdd"))
    rng = np.random.default_rng(seed + 1)
    for t in (pre, post):
        t.identity = identity
        if qmat:
            t.qmat = (0.05 * rng.standard_normal((B, T, H, H // G))).astype(np.float32)
    r = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).bfloat16().float().numpy()
    q, k, v = r(q), r(k), r(v)
    for t in (pre, post):
        for n in ("qw1", "qw2", "qdd", "qmat"):
            setattr(t, n, r(getattr(t, n)))
    dout = r(rng.standard_normal(q.shape).astype(np.float32))
    return q, k, v, pre, post, dout


def _terms(t):
    return dc.DCTerms(identity=t.identity, w=_d(t.w, torch.float32), qw1=_d(t.qw1), qw2=_d(t.qw2), qdd=_d(t.qdd),
                      qmat=_d(t.qmat))


@pytest.mark.parametrize("B,T,H,G,R,window,seq_lens,qmat", [
    (1, 70, 8, 2, 1, 24, None, False),     # HPG 4, ragged T
    (2, 64, 8, 8, 2, 16, [64, 37], False),  # HPG 1, rank 2, seq_lens
    (1, 90, 16, 8, 1, 40, None, True),     # HPG 2, per-query matrices
    (1, 48, 16, 2, 2, 20, None, True),     # HPG 8
    (1, 40, 32, 2, 1, 12, None, False),    # HPG 16
    (1, 36, 32, 1, 2, 10, None, True),     # HPG 32
    (1, 64, 8, 2, 1, None, None, False),   # full causal (short T)
    (1, 300, 8, 2, 1, 256, None, False),   # config-2 window
])
def test_backward_general_terms_vs_oracle(B, T, H, G, R, window, seq_lens, qmat):
    q, k, v, pre, post, dout = _inputs(B, T, H, G, R, seed=T + H + G, qmat=qmat)
    scale = 128 ** -0.5
    ref = dc_attn_torch_grads(q, k, v, pre, post, scale, window, G, seq_lens, dout)
    sl = None if seq_lens is None else torch.tensor(seq_lens, device=DEV)
    dq, dk, dv, gp, gq = dc.dc_attn_bwd(_d(dout), _d(q), _d(k), _d(v), _terms(pre), _terms(post), scale, window, G,
                                        sl)
    torch.cuda.synchronize()
    got = {"dq": _np(dq), "dk": _np(dk), "dv": _np(dv)}
    for name, gd in (("pre", gp), ("post", gq)):
        for n, t in gd.items():
            got[f"{name}_{n}"] = _np(t)
    assert set(got) == set(ref), (sorted(got), sorted(ref))
    for key in ref:
        assert_grad_close(got[key], ref[key], f"T{T} H{H} G{G} R{R} W{window} {key}")


def test_autograd_function_and_reference_class():
    """dc_attn is differentiable (gradients equal dc_attn_bwd's, in the input
    dtypes) and DCResidual mirrors TritonDCResidual's forward / backward."""
    case = load_grad_cases()[0]
    q, k, v = (_d(x).requires_grad_() for x in (case.q, case.k, case.v))
    ws = [_d(w).requires_grad_() for w in case.ws]
    pre, post = dc.DCTerms.residual(*ws[:3]), dc.DCTerms.residual(*ws[3:])
    out = dc.dc_attn(q, k, v, pre, post, case.scale, case.window, case.G)
    dout = _d(case.dout_btnd)
    out.backward(dout)
    dq, dk, dv, gp, gq = dc.dc_attn_bwd(dout, q.detach(), k.detach(), v.detach(), pre, post, case.scale,
                                        case.window, case.G)
    torch.cuda.synchronize()
    assert q.grad.dtype == torch.bfloat16 and ws[0].grad.dtype == torch.bfloat16
    assert torch.equal(q.grad, dq) and torch.equal(k.grad, dk.bfloat16()) and torch.equal(v.grad, dv.bfloat16())
    assert torch.equal(ws[2].grad, gp["qdd"].bfloat16())
    assert torch.equal(ws[3].grad, gq["qw1"][..., 0].bfloat16())
    # the reference class has no groups: all heads in one
    c = next(c for c in load_grad_cases() if c.G == 1)
    q, k, v = _d(c.q), _d(c.k), _d(c.v)
    ws = [_d(w) for w in c.ws]
    sl = None if c.seq_lens is None else torch.tensor(c.seq_lens, device=DEV, dtype=torch.int32)
    bufs = dc.DCResidual.alloc_buffers(q, c.window)
    out = dc.TritonDCResidual.forward(q, k, v, ws, c.scale, c.window, sl, buffers=bufs)
    assert out.data_ptr() == bufs["out"].data_ptr()
    grads = dc.TritonDCResidual.backward(_d(c.dout_btnd), q, k, v, ws, c.scale, c.window, seq_lens=sl)
    torch.cuda.synchronize()
    assert len(grads) == 9 and grads[0].dtype == torch.bfloat16 and grads[1].dtype == torch.float32
    for g, key in zip(grads, ["dq", "dk", "dv"] + [f"d_{n}" for n in WNAMES]):
        assert_grad_close(_np(g), c.grads[key], f"TritonDCResidual {key}")


def test_backward_rejects_keywise_terms():
    q = torch.zeros(1, 16, 8, 128, device=DEV, dtype=torch.bfloat16)
    kd = torch.zeros(1, 16, 8, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="key-wise"):
        dc.dc_attn_bwd(q, q, q, q, dc.DCTerms(kdd=kd), None, None, 8, 1)
