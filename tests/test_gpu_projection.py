"""Composition-weight producer (``dc_proj_weights``) against the oracle's
restatement (``oracle.dc_oracle.project_weights``).  Parity unpinned: the
reference project has no code for this step, which produces the weights its
DC-attention functions take as inputs."""

import numpy as np
import pytest
import torch

import dc_triton_opt_b200 as dc
from oracle import dc_oracle as O
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _inputs(lead, Dm, I, H, R, seed, dt):
    rng = np.random.default_rng(seed)
    r = lambda *s, std: torch.from_numpy((std * rng.standard_normal(s)).astype(np.float32)).to(DEV).to(dt)
    x = r(*lead, Dm, std=1.0)
    w1 = r(Dm, I, std=Dm ** -0.5)
    w2 = r(I, 8 * H * R, std=0.1 * I ** -0.5)
    wdd = r(Dm, 4 * H, std=0.1 * Dm ** -0.5)
    return x, w1, w2, wdd


@pytest.mark.parametrize("lead,Dm,I,H,R,dtype", [
    ((2, 100), 256, 64, 8, 1, torch.bfloat16),     # ragged M (200 tokens), mma.sync path (4H = 32)
    ((2, 100), 256, 64, 16, 1, torch.bfloat16),    # ragged M, tcgen05 path for both GEMMs (N 128, 128)
    ((1, 384), 512, 128, 32, 1, torch.float16),    # tcgen05 path, N 256 (x [W1 | Wdd]) and 256 (hidden W2)
    ((1, 300), 512, 128, 32, 2, torch.bfloat16),
    ((3, 64), 128, 32, 4, 2, torch.float16),
])
def test_projection_matches_oracle(lead, Dm, I, H, R, dtype):
    x, w1, w2, wdd = _inputs(lead, Dm, I, H, R, seed=Dm + H, dt=dtype)
    pre, post = dc.dc_proj_weights(x, w1, w2, wdd, H, R)
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy()
    rpre, rpost, _ = O.project_weights(f(x), f(w1), f(w2), f(wdd), H, R)
    for got, ref in ((pre, rpre), (post, rpost)):
        for n in ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd"):
            g, r = f(getattr(got, n)), getattr(ref, n)
            # weights rounded to the input dtype; the hidden activations too
            assert_close(g, r, n, max_abs=2e-2 * max(1.0, float(np.abs(r).max())), max_rel=2e-2)


def test_projection_feeds_the_forward():
    """The producer's outputs go straight into dc_attn_fwd (shapes and layout)."""
    B, T, H, D, G, R = 1, 128, 32, 128, 8, 1
    x, w1, w2, wdd = _inputs((B, T), 256, 64, H, R, seed=3, dt=torch.bfloat16)
    pre, post = dc.dc_proj_weights(x, w1, w2, wdd, H, R)
    q, k, v = (torch.randn(B, T, H, D, device=DEV).bfloat16() for _ in range(3))
    out = dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, 64, G)
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy()
    cv = lambda tm: O.Terms(identity=True, **{n: f(getattr(tm, n)) for n in ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd")})
    ref = O.dc_attn_oracle(f(q), f(k), f(v), cv(pre), cv(post), D ** -0.5, 64, G, None)
    assert_close(f(out), ref, "forward on produced weights")
