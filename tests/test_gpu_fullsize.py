"""BASELINE full sizes, checked through size-independent properties.

The fp64 oracle cannot evaluate a B16 T4096 layer in test time, but two
properties of the operator let the full-size device result be checked against
it row by row:

* window locality: with a causal window W, output rows [t0, t1) depend only
  on the tokens [t0 - W + 1, t1) (keys, per-key weights) and on the rows'
  own queries and per-query weights, so the oracle run on that slice alone
  must give the same rows;
* causal prefix: in a full-causal layer rows [0, t1) depend only on tokens
  [0, t1);

plus batch independence (the multi-GPU partition): the full batch must equal
its slices computed separately, bit for bit.
"""

import numpy as np
import pytest
import torch

import dc_triton_opt_b200 as dc
from oracle import dc_oracle as O
from tests.tolerances import assert_close

DEV = "cuda:0"
pytestmark = pytest.mark.gpu
PER_TOKEN = ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _inputs(B, T, H, D, G, R, seed):
    """BASELINE distributions, generated on the device (bf16 inputs, fp32 static mix)."""
    gen = torch.Generator(device=DEV).manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=gen, device=DEV)
    bf = torch.bfloat16
    hpg = H // G
    q, k, v = (rn(B, T, H, D).to(bf) for _ in range(3))
    sets = []
    for _ in range(2):
        sets.append(dc.DCTerms(identity=False, w=torch.eye(hpg, device=DEV)[None] + 0.02 * rn(G, hpg, hpg),
                               qw1=(0.1 * rn(B, T, H, R)).to(bf), qw2=(0.1 * rn(B, T, R, H)).to(bf),
                               kw1=(0.1 * rn(B, T, H, R)).to(bf), kw2=(0.1 * rn(B, T, R, H)).to(bf),
                               qdd=(0.1 * rn(B, T, H)).to(bf), kdd=(0.1 * rn(B, T, H)).to(bf)))
    return q, k, v, sets[0], sets[1]


def _np(t):
    return t.float().cpu().numpy()


def _oracle_rows(q, k, v, pre, post, b, a, t0, t1, window, G):
    """Oracle on batch b's tokens [a, t1); returns its rows [t0, t1)."""
    def terms(tm):
        r = O.Terms(identity=tm.identity, w=tm.w.float().cpu().numpy())
        for f in PER_TOKEN:
            setattr(r, f, _np(getattr(tm, f)[b:b + 1, a:t1]))
        return r
    ref = O.dc_attn_oracle(_np(q[b:b + 1, a:t1]), _np(k[b:b + 1, a:t1]), _np(v[b:b + 1, a:t1]), terms(pre),
                           terms(post), q.shape[-1] ** -0.5, window, G)
    return ref[0, t0 - a:]


@pytest.mark.parametrize("G", [8, 1, 2, 4, 16, 32])
def test_config1_full_size_window_locality(G):
    """config1 (B16 T4096 H32 D128 W128 R1, every term) over the G sweep
    (persistent TC kernel for G >= 4, tensor-core-mix kernel for G <= 2):
    rows at the sequence start, in the middle and at the end of the last
    batch against the oracle on their key windows."""
    B, T, H, D, R, W = 16, 4096, 32, 128, 1, 128
    q, k, v, pre, post = _inputs(B, T, H, D, G, R, seed=100 + G)
    out = dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, W, G)
    torch.cuda.synchronize()
    for b, t0, t1 in ((0, 0, 64), (7, 2000, 2064), (15, 4032, 4096)):
        a = max(0, t0 - W + 1)
        ref = _oracle_rows(q, k, v, pre, post, b, a, t0, t1, W, G)
        assert_close(_np(out[b, t0:t1]), ref, f"config1 G{G} b{b} rows [{t0},{t1})")


@pytest.mark.parametrize("G", [1, 4, 32])
def test_config2_full_size_window_locality(G):
    """config2 (W256 R2) at its G values: 3-key-tile spans (single-pass TC
    kernel for G 4 and 32, tensor-core-mix kernel for G 1)."""
    B, T, H, D, R, W = 16, 4096, 32, 128, 2, 256
    q, k, v, pre, post = _inputs(B, T, H, D, G, R, seed=200 + G)
    out = dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, W, G)
    torch.cuda.synchronize()
    for b, t0, t1 in ((3, 100, 164), (15, 4040, 4096)):
        a = max(0, t0 - W + 1)
        ref = _oracle_rows(q, k, v, pre, post, b, a, t0, t1, W, G)
        assert_close(_np(out[b, t0:t1]), ref, f"config2 G{G} b{b} rows [{t0},{t1})")


def test_config3_full_size_causal_prefix():
    """config3 (full causal, B4 T4096 G4 R2): rows of the last batch's first
    512 tokens against the oracle on that prefix."""
    B, T, H, D, G, R = 4, 4096, 32, 128, 4, 2
    q, k, v, pre, post = _inputs(B, T, H, D, G, R, seed=301)
    out = dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, None, G)
    torch.cuda.synchronize()
    ref = _oracle_rows(q, k, v, pre, post, 3, 0, 0, 512, None, G)
    for t0, t1 in ((0, 64), (448, 512)):
        assert_close(_np(out[3, t0:t1]), ref[t0:t1], f"config3 b3 rows [{t0},{t1})")


@pytest.mark.parametrize("G", [8, 1])
def test_config1_full_size_batch_shards_are_exact(G):
    """The full batch equals its two halves computed separately, bit for bit
    (the batch partition of the multi-GPU runs)."""
    B, T, H, D, R, W = 16, 4096, 32, 128, 1, 128
    q, k, v, pre, post = _inputs(B, T, H, D, G, R, seed=400 + G)
    full = dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, W, G)

    def half(tm, b0, b1):
        return dc.DCTerms(identity=tm.identity, w=tm.w, **{f: getattr(tm, f)[b0:b1] for f in PER_TOKEN})

    for b0, b1 in ((0, 7), (7, 16)):
        part = dc.dc_attn_fwd(q[b0:b1], k[b0:b1], v[b0:b1], half(pre, b0, b1), half(post, b0, b1), D ** -0.5, W, G)
        torch.cuda.synchronize()
        assert torch.equal(part, full[b0:b1]), f"G{G} batch slice [{b0},{b1}) differs"


def test_config4_full_size_window_locality_and_shard():
    """config4 (B64 T8192 W256 G1 R2, the multi-GPU scaling layer) on one GPU:
    rows at both ends of the sequence against the oracle on their windows, and
    the rank-3-of-8 batch shard equal to the same rows of the full batch."""
    B, T, H, D, G, R, W = 64, 8192, 32, 128, 1, 2, 256
    q, k, v, pre, post = _inputs(B, T, H, D, G, R, seed=501)
    out = dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, W, G)
    torch.cuda.synchronize()
    for b, t0, t1 in ((0, 0, 32), (63, 8160, 8192)):
        a = max(0, t0 - W + 1)
        ref = _oracle_rows(q, k, v, pre, post, b, a, t0, t1, W, G)
        assert_close(_np(out[b, t0:t1]), ref, f"config4 b{b} rows [{t0},{t1})")
    b0, b1 = 24, 32
    part = dc.dc_attn_fwd(q[b0:b1], k[b0:b1], v[b0:b1],
                          dc.DCTerms(identity=pre.identity, w=pre.w, **{f: getattr(pre, f)[b0:b1] for f in PER_TOKEN}),
                          dc.DCTerms(identity=post.identity, w=post.w, **{f: getattr(post, f)[b0:b1] for f in PER_TOKEN}),
                          D ** -0.5, W, G)
    torch.cuda.synchronize()
    assert torch.equal(part, out[b0:b1])
