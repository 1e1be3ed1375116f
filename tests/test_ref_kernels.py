"""The reference's own CUDA kernels, built for sm_100a from its sources by
``oracle/build_ref.py``, against the oracle and against this library.

They are the same-box comparator of ``bench.py``'s ``repo_best`` block, so
before their times mean anything their outputs must be right on a B200:

* ``dc_fused_cuda.onekernel_v4_forward`` (``dc_fused_cuda/kernel.cu:1350-1431``,
  the CUDA port of the one-kernel V4): fp16, N 32, D 128, G 4 or 8,
  chunk 16/32, BM+W <= 128;
* ``_dc_hopper_cuda.forward_hpg4_wide_opt`` (WMMA, BM16 W240) and
  ``forward_hpg4_wide_ref`` (scalar, BM32 W224 and BM16 W240)
  (``dc_hopper_kernel.cu:639-760``), G 8.

The reference's own gate applies to them (``test_dc_hopper_cuda.py:123-124``:
max <= 1.2e-1, mean <= 1e-3; 2e-1 / 2e-3 for the opt kernel); this library is
held to its own, tighter tolerance against the oracle on the same inputs.
Skipped where the modules were not built (no reference checkout at build time).
"""

import numpy as np
import pytest
import torch

import dc_triton_opt_b200 as dc
from oracle import dc_oracle as O
from oracle.build_ref import built, import_module
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(B, T, seed):
    rng = np.random.default_rng(seed)
    q, k, v = (rng.standard_normal((B, T, 32, 128)).astype(np.float32) for _ in range(3))
    ws = [(0.1 * rng.standard_normal((B, T, 32))).astype(np.float32) for _ in range(6)]
    h = lambda a: torch.from_numpy(a).to(DEV).half()
    qd, kd, vd = h(q), h(k), h(v)
    wd = [h(w) for w in ws]
    back = lambda t: t.float().cpu().numpy()
    return qd, kd, vd, wd, [back(t) for t in (qd, kd, vd)], [back(w) for w in wd]


def _ref_gate(got, ref, what, max_lim=1.2e-1, mean_lim=1e-3):
    d = np.abs(got.astype(np.float64) - ref)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert d.max() <= max_lim and d.mean() <= mean_lim, f"{what}: max={d.max():.3e} mean={d.mean():.3e}"


def _need(name):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if built(name) is None:
        pytest.skip(f"{name} not built (oracle/build_ref.py needs the reference checkout)")
    return import_module(name)


@pytest.mark.parametrize("B,T,G,chunk,W", [(1, 256, 8, 16, 112), (2, 384, 8, 16, 112),
                                           (1, 256, 4, 16, 112), (1, 320, 8, 32, 96)])
def test_onekernel_v4_vs_oracle_and_ours(B, T, G, chunk, W):
    m = _need("dc_fused_cuda")
    qd, kd, vd, wd, (q, k, v), ws = _inputs(B, T, seed=B * 1000 + T + G + W)
    scale = 128 ** -0.5
    sl = torch.full((B,), T, dtype=torch.int32, device=DEV)
    theirs = m.onekernel_v4_forward(qd, kd, vd, *wd, sl, scale, W, G, chunk)
    ours = dc.dc_attention_window_chunked_residual_grouped(qd, kd, vd, wd, scale, W, G=G)
    torch.cuda.synchronize()
    ref = O.grouped_residual(q, k, v, ws, scale, W, G=G).transpose(0, 2, 1, 3)  # [B,T,N,D]
    _ref_gate(theirs.float().cpu().numpy(), ref, "onekernel_v4")
    assert_close(ours.float().cpu().numpy().transpose(0, 2, 1, 3), ref, "ours")


@pytest.mark.parametrize("fn,B,T,BM,W", [("forward_hpg4_wide_opt", 1, 256, 16, 240),
                                         ("forward_hpg4_wide_opt", 2, 512, 16, 240),
                                         ("forward_hpg4_wide_ref", 1, 256, 32, 224),
                                         ("forward_hpg4_wide_ref", 1, 512, 16, 240)])
def test_hopper_wide_vs_oracle_and_ours(fn, B, T, BM, W):
    m = _need("_dc_hopper_cuda")
    qd, kd, vd, wd, (q, k, v), ws = _inputs(B, T, seed=7 * B + T + BM)
    scale = 128 ** -0.5
    theirs = getattr(m, fn)(qd, kd, vd, *wd, scale, W, BM)
    ours = dc.dc_attention_window_chunked_residual_grouped(qd, kd, vd, wd, scale, W, G=8)
    torch.cuda.synchronize()
    ref = O.grouped_residual(q, k, v, ws, scale, W, G=8).transpose(0, 2, 1, 3)
    lim = (2e-1, 2e-3) if fn.endswith("opt") else (1.2e-1, 1e-3)
    _ref_gate(theirs.float().cpu().numpy(), ref, fn, *lim)
    assert_close(ours.float().cpu().numpy().transpose(0, 2, 1, 3), ref, "ours")
