"""Numerical tolerances of the CUDA kernels against the fp32/fp64 oracle on
identical (bf16- or fp16-rounded) inputs.

bf16/fp16 inputs, fp32 accumulation and fp32 softmax/composition; the output
and the probabilities fed to the P'V product are rounded to the input type.
Gate (all must hold): max|d| <= MAX_ABS, max|d| / max|ref| <= MAX_REL and
mean|d| <= max(MEAN_ABS, MEAN_REL * mean|ref|) (rounding the output itself to
bf16 already costs ~1e-3 of its magnitude on average).  The reference's own fp16 gate was max <= 1.2e-1,
mean <= 1e-3 (test_dc_hopper_cuda.py:123-124); these are tighter.
"""

import numpy as np

MAX_ABS = 3e-2
MAX_REL = 1e-2
MEAN_ABS = 1e-3
MEAN_REL = 4e-3


def assert_close(got, ref, what="", max_abs=MAX_ABS, max_rel=MAX_REL, mean_abs=MEAN_ABS, mean_rel=MEAN_REL):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    d = np.abs(got - ref)
    mx, mean = float(d.max()) if d.size else 0.0, float(d.mean()) if d.size else 0.0
    scale = max(float(np.abs(ref).max()) if ref.size else 0.0, 1e-6)
    msg = f"{what}: max|d|={mx:.3e} rel={mx / scale:.3e} mean|d|={mean:.3e}"
    mean_gate = max(mean_abs, mean_rel * (float(np.abs(ref).mean()) if ref.size else 0.0))
    assert mx <= max_abs and mx / scale <= max_rel and mean <= mean_gate, msg
    return mx, mean


# Gradients (backward kernel, fp32 arithmetic; dq rounded to the input dtype,
# dk / dv / weight gradients fp32) against the float64 autograd oracle or the
# reference's fp32 autograd on the same inputs.  Gradient magnitudes differ by
# orders between tensors, so the gate is relative to each tensor's largest
# entry: max|d| <= GRAD_MAX_REL * max|ref| and
# mean|d| <= GRAD_MEAN_REL * mean|ref| + 1e-4 * max|ref|.
GRAD_MAX_REL = 1e-2
GRAD_MEAN_REL = 4e-3


def assert_grad_close(got, ref, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite gradient"
    d = np.abs(got - ref)
    scale = max(float(np.abs(ref).max()), 1e-12)
    mx, mean = float(d.max()), float(d.mean())
    msg = f"{what}: max|d|={mx:.3e} (max|ref|={scale:.3e}) mean|d|={mean:.3e}"
    assert mx <= GRAD_MAX_REL * scale and mean <= GRAD_MEAN_REL * float(np.abs(ref).mean()) + 1e-4 * scale, msg
