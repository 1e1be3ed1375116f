"""Class-style entry point of the reference's fused kernels:
``Cls.forward(q, k, v, dc_weights, scaling, window, seq_lens=None, G=..., chunk_size=...)``
returning [B,T,N,D] (``triton_dc_onekernel_v4_h100.py:864-1168``,
``cuda_dc_onekernel_v4.py:20-67``).

The reference has one class per kernel experiment, each with its own shape
gate and a fallback chain to older kernels (``triton_dc_onekernel_v4_h100.py:881-883``).
Here one class covers every shape; the reference's class names are kept as
aliases so existing call sites switch by changing the import only.
"""

from __future__ import annotations

from .api import DCTerms, dc_attn_fwd


class DCOneKernel:
    """Fused DC-attention forward: residual rank-1 pre/post composition inside
    head groups of H/G heads, causal sliding window."""

    @staticmethod
    def forward(q, k, v, dc_weights, scaling, window, seq_lens=None, G=16, chunk_size=16):
        pw1, pw2, pdd, qw1, qw2, qdd = dc_weights
        B, T, N, D = q.shape
        if N % G != 0:
            raise RuntimeError(f"N={N} must be divisible by G={G}")
        W = min(int(window), T)  # triton_dc_onekernel_v4_h100.py:873
        return dc_attn_fwd(q, k, v, DCTerms.residual(pw1, pw2, pdd), DCTerms.residual(qw1, qw2, qdd),
                           scaling, W, G, seq_lens)


# reference class names (same call signature, same result)
TritonDCOneKernel = DCOneKernel
TritonDCOneKernelCombined = DCOneKernel
TritonDCOneKernelCombinedProbs = DCOneKernel
TritonDCOneKernelMixedProbs = DCOneKernel
TritonDCOneKernelMixedProbs256 = DCOneKernel
CudaDCOneKernelV4 = DCOneKernel
