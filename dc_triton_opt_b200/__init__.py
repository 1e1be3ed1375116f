"""B200-native (sm_100a) DC-attention forward and backward.

Drop-in replacements for the reference project's torch-callable DC-attention
entry points, backed by hand-written CUDA kernels behind a C ABI
(``include/dc_attn.h``).  See :mod:`dc_triton_opt_b200.api`.
"""

from .api import (DCTerms, dc_attn_fwd, dc_attn_fwd_fp8qk, dc_attn_fwd_host, dc_attn_fwd_varlen, quantize_e4m3, device_error, dc_attention_decomposed_window_chunked,
                  dc_attention_window_chunked_residual,
                  dc_attention_window_chunked_residual_grouped, select_kernel)
from .projection import dc_proj_weights
from .backward import DCResidual, TritonDCResidual, dc_attn, dc_attn_bwd

__all__ = ["DCTerms", "dc_attn_fwd", "dc_attn_fwd_host", "dc_attention_window_chunked_residual_grouped",
           "dc_attention_window_chunked_residual", "dc_attention_decomposed_window_chunked",
           "select_kernel", "device_error", "dc_attn_fwd_varlen", "dc_proj_weights", "dc_attn_fwd_fp8qk", "quantize_e4m3", "dc_attn", "dc_attn_bwd", "DCResidual", "TritonDCResidual"]
