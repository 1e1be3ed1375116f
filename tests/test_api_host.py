"""Host-side argument checks of the torch API (no GPU needed): the same
conditions the reference rejects with TORCH_CHECK raise RuntimeError here."""

import pytest
import torch

import dc_triton_opt_b200 as dc
from dc_triton_opt_b200 import dc_hopper_cuda, onekernel


def _inputs(B=1, T=16, N=32, D=128, dtype=torch.float16):
    q = torch.randn(B, T, N, D).to(dtype)
    ws = tuple(torch.randn(B, T, N).to(dtype) for _ in range(6))
    return q, q.clone(), q.clone(), ws


def test_cpu_tensors_rejected():
    q, k, v, ws = _inputs()
    with pytest.raises(RuntimeError, match="CUDA"):
        dc.dc_attention_window_chunked_residual_grouped(q, k, v, ws, 0.1, 8, G=8)


def test_fp32_rejected():
    q, k, v, ws = _inputs(dtype=torch.float32)
    with pytest.raises(RuntimeError):
        dc.dc_attn_fwd(q, k, v)


def test_hopper_api_checks():
    q, k, v, ws = _inputs()
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        dc_hopper_cuda.forward_hpg4_wide_ref(q, k, v, *ws, 0.1, 224, 32)


def test_onekernel_group_check():
    q, k, v, ws = _inputs(N=30)
    with pytest.raises(RuntimeError, match="divisible"):
        onekernel.DCOneKernel.forward(q, k, v, ws, 0.1, 16, G=8)


def test_reference_class_aliases():
    for name in ("TritonDCOneKernelMixedProbs", "TritonDCOneKernelMixedProbs256", "CudaDCOneKernelV4",
                 "TritonDCOneKernel"):
        assert getattr(onekernel, name) is onekernel.DCOneKernel
