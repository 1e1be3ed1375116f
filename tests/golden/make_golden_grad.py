"""Generate golden gradients from the reference's own torch implementation.

Run where the reference project (Lisennlp/dc_triton_opt) is checked out:

    python tests/golden/make_golden_grad.py <path-to-reference-checkout>

The reference has no CPU backward of its own; its GPU backward
(TritonDCResidual.backward, triton_dc_residual.py:1707-1892) differentiates
``dc_attention_window_chunked_residual_grouped`` (dc_attention_torch.py:159-258).
This script runs torch autograd through that reference function (fp32, inputs
rounded to the kernel dtype first) with a seeded output gradient and stores
the gradients of q, k, v and the six [B,T,N] weights in
``tests/golden/golden_grad.npz`` (not needed at test time).
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "golden_grad.npz"
WNAMES = ("pre_w1", "pre_w2", "pre_dd", "post_w1", "post_w2", "post_dd")


def main(ref_dir: str):
    sys.path.insert(0, ref_dir)
    import dc_attention_torch as ref  # noqa: E402  (reference module)

    blob, cases = {}, []

    def case(name, B, T, H, D, G, window, seq_lens, wstd, dtype, seed):
        g = torch.Generator().manual_seed(seed)
        rnd = lambda *s, std=1.0: (std * torch.randn(*s, generator=g)).to(dtype).to(torch.float32)
        q, k, v = (rnd(B, T, H, D).requires_grad_() for _ in range(3))
        ws = [rnd(B, T, H, std=wstd).requires_grad_() for _ in range(6)]
        dout = rnd(B, H, T, D)  # the reference returns [B,N,T,D]
        sl = None if seq_lens is None else torch.tensor(seq_lens, dtype=torch.int32)
        out = ref.dc_attention_window_chunked_residual_grouped(q, k, v, ws, 1.0 / math.sqrt(D), window=window,
                                                               seq_lens=sl, chunk_size=16, G=G)
        (out * dout).sum().backward()
        to16 = lambda t: t.detach().to(dtype).view(torch.int16).numpy().view(np.uint16)
        for key, t in (("q", q), ("k", k), ("v", v)):
            blob[f"{name}/{key}"] = to16(t)
        for n, t in zip(WNAMES, ws):
            blob[f"{name}/{n}"] = to16(t)
            blob[f"{name}/d_{n}"] = t.grad.numpy().astype(np.float32)
        blob[f"{name}/dout"] = to16(dout)
        for key, t in (("dq", q), ("dk", k), ("dv", v)):
            blob[f"{name}/{key}"] = t.grad.numpy().astype(np.float32)
        blob[f"{name}/meta"] = np.array([B, T, H, D, G, window], dtype=np.int64)
        blob[f"{name}/seq_lens"] = np.array(seq_lens if seq_lens is not None else [], dtype=np.int32)
        cases.append(name)

    bf = torch.bfloat16
    # HPG 4 (the reference's grouping), window edge and ragged T
    case("grad_g2_w24", 1, 80, 8, 128, 2, 24, None, 0.1, bf, 11)
    # G = 1 (all heads mix), seq_lens shorter than T
    case("grad_g1_seqlens", 2, 48, 8, 128, 1, 16, [48, 29], 0.1, bf, 12)
    # HPG 1 and std-1 weights (negative (1 + dd) gates)
    case("grad_hpg1_std1", 1, 40, 4, 128, 4, 12, None, 1.0, bf, 13)
    blob["cases"] = np.array(cases)
    np.savez_compressed(OUT, **blob)
    print(f"wrote {OUT} ({len(cases)} cases)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
