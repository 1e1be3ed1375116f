"""Load the committed golden vectors (made by tests/golden/make_golden.py from
the reference's own torch functions) into numpy arrays and oracle term sets."""

from __future__ import annotations

import os

import numpy as np

from oracle.dc_oracle import Terms, residual_terms

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")


def _load_input(z, key):
    a = z[key]
    if a.dtype == np.uint16:  # bf16 bit patterns
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


class Case:
    def __init__(self, z, name):
        self.name = name
        B, T, H, D, G, window, chunk, is_bf16 = (int(x) for x in z[f"{name}/meta"])
        self.B, self.T, self.H, self.D, self.G = B, T, H, D, G
        self.kind = name.split("_")[0]
        self.window = None if window < 0 else window
        self.chunk = None if chunk < 0 else chunk
        self.dtype = "bf16" if is_bf16 else "fp16"
        sl = z[f"{name}/seq_lens"]
        self.seq_lens = None if sl.size == 0 else sl.astype(np.int32)
        self.scale = float(z[f"{name}/scale"][0])
        self.q, self.k, self.v = (_load_input(z, f"{name}/{x}") for x in "qkv")
        self.out = z[f"{name}/out"]
        if self.kind in ("grouped", "residual"):
            self.ws = [_load_input(z, f"{name}/w{i}") for i in range(6)]
            self.pre = residual_terms(*self.ws[:3])
            self.post = residual_terms(*self.ws[3:])
        elif self.kind == "decomposed":
            self.pre_w = _load_input(z, f"{name}/pre_w")
            self.post_w = _load_input(z, f"{name}/post_w")
            self.pre = Terms(identity=False, qmat=self.pre_w)
            self.post = Terms(identity=False, qmat=self.post_w)
        elif self.kind == "terms":
            self.R = chunk
            sets = []
            for side in ("pre", "post"):
                sets.append(Terms(identity=False, w=z[f"{name}/{side}_w"],
                                  qw1=_load_input(z, f"{name}/{side}_qw1"),
                                  qw2=_load_input(z, f"{name}/{side}_qw2"),
                                  qdd=_load_input(z, f"{name}/{side}_qdd")))
            self.pre, self.post = sets
        else:
            raise ValueError(name)

    @property
    def out_btnd(self):
        """Reference output in [B,T,N,D] (the grouped/residual fns return [B,N,T,D])."""
        if self.kind in ("grouped", "residual"):
            return self.out.transpose(0, 2, 1, 3)
        return self.out

    @property
    def eff_window(self):
        if self.kind in ("grouped", "residual") and self.window is None:
            return 256
        return self.window


def load_cases():
    z = np.load(PATH)
    return [Case(z, str(n)) for n in z["cases"]]


GRAD_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_grad.npz")
WNAMES = ("pre_w1", "pre_w2", "pre_dd", "post_w1", "post_w2", "post_dd")


class GradCase:
    """One golden backward case (tests/golden/make_golden_grad.py): bf16 inputs,
    the output gradient dout [B,N,T,D] of the reference's grouped function, and
    the reference's autograd gradients (fp32)."""

    def __init__(self, z, name):
        self.name = name
        self.B, self.T, self.H, self.D, self.G, self.window = (int(x) for x in z[f"{name}/meta"])
        sl = z[f"{name}/seq_lens"]
        self.seq_lens = None if sl.size == 0 else sl.astype(np.int32)
        self.q, self.k, self.v = (_load_input(z, f"{name}/{k}") for k in ("q", "k", "v"))
        self.ws = [_load_input(z, f"{name}/{n}") for n in WNAMES]
        self.dout = _load_input(z, f"{name}/dout")               # [B,N,T,D]
        self.dout_btnd = self.dout.transpose(0, 2, 1, 3).copy()  # [B,T,N,D]
        self.grads = {k: z[f"{name}/{k}"] for k in ("dq", "dk", "dv")}
        for n in WNAMES:
            self.grads[f"d_{n}"] = z[f"{name}/d_{n}"]
        self.scale = 1.0 / np.sqrt(self.D)


def load_grad_cases():
    with np.load(GRAD_PATH) as z:
        return [GradCase(z, str(n)) for n in z["cases"]]
