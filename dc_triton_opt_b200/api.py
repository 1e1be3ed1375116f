"""Torch-callable DC-attention forward on B200, backed by ``libdcattn.so``.

Entry points (each a drop-in for the reference call it names):

* :func:`dc_attn_fwd` — general form: static head mix W, query- and key-wise
  rank-R weights, qdd/kdd gates, per-query matrices; window or full causal.
* :func:`dc_attn_fwd_host` — the same for inputs and output in host memory,
  with the batch pipelined over copy / compute streams.
* :func:`dc_attention_window_chunked_residual_grouped` —
  ``dc_attention_torch.py:159`` (same signature, defaults, output [B,N,T,D]).
* :func:`dc_attention_window_chunked_residual` — ``dc_attention_torch.py:88``.
* :func:`dc_attention_decomposed_window_chunked` — ``dc_attention_torch.py:22``
  (per-query N x N mixing matrices, output [B,T,N,D]).

All of them run the CUDA kernels on the tensors' device and current stream,
asynchronously, and raise ``RuntimeError`` for bad arguments (the reference
raises through ``TORCH_CHECK``, which surfaces as ``RuntimeError`` too).
"""

from __future__ import annotations

import ctypes
import warnings
from dataclasses import dataclass, fields
from typing import Optional, Sequence

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.DC_DTYPE_BF16, torch.float16: _lib.DC_DTYPE_FP16}


@dataclass
class DCTerms:
    """One composition term set (pre on logits, post on probabilities).

    Shapes (B,T,H heads, G groups, HPG=H/G, rank R):
      w [G,HPG,HPG] (any float dtype, used as fp32): a'[h] += sum_h' a[h'] w[g,h',h]
      qw1/kw1 [B,T,H,R]; qw2/kw2 [B,T,R,H]; qdd/kdd [B,T,H]; qmat [B,T,H,HPG].
    ``identity`` adds a[h] itself (the reference's residual term).
    """

    identity: bool = False
    w: Optional[torch.Tensor] = None
    qw1: Optional[torch.Tensor] = None
    qw2: Optional[torch.Tensor] = None
    kw1: Optional[torch.Tensor] = None
    kw2: Optional[torch.Tensor] = None
    qdd: Optional[torch.Tensor] = None
    kdd: Optional[torch.Tensor] = None
    qmat: Optional[torch.Tensor] = None

    @staticmethod
    def residual(w1, w2, dd) -> "DCTerms":
        """The reference's residual rank-1 set from three [B,T,N] tensors
        (``dc_attention_torch.py:217-225``): a + dd*a + w2 * sum(w1*a)."""
        return DCTerms(identity=True, qw1=w1.unsqueeze(-1), qw2=w2.unsqueeze(-2), qdd=dd)


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _prep(t: Optional[torch.Tensor], name: str, shape, dtype, device, keep):
    if t is None:
        return None
    _check(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor")
    _check(t.device == device, f"{name} must be on {device} (got {t.device})")
    _check(tuple(t.shape) == tuple(shape), f"{name} must have shape {list(shape)} (got {list(t.shape)})")
    t = t.to(dtype).contiguous()
    keep.append(t)
    return t


def _terms_struct(tm: Optional[DCTerms], name, B, T, H, G, R, dtype, device, keep) -> _lib.DcTerms:
    s = _lib.DcTerms()
    if tm is None:
        s.identity = 1
        return s
    hpg = H // G
    s.identity = 1 if tm.identity else 0
    shapes = {"w": (G, hpg, hpg), "qw1": (B, T, H, R), "qw2": (B, T, R, H), "kw1": (B, T, H, R),
              "kw2": (B, T, R, H), "qdd": (B, T, H), "kdd": (B, T, H), "qmat": (B, T, H, hpg)}
    for f in fields(DCTerms):
        if f.name == "identity":
            continue
        t = getattr(tm, f.name)
        dt = torch.float32 if f.name == "w" else dtype
        t = _prep(t, f"{name}.{f.name}", shapes[f.name], dt, device, keep)
        setattr(s, f.name, None if t is None else t.data_ptr())
    return s


def _infer_rank(*sets: Optional[DCTerms]) -> int:
    R = 0
    for tm in sets:
        if tm is None:
            continue
        for a in (tm.qw1, tm.kw1):
            if a is not None:
                R = max(R, a.shape[-1])
    return R


def _params(q, k, v, pre, post, scaling, window, G, seq_lens, out, kernel, wait_us=0, test_flags=0):
    """Validate a forward call and build its dc_attn_params; returns
    (params, out, keep) where `keep` holds converted temporaries alive."""
    _check(q.dim() == 4, f"q must be [B,T,H,D] (got {list(q.shape)})")
    _check(k.shape == q.shape and v.shape == q.shape, "k and v must match q's shape")
    _check(q.dtype in _DTYPES, f"q must be bfloat16 or float16 (got {q.dtype})")
    _check(k.dtype == q.dtype and v.dtype == q.dtype, "q, k, v must share one dtype")
    _check(q.is_cuda and k.device == q.device and v.device == q.device,
           "q, k, v must be CUDA tensors on one device")
    B, T, H, D = q.shape
    _check(G >= 1 and H % G == 0, f"H={H} must be divisible by G={G}")
    R = _infer_rank(pre, post)
    device, dtype = q.device, q.dtype
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    keep = [q, k, v]
    if out is None:
        out = torch.empty((B, T, H, D), device=device, dtype=dtype)
    _check(out.shape == (B, T, H, D) and out.dtype == dtype and out.device == device,
           "out must be a [B,T,H,D] tensor of q's dtype and device")
    _check(out.stride(3) == 1, "out must be contiguous in its last dim")
    p = _lib.DcAttnParams()
    p.abi_version = _lib.ABI_VERSION
    p.B, p.T, p.H, p.D, p.G, p.R = B, T, H, D, G, R
    p.window = 0 if window is None else int(window)
    _check(window is None or int(window) >= 1, f"window must be >= 1 or None (got {window})")
    p.scale = float(D ** -0.5 if scaling is None else scaling)
    p.dtype = _DTYPES[dtype]
    _check(kernel in _lib.KERNELS, f"kernel must be one of {sorted(_lib.KERNELS)}")
    p.kernel = _lib.KERNELS[kernel]
    p.q, p.k, p.v, p.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.out_sb, p.out_st, p.out_sh = out.stride(0), out.stride(1), out.stride(2)
    if seq_lens is not None:
        _check(seq_lens.shape == (B,), f"seq_lens must be [B]={B} (got {list(seq_lens.shape)})")
        seq_lens = seq_lens.to(device=device, dtype=torch.int32).contiguous()
        keep.append(seq_lens)
        p.seq_lens = seq_lens.data_ptr()
    p.pre = _terms_struct(pre, "pre", B, T, H, G, R, dtype, device, keep)
    p.post = _terms_struct(post, "post", B, T, H, G, R, dtype, device, keep)
    _check(0 <= int(wait_us) < 2 ** 32, "wait_us must be in [0, 2^32)")
    p.wait_us = int(wait_us)
    p.test_flags = int(test_flags)
    return p, out, keep


def dc_attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                pre: Optional[DCTerms] = None, post: Optional[DCTerms] = None,
                scaling: Optional[float] = None, window: Optional[int] = None, G: int = 1,
                seq_lens: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                kernel: str = "auto", check: bool = False, wait_us: int = 0,
                test_flags: int = 0) -> torch.Tensor:
    """General DC-attention forward.  q,k,v [B,T,H,D] (bf16 or fp16) -> [B,T,H,D].

    ``window=None`` is full causal; otherwise key s is visible from query t iff
    t - window < s <= t.  ``pre``/``post`` default to the identity (plain
    attention).  ``out`` may be any tensor whose last dim is contiguous and whose
    [b,t,h] strides are positive (e.g. a [B,N,T,D] tensor permuted to
    [B,T,N,D]); it is written in place and returned.

    Every wait inside the kernels is bounded (``wait_us``, default 2 s); a wait
    that runs out makes the kernel skip the rest of its work and write a code
    to the device error word.  ``check=True`` synchronises with the stream and
    raises ``RuntimeError`` if that happened (otherwise read it later with
    :func:`device_error`).  ``test_flags`` is for tests only.
    """
    p, out, keep = _params(q, k, v, pre, post, scaling, window, G, seq_lens, out, kernel, wait_us, test_flags)
    device = q.device
    B, T, H, D = q.shape
    R = p.R
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(lib.dc_attn_fwd(ctypes.byref(p), ctypes.c_void_p(stream)))
        if kernel == "auto" and lib.dc_attn_last_kernel() == _lib.DC_KERNEL_SIMT:
            _warn_simt(T, H, D, G, R, window, pre, post)
        if check:
            _raise_device_error(lib, stream)
    # Converted temporaries in `keep` may be freed on return: the caching
    # allocator only hands their blocks to later work on this same stream.
    return out


def dc_attn_fwd_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens,
                       pre: Optional[DCTerms] = None, post: Optional[DCTerms] = None,
                       scaling: Optional[float] = None, window: Optional[int] = None, G: int = 1,
                       out: Optional[torch.Tensor] = None, kernel: str = "auto") -> torch.Tensor:
    """Forward over a packed batch of variable-length sequences.

    q, k, v are [total, H, D] (the sequences back to back); per-token weights
    are packed the same way ([total, H, R], [total, R, H], [total, H],
    [total, H, HPG]).  Sequence i is tokens [cu_seqlens[i], cu_seqlens[i+1]);
    attention never crosses a sequence boundary.  ``cu_seqlens`` is read on the
    host (a CUDA tensor is copied, which synchronises).  Returns [total, H, D]."""
    _check(q.dim() == 3, f"q must be [total, H, D] (got {list(q.shape)})")
    cu = torch.as_tensor(cu_seqlens).to("cpu", torch.int32).contiguous()
    _check(cu.dim() == 1 and cu.numel() >= 2, "cu_seqlens must be a 1-D list of nseq + 1 offsets")
    unsq = lambda t: None if t is None else t.unsqueeze(0)
    lift = lambda tm: None if tm is None else DCTerms(
        identity=tm.identity, w=tm.w, **{f: unsq(getattr(tm, f)) for f in _PER_TOKEN})
    q4, k4, v4 = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0)
    o4 = None if out is None else out.unsqueeze(0)
    p, o4, keep = _params(q4, k4, v4, lift(pre), lift(post), scaling, window, G, None, o4, kernel)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(lib.dc_attn_fwd_varlen(ctypes.byref(p), cu.data_ptr(), cu.numel() - 1, ctypes.c_void_p(stream)),
                   "dc_attn_fwd_varlen")
    return o4[0]


E4M3_MAX = 448.0


def quantize_e4m3(x: torch.Tensor):
    """Per-tensor e4m3 quantization for :func:`dc_attn_fwd_fp8qk`:
    returns (x8, scale) with x ~= x8.float() * scale and |x8| <= 448."""
    amax = x.detach().abs().amax().float().clamp_min(1e-12)
    scale = amax / E4M3_MAX
    return (x.float() / scale).to(torch.float8_e4m3fn), float(scale)


def dc_attn_fwd_fp8qk(q8: torch.Tensor, k8: torch.Tensor, v: torch.Tensor, q_scale: float, k_scale: float,
                      pre: Optional[DCTerms] = None, post: Optional[DCTerms] = None,
                      scaling: Optional[float] = None, window: int = 128, G: int = 1,
                      seq_lens: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Forward with q and k in e4m3 (``torch.float8_e4m3fn``, [B,T,H,D]) and
    per-tensor scales (q ~= q8 * q_scale): QK^T on the tensor cores in fp8,
    everything else as :func:`dc_attn_fwd` in v's dtype (bf16 / fp16).  Windowed
    layers with 1-8 heads per group (the single-pass tensor-core kernel)."""
    _check(q8.dtype == torch.float8_e4m3fn and k8.dtype == torch.float8_e4m3fn,
           "q8 and k8 must be torch.float8_e4m3fn")
    _check(q8.shape == v.shape and k8.shape == v.shape, "q8, k8 and v must share one shape")
    _check(window is not None, "the fp8 path needs a sliding window")
    p, out, keep = _params(v, v, v, pre, post, scaling, window, G, seq_lens, out, "tc")
    q8, k8 = q8.contiguous(), k8.contiguous()
    keep += [q8, k8]
    p.q, p.k = q8.data_ptr(), k8.data_ptr()
    lib = _lib.load()
    with torch.cuda.device(v.device):
        stream = torch.cuda.current_stream(v.device).cuda_stream
        _lib.check(lib.dc_attn_fwd_fp8qk(ctypes.byref(p), float(q_scale), float(k_scale), ctypes.c_void_p(stream)),
                   "dc_attn_fwd_fp8qk")
    return out


_SIMT_WARNED = set()


def _warn_simt(T, H, D, G, R, window, pre, post):
    """One warning per distinct request shape that AUTO had to run on the
    CUDA-core kernel (two orders of magnitude slower than the tensor-core ones)."""
    key = (T, H, D, G, R, window)
    if key in _SIMT_WARNED:
        return
    _SIMT_WARNED.add(key)
    why = f"D={D}, heads per group={H // G}, R={R}, window={window}"
    warnings.warn(f"dc_attn_fwd: no tensor-core kernel supports this call ({why}); "
                  "it runs on the CUDA-core kernel, which is much slower", RuntimeWarning, stacklevel=3)


def _raise_device_error(lib, stream):
    code = lib.dc_attn_read_error(None, 1, ctypes.c_void_p(stream))
    if code < 0:
        _lib.check(code, "dc_attn_read_error")
    if code > 0:
        raise RuntimeError(f"dc_attn_fwd: device error {_lib.DEV_ERRORS.get(code, code)} "
                           "(a wait inside the kernel ran out; the output is not valid)")


def device_error(device=None, clear: bool = True) -> int:
    """Code in the library's device error word of ``device`` (0 = none) after
    the work queued so far on its current stream (this synchronises with that
    stream).  Non-zero means a kernel's bounded wait ran out and that launch's
    output is not valid; ``clear`` resets the word."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        code = lib.dc_attn_read_error(None, 1 if clear else 0, ctypes.c_void_p(stream))
    if code < 0:
        _lib.check(code, "dc_attn_read_error")
    return code


_PER_TOKEN = ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd", "qmat")


class _HostWorkspace:
    """Device staging buffers of :func:`dc_attn_fwd_host` for one device: two
    slots of inputs and output, the copy streams, and per slot the events of
    its last use.  The events are kept across calls, so a call never
    overwrites a slot that an earlier call's forward or copy-back still uses.
    One buffer set per device is retained (two batch slices of q, k, v, out and
    the per-token weights); a call with other slice shapes first waits for the
    old buffers' last use, then replaces them."""

    def __init__(self, device):
        self.device = device
        self.key = None
        self.bufs = {}
        self.ev_comp = [None, None]  # slot's inputs / output buffer in use by a forward until then
        self.ev_out = [None, None]   # slot's output copied back to the host
        self.slot = 0
        self.s_in = torch.cuda.Stream(device)
        self.s_out = torch.cuda.Stream(device)

    def reset(self, key):
        if key == self.key:
            return
        for ev in self.ev_comp + self.ev_out:
            if ev is not None:
                ev.synchronize()
        self.bufs.clear()
        self.ev_comp, self.ev_out = [None, None], [None, None]
        self.key = key

    def buf(self, slot, name, shape, dtype):
        b = self.bufs.get((slot, name))
        if b is None:
            b = torch.empty(shape, device=self.device, dtype=dtype)
            self.bufs[(slot, name)] = b
        return b


_host_ws = {}  # device -> _HostWorkspace


def dc_attn_fwd_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     pre: Optional[DCTerms] = None, post: Optional[DCTerms] = None,
                     scaling: Optional[float] = None, window: Optional[int] = None, G: int = 1,
                     seq_lens: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                     device=None, chunks: int = 4, kernel: str = "auto") -> torch.Tensor:
    """:func:`dc_attn_fwd` for inputs in host memory (ideally pinned).

    q, k, v [B,T,H,D] and the per-token weights of ``pre``/``post`` are CPU
    tensors; the output is written to ``out`` (a [B,T,H,D] CPU tensor; a pinned
    one is allocated if None).  The batch is processed in ``chunks`` slices
    whose host-to-device copies, forward and device-to-host copies run on three
    streams, so the transfers of neighbouring slices overlap each other and the
    compute (two device buffers per stream stage).  Asynchronous like the
    device entry point: the caller's current stream waits for the last copy,
    so a ``torch.cuda.synchronize()`` (or a sync of that stream) makes ``out``
    valid.
    """
    _check(q.dim() == 4 and not q.is_cuda and not k.is_cuda and not v.is_cuda,
           "q, k, v must be [B,T,H,D] host tensors")
    _check(k.shape == q.shape and v.shape == q.shape, "k and v must match q's shape")
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    B, T, H, D = q.shape
    dtype = q.dtype
    if out is None:
        out = torch.empty((B, T, H, D), dtype=dtype, pin_memory=True)
    _check(out.shape == (B, T, H, D) and out.dtype == dtype and not out.is_cuda and out.is_contiguous(),
           "out must be a contiguous [B,T,H,D] host tensor of q's dtype")
    nch = max(1, min(int(chunks), B))
    cb = -(-B // nch)
    comp = torch.cuda.current_stream(device)
    ws = _host_ws.get(device)
    if ws is None:
        ws = _host_ws[device] = _HostWorkspace(device)
    tok_shapes = tuple((side, f, tuple(getattr(tm, f).shape[1:]), getattr(tm, f).dtype)
                       for side, tm in (("pre", pre), ("post", post)) if tm is not None
                       for f in _PER_TOKEN if getattr(tm, f) is not None)
    ws.reset((cb, T, H, D, dtype, tok_shapes))
    s_in, s_out = ws.s_in, ws.s_out
    # static mixes (small) go to the device once per call
    w_dev = {}
    for side, tm in (("pre", pre), ("post", post)):
        if tm is not None and tm.w is not None:
            w_dev[side] = tm.w.to(device=device, dtype=torch.float32, non_blocking=True)
    sl_dev = None
    if seq_lens is not None:
        sl_dev = seq_lens.to(device=device, dtype=torch.int32, non_blocking=True)
    last = None
    with torch.cuda.device(device):
        for c in range(nch):
            b0, b1 = c * cb, min(B, (c + 1) * cb)
            if b0 >= b1:
                break
            n, slot = b1 - b0, ws.slot
            ws.slot ^= 1

            def dev(name, t):
                buf = ws.buf(slot, name, (cb,) + tuple(t.shape[1:]), t.dtype)[:n]
                buf.copy_(t[b0:b1], non_blocking=True)
                return buf

            with torch.cuda.stream(s_in):
                # the slot's previous forward (of this call or an earlier one) has read its inputs
                if ws.ev_comp[slot] is not None:
                    s_in.wait_event(ws.ev_comp[slot])
                dq, dk, dv = dev("q", q), dev("k", k), dev("v", v)
                terms = {}
                for side, tm in (("pre", pre), ("post", post)):
                    if tm is None:
                        terms[side] = None
                        continue
                    kw = {"identity": tm.identity, "w": w_dev.get(side)}
                    for f in _PER_TOKEN:
                        t = getattr(tm, f)
                        kw[f] = None if t is None else dev(f"{side}.{f}", t)
                    terms[side] = DCTerms(**kw)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            comp.wait_event(ev_in)
            if ws.ev_out[slot] is not None:
                comp.wait_event(ws.ev_out[slot])  # the slot's previous output has been copied back
            dout = ws.buf(slot, "out", (cb, T, H, D), dtype)[:n]
            dc_attn_fwd(dq, dk, dv, terms["pre"], terms["post"], scaling, window, G,
                        None if sl_dev is None else sl_dev[b0:b1], out=dout, kernel=kernel)
            ev = torch.cuda.Event()
            ev.record(comp)
            ws.ev_comp[slot] = ev
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                out[b0:b1].copy_(dout, non_blocking=True)
                ev_o = torch.cuda.Event()
                ev_o.record(s_out)
                ws.ev_out[slot] = last = ev_o
        if last is not None:
            comp.wait_event(last)
    return out


def select_kernel(q, k, v, pre=None, post=None, window=None, G=1) -> str:
    """Which kernel ``kernel='auto'`` runs for these arguments ('tc', 'tcm', 'tcs' or 'simt')."""
    B, T, H, D = q.shape
    p = _lib.DcAttnParams()
    p.abi_version = _lib.ABI_VERSION
    p.B, p.T, p.H, p.D, p.G, p.R = B, T, H, D, G, _infer_rank(pre, post)
    p.window = 0 if window is None else int(window)
    p.scale = 1.0
    p.dtype = _DTYPES.get(q.dtype, -1)
    p.q = p.k = p.v = p.out = 16  # placeholders: selection reads only sizes and term presence
    p.out_sb, p.out_st, p.out_sh = T * H * D, H * D, D
    for side, tm in (("pre", pre), ("post", post)):
        st = getattr(p, side)
        st.identity = 1 if (tm is None or tm.identity) else 0
        if tm is not None:
            for f in fields(DCTerms):
                if f.name != "identity" and getattr(tm, f.name) is not None:
                    setattr(st, f.name, 16)
    rc = _lib.load().dc_attn_select_kernel(ctypes.byref(p))
    _lib.check(rc if rc < 0 else 0, "dc_attn_select_kernel")
    return {1: "simt", 2: "tc", 3: "tcs", 4: "tcm"}[rc]


def _residual_call(q, k, v, dc_weights, scaling, window, seq_lens, G, out):
    _check(len(dc_weights) == 6, "dc_weights must be (pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd)")
    pw1, pw2, pdd, qw1, qw2, qdd = dc_weights
    B, T, N, D = q.shape
    for name, w in zip(("pre_w1", "pre_w2", "pre_dd", "post_w1", "post_w2", "post_dd"), dc_weights):
        _check(tuple(w.shape) == (B, T, N), f"{name} must be [B,T,N]")
    return dc_attn_fwd(q, k, v, DCTerms.residual(pw1, pw2, pdd), DCTerms.residual(qw1, qw2, qdd),
                       scaling, window, G, seq_lens, out)


def _fp32_to_bf16(*ts):
    """The reference's torch functions accept any float dtype.  fp32 inputs are
    rounded to bf16 here (the kernels take bf16/fp16 operands and accumulate in
    fp32); the caller then gets its result back in fp32."""
    return [None if t is None else (t.to(torch.bfloat16) if t.dtype == torch.float32 else t) for t in ts]


def dc_attention_window_chunked_residual_grouped(
        q, k, v, dc_weights: Sequence[torch.Tensor], scaling: float, window: Optional[int] = None,
        seq_lens: Optional[torch.Tensor] = None, chunk_size: Optional[int] = None, G: int = 1):
    """Drop-in for ``dc_attention_torch.dc_attention_window_chunked_residual_grouped``
    (``dc_attention_torch.py:159-258``): q,k,v [B,T,N,D], six [B,T,N] weights,
    window default 256, returns a contiguous [B,N,T,D] tensor of q's dtype.
    ``chunk_size`` is accepted and ignored (the reference's mask is exact).
    fp32 inputs are computed from their bf16 rounding, output in fp32."""
    B, T, N, D = q.shape
    if window is None:
        window = 256
    if q.dtype == torch.float32:
        q, k, v, *ws = _fp32_to_bf16(q, k, v, *dc_weights)
        return dc_attention_window_chunked_residual_grouped(q, k, v, ws, scaling, window, seq_lens,
                                                            chunk_size, G).float()
    out = torch.empty((B, N, T, D), device=q.device, dtype=q.dtype)
    _residual_call(q, k, v, dc_weights, scaling, window, seq_lens, G, out.permute(0, 2, 1, 3))
    return out


def dc_attention_window_chunked_residual(q, k, v, dc_weights, scaling, window=None, seq_lens=None,
                                         chunk_size=None):
    """Drop-in for ``dc_attention_torch.dc_attention_window_chunked_residual``
    (``dc_attention_torch.py:88-156``): the G=1 case, output [B,N,T,D]."""
    return dc_attention_window_chunked_residual_grouped(q, k, v, dc_weights, scaling, window,
                                                        seq_lens, chunk_size, G=1)


def dc_attention_decomposed_window_chunked(q, k, v, pre_w, post_w, scaling, window, seq_lens,
                                           chunk_size):
    """Drop-in for ``dc_attention_torch.dc_attention_decomposed_window_chunked``
    (``dc_attention_torch.py:22-84``): per-query N x N matrices
    (``mixed[i] = sum_j pre_w[b,t,i,j] L[j]``), no residual, output [B,T,N,D].
    ``window`` is clamped to [1, T] as in the reference (``:38``).  fp32 inputs
    are computed from their bf16 rounding, output in fp32."""
    B, T, N, D = q.shape
    window = max(1, min(int(window), T))
    if q.dtype == torch.float32:
        q, k, v, pre_w, post_w = _fp32_to_bf16(q, k, v, pre_w, post_w)
        return dc_attention_decomposed_window_chunked(q, k, v, pre_w, post_w, scaling, window, seq_lens,
                                                      chunk_size).float()
    return dc_attn_fwd(q, k, v, DCTerms(qmat=pre_w), DCTerms(qmat=post_w), scaling, window, 1, seq_lens)
