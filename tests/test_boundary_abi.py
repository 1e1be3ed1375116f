"""The C entry points exactly as a reference-side maintainer binds them.

``dc_attn_fwd_residual`` is called through the ctypes stub that INTEGRATION.md
gives for the reference's ``dc_hopper_cuda/__init__.py`` (same argtypes, same
argument order, G=8, dtype code, caller's stream), on the golden vectors made
by the reference's own torch functions and on the reference test's shapes
(``test_dc_hopper_cuda.py:171-175``: N=32, G=8, B in {1, 2} x (T, BM, W) in
{(256,32,224), (512,32,224), (256,16,240), (512,16,240)}), with a
contiguous [B,T,N,D] output and with a strided [B,N,T,D] one on a non-default
stream.  Also: the device error word (a launch whose loads never arrive must
report a timeout code, then the next launch must be clean) and the host-memory
entry point called back to back without a sync.
"""

import ctypes

import numpy as np
import pytest
import torch

import dc_triton_opt_b200 as dc
from dc_triton_opt_b200 import _lib
from oracle import dc_oracle as O
from tests.golden_cases import load_cases
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def stub():
    """The reference-side binding of INTEGRATION.md, verbatim in its argtypes."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = ctypes.CDLL(_lib.LIB_PATH)
    lib.dc_attn_fwd_residual.restype = ctypes.c_int
    lib.dc_attn_last_error.restype = ctypes.c_char_p
    _vp, _i64, _i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    lib.dc_attn_fwd_residual.argtypes = [_vp] * 10 + [_i64] * 3 + [_vp] + [_i32] * 5 + \
        [ctypes.c_float, _i32, _i32, _i32, _vp]

    def forward(q, k, v, pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd, scaling, window, chunk_size,
                out=None, seq_lens=None, G=8):
        B, T, N, D = q.shape
        if out is None:
            out = torch.empty_like(q)
        ws = [w.contiguous() for w in (pre_w1, pre_w2, pre_dd, post_w1, post_w2, post_dd)]
        rc = lib.dc_attn_fwd_residual(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), *[w.data_ptr() for w in ws],
            out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
            None if seq_lens is None else seq_lens.data_ptr(),
            B, T, N, D, G, float(scaling), int(window), int(chunk_size),
            0 if q.dtype == torch.bfloat16 else 1,
            torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(lib.dc_attn_last_error().decode())
        return out

    return forward


def _dev(x, dt):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV).to(dt)


GOLDEN = [c for c in load_cases() if c.kind in ("grouped", "residual")]


@pytest.mark.parametrize("case", GOLDEN, ids=lambda c: c.name)
def test_stub_golden(stub, case):
    dt = torch.bfloat16 if case.dtype == "bf16" else torch.float16
    q, k, v = (_dev(x, dt) for x in (case.q, case.k, case.v))
    ws = [_dev(w, dt) for w in case.ws]
    sl = None if case.seq_lens is None else torch.tensor(case.seq_lens, dtype=torch.int32, device=DEV)
    window = case.eff_window
    ref = case.out_btnd
    got = stub(q, k, v, *ws, case.scale, window, case.chunk or 16, seq_lens=sl, G=case.G)
    torch.cuda.synchronize()
    assert_close(got.float().cpu().numpy(), ref, f"stub {case.name}")


@pytest.mark.parametrize("B", [1, 2])
@pytest.mark.parametrize("T,BM,W", [(256, 32, 224), (512, 32, 224), (256, 16, 240), (512, 16, 240)])
def test_stub_reference_test_shapes(stub, B, T, BM, W):
    g = torch.Generator().manual_seed(1000 * B + T + W)
    dt = torch.float16
    q, k, v = (torch.randn(B, T, 32, 128, generator=g).to(dt) for _ in range(3))
    ws = [torch.randn(B, T, 32, generator=g).to(dt) for _ in range(6)]
    f = lambda x: x.float().numpy()
    ref = O.grouped_residual(f(q), f(k), f(v), [f(w) for w in ws], 128 ** -0.5, W, None, None, 8)  # [B,N,T,D]
    qd, kd, vd = (x.to(DEV) for x in (q, k, v))
    wd = [w.to(DEV) for w in ws]
    # contiguous [B,T,N,D] output on the current stream
    got = stub(qd, kd, vd, *wd, 128 ** -0.5, W, BM)
    torch.cuda.synchronize()
    assert_close(got.float().cpu().numpy(), ref.transpose(0, 2, 1, 3), f"stub B{B} T{T} BM{BM} W{W}")
    # strided output: a [B,N,T,D] buffer written through its [B,T,N,D] view, on a side stream
    side = torch.cuda.Stream()
    out_bntd = torch.full((B, 32, T, 128), float("nan"), dtype=dt, device=DEV)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        stub(qd, kd, vd, *wd, 128 ** -0.5, W, BM, out=out_bntd.permute(0, 2, 1, 3))
    side.synchronize()
    assert_close(out_bntd.float().cpu().numpy(), ref, f"stub strided B{B} T{T} BM{BM} W{W}")


# ---------------------------------------------------------------- device error word

@pytest.mark.parametrize("G,window,kernel", [(8, 112, "tc"), (8, 256, "tc"), (4, None, "tcs"), (1, 128, "tcm")])
def test_timed_out_wait_is_reported(G, window, kernel):
    """With the test flag set, the loading warp issues nothing: every consumer's
    bounded wait runs out after wait_us, the kernel skips its work and writes a
    timeout code.  The check raises, the word is cleared, and the next normal
    launch on the same context is correct and clean."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dt = torch.bfloat16
    B, T = 1, 256
    q, k, v, pre, post = O.make_inputs(B, T, 32, 128, G, 1, seed=77)
    to = lambda x: _dev(x, torch.float32).to(dt)
    terms = lambda t: dc.DCTerms(identity=t.identity, w=torch.from_numpy(t.w).to(DEV), qw1=to(t.qw1),
                                 qw2=to(t.qw2), kw1=to(t.kw1), kw2=to(t.kw2), qdd=to(t.qdd), kdd=to(t.kdd))
    qd, kd, vd = to(q), to(k), to(v)
    assert dc.device_error() == 0
    with pytest.raises(RuntimeError, match="TIMEOUT"):
        dc.dc_attn_fwd(qd, kd, vd, terms(pre), terms(post), 128 ** -0.5, window, G, kernel=kernel,
                       check=True, wait_us=2000, test_flags=_lib.DC_TEST_SKIP_LOADS)
    assert dc.device_error() == 0  # the check cleared it
    # the same launch again, read through the explicit poll instead of check=True
    dc.dc_attn_fwd(qd, kd, vd, terms(pre), terms(post), 128 ** -0.5, window, G, kernel=kernel,
                   wait_us=2000, test_flags=_lib.DC_TEST_SKIP_LOADS)
    code = dc.device_error(clear=False)
    assert code in _lib.DEV_ERRORS and code != 0
    assert dc.device_error(clear=True) == code
    assert dc.device_error() == 0
    got = dc.dc_attn_fwd(qd, kd, vd, terms(pre), terms(post), 128 ** -0.5, window, G, kernel=kernel, check=True)
    rd = lambda x: to(x).float().cpu().numpy()
    rt = lambda t: O.Terms(identity=t.identity, w=t.w, qw1=rd(t.qw1), qw2=rd(t.qw2), kw1=rd(t.kw1),
                           kw2=rd(t.kw2), qdd=rd(t.qdd), kdd=rd(t.kdd))
    ref = O.dc_attn_oracle(rd(q), rd(k), rd(v), rt(pre), rt(post), 128 ** -0.5, window, G)
    assert_close(got.float().cpu().numpy(), ref, f"after timeout {kernel}")


# ---------------------------------------------------------------- host entry point, back to back

def test_host_entry_back_to_back_calls():
    """Two dc_attn_fwd_host calls with different inputs, issued back to back
    with no synchronisation in between, reuse the same staging slots: each
    output must equal the device entry point's bit for bit."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dt = torch.bfloat16
    outs, refs = [], []
    calls = []
    for seed in (11, 12, 13):
        q, k, v, pre, post = O.make_inputs(4, 128, 32, 128, 8, 1, seed=seed)
        to = lambda x: _dev(x, torch.float32).to(dt)
        terms = lambda t: dc.DCTerms(identity=t.identity, w=torch.from_numpy(t.w).to(DEV), qw1=to(t.qw1),
                                     qw2=to(t.qw2), kw1=to(t.kw1), kw2=to(t.kw2), qdd=to(t.qdd), kdd=to(t.kdd))
        qd, kd, vd, pre_d, post_d = to(q), to(k), to(v), terms(pre), terms(post)
        refs.append(dc.dc_attn_fwd(qd, kd, vd, pre_d, post_d, 128 ** -0.5, 112, 8).cpu())
        host = lambda tm: dc.DCTerms(identity=tm.identity, w=tm.w.cpu(), **{
            f: getattr(tm, f).cpu().pin_memory() for f in ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd")})
        calls.append((qd.cpu().pin_memory(), kd.cpu().pin_memory(), vd.cpu().pin_memory(), host(pre_d),
                      host(post_d)))
    torch.cuda.synchronize()
    for qh, kh, vh, pre_h, post_h in calls:  # no sync between the calls
        outs.append(dc.dc_attn_fwd_host(qh, kh, vh, pre_h, post_h, 128 ** -0.5, 112, 8, chunks=2))
    torch.cuda.synchronize()
    for i, (o, r) in enumerate(zip(outs, refs)):
        assert torch.equal(o, r), f"call {i}"
