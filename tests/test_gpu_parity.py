"""Parity of the CUDA kernels with the oracle and the reference's golden vectors.

Every call goes through the library's C ABI (ctypes -> libdcattn.so); the
oracle in oracle/dc_oracle.py is only the checker.  Tolerances: tests/tolerances.py.
"""

import numpy as np
import pytest
import torch

import dc_triton_opt_b200 as dc
from dc_triton_opt_b200 import dc_hopper_cuda, onekernel
from oracle import dc_oracle as O
from tests.golden_cases import load_cases
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TORCH_DT = {"bf16": torch.bfloat16, "fp16": torch.float16}
KERNELS = ["simt", "auto"]


def T_(x, dt):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to(DEV).to(dt)


def to_dcterms(t: O.Terms, dt) -> dc.DCTerms:
    return dc.DCTerms(identity=t.identity, w=T_(t.w, torch.float32), qw1=T_(t.qw1, dt), qw2=T_(t.qw2, dt),
                      kw1=T_(t.kw1, dt), kw2=T_(t.kw2, dt), qdd=T_(t.qdd, dt), kdd=T_(t.kdd, dt),
                      qmat=T_(t.qmat, dt))


def round_terms(t: O.Terms, dt) -> O.Terms:
    """Round a term set's per-token tensors to the kernel dtype (w stays fp32)."""
    r = O.Terms(identity=t.identity, w=t.w)
    for n in ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd", "qmat"):
        a = getattr(t, n)
        if a is not None:
            setattr(r, n, torch.from_numpy(np.ascontiguousarray(a)).to(dt).float().numpy())
    return r


def rnd(x, dt):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dt).float().numpy()


def run_general(q, k, v, pre, post, scale, window, G, seq_lens=None, dtype="bf16", kernel="auto"):
    dt = TORCH_DT[dtype]
    out = dc.dc_attn_fwd(T_(q, dt), T_(k, dt), T_(v, dt), to_dcterms(pre, dt), to_dcterms(post, dt), scale,
                         window, G, None if seq_lens is None else torch.tensor(seq_lens, device=DEV),
                         kernel=kernel)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


# ---------------------------------------------------------------- golden vectors

@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("case", load_cases(), ids=lambda c: c.name)
def test_golden(case, kernel):
    dt = TORCH_DT[case.dtype]
    q, k, v = (T_(x, dt) for x in (case.q, case.k, case.v))
    sl = None if case.seq_lens is None else torch.tensor(case.seq_lens, device=DEV)
    if case.kind in ("grouped", "residual"):
        ws = tuple(T_(w, dt) for w in case.ws)
        if kernel == "auto" and case.kind == "grouped":
            got = dc.dc_attention_window_chunked_residual_grouped(q, k, v, ws, case.scale, case.window, sl,
                                                                  case.chunk, G=case.G)
        elif kernel == "auto":
            got = dc.dc_attention_window_chunked_residual(q, k, v, ws, case.scale, case.window, sl, case.chunk)
        else:
            got = dc.dc_attn_fwd(q, k, v, dc.DCTerms.residual(*ws[:3]), dc.DCTerms.residual(*ws[3:]),
                                 case.scale, case.eff_window, case.G, sl, kernel=kernel).permute(0, 2, 1, 3)
    elif case.kind == "decomposed":
        pw, qw = T_(case.pre_w, dt), T_(case.post_w, dt)
        if kernel == "auto":
            got = dc.dc_attention_decomposed_window_chunked(q, k, v, pw, qw, case.scale, case.window, sl,
                                                            case.chunk)
        else:
            got = dc.dc_attn_fwd(q, k, v, dc.DCTerms(qmat=pw), dc.DCTerms(qmat=qw), case.scale,
                                 min(case.window, case.T), 1, sl, kernel=kernel)
    else:
        got = dc.dc_attn_fwd(q, k, v, to_dcterms(case.pre, dt), to_dcterms(case.post, dt), case.scale,
                             case.window, case.G, sl, kernel=kernel)
    torch.cuda.synchronize()
    assert_close(got.float().cpu().numpy(), case.out, case.name)


# ---------------------------------------------------------------- general terms

GENERAL = [
    # B, T, H, G, R, window, terms, seq_lens
    (1, 96, 8, 2, 1, 32, ("w", "qw", "kw", "qdd", "kdd"), None),
    (2, 80, 8, 1, 2, 24, ("w", "qw", "kw", "qdd", "kdd"), [80, 41]),
    (1, 64, 8, 8, 2, 16, ("w", "qw", "kw", "qdd", "kdd"), None),   # HPG=1
    (1, 130, 8, 2, 1, None, ("w", "qw", "kw", "qdd", "kdd"), None),  # full causal, ragged T
    (1, 64, 16, 1, 1, 1, ("w", "qw", "kw", "qdd", "kdd"), None),   # window 1 (self only)
    (1, 72, 8, 2, 2, 40, ("qw", "kw"), None),                      # identity + rank terms only
]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("B,T,H,G,R,window,terms,seq_lens", GENERAL)
def test_general_terms(B, T, H, G, R, window, terms, seq_lens, kernel, dtype):
    dt = TORCH_DT[dtype]
    q, k, v, pre, post = O.make_inputs(B, T, H, 128, G, R, seed=B * 1000 + T + G, terms=terms)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.dc_attn_oracle(q, k, v, pre, post, 128 ** -0.5, window, G, seq_lens)
    got = run_general(q, k, v, pre, post, 128 ** -0.5, window, G, seq_lens, dtype, kernel)
    assert_close(got, ref, f"B{B} T{T} H{H} G{G} R{R} W{window} {kernel} {dtype}")


@pytest.mark.parametrize("kernel", KERNELS)
def test_config0_shape(kernel):
    """BASELINE config 0 shape (B2 T512 H32 D128 G1 W128 R1, every term), bf16 inputs."""
    dt = torch.bfloat16
    q, k, v, pre, post = O.make_inputs(2, 512, 32, 128, 1, 1, seed=0)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.dc_attn_oracle(q, k, v, pre, post, 128 ** -0.5, 128, 1, None, chunk=128)
    got = run_general(q, k, v, pre, post, 128 ** -0.5, 128, 1, None, "bf16", kernel)
    assert_close(got, ref, f"config0 {kernel}")


@pytest.mark.parametrize("G", [1, 2, 4, 8, 16, 32])
def test_group_sweep_small(G):
    """Every G of the BASELINE sweep (HPG = 32/G) at a small T, auto kernel."""
    dt = torch.bfloat16
    q, k, v, pre, post = O.make_inputs(1, 160, 32, 128, G, 1, seed=G)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.dc_attn_oracle(q, k, v, pre, post, 128 ** -0.5, 64, G, None)
    got = run_general(q, k, v, pre, post, 128 ** -0.5, 64, G)
    assert_close(got, ref, f"G{G}")


# ---------------------------------------------------------------- API surfaces

def _residual_inputs(B, T, N, std, dt, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, T, N, 128, generator=g).to(dt).to(DEV) for _ in range(3))
    ws = tuple((std * torch.randn(B, T, N, generator=g)).to(dt).to(DEV) for _ in range(6))
    return q, k, v, ws


def _oracle_residual(q, k, v, ws, scale, window, G):
    f = lambda x: x.float().cpu().numpy()
    return O.grouped_residual(f(q), f(k), f(v), [f(w) for w in ws], scale, window, None, None, G)


def test_hopper_api_matches_oracle():
    """dc_hopper_cuda.forward_hpg4_wide_* with the reference test's own cases
    (test_dc_hopper_cuda.py:171-175 shapes at B=1, std-1 weights, fp16)."""
    for T, BM, W in ((256, 32, 224), (256, 16, 240)):
        q, k, v, ws = _residual_inputs(1, T, 32, 1.0, torch.float16, T + BM)
        ref = _oracle_residual(q, k, v, ws, 128 ** -0.5, W, 8).transpose(0, 2, 1, 3)
        for fn in (dc_hopper_cuda.forward_hpg4_wide_ref, dc_hopper_cuda.forward_hpg4_wide_opt,
                   dc_hopper_cuda.forward_hpg4_wide_cluster):
            got = fn(q, k, v, *ws, 128 ** -0.5, W, BM)
            torch.cuda.synchronize()
            assert got.shape == (1, T, 32, 128)
            assert_close(got.float().cpu().numpy(), ref, f"{fn.__name__} T{T} BM{BM} W{W}")


def test_onekernel_class_matches_grouped():
    q, k, v, ws = _residual_inputs(2, 192, 32, 0.1, torch.bfloat16, 11)
    a = onekernel.TritonDCOneKernelMixedProbs.forward(q, k, v, ws, 128 ** -0.5, 112, None, G=8, chunk_size=16)
    b = dc.dc_attention_window_chunked_residual_grouped(q, k, v, ws, 128 ** -0.5, 112, G=8)
    torch.cuda.synchronize()
    assert torch.equal(a, b.permute(0, 2, 1, 3))


def test_output_layout_strided():
    q, k, v, ws = _residual_inputs(1, 64, 8, 0.1, torch.bfloat16, 12)
    out = dc.dc_attention_window_chunked_residual_grouped(q, k, v, ws, 0.1, 16, G=2)
    assert out.shape == (1, 8, 64, 128) and out.is_contiguous()
    flat = dc.dc_attn_fwd(q, k, v, dc.DCTerms.residual(*ws[:3]), dc.DCTerms.residual(*ws[3:]), 0.1, 16, 2)
    torch.cuda.synchronize()
    assert torch.equal(out.permute(0, 2, 1, 3), flat)


def test_all_masked_rows_zero():
    """seq_len 3 with window 4: queries t >= 6 see no key -> exact zeros (NaN-free)."""
    q, k, v, ws = _residual_inputs(1, 32, 8, 0.1, torch.bfloat16, 13)
    out = dc.dc_attn_fwd(q, k, v, dc.DCTerms.residual(*ws[:3]), dc.DCTerms.residual(*ws[3:]), 0.1, 4, 2,
                         torch.tensor([3], device=DEV))
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert (out[0, 6:] == 0).all()


def test_bad_arguments_raise():
    q, k, v, ws = _residual_inputs(1, 32, 8, 0.1, torch.bfloat16, 14)
    with pytest.raises(RuntimeError, match="divisible"):
        dc.dc_attn_fwd(q, k, v, G=3)
    with pytest.raises(RuntimeError, match="shape"):
        dc.dc_attn_fwd(q, k, v, dc.DCTerms(qdd=ws[0][:, :16]))
    with pytest.raises(RuntimeError, match="only N=32"):
        dc_hopper_cuda.forward_hpg4_wide_ref(q, k, v, *ws, 0.1, 224, 32)


def test_stream_semantics():
    """The launch goes on the caller's current stream."""
    q, k, v, ws = _residual_inputs(1, 128, 32, 0.1, torch.bfloat16, 15)
    ref = dc.dc_attention_window_chunked_residual_grouped(q, k, v, ws, 0.1, 64, G=8)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        got = dc.dc_attention_window_chunked_residual_grouped(q, k, v, ws, 0.1, 64, G=8)
    s.synchronize()
    assert torch.equal(ref, got)


@pytest.mark.parametrize("G,window,expect", [(8, 128, "tc"), (4, 256, "tc"), (32, 128, "tc"), (16, 200, "tc"),
                                              (1, 128, "tcm"), (1, None, "tcm"), (8, None, "tcs"), (2, 128, "tcm"),
                                              (8, 1024, "tcs")])
def test_auto_dispatch(G, window, expect):
    """AUTO picks the single-pass tensor-core kernel for windows within three key
    tiles and <= 8 heads per group, the tensor-core-mix streaming kernel for 16
    or 32 heads per group, and the streaming kernel for the other full-causal
    layers and long windows."""
    q = torch.empty(1, 64, 32, 128, dtype=torch.bfloat16, device=DEV)
    pre = dc.DCTerms(qw1=torch.empty(1, 64, 32, 1, dtype=torch.bfloat16, device=DEV),
                     qw2=torch.empty(1, 64, 1, 32, dtype=torch.bfloat16, device=DEV))
    assert dc.select_kernel(q, q, q, pre, pre, window, G) == expect


@pytest.mark.parametrize("G,R,window,T", [(8, 1, 128, 320), (4, 2, 256, 300), (32, 1, 96, 200), (32, 2, 128, 260),
                                          (16, 1, 240, 280), (8, 2, 1, 64)])
def test_tc_kernel_vs_oracle(G, R, window, T):
    """Tensor-core kernel, every term, ragged T, BASELINE distributions."""
    dt = torch.bfloat16
    q, k, v, pre, post = O.make_inputs(1, T, 32, 128, G, R, seed=G * 7 + R)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.dc_attn_oracle(q, k, v, pre, post, 128 ** -0.5, window, G, None)
    got = run_general(q, k, v, pre, post, 128 ** -0.5, window, G, None, "bf16", "tc")
    assert_close(got, ref, f"tc G{G} R{R} W{window} T{T}")


@pytest.mark.parametrize("G,R,window,T,B,seq_lens", [
    (8, 1, None, 300, 1, None),      # full causal, HPG 4, ragged T, 3 key tiles at the end
    (4, 2, None, 260, 2, [260, 131]),  # full causal, HPG 8, seq_lens
    (4, 1, 128, 200, 1, None),       # HPG 8 windowed
    (32, 1, 500, 700, 1, None),      # HPG 1, window longer than three key tiles
    (16, 2, 64, 96, 1, None),        # HPG 2, one key tile
    (8, 1, 1, 64, 1, None),          # window 1
])
def test_tcs_kernel_vs_oracle(G, R, window, T, B, seq_lens):
    """Two-pass streaming tensor-core kernel, every term, BASELINE distributions."""
    dt = torch.bfloat16
    q, k, v, pre, post = O.make_inputs(B, T, 32, 128, G, R, seed=G * 11 + R + T)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.dc_attn_oracle(q, k, v, pre, post, 128 ** -0.5, window, G, seq_lens)
    got = run_general(q, k, v, pre, post, 128 ** -0.5, window, G, seq_lens, "bf16", "tcs")
    assert_close(got, ref, f"tcs G{G} R{R} W{window} T{T}")


def test_tcs_matches_tc_on_windowed_layer():
    """Both tensor-core kernels on the same windowed layer agree closely."""
    dt = torch.bfloat16
    q, k, v, pre, post = O.make_inputs(1, 384, 32, 128, 8, 1, seed=99)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    a = run_general(q, k, v, pre, post, 128 ** -0.5, 128, 8, None, "bf16", "tc")
    b = run_general(q, k, v, pre, post, 128 ** -0.5, 128, 8, None, "bf16", "tcs")
    assert_close(a, b, "tc vs tcs", max_abs=2e-2)


@pytest.mark.parametrize("H,G,R,window,T,B,seq_lens,dtype", [
    (32, 1, 1, 128, 200, 1, None, "bf16"),          # config-0 layer shape, ragged T
    (32, 1, 2, None, 300, 1, None, "bf16"),         # full causal, five key tiles at the end
    (32, 1, 1, 64, 150, 2, [150, 77], "fp16"),      # seq_lens, fp16
    (64, 2, 1, 100, 130, 1, None, "bf16"),          # two groups of 32 (head offset of the key weights)
    (32, 1, 2, 1, 40, 1, None, "bf16"),             # window 1
    (32, 2, 1, 128, 260, 1, None, "bf16"),          # 16 heads per group
    (32, 2, 2, None, 200, 2, [200, 90], "fp16"),    # 16 heads per group, full causal, seq_lens
    (32, 2, 2, 256, 300, 1, None, "bf16"),          # 16 heads per group, config-2 window
])
def test_tcm_kernel_vs_oracle(H, G, R, window, T, B, seq_lens, dtype):
    """Streaming kernel with the static head mix as a tcgen05 MMA, every term."""
    dt = TORCH_DT[dtype]
    q, k, v, pre, post = O.make_inputs(B, T, H, 128, G, R, seed=H + G * 3 + R + T)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.dc_attn_oracle(q, k, v, pre, post, 128 ** -0.5, window, G, seq_lens)
    got = run_general(q, k, v, pre, post, 128 ** -0.5, window, G, seq_lens, dtype, "tcm")
    assert_close(got, ref, f"tcm H{H} G{G} R{R} W{window} T{T}")


@pytest.mark.parametrize("G,B,seq_lens,chunks", [(8, 5, [64, 30, 64, 1, 50], 4), (1, 3, None, 2), (8, 1, None, 4)])
def test_host_entry_point_matches_device(G, B, seq_lens, chunks):
    """dc_attn_fwd_host (host tensors, batch pipelined over streams) equals the
    device entry point bit for bit, ragged last chunk and seq_lens included."""
    dt = torch.bfloat16
    q, k, v, pre, post = O.make_inputs(B, 64, 32, 128, G, 1, seed=G + B)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    sl = None if seq_lens is None else torch.tensor(seq_lens, dtype=torch.int32)
    qd, kd, vd = (T_(x, dt) for x in (q, k, v))
    pre_d, post_d = to_dcterms(pre, dt), to_dcterms(post, dt)
    ref = dc.dc_attn_fwd(qd, kd, vd, pre_d, post_d, 128 ** -0.5, 48, G, None if sl is None else sl.to(DEV))
    host = lambda tm: dc.DCTerms(identity=tm.identity, w=tm.w, **{f: (None if getattr(tm, f) is None else
                                 getattr(tm, f).cpu().pin_memory()) for f in ("qw1", "qw2", "kw1", "kw2",
                                                                             "qdd", "kdd")})
    got = dc.dc_attn_fwd_host(qd.cpu().pin_memory(), kd.cpu().pin_memory(), vd.cpu().pin_memory(),
                              host(pre_d), host(post_d), 128 ** -0.5, 48, G, sl, chunks=chunks)
    torch.cuda.synchronize()
    assert torch.equal(got, ref.cpu())


@pytest.mark.parametrize("G", [8, 32, 4, 16])
def test_persistent_kernel_many_tiles_per_cta(G):
    """More tiles than SMs, so each persistent CTA walks tiles of several batches
    and head groups (each group with its own static mix): every tile must use
    its own group's weights."""
    dt = torch.bfloat16
    B, T = 8, 640
    q, k, v, pre, post = O.make_inputs(B, T, 32, 128, G, 1, seed=500 + G, mix_std=0.05)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.dc_attn_oracle(q, k, v, pre, post, 128 ** -0.5, 128, G, None)
    got = run_general(q, k, v, pre, post, 128 ** -0.5, 128, G, None, "bf16", "tc")
    assert_close(got, ref, f"persistent G{G} B{B} T{T}")


# ---------------------------------------------------------------- per-query mixing matrices (qmat)

def _with_qmat(pre, post, B, T, H, G, seed, decomposed=False):
    """Add a per-query mix qmat [B,T,H,HPG] to both sets.  decomposed=True gives
    the reference's decomposed form instead: no identity, no other term, and
    qmat = I + N(0, 0.05) (dc_attention_torch.py:22-84 folds the residual into
    its matrices)."""
    rng = np.random.default_rng(seed)
    hpg = H // G
    out = []
    for t in (pre, post):
        qm = (0.05 * rng.standard_normal((B, T, H, hpg))).astype(np.float32)
        if decomposed:
            qm += np.tile(np.eye(hpg, dtype=np.float32), (G, 1))[None, None]
            t = O.Terms(identity=False)
        t.qmat = qm
        out.append(t)
    return out


@pytest.mark.parametrize("kernel,G,window,T,R", [
    ("tc", 8, 128, 200, 1),    # persistent kernel, HPG 4
    ("tc", 32, 96, 150, 1),    # persistent kernel, HPG 1
    ("tc", 16, 128, 300, 2),   # persistent kernel, HPG 2
    ("tc", 4, 256, 300, 2),    # one-tile-per-CTA kernel, three key tiles, HPG 8
    ("tcs", 8, None, 260, 1),  # streaming kernel, full causal
    ("tcm", 1, 128, 200, 1),   # tensor-core mix, 32 heads per group
    ("tcm", 2, None, 150, 2),  # tensor-core mix, 16 heads per group, full causal
])
@pytest.mark.parametrize("decomposed", [False, True])
def test_qmat_tensor_core_kernels(kernel, G, window, T, R, decomposed):
    """Per-query mixing matrices on every tensor-core kernel: folded into the
    per-query matrices (tc, tcs) or, at 16/32 heads per group, a per-query mix
    operand of the tcgen05 mix MMA (off-diagonal entries in fp16, diagonal in
    fp32)."""
    dt = torch.bfloat16
    q, k, v, pre, post = O.make_inputs(1, T, 32, 128, G, R, seed=G * 13 + T)
    pre, post = _with_qmat(pre, post, 1, T, 32, G, seed=T + G, decomposed=decomposed)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.dc_attn_oracle(q, k, v, pre, post, 128 ** -0.5, window, G, None)
    got = run_general(q, k, v, pre, post, 128 ** -0.5, window, G, None, "bf16", kernel)
    assert_close(got, ref, f"qmat {kernel} G{G} W{window} T{T} decomposed={decomposed}")


def test_decomposed_form_runs_on_tensor_cores():
    """The reference's decomposed entry point (N x N per-query matrices, G = 1)
    at the config-0 layer shape goes to the tensor-core mix kernel, not the
    CUDA-core one, and matches the oracle."""
    dt = torch.bfloat16
    B, T, N, W = 1, 512, 32, 128
    q, k, v, pre, post = O.make_inputs(B, T, N, 128, 1, 1, seed=5)
    pre, post = _with_qmat(pre, post, B, T, N, 1, seed=6, decomposed=True)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    ref = O.decomposed(q, k, v, pre.qmat, post.qmat, 128 ** -0.5, W, np.full(B, T))
    qd, kd, vd = T_(q, dt), T_(k, dt), T_(v, dt)
    pw, qw = T_(pre.qmat, dt), T_(post.qmat, dt)
    assert dc.select_kernel(qd, kd, vd, dc.DCTerms(qmat=pw), dc.DCTerms(qmat=qw), W, 1) == "tcm"
    got = dc.dc_attention_decomposed_window_chunked(qd, kd, vd, pw, qw, 128 ** -0.5, W,
                                                    torch.full((B,), T, device=DEV, dtype=torch.int32), 64)
    torch.cuda.synchronize()
    assert_close(got.float().cpu().numpy(), ref, "decomposed on tcm")


def test_fp32_inputs_through_the_drop_ins():
    """The reference's torch functions are dtype-generic; fp32 callers of the
    drop-ins get an fp32 result computed from the bf16-rounded inputs."""
    case = next(c for c in load_cases() if c.kind == "grouped")
    f32 = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV).float()
    q, k, v = f32(case.q), f32(case.k), f32(case.v)
    ws = [f32(w) for w in case.ws]
    got = dc.dc_attention_window_chunked_residual_grouped(q, k, v, ws, case.scale, case.window, None,
                                                          case.chunk, G=case.G)
    assert got.dtype == torch.float32
    bq, bk, bv = (x.bfloat16() for x in (q, k, v))
    want = dc.dc_attention_window_chunked_residual_grouped(bq, bk, bv, [w.bfloat16() for w in ws], case.scale,
                                                           case.window, None, case.chunk, G=case.G)
    torch.cuda.synchronize()
    assert torch.equal(got, want.float())
    if case.seq_lens is None:
        assert_close(got.cpu().numpy(), case.out, "fp32 drop-in")
    case = next(c for c in load_cases() if c.kind == "decomposed")
    sl = torch.tensor(case.seq_lens if case.seq_lens is not None else [case.T] * case.q.shape[0], device=DEV)
    got = dc.dc_attention_decomposed_window_chunked(f32(case.q), f32(case.k), f32(case.v), f32(case.pre_w),
                                                    f32(case.post_w), case.scale, case.window, sl, case.chunk)
    torch.cuda.synchronize()
    assert got.dtype == torch.float32
    assert_close(got.cpu().numpy(), case.out, "fp32 decomposed drop-in")


# ---------------------------------------------------------------- packed variable-length batches

@pytest.mark.parametrize("lens,H,G,R,window", [
    ([37, 64, 64, 0, 130, 5], 32, 8, 1, 128),   # tc, equal-length run, empty and 5-token sequences
    ([90, 33, 33, 33], 32, 1, 2, 64),           # tcm (32 heads per group)
    ([200, 77], 32, 8, 2, None),                # full causal (streaming kernel)
])
def test_varlen_matches_each_sequence(lens, H, G, R, window):
    """dc_attn_fwd_varlen on a packed batch equals the oracle run on every
    sequence alone (no attention across sequence boundaries)."""
    dt = torch.bfloat16
    total = sum(lens)
    q, k, v, pre, post = O.make_inputs(1, total, H, 128, G, R, seed=total + G)
    q, k, v = rnd(q, dt), rnd(k, dt), rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    sq = lambda t: dc.DCTerms(identity=t.identity, w=T_(t.w, torch.float32),
                              **{f: (None if getattr(t, f) is None else T_(getattr(t, f)[0], dt))
                                 for f in ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd")})
    got = dc.dc_attn_fwd_varlen(T_(q[0], dt), T_(k[0], dt), T_(v[0], dt), cu, sq(pre), sq(post), 128 ** -0.5,
                                window, G)
    torch.cuda.synchronize()
    got = got.float().cpu().numpy()
    for i, L in enumerate(lens):
        if L == 0:
            continue
        a, b = cu[i], cu[i + 1]
        cut = lambda t: O.Terms(identity=t.identity, w=t.w, **{f: (None if getattr(t, f) is None else
                                                                   getattr(t, f)[:, a:b])
                                                                for f in ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd")})
        ref = O.dc_attn_oracle(q[:, a:b], k[:, a:b], v[:, a:b], cut(pre), cut(post), 128 ** -0.5, window, G, None)
        assert_close(got[a:b], ref[0], f"varlen seq {i} len {L}")


# ---------------------------------------------------------------- fp8 (e4m3) q and k

@pytest.mark.parametrize("G,R,window,T,B", [(8, 1, 128, 300, 1), (32, 2, 96, 200, 2), (4, 2, 256, 260, 1),
                                             (16, 1, 128, 130, 1)])
def test_fp8_qk_matches_oracle_on_dequantized_inputs(G, R, window, T, B):
    """QK^T in e4m3 on the tensor cores: the result equals the oracle run on the
    dequantized q and k (q8 * q_scale), under the usual tolerance."""
    dt = torch.bfloat16
    q, k, v, pre, post = O.make_inputs(B, T, 32, 128, G, R, seed=G + T + R)
    v = rnd(v, dt)
    pre, post = round_terms(pre, dt), round_terms(post, dt)
    q8, qs = dc.quantize_e4m3(torch.from_numpy(q).to(DEV))
    k8, ks = dc.quantize_e4m3(torch.from_numpy(k).to(DEV))
    qd = (q8.float() * qs).cpu().numpy()
    kd = (k8.float() * ks).cpu().numpy()
    ref = O.dc_attn_oracle(qd, kd, v, pre, post, 128 ** -0.5, window, G, None)
    got = dc.dc_attn_fwd_fp8qk(q8, k8, T_(v, dt), qs, ks, to_dcterms(pre, dt), to_dcterms(post, dt), 128 ** -0.5,
                               window, G)
    torch.cuda.synchronize()
    assert_close(got.float().cpu().numpy(), ref, f"fp8 G{G} R{R} W{window} T{T}")


def test_golden_h32_case_runs_on_the_tensor_core_mix_kernel():
    """The 32-heads-per-group golden case (made by the reference's own function)
    pins the tensor-core-mix kernel directly: AUTO picks it for that shape."""
    case = next(c for c in load_cases() if c.name == "residual_h32")
    q = T_(case.q, torch.bfloat16)
    ws = tuple(T_(w, torch.bfloat16) for w in case.ws)
    assert dc.select_kernel(q, q, q, dc.DCTerms.residual(*ws[:3]), dc.DCTerms.residual(*ws[3:]),
                            case.eff_window, 1) == "tcm"
