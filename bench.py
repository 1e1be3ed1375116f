"""Benchmark of the B200 DC-attention forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config1|config2|config3|config4] [--G g] [--window w]

A step is one fused DC-attention forward over one batch of the workload (the
metric of the reference: µs/call and effective TFLOP/s).  ``value`` is the
whole-job TFLOP/s (algorithmic FLOPs of every rank / max-over-ranks device
time), inputs resident in HBM (2.2 GB at the default workload: larger than
L2, so no flush is needed).  ``e2e`` is the same metric through the public
API with pinned host buffers copied in and the output copied back inside the
timed region.  ``--impl reference`` times the CPU restatement of the
reference algorithm (oracle/dc_oracle_torch.py, fp32, all host threads) on a
bounded sample of the same workload; under torchrun only rank 0 runs it.

Workloads (synthetic, seeded, BASELINE distributions):
  config1  B16 T4096 H32 D128 window 128, R1, G8 (HPG 4; G sweep via --G)
  config2  B16 T4096 H32 D128 window 256, R2 (--G in {1,4,32})
  config3  B4  T4096 H32 D128 full causal, G4, R2
  config4  B64 T8192 H32 D128 window 256, G1, R2, batch split over the ranks
Multi-GPU: configs 1-3 give every rank the full workload (weak scaling);
config4 splits its batch (strong scaling).  No collective touches the data
path: the op has no cross-batch dependency.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

WORKLOADS = {
    "config1": dict(B=16, T=4096, H=32, D=128, window=128, G=8, R=1),
    "config2": dict(B=16, T=4096, H=32, D=128, window=256, G=1, R=2),
    "config3": dict(B=4, T=4096, H=32, D=128, window=None, G=4, R=2),
    "config4": dict(B=64, T=8192, H=32, D=128, window=256, G=1, R=2),
    # the reference's decomposed form (dc_attention_torch.py:22-84): per-query
    # N x N mixing matrices (qmat = I + N(0, 0.05)) and no other term, at the
    # config-1 layer shape
    "decomposed": dict(B=16, T=4096, H=32, D=128, window=128, G=1, R=0, qmat=True),
}
FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS = 6650.0, 1590.0


def pairs(T, W):
    if W is None or W >= T:
        return T * (T + 1) // 2
    return T * W - W * (W - 1) // 2


def pairs_range(t0, t1, W):
    return sum(t + 1 if (W is None or t + 1 < W) else W for t in range(t0, t1))


def flops(B, H, D, G, R, npairs, qmat=False):
    """Algorithmic FLOPs: QK^T + PV, plus pre+post composition (static mix 2*HPG,
    query- and key-wise rank-R aggregate+apply 8R, qdd/kdd 4) per (b,h,t,s);
    with qmat (the decomposed form) the composition is the per-query mix alone
    (2*HPG per set)."""
    hpg = H // G
    comp = 2 * hpg if qmat else 2 * hpg + 8 * R + 4
    return 4 * D * H * B * npairs + 2 * comp * H * B * npairs


def algo_bytes(B, T, H, D, R, esize=2):
    """q,k,v read once + out written once, plus the two sets of per-token
    weights (qw1, qw2, kw1, kw2: R each; qdd, kdd)."""
    return 4 * B * T * H * D * esize + 2 * (4 * R + 2) * B * T * H * esize


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), float(m["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def make_inputs(cfg, device, dtype=torch.bfloat16, seed=0):
    from dc_triton_opt_b200 import DCTerms
    B, T, H, D, G, R = (cfg[k] for k in ("B", "T", "H", "D", "G", "R"))
    hpg = H // G
    g = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g, device=device, dtype=torch.float32)
    q, k, v = (rn(B, T, H, D).to(dtype) for _ in range(3))
    sets = []
    if cfg.get("qmat"):
        eye = torch.eye(hpg, device=device).repeat(G, 1)
        for _ in range(2):
            sets.append(DCTerms(identity=False, qmat=(eye + 0.05 * rn(B, T, H, hpg)).to(dtype)))
        return q, k, v, sets[0], sets[1]
    for _ in range(2):
        sets.append(DCTerms(
            identity=False, w=torch.eye(hpg, device=device)[None] + 0.02 * rn(G, hpg, hpg),
            qw1=(0.1 * rn(B, T, H, R)).to(dtype), qw2=(0.1 * rn(B, T, R, H)).to(dtype),
            kw1=(0.1 * rn(B, T, H, R)).to(dtype), kw2=(0.1 * rn(B, T, R, H)).to(dtype),
            qdd=(0.1 * rn(B, T, H)).to(dtype), kdd=(0.1 * rn(B, T, H)).to(dtype)))
    return q, k, v, sets[0], sets[1]


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, val in zip(names, r[5:9]) if "Active" in val
                          and "Not" not in val})
        load = [s for s in sm if s > 0.5 * (max(mx) if mx else 1)] or sm
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


from dc_triton_opt_b200.shard import max_over_ranks, shard_batch  # noqa: E402


_CPU_INPUTS = {}


def cpu_port_sample(cfg, target_s=12.0, threads=None):
    """Time the torch-CPU restatement on batch 0, a bounded query range, repeated
    until ~target_s seconds; returns (TFLOP/s, cores, sample description)."""
    from oracle.dc_oracle import make_inputs as np_inputs
    from oracle.dc_oracle_torch import dc_attn_torch_cpu
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    T, H, D, G, R, W = cfg["T"], cfg["H"], cfg["D"], cfg["G"], cfg["R"], cfg["window"]
    t0, t1 = (T - 512, T) if W is not None else (T - 256, T)
    key = (T, H, D, G, R)
    if key not in _CPU_INPUTS:
        _CPU_INPUTS[key] = np_inputs(1, T, H, D, G, R, seed=0)
        q, k, v, pre, post = _CPU_INPUTS[key]
        dc_attn_torch_cpu(q, k, v, pre, post, D ** -0.5, W, G, None, t_range=(t1 - 64, t1))  # warm
    q, k, v, pre, post = _CPU_INPUTS[key]
    scale = D ** -0.5
    n, start = 0, time.perf_counter()
    while True:
        dc_attn_torch_cpu(q, k, v, pre, post, scale, W, G, None, t_range=(t0, t1))
        n += 1
        el = time.perf_counter() - start
        if el >= target_s:
            break
    fl = flops(1, H, D, G, R, pairs_range(t0, t1, W)) * n
    sample = (f"batch 1 of {cfg['B']}, queries [{t0},{t1}) of T={T}, all {H} heads; "
              f"{n} calls in {el:.1f} s (fp32 torch CPU, oracle/dc_oracle_torch.py)")
    return fl / el / 1e12, threads, sample


def run_reference(args, cfg, world, rank):
    if world > 1 and rank != 0:
        return
    vals = []
    for _ in range(args.warmup + args.steps):
        v, cores, sample = cpu_port_sample(cfg, target_s=max(2.0, 30.0 / max(1, args.steps + args.warmup)))
        vals.append(v)
    val = statistics.median(vals[args.warmup:]) if len(vals) > args.warmup else vals[-1]
    line = {
        "impl": "reference", "metric": "DC-attn fwd effective TFLOP/s", "value": val, "unit": "TFLOP/s",
        "n_gpus": 0, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "dtype": "f32", "data": "synthetic", "config": config_desc(args, cfg, world),
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }
    print(json.dumps(line), flush=True)


def config_desc(args, cfg, world):
    d = {"workload": args.workload, "B": cfg["B"], "T": cfg["T"], "H": cfg["H"], "D": cfg["D"],
         "window": cfg["window"] if cfg["window"] is not None else "full_causal", "G": cfg["G"],
         "HPG": cfg["H"] // cfg["G"], "R": cfg["R"],
         "terms": ("per-query N x N mixing matrices only (decomposed form, pre and post)" if cfg.get("qmat") else
                   "static W + query- and key-wise rank R + qdd + kdd (pre and post)"),
         "l2": "inputs larger than L2 (no flush)", "parallelism": f"batch-sharded x{world}, no collectives"}
    return d


def load_traffic(workload_key):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload_key)
    except Exception:
        return None


def run_ours(args, cfg, world, rank, local):
    import dc_triton_opt_b200 as dc
    from dc_triton_opt_b200 import _lib
    _lib.load()
    device = torch.device("cuda", local)
    rcfg = dict(cfg)
    if args.workload == "config4":
        b0, b1 = shard_batch(cfg["B"], world, rank)
        rcfg["B"] = b1 - b0
    q, k, v, pre, post = make_inputs(rcfg, device, seed=1234 + rank)
    B, T, H, D, G, R, W = (rcfg[k] for k in ("B", "T", "H", "D", "G", "R", "window"))
    stream = torch.cuda.current_stream(device)
    out = torch.empty_like(q)
    call = lambda: dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, W, G, out=out, kernel=args.kernel)
    kernel_used = dc.select_kernel(q, k, v, pre, post, W, G) if args.kernel == "auto" else args.kernel
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            call()
        ev1.record(stream)
        barrier()
    ms_max = max_over_ranks(ev0.elapsed_time(ev1), device)
    ms_step = ms_max / args.steps

    # end to end through the host-memory entry point: pinned host inputs ->
    # device, forward, output -> host, every step (the batch is pipelined
    # over copy / compute streams inside dc_attn_fwd_host)
    from dataclasses import replace
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    h2d = sum(t.numel() * t.element_size() for t in (qh, kh, vh))
    host_sets = []
    for tm in (pre, post):
        kw = {}
        for f in ("qw1", "qw2", "kw1", "kw2", "qdd", "kdd", "qmat"):
            t = getattr(tm, f)
            if t is not None:
                kw[f] = t.cpu().pin_memory()
                h2d += kw[f].numel() * kw[f].element_size()
        host_sets.append(replace(tm, **kw))
    out_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    d2h = out_host.numel() * out_host.element_size()
    e2e_steps = max(1, min(args.steps, 10))

    def e2e_step():
        dc.dc_attn_fwd_host(qh, kh, vh, host_sets[0], host_sets[1], D ** -0.5, W, G, out=out_host,
                            device=device, kernel=args.kernel)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    ev0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    ev1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1) / e2e_steps, device)

    fl_rank = flops(B, H, D, G, R, pairs(T, W), qmat=bool(rcfg.get("qmat")))
    total_fl = fl_rank * world
    value = total_fl / (ms_step * 1e-3) / 1e12
    e2e_val = total_fl / (e2e_ms * 1e-3) / 1e12
    hbm, tc_peak, peak_src = peaks()
    by = algo_bytes(B, T, H, D, R)
    if rcfg.get("qmat"):  # two [B,T,H,HPG] qmat tensors instead of the rank/gate weights
        by = 4 * B * T * H * D * 2 + 2 * B * T * H * (H // G) * 2
    achieved = by / (ms_step * 1e-3) / 1e9
    tflops_rank = fl_rank / (ms_step * 1e-3) / 1e12
    strong = best = others = bwd = prj = f8 = None
    if not args.no_extra:
        del qh, kh, vh, host_sets, out_host
        strong = strong_scaling_config4(world, rank, local)
        if rank == 0:
            best = repo_best(local)
            others = other_layers(local)
            bwd = backward_layer(local)
            prj = projection_layer(local)
            f8 = fp8_layer(local)
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline and not cfg.get("qmat"):
        v_cpu, cores, sample = cpu_port_sample(cfg, target_s=12.0)
        cpu = {"value": v_cpu, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}
    wl_key = f"{args.workload}_G{G}_W{W}"
    line = {
        "metric": "DC-attn fwd effective TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "us_per_call": ms_step * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if args.workload == "config4" else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded; BASELINE distributions)",
        "config": config_desc(args, cfg, world), "kernel": kernel_used,
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_source": peak_src,
                     "traffic": load_traffic(wl_key), "algo_bytes_per_launch": by,
                     "tensor_tflops": tflops_rank, "tensor_peak": tc_peak,
                     "tensor_frac": tflops_rank / tc_peak},
        "e2e": {"value": e2e_val, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms},
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    if not args.no_extra:
        line["strong_scaling"] = strong
        line["repo_best"] = best
        line["other_layers"] = others
        line["backward"] = bwd
        line["projection"] = prj
        line["fp8"] = f8
    print(json.dumps(line), flush=True)


def time_calls(call, steps, warmup, stream, world):
    """Device time per call (CUDA events on `stream`, max over ranks), after warm-up."""
    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        call()
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    # world == 1: a measurement on this rank alone (rank 0's extra blocks run
    # while the other ranks have finished), so no collective
    return max_over_ranks(ms, stream.device) if world > 1 else ms


# The other BASELINE layers, timed in the same run (device time only): the
# W256 half of the headline metric at the reference's best grouping (G8), its
# G sweep ends, the full-causal layer and the decomposed form.
OTHER_LAYERS = [("config2", dict(G=8)), ("config2", dict(G=32)), ("config2", dict(G=1)),
                ("config3", {}), ("decomposed", {})]


def other_layers(local, steps=5, warmup=3):
    import dc_triton_opt_b200 as dc
    device = torch.device("cuda", local)
    res = {}
    hbm, tc_peak, _ = peaks()
    for name, over in OTHER_LAYERS:
        cfg = dict(WORKLOADS[name], **over)
        q, k, v, pre, post = make_inputs(cfg, device, seed=99)
        B, T, H, D, G, R, W = (cfg[x] for x in ("B", "T", "H", "D", "G", "R", "window"))
        out = torch.empty_like(q)
        call = lambda: dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, W, G, out=out)
        ms = time_calls(call, steps, warmup, torch.cuda.current_stream(device), 1)
        fl = flops(B, H, D, G, R, pairs(T, W), qmat=bool(cfg.get("qmat")))
        by = (4 * B * T * H * D * 2 + 2 * B * T * H * (H // G) * 2) if cfg.get("qmat") else algo_bytes(B, T, H, D, R)
        key = f"{name}_G{G}_W{W if W is not None else 'causal'}"
        res[key] = {"B": B, "T": T, "window": W if W is not None else "full_causal", "G": G, "R": R,
                    "kernel": dc.select_kernel(q, k, v, pre, post, W, G), "ms_per_call": ms,
                    "tflops": fl / (ms * 1e-3) / 1e12, "tensor_frac": fl / (ms * 1e-3) / 1e12 / tc_peak,
                    "hbm_gbs": by / (ms * 1e-3) / 1e9, "hbm_frac": by / (ms * 1e-3) / 1e9 / hbm}
        del q, k, v, pre, post, out
        torch.cuda.empty_cache()
    res["timing"] = f"CUDA events, {warmup} warm-up + {steps} calls, inputs larger than L2"
    return res


def backward_layer(local, steps=3, warmup=2):
    """The backward (dc_attn_bwd) at the headline layer (config1 G8 W128, the
    query-side terms: static W, rank-1 query-wise weights, qdd; key-wise terms
    have no backward).  FLOPs counted: QK^T recompute, dP' = dO V^T, dV, dQ and
    dK (10 D per (b, h, t, s) pair) plus twice the forward's composition."""
    import dc_triton_opt_b200 as dc
    device = torch.device("cuda", local)
    cfg = dict(WORKLOADS["config1"])
    q, k, v, pre, post = make_inputs(cfg, device, seed=5)
    for t in (pre, post):
        t.kw1 = t.kw2 = t.kdd = None
    dout = torch.randn_like(q)
    B, T, H, D, G, R, W = (cfg[x] for x in ("B", "T", "H", "D", "G", "R", "window"))
    call = lambda: dc.dc_attn_bwd(dout, q, k, v, pre, post, D ** -0.5, W, G)
    ms = time_calls(call, steps, warmup, torch.cuda.current_stream(device), 1)
    npairs = pairs(T, W)
    fl = 10 * D * H * B * npairs + 2 * (flops(B, H, D, G, R, npairs) - 4 * D * H * B * npairs)
    del q, k, v, pre, post, dout
    torch.cuda.empty_cache()
    return {"workload": "config1", "G": G, "window": W, "R": R, "ms_per_call": ms,
            "tflops": fl / (ms * 1e-3) / 1e12, "kernel": "dc_bwd_kernel (mma.sync tensor-core products, fp32 composition)",
            "timing": f"CUDA events, {warmup} warm-up + {steps} calls"}


def projection_layer(local, steps=5, warmup=3, M=16 * 4096):
    """The composition-weight producer (dc_proj_weights) for the headline
    layer's tokens: M = B*T = 65536, hidden size Dm = H*D = 4096, MLP width
    I = 128, H = 32, R = 1.  FLOPs: 2 M Dm I + 2 M Dm 4H + 2 M I 8HR."""
    import dc_triton_opt_b200 as dc
    device = torch.device("cuda", local)
    Dm, I, H, R = 4096, 128, 32, 1
    g = torch.Generator(device=device).manual_seed(11)
    rn = lambda *sh, std: (std * torch.randn(*sh, generator=g, device=device)).to(torch.bfloat16)
    x = rn(M, Dm, std=1.0)
    w1, w2, wdd = rn(Dm, I, std=Dm ** -0.5), rn(I, 8 * H * R, std=0.01), rn(Dm, 4 * H, std=0.01)
    hidden = torch.empty(M, I, device=device, dtype=torch.bfloat16)
    call = lambda: dc.dc_proj_weights(x, w1, w2, wdd, H, R, hidden=hidden)
    ms = time_calls(call, steps, warmup, torch.cuda.current_stream(device), 1)
    fl = 2 * M * Dm * I + 2 * M * Dm * 4 * H + 2 * M * I * 8 * H * R
    by = 2 * M * Dm * 2 + 2 * M * I * 2 + M * (8 * H * R + 4 * H) * 2
    hbm, tc_peak, _ = peaks()
    del x, hidden
    torch.cuda.empty_cache()
    return {"M": M, "Dm": Dm, "I": I, "H": H, "R": R, "ms_per_call": ms, "tflops": fl / (ms * 1e-3) / 1e12,
            "tensor_frac": fl / (ms * 1e-3) / 1e12 / tc_peak, "hbm_gbs": by / (ms * 1e-3) / 1e9,
            "kernel": "dc_proj_tc_gemm (tcgen05, TMA), 2 launches (x [W1 | Wdd], hidden W2)", "timing": f"CUDA events, {warmup} warm-up + {steps} calls"}


def fp8_layer(local, steps=5, warmup=3):
    """The headline layer (config1 G8 W128, every term) with q and k in e4m3
    (per-tensor scales, QK^T in fp8 on the tensor cores, one-tile-per-CTA
    kernel) beside the bf16 forward on the same inputs; error of the fp8 result
    against the bf16 one as max|d| / max|bf16 out|."""
    import dc_triton_opt_b200 as dc
    device = torch.device("cuda", local)
    cfg = dict(WORKLOADS["config1"])
    q, k, v, pre, post = make_inputs(cfg, device, seed=21)
    B, T, H, D, G, R, W = (cfg[x] for x in ("B", "T", "H", "D", "G", "R", "window"))
    q8, qs = dc.quantize_e4m3(q)
    k8, ks = dc.quantize_e4m3(k)
    out8, out16 = torch.empty_like(v), torch.empty_like(v)
    f8 = lambda: dc.dc_attn_fwd_fp8qk(q8, k8, v, qs, ks, pre, post, D ** -0.5, W, G, out=out8)
    f16 = lambda: dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, W, G, out=out16)
    stream = torch.cuda.current_stream(device)
    ms8 = time_calls(f8, steps, warmup, stream, 1)
    ms16 = time_calls(f16, steps, warmup, stream, 1)
    err = ((out8.float() - out16.float()).abs().max() / out16.float().abs().max()).item()
    fl = flops(B, H, D, G, R, pairs(T, W))
    del q, k, v, pre, post, q8, k8, out8, out16
    torch.cuda.empty_cache()
    return {"workload": "config1", "G": G, "window": W, "fp8_qk_ms": ms8, "fp8_qk_tflops": fl / (ms8 * 1e-3) / 1e12,
            "bf16_ms": ms16, "max_rel_diff_vs_bf16": err, "quantization": "e4m3, per-tensor scales for q and k",
            "kernel": "dc_tc_kernel (one tile per CTA), QK^T kind::f8f6f4"}


def strong_scaling_config4(world, rank, local, steps=5, warmup=3):
    """BASELINE config 4 (B64 T8192 W256 G1 R2) with its batch split over the
    ranks (shard_work: contiguous batch slices, no collective): per-GPU and
    whole-box ms and TFLOP/s, time = max over ranks."""
    import dc_triton_opt_b200 as dc
    from dc_triton_opt_b200.shard import shard_work
    cfg = dict(WORKLOADS["config4"])
    b0, b1, g0, g1 = shard_work(cfg["B"], cfg["G"], world, rank)
    device = torch.device("cuda", local)
    rcfg = dict(cfg, B=max(1, b1 - b0))
    q, k, v, pre, post = make_inputs(rcfg, device, seed=4321 + rank)
    D, W, G = cfg["D"], cfg["window"], cfg["G"]
    out = torch.empty_like(q)
    call = lambda: dc.dc_attn_fwd(q, k, v, pre, post, D ** -0.5, W, G, out=out)
    ms = time_calls(call, steps, warmup, torch.cuda.current_stream(device), world)
    fl = flops(cfg["B"], cfg["H"], D, G, cfg["R"], pairs(cfg["T"], W))
    del q, k, v, pre, post, out
    torch.cuda.empty_cache()
    return {"workload": "config4", "B": cfg["B"], "T": cfg["T"], "window": W, "G": G, "R": cfg["R"],
            "n_gpus": world, "batch_per_gpu": b1 - b0, "ms_per_step": ms,
            "tflops_whole_box": fl / (ms * 1e-3) / 1e12, "tflops_per_gpu": fl / world / (ms * 1e-3) / 1e12,
            "steps": steps, "warmup": warmup, "timing": "CUDA events, max over ranks"}


# Published forward times of the reference's best kernels (H100, fp16, rank-1
# query-wise residual terms, no static mix, no key-wise terms): BASELINE.md §1.
PUBLISHED_H100 = {
    "w112": {"kernel": "V4HCM (TritonDCOneKernelMixedProbs), BM16 W112, G8", "B": 8, "us": 958.0,
             "source": "onekernel_opt_summary.md:766 (B not stated, about 8)"},
    "w240": {"kernel": "V4HCM256 (TritonDCOneKernelMixedProbs256), BM16 W240, G8", "B": 16, "us": 4403.0,
             "source": "fa3_dc_hopper_plan.md:294"},
}

# The reference's CUDA kernels built from its own sources for sm_100a
# (oracle/build_ref.py) and the case each one times: (module, function, G,
# chunk, window).  Both sides get the same fp16 inputs, the same residual
# rank-1 weights and return the same [B,T,N,D] layout.
REPO_BEST = {
    "w112_g8": ("dc_fused_cuda", "onekernel_v4_forward", 8, 16, 112),
    "w112_g4": ("dc_fused_cuda", "onekernel_v4_forward", 4, 16, 112),
    "w240_g8": ("_dc_hopper_cuda", "forward_hpg4_wide_opt", 8, 16, 240),
}


def repo_best(local, steps=10, warmup=3):
    """The reference's best GPU kernels that can run here against this library,
    on one box, on the exact work they do: fp16, B16 T4096 N32 D128, the
    residual rank-1 weights only (no static mix, no key-wise terms).  The
    reference kernels are its CUDA ones (one-kernel V4 port, BM+W <= 128; the
    HPG-4 WMMA wide kernel, BM16 W240), compiled from its sources for sm_100a
    with its own flags.  Its Triton kernels (V4HCM / V4HCM256) are Python
    sources that do not travel to the GPU host; their published H100 times are
    listed beside.  FLOP/s count QK^T + PV only (the reference's convention)."""
    import dc_triton_opt_b200 as dc
    from dc_triton_opt_b200.onekernel import DCOneKernel
    from oracle.build_ref import import_module
    device = torch.device("cuda", local)
    g = torch.Generator(device=device).manual_seed(7)
    B, T, N, D = 16, 4096, 32, 128
    rn = lambda *sh: torch.randn(*sh, generator=g, device=device, dtype=torch.float32).to(torch.float16)
    q, k, v = rn(B, T, N, D), rn(B, T, N, D), rn(B, T, N, D)
    ws = [0.1 * rn(B, T, N) for _ in range(6)]
    sl = torch.full((B,), T, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    scale = D ** -0.5
    res = {"dtype": "fp16", "B": B, "T": T, "N": N, "D": D, "terms": "residual rank-1 (pre and post)",
           "timing": f"CUDA events, {warmup} warm-up + {steps} calls", "flops": "QK^T + PV only"}
    for key, (mod, fn, G, chunk, W) in REPO_BEST.items():
        fl = 4 * D * N * B * pairs(T, W)
        ours = lambda: DCOneKernel.forward(q, k, v, ws, scale, W, G=G, chunk_size=chunk)
        ms = time_calls(ours, steps, warmup, stream, 1)
        ent = {"window": W, "G": G, "chunk": chunk,
               "ours": {"us_per_call": ms * 1e3, "tflops": fl / (ms * 1e-3) / 1e12}}
        try:
            m = import_module(mod)
            f = getattr(m, fn)
            if mod == "dc_fused_cuda":
                theirs = lambda: f(q, k, v, *ws, sl, scale, W, G, chunk)
            else:
                theirs = lambda: f(q, k, v, *ws, scale, W, chunk)
            a, b = ours(), theirs()
            torch.cuda.synchronize()
            rms = ((a.float() - b.float()) ** 2).mean().sqrt().item()
            del a, b
            ms_r = time_calls(theirs, steps, warmup, stream, 1)
            ent["reference"] = {"kernel": f"{mod}.{fn}", "us_per_call": ms_r * 1e3,
                                "tflops": fl / (ms_r * 1e-3) / 1e12, "rms_diff_vs_ours": rms}
            ent["speedup"] = ms_r / ms
        except Exception as e:  # not built (no reference checkout at build time) or failed
            ent["reference"] = {"kernel": f"{mod}.{fn}", "unavailable": f"{type(e).__name__}: {e}"[:300]}
        pk = key.split("_")[0]
        if G == 8 and pk in PUBLISHED_H100:
            pub = PUBLISHED_H100[pk]
            ent["published_h100"] = dict(pub, us_scaled_to_B16=pub["us"] * B / pub["B"])
        res[key] = ent
        torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config1", choices=sorted(WORKLOADS))
    ap.add_argument("--G", type=int, default=None)
    ap.add_argument("--window", type=int, default=None)
    ap.add_argument("--B", type=int, default=None)
    ap.add_argument("--T", type=int, default=None)
    ap.add_argument("--kernel", default="auto", choices=["auto", "simt", "tc", "tcs", "tcm"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the config-4 strong-scaling, repo-best and other-layer blocks")
    ap.add_argument("--op", default=None, choices=["backward", "projection"],
                    help="run only this op a few times at a reduced size (B=2: 8192 tokens for the projection, "
                         "--B sets it), "
                         "for profiling; prints its ms per call")
    args = ap.parse_args()
    if args.op is not None:
        torch.cuda.set_device(0)
        if args.op == "backward":
            WORKLOADS["config1"] = dict(WORKLOADS["config1"], B=2)
            print(json.dumps(backward_layer(0, steps=args.steps, warmup=args.warmup)))
        else:
            print(json.dumps(projection_layer(0, steps=args.steps, warmup=args.warmup, M=4096 * (args.B or 2))))
        return
    cfg = dict(WORKLOADS[args.workload])
    for k in ("G", "window", "B", "T"):
        if getattr(args, k) is not None:
            cfg[k] = getattr(args, k)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, cfg, world, int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup()
    try:
        run_ours(args, cfg, world, rank, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
