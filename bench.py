#!/usr/bin/env python
"""Benchmark of the B200 DeepSeek-V3 FP8 MoE layer (the hot path of plops655/GEMMS).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gemms|reference]

One *step* is one full MoE layer forward (router GEMM -> routing -> permute +
1x128 quant -> grouped FP8 GEMM1 + SwiGLU -> grouped FP8 GEMM2 -> weighted
combine + shared expert -> bf16) over one batch of synthetic tokens.

* N=1: BASELINE config c1 -- T=4096, H=7168, I=2048, E=256, 8 groups /
  top-4 groups / top-8, scaling 2.5, + 1 shared expert.  Inputs are resident in
  HBM; every step streams 11.3 GB of expert weights, far larger than the 126 MB
  L2, so no flush is needed between steps.
* N>1 (torchrun): BASELINE config c3 -- expert parallel over N ranks, T=32768
  tokens in total (32768/N per rank), E/N experts per rank; rows exchanged
  by NCCL all-to-all or by the device-driven exchange over symmetric memory
  (``--ep-exchange``).  Total work is fixed as N grows ("strong" scaling).

Rank 0 prints one JSON line.  ``--impl reference`` times the reference's CPU
implementation of the path (the oracle restatement in ``oracle/``, bit-identical
to ``flashinfer_baseline.run``) on the host cores instead, on the same inputs
(drawn through the same generator path on GPU 0 and copied to the host) and
with the same ``config`` dict as the GPU arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE layer tokens/s and FP8 TFLOP/s (frac of peak) at T=4096, 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["gemms", "reference"], default="gemms")
    p.add_argument("--config", default=None, help="c1 (N=1 default), c2:<T> decode, c3 (N>1 default), c4")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-launch-count", action="store_true", help="skip the torch.profiler launch count (for ncu)")
    p.add_argument("--ep-exchange", choices=["nccl", "peer"], default=None,
                   help="N>1: rows exchanged by NCCL all-to-all or device-driven over symmetric memory "
                        "(default: GEMMS_EP_EXCHANGE, else peer)")
    return p.parse_args()


def parse_config(spec: str):
    """'c1', 'c2:128' (decode T) or 'c1:T=1024,E=64' (overrides for profiling)."""
    from gemms_b200 import workloads as W

    name, _, rest = spec.partition(":")
    base = W.CONFIGS[name]
    if rest:
        if "=" not in rest:
            return base.replace(T=int(rest))
        kv = {}
        for item in rest.split(","):
            k, v = item.split("=")
            kv[k] = type(getattr(base, k))(v) if not isinstance(getattr(base, k), bool) else v.lower() in ("1", "true")
        base = base.replace(**kv)
    return base


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                pw.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        # samples under load: power within 70% of the region's max
        pmax = max(pw)
        loaded = [s for s, p in zip(sm, pw) if p >= 0.7 * pmax] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": pmax}


# ------------------------------------------------------------ workload sizes
def algorithmic_bytes(sh, counts, planes: int, world: int = 1):
    """HBM bytes the two grouped GEMMs must move per launch (not counting
    re-reads): weights + scales of every expert that received rows (+ shared),
    the grouped activation rows (one per routed pair, as GEMM1 reads them),
    the SwiGLU intermediate (written by GEMM1, read by GEMM2) and GEMM2's fp32
    output accumulation."""
    H, I = sh.H, sh.I
    hit = int((counts > 0).sum())
    rows = int(counts.sum()) + (sh.T if sh.shared else 0)
    n_exp = hit + (1 if sh.shared else 0)
    w13 = 2 * I * H + 4 * (2 * I // 128) * (H // 128)
    w2 = H * I + 4 * (H // 128) * (I // 128)
    a_rows = rows * (H + 4 * H // 128)
    inter = rows * (planes * I + 4 * I // 128)
    out_acc = sh.T * H * 4 * 2  # fp32 accumulation target, read+write once
    g1 = n_exp * w13 + a_rows + inter
    g2 = n_exp * w2 + inter + out_acc
    return {"gemm1": g1, "gemm2": g2, "experts_hit": hit, "rows": rows}


def _traffic(kernel: str, algorithmic_bytes: float):
    """DRAM bytes per launch from the committed ncu capture (profiles/dram_traffic.json):
    the measured traffic/algorithmic ratio of that capture times this launch's
    algorithmic bytes.  None if there is no capture for the kernel."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d[kernel]["ratio"]) * algorithmic_bytes
    except Exception:
        return None


# ------------------------------------------------------------- CPU baseline
def cpu_baseline(sh, d_dev, logits_dev, n_experts_sample: int, threads: int | None = None):
    """Time the oracle port (== reference run(), bit for bit) on host cores for
    a bounded sample: ``n_experts_sample`` of the E routed experts over all T
    tokens, plus the shared expert; scaled to the full layer."""
    import torch

    from oracle import reference_moe as R

    if threads:
        torch.set_num_threads(threads)
    nt = torch.get_num_threads()
    x = d_dev["x"].cpu()
    logits = logits_dev.cpu()
    bias = d_dev["router_bias"].cpu()
    hs, hss = R.quantize_1x128(x)
    n = n_experts_sample
    w13 = d_dev["w13"][:n].cpu()
    w13s = d_dev["w13_scale"][:n].cpu()
    w2 = d_dev["w2"][:n].cpu()
    w2s = d_dev["w2_scale"][:n].cpu()
    t0 = time.perf_counter()
    R.run_local(logits, bias, hs, hss, w13, w13s, w2, w2s, 0, sh.rsf, n_group=sh.n_group,
                topk_group=sh.topk_group, top_k=sh.top_k, return_fp32=True)
    t_chunk = time.perf_counter() - t0
    t_shared = 0.0
    if sh.shared:
        A = R.dequant_hidden(hs, hss)
        sw = [d_dev[k].cpu() for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")]
        t0 = time.perf_counter()
        R.shared_expert(A, *sw)
        t_shared = time.perf_counter() - t0
    t_layer = t_chunk * (sh.E / n) + t_shared
    return {"value": sh.T / t_layer, "unit": "tokens/s", "cores": nt, "kind": "port",
            "sample": f"oracle run_local (== reference run()) over all T={sh.T} tokens for {n} of {sh.E} experts "
                      f"({t_chunk:.2f} s) + shared expert ({t_shared:.2f} s), scaled x{sh.E / n:.0f} to the full "
                      f"layer ({t_layer:.1f} s)",
            "os_cpu_count": os.cpu_count()}


def bench_setup(a, world: int, rank: int, dev):
    """Config and seeded inputs of this rank, shared by both arms.  Returns
    (cfg name, base shape, per-rank shape, local expert count, inputs on dev,
    Zipf histogram or None)."""
    import torch

    import gemms_b200
    from gemms_b200 import workloads as W

    cfg = a.config or ("c1" if world == 1 else "c3")
    base = parse_config(cfg)
    T_rank = base.T // world if world > 1 else base.T
    sh = base.replace(T=T_rank)
    n_local = sh.E // world
    zipf_hist = None
    d = W.make_inputs(sh, seed=rank, device=dev, experts=n_local)
    # every rank must hold the same router weights/bias and shared expert
    g = torch.Generator(device=dev).manual_seed(12345)
    d["router_w"] = torch.randn((sh.E, sh.H), generator=g, device=dev) * 0.02
    d["router_bias"] = torch.rand((sh.E,), generator=g, device=dev) * 0.2 - 0.1
    if sh.shared:
        d["shared_w13"] = torch.randn((2 * sh.I, sh.H), generator=g, device=dev).clamp_(-448, 448).to(torch.float8_e4m3fn)
        d["shared_w13_scale"] = torch.rand((2 * sh.I // 128, sh.H // 128), generator=g, device=dev) * 2e-3 + 1e-3
        d["shared_w2"] = torch.randn((sh.H, sh.I), generator=g, device=dev).clamp_(-448, 448).to(torch.float8_e4m3fn)
        d["shared_w2_scale"] = torch.rand((sh.H // 128, sh.I // 128), generator=g, device=dev) * 2e-3 + 1e-3
    if cfg.startswith("c4"):
        # BASELINE c4: router bias calibrated so expert popularity follows
        # Zipf(1.2) over a seeded permutation, hottest experts on ranks 0-1.
        route_fn = lambda lg, b: gemms_b200.route(lg, b, n_group=sh.n_group, topk_group=sh.topk_group,
                                                  top_k=sh.top_k, routed_scaling_factor=sh.rsf, counts=False)[0]
        bias, frac = W.zipf_bias(sh, route_fn, router_w=d["router_w"], s=1.2, seed=0, hot_ranks=2, world=8,
                                 device=dev)
        d["router_bias"] = bias
        zipf_hist = frac.cpu()
    return cfg, base, sh, n_local, d, zipf_hist


def config_dict(cfg, base, sh, n_local, planes, world, zipf_hist=None):
    c = {"workload": (f"{cfg}: DeepSeek-V3 MoE layer T={base.T} H={sh.H} I={sh.I} E={sh.E} "
                      f"groups {sh.n_group}/{sh.topk_group} top-{sh.top_k}" + (" + shared expert" if sh.shared else "")),
         "tokens_per_rank": sh.T, "experts_per_rank": n_local, "inter_planes": planes,
         "parallelism": f"ep{world}" if world > 1 else "single GPU",
         **({"ep_exchange": os.environ.get("GEMMS_EP_EXCHANGE", "peer")} if world > 1 else {}),
         "l2": "inputs larger than L2 (11.3 GB of expert weights streamed per step)"}
    if zipf_hist is not None:
        per_rank = zipf_hist.reshape(8, -1).sum(1)
        c["zipf"] = {"s": 1.2, "top_expert_share": float(zipf_hist.max()),
                     "rank_share_of_routed_pairs": [round(float(v), 4) for v in per_rank]}
    return c


REF_E_LOCAL = 32     # the reference's own E_local (flashinfer_baseline.py:45)
REF_TOKENS = 4096    # tokens per reference call (one rank's c1 batch)


def reference_arm(a):
    """--impl reference: the reference's CPU path (the oracle port, bit-identical
    to flashinfer_baseline.run) on the host cores, on the GPU arm's inputs and
    config.  One step = one reference run() call over up to 4096 of rank 0's
    tokens with E_local=32 local experts, as the reference calls it; the
    layer's throughput is that call's time scaled to all tokens and all E
    experts, plus the shared expert (timed once on the same tokens)."""
    import torch

    from oracle import reference_moe as R

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    planes = 2
    cfg, base, sh, n_local, d, zipf_hist = bench_setup(a, world, 0, dev)
    ts = min(sh.T, REF_TOKENS)
    el = min(REF_E_LOCAL, n_local)
    x = d["x"][:ts].cpu()
    cw = {k: d[k][:el].cpu() for k in ("w13", "w13_scale", "w2", "w2_scale")}
    router_w, bias = d["router_w"].cpu(), d["router_bias"].cpu()
    shared = [d[k].cpu() for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")] \
        if sh.shared else None
    del d
    torch.cuda.empty_cache()
    logits = R.router_logits(x, router_w)
    hs, hss = R.quantize_1x128(x)
    times = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        R.run_local(logits, bias, hs, hss, cw["w13"], cw["w13_scale"], cw["w2"], cw["w2_scale"], 0, sh.rsf,
                    n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, return_fp32=True)
        dt = time.perf_counter() - t0
        if i >= a.warmup:
            times.append(dt)
    t_shared = 0.0
    if shared is not None:
        A = R.dequant_hidden(hs, hss)
        t0 = time.perf_counter()
        R.shared_expert(A, *shared)
        t_shared = time.perf_counter() - t0
    t_call = statistics.mean(times)
    token_scale = base.T / ts
    t_layer = t_call * token_scale * (sh.E / el) + t_shared * token_scale
    value = base.T / t_layer
    cores = torch.get_num_threads()
    sample = (f"per step: one oracle run() call (== reference flashinfer_baseline.run) over {ts} of rank 0's "
              f"tokens with E_local={el} local experts ({t_call:.2f} s); layer = call x {token_scale:g} token "
              f"slices x {sh.E // el} expert slices + shared expert ({t_shared:.2f} s per slice) = {t_layer:.1f} s")
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": t_call * 1e3, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32 (fp8 dequantised)",
            "data": "synthetic (seeded; BASELINE distributions; random-init weights)",
            "config": config_dict(cfg, base, sh, n_local, planes, world, zipf_hist),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
                             "os_cpu_count": os.cpu_count()},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def fp8_peak_tflops(dev, n: int = 8192, reps: int = 10):
    """Dense FP8 tensor peak of this GPU measured with a library GEMM:
    torch._scaled_mm (cuBLAS) on e4m3 n x n x n, bf16 out, best of `reps`."""
    import torch

    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=dev)
    for _ in range(3):
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


# --------------------------------------------------------------- GPU arm
def count_kernels_per_step(step_fn) -> int:
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    n = 0
    for ev in prof.events():
        if ev.device_type.name == "CUDA" and "gemms::" in ev.name:
            n += 1
    return n


def decode_sweep(d, kw, sh, hbm, Ts=(1, 2, 4, 8, 32, 128), steps=50, warmup=5):
    """BASELINE config c2: the same full layer (same weights) on the first T
    tokens, T in Ts, one GPU.  Decode streams the weights of every expert the
    batch hits (+ the shared expert), so each line reports that weight traffic
    per layer as HBM GB/s; the experts hit are counted from the batch's own
    routing.  For T <= 2 the graph is also timed with the CUDA-core expert
    GEMMs forced on and off (``gemms_set_decode_max_t``), an A/B on one box.  Every step reads >= 396 MB of weights (T=1: 8 experts + shared),
    more than the 126 MB L2.  Each time is the median of three batches of
    ``steps`` steps (a decode step is ~0.1 ms: one disturbed batch would
    otherwise decide the figure)."""
    import torch

    import gemms_b200

    args = (d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):  # median over three batches of `steps` calls, ms per call
        per = []
        for _ in range(3):
            e0.record()
            for _ in range(steps):
                fn()
            e1.record()
            e1.synchronize()
            per.append(e0.elapsed_time(e1) / steps)
        return statistics.median(per)

    res = {}
    for T in Ts:
        x = d["x"][:T].contiguous()
        counts = gemms_b200.moe(x, *args, return_routing=True, **kw)[3]
        hit = int((counts > 0).sum())
        for _ in range(warmup):
            gemms_b200.moe(x, *args, **kw)
        torch.cuda.synchronize()
        ms = timed(lambda: gemms_b200.moe(x, *args, **kw))
        # the same layer captured in a CUDA graph (gemms_b200.MoeGraph): one
        # launch per step instead of one per kernel
        graph = gemms_b200.MoeGraph(d, T, **kw)
        for _ in range(warmup):
            graph(x)
        torch.cuda.synchronize()
        ms_g = timed(lambda: graph(x))
        del graph
        ab = {}
        if T <= 2:  # A/B on this box: the graph with the CUDA-core and with the tensor-core expert GEMMs
            L = gemms_b200.load_library()
            for name, limit in (("graph_cuda_core_gemms_ms", 2), ("graph_tensor_core_gemms_ms", 0)):
                prev = L.gemms_set_decode_max_t(limit)
                try:
                    graph = gemms_b200.MoeGraph(d, T, **kw)
                    for _ in range(warmup):
                        graph(x)
                    torch.cuda.synchronize()
                    ab[name] = round(timed(lambda: graph(x)), 5)
                    del graph
                finally:
                    L.gemms_set_decode_max_t(prev)
        nbytes = (hit + (1 if sh.shared else 0)) * sh.expert_bytes()
        gbs = nbytes / (ms / 1e3) / 1e9
        gbs_g = nbytes / (ms_g / 1e3) / 1e9
        res[f"T={T}"] = {"ms_per_step": round(ms, 5), "tokens_per_s": round(T / (ms / 1e3), 1), "experts_hit": hit,
                         "weight_bytes": nbytes, "GB/s": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
                         **ab,
                         "graph": {"ms_per_step": round(ms_g, 5), "tokens_per_s": round(T / (ms_g / 1e3), 1),
                                   "GB/s": round(gbs_g, 1), "hbm_frac": round(gbs_g / hbm, 4)}}
    return res


def gpu_arm(a):
    # N>1 default: the device-driven exchange (no host synchronisation; every
    # rank runs the same token count here)
    os.environ["GEMMS_EP_EXCHANGE"] = a.ep_exchange or os.environ.get("GEMMS_EP_EXCHANGE") or "peer"
    import torch
    import torch.distributed as dist

    import gemms_b200
    from gemms_b200 import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD
    planes = 2
    cfg, base, sh, n_local, d, zipf_hist = bench_setup(a, world, rank, dev)
    shared_kw = {k: d[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale") if k in d}
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf,
              inter_planes=planes, ep_group=group, **shared_kw)

    def step(x, events=None):
        # NVTX range per step: `ncu --nvtx --nvtx-include moe_step/` selects the layer's launches.
        torch.cuda.nvtx.range_push("moe_step")
        try:
            if group is None:
                return gemms_b200.moe(x, d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                                      d["w2_scale"], profile_events=events, **kw)
            return gemms_b200.moe(x, d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                                  d["w2_scale"], **kw)
        finally:
            torch.cuda.nvtx.range_pop()

    def barrier():
        if group is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # routing statistics for the algorithmic byte count
    if group is None:
        out, idx, wts, counts, logits = gemms_b200.moe(d["x"], d["router_w"], d["router_bias"], d["w13"],
                                                       d["w13_scale"], d["w2"], d["w2_scale"], return_routing=True,
                                                       **{k: v for k, v in kw.items() if k != "ep_group"})
        gemms_b200.check_device_errors(tag="moe")
        counts_cpu = counts.cpu()
    for _ in range(a.warmup):
        step(d["x"])
    barrier()
    launches_per_step = None
    if not a.no_launch_count:
        launches_per_step = count_kernels_per_step(lambda: step(d["x"]))
    barrier()

    # ---- device-resident timed region
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    nev = a.steps if group is None else 0
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(nev)]
    for e3 in evs:
        for e in e3:
            e.record()  # materialise the CUDA events before they are handed to the C ABI
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(a.steps):
        step(d["x"], evs[i] if nev else None)
    t1.record()
    barrier()
    ms_total = t0.elapsed_time(t1)
    if group is not None:
        tt = torch.tensor([ms_total], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_total = float(tt.item())
    ms = ms_total / a.steps

    ep_timeline = None
    if group is not None:
        # per-phase device time of the expert-parallel step (rank 0's stream),
        # measured on extra steps after the timed region
        from gemms_b200 import ep as ep_mod
        marks = []
        for _ in range(5):
            tl = []
            ep_mod.moe_ep(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                          d["w2_scale"], group=group, timeline=tl,
                          **{k: v for k, v in kw.items() if k != "ep_group"})
            marks.append(tl)
        barrier()
        info = {n: v for n, v in marks[0] if n in ("recv_rows", "pair_rows", "experts_hit")}
        marks = [[(n, e) for n, e in tl if n not in info] for tl in marks]
        names = [n for n, _ in marks[0]]
        ep_timeline = {names[j]: round(statistics.median(tl[j - 1][1].elapsed_time(tl[j][1]) for tl in marks), 4)
                       for j in range(1, len(names))}
        ep_timeline.update(info)
    g1_ms = statistics.mean(evs[i][0].elapsed_time(evs[i][1]) for i in range(nev)) if nev else None
    g2_ms = statistics.mean(evs[i][1].elapsed_time(evs[i][2]) for i in range(nev)) if nev else None
    if group is None:
        gemms_b200.check_device_errors(tag="moe")

    # ---- end-to-end through the public API with host buffers: gemms_b200.MoePipeline
    # copies every step's x in from pinned host memory and its result back out,
    # overlapping the copies of neighbouring steps with the layer.
    e2e = None
    if not a.no_e2e:
        x_host = d["x"].cpu().pin_memory()
        outs = [torch.empty((sh.T, sh.H), dtype=torch.bfloat16).pin_memory() for _ in range(4)]
        pipe = gemms_b200.MoePipeline(d, device=dev, **kw)
        pipe.run([x_host] * 2, outs[:2])  # warm-up (allocates the device slots)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        pipe.run([x_host] * a.steps, [outs[i % 4] for i in range(a.steps)])
        e1.record()
        barrier()
        e2e_ms = e0.elapsed_time(e1)
        if group is not None:
            tt = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_ms = float(tt.item())
        e2e_ms /= a.steps
        e2e = {"value": base.T / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": x_host.numel() * x_host.element_size() * world,
               "d2h_bytes_per_step": outs[0].numel() * outs[0].element_size() * world,
               "path": "pinned host x -> gemms_b200.MoePipeline (public API; copies overlapped with the "
                       "layer on side streams) -> pinned host out, every step, every rank"}
    decode = None
    det = None
    if group is None and cfg == "c1":
        hbm_peak = _peaks()[0]
        decode = decode_sweep(d, {k: v for k, v in kw.items() if k != "ep_group"}, sh, hbm_peak)
        # the same step with the deterministic (fixed-order) combine
        kw1 = {k: v for k, v in kw.items() if k != "ep_group"}
        for _ in range(2):
            gemms_b200.moe(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                           deterministic=True, **kw1)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dev_evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(a.steps)]
        for e3 in dev_evs:
            for e in e3:
                e.record()
        torch.cuda.synchronize()
        e0.record()
        for i in range(a.steps):
            gemms_b200.moe(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                           deterministic=True, profile_events=dev_evs[i], **kw1)
        e1.record()
        torch.cuda.synchronize()
        ms_det = e0.elapsed_time(e1) / a.steps
        g2_det = statistics.mean(e3[1].elapsed_time(e3[2]) for e3 in dev_evs)
        det = {"what": "same c1 step with deterministic=True (per-token fixed-order combine, bit-reproducible)",
               "ms_per_step": round(ms_det, 4), "tokens_per_s": round(base.T / (ms_det / 1e3), 1),
               "gemm2_ms": round(g2_det, 4)}
    clocks = sampler.stop() if sampler else None

    tokens_total = base.T
    value = tokens_total / (ms / 1e3)
    flops = 6.0 * sh.H * sh.I * (base.T * sh.top_k + (base.T if sh.shared else 0))
    if rank != 0:
        if group is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    hbm, bf16, src = _peaks()
    tflops = flops / (ms / 1e3) / 1e12
    fp8_peak = fp8_peak_tflops(dev)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "fp8_e4m3 (fp32 accumulate)",
            "data": "synthetic (seeded; BASELINE distributions; random-init weights)",
            "config": config_dict(cfg, base, sh, n_local, planes, world, zipf_hist),
            "tflops": tflops,
            "fp8": {"tflops": tflops, "tflops_per_gpu": tflops / world, "peak_tflops": fp8_peak * world,
                    "frac": tflops / (fp8_peak * world),
                    "peak_source": "measured in this run: torch._scaled_mm (cuBLAS) e4m3 8192^3, bf16 out, "
                                   "best of 10 on rank 0's GPU, times the GPU count"},
            "gpu_launches": (launches_per_step * a.steps) if launches_per_step is not None else None,
            "e2e": e2e, "clocks": clocks}
    if det is not None:
        det["vs_default"] = round(ms / det["ms_per_step"], 4)
        line["deterministic"] = det
    if decode is not None:
        line["decode_c2"] = {"what": "BASELINE config c2 on the same GPU and weights: full layer (router GEMM, "
                                     "routing, quantisation, grouped GEMMs, combine, shared expert) on the first T "
                                     "tokens; GB/s = weight bytes of the experts hit (+ shared) per layer / time; "
                                     "hbm_frac against the measured HBM copy bandwidth; 'graph': the same call "
                                     "replayed from a CUDA graph (gemms_b200.MoeGraph)",
                             **decode}
    if group is not None:
        # Dominant phase at N>1: the grouped GEMMs over the received rows
        # (GEMM1 + GEMM2 of the rank's E/N experts, all of them hit at c3).
        # same model as algorithmic_bytes: weights (+ scales) of the local
        # experts hit (+ shared), the grouped rows (one per received row and
        # local expert), the intermediate written and read, the fp32 result
        # rows (received rows; the shared expert's T rows) read and written
        H, I = sh.H, sh.I
        w_exp = 3 * I * H + 4 * (2 * I // 128) * (H // 128) + 4 * (H // 128) * (I // 128)
        row_b = H + 4 * H // 128
        inter_b = 2 * (planes * I + 4 * I // 128)
        R, P = ep_timeline["recv_rows"], ep_timeline["pair_rows"]
        # the shared expert is in the roofline only where it has its own phase
        # (with the device exchange it runs beside the gather, `shared_and_gather`)
        shared_timed = sh.shared and ("shared_ffn" in ep_timeline or "shared_ffn_2" in ep_timeline)
        ffn_bytes = (ep_timeline["experts_hit"] * w_exp + P * (row_b + inter_b) + R * H * 4 * 2
                     + ((w_exp + sh.T * (row_b + inter_b) + sh.T * H * 4 * 2) if shared_timed else 0))
        ffn_ms = ep_timeline["expert_ffn"] + (ep_timeline.get("shared_ffn", 0.0) + ep_timeline.get("shared_ffn_2", 0.0)
                                              if shared_timed else 0.0)
        ach = ffn_bytes / (ffn_ms / 1e3) / 1e9
        # at c3 the grouped rows per rank (>= 32k) make the FFN compute-bound:
        # its roof is the tensor pipe (FP8 work of rank 0's grouped rows and
        # shared rows over the same phases)
        ffn_flops = 6.0 * H * I * (P + (sh.T if shared_timed else 0))
        ach_tf = ffn_flops / (ffn_ms / 1e3) / 1e12
        line["roofline"] = {"bound": "tensor", "kernel": "grouped GEMM1+GEMM2 over received rows" +
                                                         (" + shared expert (rank 0, expert_ffn + shared_ffn phases)"
                                                          if shared_timed else " (rank 0, expert_ffn phase)"),
                            "achieved": ach_tf, "peak": fp8_peak, "unit": "TFLOP/s", "frac": ach_tf / fp8_peak,
                            "peak_source": "dense FP8 measured in this run (torch._scaled_mm, cuBLAS, e4m3 8192^3); "
                                           "MEASURED_PEAKS.json has no FP8 entry",
                            "traffic": None, "algorithmic_flops": ffn_flops, "launch_ms": ffn_ms,
                            "hbm": {"algorithmic_bytes": ffn_bytes, "achieved_gbs": ach, "peak_gbs": hbm,
                                    "frac": ach / hbm}}
        line["ep_timeline_ms"] = ep_timeline
    if group is None:
        ab = algorithmic_bytes(sh, counts_cpu, planes)
        g1_gbs = ab["gemm1"] / (g1_ms / 1e3) / 1e9
        g2_gbs = ab["gemm2"] / (g2_ms / 1e3) / 1e9
        tr = _traffic("gemm1", ab["gemm1"])
        line["roofline"] = {"bound": "hbm", "kernel": "grouped_gemm_kernel<0,1,2> (GEMM1 + SwiGLU + requant)",
                            "achieved": g1_gbs, "peak": hbm, "unit": "GB/s", "frac": g1_gbs / hbm,
                            "peak_source": f"{src} hbm_gbs (MEASURED_PEAKS.json)" if src == "measured" else
                            "fallback 6650 GB/s", "traffic": tr,
                            "algorithmic_bytes": ab["gemm1"], "launch_ms": g1_ms}
        line["kernels"] = {"gemm1": {"ms": g1_ms, "GB/s": g1_gbs, "bytes": ab["gemm1"]},
                           "gemm2": {"ms": g2_ms, "GB/s": g2_gbs, "bytes": ab["gemm2"], "traffic": _traffic("gemm2", ab["gemm2"])},
                           "layer": {"ms": ms, "hbm_frac_of_layer_floor":
                                     (ab["gemm1"] + ab["gemm2"]) / 1e9 / hbm / (ms / 1e3)},
                           "experts_hit": ab["experts_hit"], "rows": ab["rows"]}
        if not a.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(sh, d, logits, n_experts_sample=32)
    print(json.dumps(line), flush=True)
    if group is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    a = _args()
    if a.impl == "reference":
        reference_arm(a)
        return
    gpu_arm(a)


if __name__ == "__main__":
    main()
