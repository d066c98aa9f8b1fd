"""Seeded synthetic workloads for the DeepSeek-V3 FP8 MoE layer.

The reference ships no datasets or fixtures; its harnesses fill random data
(``modal_ncu.py:64-94``, ``benchmark_moe_triton.py:77-142``).  This module
defines the shapes and value distributions of the benchmark configurations so
that tests, ``bench.py`` and the golden-fixture script draw identical inputs:

* activations ``x`` bf16 ~ N(0, 1)                      [T, H]
* router weights fp32 ~ N(0, 0.02^2)                    [E, H]
* router bias fp32 ~ U(-0.1, 0.1)                       [E]
* ``w13`` e4m3 from N(0, 1) clamped to +-448            [E, 2I, H]
* ``w2``  e4m3 from N(0, 1) clamped to +-448            [E, H, I]
* 128x128 fp32 block scales ~ U(1e-3, 3e-3)             [E, 2I/128, H/128], [E, H/128, I/128]
* optional shared expert with the same layouts (one expert, no leading dim)

Generation order is fixed (x, router_w, bias, w13, w13_scale, w2, w2_scale,
shared_w13, shared_w13_scale, shared_w2, shared_w2_scale) and seeded with a
``torch.Generator`` on the requested device, so CPU draws are reproducible
across machines that run the same torch build.  Weights are drawn one expert
at a time to bound host memory at full DeepSeek-V3 shapes.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass

import torch

BLOCK = 128
FP8_MAX = 448.0


@dataclass(frozen=True)
class MoeShape:
    """Geometry of one MoE layer call (one rank's view when ``E_local < E``)."""

    T: int
    H: int
    I: int
    E: int
    n_group: int
    topk_group: int
    top_k: int
    rsf: float = 2.5
    shared: bool = False

    def replace(self, **kw) -> "MoeShape":
        return dataclasses.replace(self, **kw)

    def validate(self) -> None:
        if self.H % BLOCK or self.I % BLOCK:
            raise ValueError(f"H ({self.H}) and I ({self.I}) must be multiples of {BLOCK}")
        if self.E % self.n_group:
            raise ValueError(f"E ({self.E}) must be divisible by n_group ({self.n_group})")
        gs = self.E // self.n_group
        if gs < 2 or gs > 32:
            raise ValueError(f"group size E/n_group = {gs} must be in [2, 32]")
        if not (1 <= self.topk_group <= self.n_group):
            raise ValueError("topk_group must be in [1, n_group]")
        if not (1 <= self.top_k <= self.topk_group * gs):
            raise ValueError("top_k must be in [1, topk_group * group_size]")
        if self.top_k > 16:
            raise ValueError("top_k must be <= 16")

    # ---- algorithmic work (used by bench.py's roofline) -------------------
    def flops(self, pairs: int, shared_rows: int | None = None) -> float:
        """FP8 GEMM FLOPs for ``pairs`` routed (token, expert) rows plus shared rows."""
        rows = pairs + (self.T if (self.shared and shared_rows is None) else (shared_rows or 0))
        return 6.0 * rows * self.H * self.I

    def expert_bytes(self) -> int:
        """FP8 weight bytes + fp32 block scales of one expert (w13 and w2)."""
        w = 3 * self.H * self.I
        s = 4 * ((2 * self.I // BLOCK) * (self.H // BLOCK) + (self.H // BLOCK) * (self.I // BLOCK))
        return w + s


CONFIGS: dict[str, MoeShape] = {
    # scaled-down, CPU-runnable correctness config.
    "c0": MoeShape(T=64, H=2048, I=768, E=32, n_group=4, topk_group=2, top_k=4, rsf=2.5, shared=False),
    # full DeepSeek-V3 layer, prefill T=4096, 1 GPU, + shared expert.
    "c1": MoeShape(T=4096, H=7168, I=2048, E=256, n_group=8, topk_group=4, top_k=8, rsf=2.5, shared=True),
    # decode sweep (T overridden to 1, 8, 32, 128).
    "c2": MoeShape(T=128, H=7168, I=2048, E=256, n_group=8, topk_group=4, top_k=8, rsf=2.5, shared=True),
    # EP over 2/4/8 GPUs, T=32768 total (per-rank T = 32768 / W).
    "c3": MoeShape(T=32768, H=7168, I=2048, E=256, n_group=8, topk_group=4, top_k=8, rsf=2.5, shared=True),
    # EP8 skewed routing, T=16384 total.
    "c4": MoeShape(T=16384, H=7168, I=2048, E=256, n_group=8, topk_group=4, top_k=8, rsf=2.5, shared=True),
}


def _fp8_weights(n: int, rows: int, cols: int, g: torch.Generator, device) -> torch.Tensor:
    out = torch.empty((n, rows, cols), dtype=torch.float8_e4m3fn, device=device)
    for e in range(n):
        w = torch.randn((rows, cols), generator=g, device=device, dtype=torch.float32)
        out[e] = w.clamp_(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
        del w
    return out


def _scales(shape, g: torch.Generator, device) -> torch.Tensor:
    return torch.rand(shape, generator=g, device=device, dtype=torch.float32) * 2e-3 + 1e-3


def make_inputs(shape: MoeShape, seed: int = 0, device="cpu", experts: int | None = None,
                with_weights: bool = True) -> dict:
    """Draw one configuration's inputs.

    ``experts`` limits how many experts' weights are drawn (a rank's local
    slice in tests); routing tensors always cover all ``shape.E`` experts.
    """
    shape.validate()
    T, H, I, E = shape.T, shape.H, shape.I, shape.E
    nE = E if experts is None else experts
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    d = {}
    d["x"] = torch.randn((T, H), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    d["router_w"] = torch.randn((E, H), generator=g, device=device, dtype=torch.float32) * 0.02
    d["router_bias"] = torch.rand((E,), generator=g, device=device, dtype=torch.float32) * 0.2 - 0.1
    if not with_weights:
        return d
    d["w13"] = _fp8_weights(nE, 2 * I, H, g, device)
    d["w13_scale"] = _scales((nE, 2 * I // BLOCK, H // BLOCK), g, device)
    d["w2"] = _fp8_weights(nE, H, I, g, device)
    d["w2_scale"] = _scales((nE, H // BLOCK, I // BLOCK), g, device)
    if shape.shared:
        d["shared_w13"] = _fp8_weights(1, 2 * I, H, g, device)[0]
        d["shared_w13_scale"] = _scales((2 * I // BLOCK, H // BLOCK), g, device)
        d["shared_w2"] = _fp8_weights(1, H, I, g, device)[0]
        d["shared_w2_scale"] = _scales((H // BLOCK, I // BLOCK), g, device)
    return d


def zipf_bias(shape: MoeShape, route_fn, router_w: torch.Tensor | None = None, s: float = 1.2, seed: int = 0,
              hot_ranks: int = 2, world: int = 8, iters: int = 60, probe_tokens: int = 4096,
              device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """Calibrate a router bias so expert popularity follows Zipf(s) (config c4).

    The popularity ranking is a seeded permutation whose hottest experts sit on
    ranks ``0 .. hot_ranks-1`` (expert-parallel ownership is contiguous:
    rank r owns experts [r*E/world, (r+1)*E/world)).  The bias is adjusted by a
    damped fixed-point iteration on a probe batch until the routed histogram
    tracks the Zipf target; returns (bias, achieved_histogram_fraction).
    ``route_fn(logits, bias) -> topk_idx [T, top_k]`` is the router to calibrate
    against (the CUDA router on a GPU box); ``router_w`` the router weights the
    bias will be used with (default: this module's seeded draw).
    """
    E = shape.E
    g = torch.Generator(device="cpu").manual_seed(seed + 7)
    per_rank = E // world
    hot = torch.arange(hot_ranks * per_rank)
    cold = torch.arange(hot_ranks * per_rank, E)
    order = torch.cat([hot[torch.randperm(hot.numel(), generator=g)],
                       cold[torch.randperm(cold.numel(), generator=g)]])
    ranks = torch.arange(1, E + 1, dtype=torch.float64)
    target_sorted = ranks.pow(-s)
    target_sorted /= target_sorted.sum()
    target = torch.empty(E, dtype=torch.float64)
    target[order] = target_sorted
    probe = make_inputs(shape.replace(T=probe_tokens), seed=seed + 11, device=device, with_weights=False)
    rw = probe["router_w"] if router_w is None else router_w.to(device)
    logits = probe["x"].float() @ rw.float().t()
    bias = torch.zeros(E, dtype=torch.float32, device=device)
    target = target.to(device)
    frac = None
    for _ in range(iters):
        idx = route_fn(logits, bias)
        hist = torch.bincount(idx.reshape(-1).long(), minlength=E).double()
        frac = hist / hist.sum()
        bias = bias + (0.05 * torch.log((target + 1e-6) / (frac + 1e-6))).float().clamp(-0.2, 0.2)
        # Routing is invariant to a common offset of the bias; keep it centred
        # so that sigmoid + bias stays near 1, where fp32 resolves the scores
        # finely (an offset of ~3 leaves 4x coarser spacing and more near-ties).
        bias = bias - bias.mean()
    return bias, frac
