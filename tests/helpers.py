"""Shared helpers of the test-suite (inputs, oracle calls, parity checks)."""
from __future__ import annotations

import os

import numpy as np
import torch

from gemms_b200 import workloads as W
from oracle import reference_moe as R

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_run_v3.npz")

# Parity bar: normwise max relative error and MAE/RMS.
MAX_REL = 2e-2
MAE_RMS = 1e-3


def load_golden():
    z = np.load(GOLDEN)
    g = {k: z[k] for k in z.files}
    g["routing_logits"] = torch.from_numpy(g["routing_logits"])
    g["routing_bias"] = torch.from_numpy(g["routing_bias"])
    g["hidden_states"] = torch.from_numpy(g["hidden_states"]).view(torch.float8_e4m3fn)
    g["hidden_states_scale"] = torch.from_numpy(g["hidden_states_scale"])
    return g


def golden_weights(g):
    sh = W.CONFIGS["c1"].replace(T=int(g["T"]), shared=False)
    return W.make_inputs(sh, seed=int(g["seed"]), experts=32)


def golden_out(g, off):
    return torch.from_numpy(g[f"out_off{off}"]).view(torch.bfloat16)


def sorted_sets(idx: torch.Tensor) -> torch.Tensor:
    return torch.sort(idx.to(torch.int64).cpu(), dim=1).values


def assert_parity(out: torch.Tensor, ref: torch.Tensor, what: str = "", rows=None):
    m = R.compare(out.cpu(), ref.cpu(), rows=rows)
    assert m["max_rel"] <= MAX_REL and m["mae_rms"] <= MAE_RMS, f"{what} parity failed: {m}"
    return m


def to_dev(d: dict, device="cuda") -> dict:
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}
