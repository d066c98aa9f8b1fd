"""CPU: the oracle restatement against the reference's own golden outputs."""
import hashlib

import numpy as np
import pytest
import torch

from gemms_b200 import workloads as W
from oracle import reference_moe as R
from tests import helpers as Hh
from tests.golden import make_golden as MG


@pytest.fixture(scope="module")
def golden():
    g = Hh.load_golden()
    d = Hh.golden_weights(g)
    return g, d


def test_golden_inputs_reproduce(golden):
    g, d = golden
    assert MG.weights_digest(d) == str(g["weights_sha256"]), "workload generator drifted from the fixture"
    # The small inputs are re-derivable from the same seed too.
    logits = R.router_logits(d["x"], d["router_w"])
    assert torch.equal(logits, g["routing_logits"])
    hs, hss = R.quantize_1x128(d["x"])
    assert torch.equal(hs.view(torch.uint8), g["hidden_states"].view(torch.uint8))
    assert torch.equal(hss, g["hidden_states_scale"])


@pytest.mark.parametrize("off", [0, 96, 224])
def test_oracle_bit_exact_vs_reference(golden, off):
    """oracle.run_local == reference flashinfer_baseline.run, bit for bit."""
    g, d = golden
    out = R.run_local(g["routing_logits"], g["routing_bias"], g["hidden_states"], g["hidden_states_scale"],
                      d["w13"], d["w13_scale"], d["w2"], d["w2_scale"], off, 2.5)
    ref = Hh.golden_out(g, off)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_exact_exp_routing_agrees_with_torch_exp():
    """Correctly-rounded sigmoid (what the CUDA router computes) selects the
    same expert sets as torch's CPU exp on seeded c1-shaped logits."""
    sh = W.CONFIGS["c1"].replace(T=2048)
    d = W.make_inputs(sh, seed=3, with_weights=False)
    logits = R.router_logits(d["x"], d["router_w"])
    a, wa, _, sb = R.route(logits, d["router_bias"], 8, 4, 8, 2.5)
    b, wb, _, _ = R.route(logits, d["router_bias"], 8, 4, 8, 2.5, exact_exp=True)
    assert torch.equal(Hh.sorted_sets(a), Hh.sorted_sets(b))
    torch.testing.assert_close(wa, wb, rtol=1e-6, atol=1e-7)
    eg, gg = R.routing_margins(sb, a, 8, 4)
    assert float(eg.min()) > 0 and float(gg.min()) > 0


def test_quantize_1x128_roundtrip():
    x = (torch.randn(16, 512) * 3).bfloat16()
    x[3, 128:256] = 0  # all-zero block -> scale 1, codes 0
    q, s = R.quantize_1x128(x)
    assert s.shape == (4, 16)
    assert float(s[1, 3]) == 1.0 and torch.all(q[3, 128:256].float() == 0)
    deq = R.dequant_hidden(q, s)
    rel = (deq - x.float()).abs().max() / x.float().abs().max()
    assert rel < 0.07  # e4m3: 3 mantissa bits
    # max of every block maps to +-448 exactly
    blk = (q.float().abs().view(16, 4, 128).amax(-1))
    assert torch.all((blk == 448) | (blk == 0))


def test_c0_oracle_runs_and_is_deterministic():
    sh = W.CONFIGS["c0"]
    d = W.make_inputs(sh, seed=0)
    a = R.moe_layer(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                    n_group=4, topk_group=2, top_k=4, rsf=2.5)
    b = R.moe_layer(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                    n_group=4, topk_group=2, top_k=4, rsf=2.5)
    assert a.shape == (64, 2048) and a.dtype == torch.bfloat16
    assert torch.equal(a, b) and torch.isfinite(a.float()).all() and a.float().abs().max() > 0


def test_token_subset_matches_full():
    sh = W.CONFIGS["c0"]
    d = W.make_inputs(sh, seed=5)
    kw = dict(n_group=4, topk_group=2, top_k=4, rsf=2.5, return_fp32=True)
    full = R.moe_layer(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"], **kw)
    rows = [0, 7, 33, 63]
    sub = R.moe_layer(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                      tokens=rows, **kw)
    torch.testing.assert_close(sub[rows], full[rows], rtol=1e-5, atol=1e-8)
    mask = torch.ones(64, dtype=torch.bool)
    mask[rows] = False
    assert torch.all(sub[mask] == 0)
