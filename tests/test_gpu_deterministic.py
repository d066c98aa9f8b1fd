"""GPU: the deterministic combine (``deterministic=True``).

Each (token, expert) result row is stored by GEMM2 and the rows are summed per
token in slot order (k routed experts, then the shared expert), so two calls
on the same inputs give the same bits; the default combine adds the rows with
fp32 atomics, whose order varies.  Checked: reruns bit-identical, parity with
the oracle (all rows) and with the reference's golden outputs, agreement with
the atomic combine to the last bf16 rounding.
"""
import pytest
import torch

import gemms_b200
from gemms_b200 import workloads as W
from oracle import reference_moe as R
from tests import helpers as Hh

pytestmark = pytest.mark.gpu


def _layer(sh, d, **extra):
    return gemms_b200.moe(
        d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
        shared_w13=d["shared_w13"], shared_w13_scale=d["shared_w13_scale"], shared_w2=d["shared_w2"],
        shared_w2_scale=d["shared_w2_scale"], n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k,
        routed_scaling_factor=sh.rsf, **extra)


def test_moe_deterministic_reruns_bit_identical_and_within_parity():
    sh = W.CONFIGS["c1"].replace(T=1024)
    d = W.make_inputs(sh, seed=11, device="cuda")
    outs = []
    for _ in range(3):
        out, idx, w, counts, logits = _layer(sh, d, deterministic=True, return_routing=True)
        outs.append(out)
    gemms_b200.check_device_errors(tag="moe(deterministic)")
    for o in outs[1:]:
        assert torch.equal(o, outs[0]), "deterministic combine changed between identical calls"
    atomic = _layer(sh, d)
    m = R.compare(outs[0].cpu(), atomic.cpu())
    print("deterministic vs atomic combine", m)
    # same products, another fp32 addition order: at most a last-bit flip of
    # a few bf16 roundings
    assert m["mae_rms"] < 5e-5 and m["max_rel"] < 8e-3, m
    cpu = {k: v.cpu() for k, v in d.items()}
    ref = R.moe_layer(cpu["x"], cpu["router_w"], cpu["router_bias"], cpu["w13"], cpu["w13_scale"], cpu["w2"],
                      cpu["w2_scale"], cpu["shared_w13"], cpu["shared_w13_scale"], cpu["shared_w2"],
                      cpu["shared_w2_scale"], n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k,
                      rsf=sh.rsf, logits=logits.cpu())
    Hh.assert_parity(outs[0], ref, "deterministic combine, c1 shapes T=1024, all rows")


def test_run_deterministic_matches_reference_golden():
    g = Hh.load_golden()
    d = {k: v.cuda() for k, v in Hh.golden_weights(g).items() if isinstance(v, torch.Tensor)}
    args = (g["routing_logits"].cuda(), g["routing_bias"].cuda(), g["hidden_states"].cuda(),
            g["hidden_states_scale"].cuda(), d["w13"], d["w13_scale"], d["w2"], d["w2_scale"], 96, 2.5)
    a = gemms_b200.run(*args, deterministic=True)
    b = gemms_b200.run(*args, deterministic=True)
    gemms_b200.check_device_errors(tag="run(deterministic)")
    assert torch.equal(a, b)
    Hh.assert_parity(a, Hh.golden_out(g, 96), "run(off=96, deterministic)")


def test_moe_block_deterministic_with_residual():
    """The fused residual add goes through the same fixed-order combine."""
    sh = W.CONFIGS["c0"].replace(T=200, shared=True)
    d = W.make_inputs(sh, seed=12, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    h = (torch.randn((sh.T, sh.H), generator=g, device="cuda") * 2).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(sh.H, generator=g, device="cuda")).to(torch.bfloat16)
    kw = dict(shared_w13=d["shared_w13"], shared_w13_scale=d["shared_w13_scale"], shared_w2=d["shared_w2"],
              shared_w2_scale=d["shared_w2_scale"], n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k,
              routed_scaling_factor=sh.rsf)
    args = (h, nw, d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"])
    a = gemms_b200.moe_block(*args, deterministic=True, **kw)
    b = gemms_b200.moe_block(*args, deterministic=True, **kw)
    c = gemms_b200.moe_block(*args, **kw)
    gemms_b200.check_device_errors(tag="moe_block(deterministic)")
    assert torch.equal(a, b)
    m = R.compare(a.cpu(), c.cpu())
    assert m["mae_rms"] < 5e-5 and m["max_rel"] < 8e-3, m
