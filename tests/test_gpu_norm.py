"""GPU: the steps either side of the layer -- RMSNorm fused with the 1x128
quantisation (gemms_rmsnorm_quant) and the residual add fused into the
layer's output cast -- against the oracle's definitions (oracle/reference_moe.py:
rmsnorm, moe_block; parity unpinned: the reference has no such code)."""
import pytest
import torch

import gemms_b200
from gemms_b200 import workloads as W
from oracle import reference_moe as R
from tests import helpers as Hh

pytestmark = pytest.mark.gpu


def _h(T, H, seed):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(T, H, generator=g) * 3
    h[0] *= 1e-3  # a nearly-zero row
    return h.to(torch.bfloat16)


@pytest.mark.parametrize("T,H,wdtype", [(1, 7168, torch.bfloat16), (77, 7168, torch.bfloat16),
                                        (4096, 7168, torch.bfloat16), (64, 2048, torch.float32)])
def test_rmsnorm_quant_matches_oracle(T, H, wdtype):
    h = _h(T, H, T + H)
    g = torch.Generator().manual_seed(5)
    wgt = (1 + 0.1 * torch.randn(H, generator=g)).to(wdtype)
    y, xq, sc = gemms_b200.rmsnorm_quant(h.cuda(), wgt.cuda(), 1e-6)
    torch.cuda.synchronize()
    ref = R.rmsnorm(h, wgt, 1e-6)
    yc = y.cpu()
    # The fp32 sum of squares runs in another order than torch's: the rsqrt
    # can move by an ulp, which can flip the bf16 rounding of h * rsqrt; the
    # product with the weight is rounded again, so y can move by up to ~2 of
    # its own bf16 ulps at such an element.
    diff = (yc.float() - ref.float()).abs()
    ulp = ref.float().abs().clamp_min(1e-30) * 2.0 ** -7
    assert bool((diff <= ulp * 2.01).all()), float((diff / ulp).max())
    assert float((diff > 0).double().mean()) < 1e-3
    # the quantisation is byte-exact on the kernel's own bf16 rows
    rq, rsc = R.quantize_1x128(yc)
    assert torch.equal(xq.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(sc.cpu(), rsc)


def test_moe_residual_is_added_once():
    sh = W.CONFIGS["c0"].replace(T=80, shared=True)
    d = Hh.to_dev(W.make_inputs(sh, seed=41))
    resid = _h(sh.T, sh.H, 9).cuda()
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf,
              **{k: d[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")})
    args = (d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"])
    out, idx, w, counts, logits = gemms_b200.moe(*args, residual=resid, return_routing=True, **kw)
    torch.cuda.synchronize()
    cpu = {k: v.cpu() for k, v in d.items()}
    ref32 = R.moe_layer(cpu["x"], cpu["router_w"], cpu["router_bias"], cpu["w13"], cpu["w13_scale"], cpu["w2"],
                        cpu["w2_scale"], cpu["shared_w13"], cpu["shared_w13_scale"], cpu["shared_w2"],
                        cpu["shared_w2_scale"], n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k,
                        rsf=sh.rsf, logits=logits.cpu(), return_fp32=True)
    ref = (ref32 + resid.cpu().float()).to(torch.bfloat16)
    Hh.assert_parity(out, ref, "moe + residual")


@pytest.mark.parametrize("cfg,T", [("c0", 96), ("c2", 8)])
def test_moe_block_matches_oracle(cfg, T):
    sh = W.CONFIGS[cfg].replace(T=T, shared=True)
    d = W.make_inputs(sh, seed=43, device="cuda")
    h = (d["x"].float() * 2).to(torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(3)
    nw = (1 + 0.1 * torch.randn(sh.H, generator=g, device="cuda")).to(torch.bfloat16)
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf)
    shared = {k: d[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")}
    out = gemms_b200.moe_block(h, nw, d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                               d["w2_scale"], eps=1e-6, **shared, **kw)
    y, _, _ = gemms_b200.rmsnorm_quant(h, nw, 1e-6)
    logits = gemms_b200.router_logits(y, d["router_w"])
    gemms_b200.check_device_errors(tag="moe_block")
    ridx = R.route(logits.cpu(), d["router_bias"].cpu(), sh.n_group, sh.topk_group, sh.top_k, sh.rsf)[0]
    experts = sorted(set(ridx.reshape(-1).tolist()))
    cw = {}
    for k in ("w13", "w13_scale", "w2", "w2_scale"):
        t = torch.empty(d[k].shape, dtype=d[k].dtype)
        for e in experts:
            t[e] = d[k][e].cpu()
        cw[k] = t
    ref = R.moe_block(h.cpu(), nw.cpu(), d["router_w"].cpu(), d["router_bias"].cpu(), cw["w13"], cw["w13_scale"],
                      cw["w2"], cw["w2_scale"], *[shared[k].cpu() for k in shared], n_group=sh.n_group,
                      topk_group=sh.topk_group, top_k=sh.top_k, rsf=sh.rsf, eps=1e-6, logits=logits.cpu())
    # the residual dominates the block's output: also check the MoE part alone
    Hh.assert_parity(out, ref, f"moe_block {cfg} T={T}")
    moe_part = out.float() - h.float()
    ref_part = ref.float() - h.cpu().float()
    m = R.compare(moe_part.cpu(), ref_part)
    print("moe part of the block", m)
    assert m["mae_rms"] <= 5e-3, m
