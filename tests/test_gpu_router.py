"""GPU: the CUDA router against the oracle's routing (flashinfer_baseline.py:95-127).

Top-k expert sets and per-expert counts must match bit for bit given identical
fp32 logits; normalised weights to fp32 rounding.
"""
import pytest
import torch

import gemms_b200
from gemms_b200 import workloads as W
from oracle import reference_moe as R
from tests import helpers as Hh

pytestmark = pytest.mark.gpu


def _check(logits, bias, ng, tg, k, rsf=2.5):
    idx, w, counts = gemms_b200.route(logits.cuda(), bias.cuda(), n_group=ng, topk_group=tg, top_k=k,
                                      routed_scaling_factor=rsf)
    torch.cuda.synchronize()
    ref_idx, ref_w, _, sb = R.route(logits.cpu(), bias.cpu().float(), ng, tg, k, rsf, exact_exp=True)
    ref_idx_t, _, _, _ = R.route(logits.cpu(), bias.cpu().float(), ng, tg, k, rsf, exact_exp=False)
    got = Hh.sorted_sets(idx)
    eg, gg = R.routing_margins(sb, ref_idx, ng, tg)
    diag = f"min expert gap {float(eg.min()):.3e}, min group gap {float(gg.min()):.3e}"
    assert torch.equal(got, Hh.sorted_sets(ref_idx)), "top-k sets differ from oracle (exact exp); " + diag
    assert torch.equal(got, Hh.sorted_sets(ref_idx_t)), "top-k sets differ from oracle (torch exp); " + diag
    E = logits.shape[1]
    ref_counts = torch.bincount(ref_idx.reshape(-1), minlength=E)
    assert torch.equal(counts.cpu().long(), ref_counts)
    # weights: gather dense oracle weights at the selected experts
    wg = torch.gather(ref_w, 1, idx.cpu().long())
    torch.testing.assert_close(w.cpu(), wg, rtol=2e-6, atol=1e-7)
    assert torch.all(w.cpu() > 0)


@pytest.mark.parametrize("cfg,T", [("c0", 64), ("c1", 4096), ("c1", 1), ("c1", 33)])
def test_router_matches_oracle(cfg, T):
    sh = W.CONFIGS[cfg].replace(T=T)
    d = W.make_inputs(sh, seed=11, with_weights=False)
    logits = R.router_logits(d["x"], d["router_w"])
    _check(logits, d["router_bias"], sh.n_group, sh.topk_group, sh.top_k)


@pytest.mark.parametrize("E,ng,tg,k", [(64, 32, 4, 4), (128, 8, 3, 6), (256, 16, 8, 16), (32, 2, 1, 3), (16, 4, 2, 2)])
def test_router_geometries(E, ng, tg, k):
    g = torch.Generator().manual_seed(E * 7 + k)
    logits = torch.randn(300, E, generator=g) * 2
    bias = (torch.rand(E, generator=g) - 0.5) * 0.2
    _check(logits, bias, ng, tg, k)


def test_router_bf16_bias():
    g = torch.Generator().manual_seed(2)
    logits = torch.randn(512, 256, generator=g) * 1.7
    bias = ((torch.rand(256, generator=g) - 0.5) * 0.2).bfloat16()
    _check(logits, bias, 8, 4, 8)


def test_router_large_logits_saturate():
    # |logit| large: sigmoid saturates to 0/1; ties among saturated scores are
    # broken by bias, all finite.
    g = torch.Generator().manual_seed(4)
    logits = torch.randn(64, 256, generator=g) * 60
    bias = (torch.rand(256, generator=g) - 0.5) * 0.2
    _check(logits, bias, 8, 4, 8)


def _logits_err(got, ref):
    d = (got.double() - ref.double()).abs()
    return float(d.max() / ref.double().abs().max())


@pytest.mark.parametrize("cfg,T", [("c0", 64), ("c1", 4096), ("c1", 1), ("c1", 130), ("c2", 32)])
def test_router_gemm_matches_fp32(cfg, T):
    """The sm_100a router GEMM (bf16 hi/lo split of router_w, fp32 accumulation
    on the tensor cores) against the oracle's fp32 x . router_w^T: normwise
    relative error <= 1e-5 and every element within 1e-5 of max|logit| (an
    fp32 sum over H=7168 products carries rounding of that order in any
    summation order; the CPU sgemm's and the tensor cores' differ); two calls
    give identical bits (split-K partials summed in a fixed order); the CUDA
    router fed these logits routes exactly like the oracle fed them."""
    sh = W.CONFIGS[cfg].replace(T=T)
    d = W.make_inputs(sh, seed=13, with_weights=False)
    x, rw = d["x"].cuda(), d["router_w"].cuda()
    got = gemms_b200.router_logits(x, rw)
    again = gemms_b200.router_logits(x, rw)
    torch.cuda.synchronize()
    ref = R.router_logits(d["x"], d["router_w"])
    err = _logits_err(got.cpu(), ref)
    print(f"{cfg} T={T}: router GEMM normwise rel err {err:.2e}")
    assert err <= 1e-5
    torch.testing.assert_close(got.cpu(), ref, rtol=1e-4, atol=1e-5 * float(ref.abs().max()))
    assert torch.equal(got, again)
    _check(got.cpu(), d["router_bias"], sh.n_group, sh.topk_group, sh.top_k)


def test_router_gemm_small_expert_count():
    """E not a multiple of 16 (MMA N padded with zero weight rows)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(77, 256, generator=g).bfloat16()
    rw = torch.randn(24, 256, generator=g) * 0.02
    got = gemms_b200.router_logits(x.cuda(), rw.cuda()).cpu()
    ref = R.router_logits(x, rw)
    assert _logits_err(got, ref) <= 1e-5
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5 * float(ref.abs().max()))


@pytest.mark.parametrize("E,ng,tg,k", [(256, 8, 4, 8), (64, 32, 4, 4), (128, 8, 3, 6), (256, 16, 8, 16), (32, 2, 1, 3),
                                       (16, 4, 2, 2), (256, 128, 16, 8)])
def test_router_small_batch_kernel_matches_large_batch_kernel(E, ng, tg, k):
    """Batches of <= 64 tokens go through the block-per-token router, larger
    ones through the warp-per-token router; routing is per token, so the
    first 48 tokens routed alone must give exactly what they give inside a
    batch of 300 (ids, weights, counts)."""
    g = torch.Generator().manual_seed(E + 13 * k)
    logits = (torch.randn(300, E, generator=g) * 2).cuda()
    bias = ((torch.rand(E, generator=g) - 0.5) * 0.2).cuda()
    idx_l, w_l, _ = gemms_b200.route(logits, bias, n_group=ng, topk_group=tg, top_k=k, routed_scaling_factor=2.5)
    idx_s, w_s, c_s = gemms_b200.route(logits[:48].contiguous(), bias, n_group=ng, topk_group=tg, top_k=k,
                                       routed_scaling_factor=2.5)
    torch.cuda.synchronize()
    assert torch.equal(idx_s, idx_l[:48])
    assert torch.equal(w_s, w_l[:48])
    assert torch.equal(c_s.cpu().long(), torch.bincount(idx_s.reshape(-1).cpu().long(), minlength=E))


@pytest.mark.parametrize("E,ng,tg,k", [(256, 8, 4, 8), (128, 8, 3, 6), (256, 16, 8, 16)])
def test_router_exact_ties_same_in_both_kernels(E, ng, tg, k):
    """Logits on a coarse grid and a zero bias make many experts (and groups)
    score exactly the same.  Both routers break every tie towards the lower
    expert (and group) index; the block-per-token router (<= 64 tokens) and
    the warp-per-token router (larger batches) implement that order
    differently, so on tied inputs they must still agree bit for bit.  (torch's
    topk gives no order for ties, so the oracle cannot judge these cases.)"""
    g = torch.Generator().manual_seed(101 + E + k)
    logits = (torch.randint(-3, 4, (300, E), generator=g).float() * 0.5).cuda()
    bias = torch.zeros(E).cuda()
    idx_l, w_l, c_l = gemms_b200.route(logits, bias, n_group=ng, topk_group=tg, top_k=k, routed_scaling_factor=2.5)
    idx_s, w_s, _ = gemms_b200.route(logits[:48].contiguous(), bias, n_group=ng, topk_group=tg, top_k=k,
                                     routed_scaling_factor=2.5)
    torch.cuda.synchronize()
    assert torch.equal(idx_s, idx_l[:48])
    assert torch.equal(w_s, w_l[:48])
    assert torch.equal(c_l.cpu().long(), torch.bincount(idx_l.reshape(-1).cpu().long(), minlength=E))
    # every token's k experts are distinct
    assert all(len(set(row.tolist())) == k for row in idx_l.cpu())
