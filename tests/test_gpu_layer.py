"""GPU: full MoE layer parity against the oracle and the reference's golden outputs."""
import pytest
import torch

import gemms_b200
from gemms_b200 import workloads as W
from oracle import reference_moe as R
from tests import helpers as Hh

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden():
    g = Hh.load_golden()
    d = Hh.golden_weights(g)
    return g, d


@pytest.mark.parametrize("off", [0, 96, 224])
def test_run_matches_reference_golden(golden, off):
    """gemms_b200.run on the inputs the reference's own run() produced outputs for."""
    g, d = golden
    dev = {k: v.cuda() for k, v in d.items() if isinstance(v, torch.Tensor)}
    out, idx, w, counts = gemms_b200.run(g["routing_logits"].cuda(), g["routing_bias"].cuda(),
                                         g["hidden_states"].cuda(), g["hidden_states_scale"].cuda(), dev["w13"],
                                         dev["w13_scale"], dev["w2"], dev["w2_scale"], off, 2.5,
                                         return_routing=True)
    gemms_b200.check_device_errors(tag="run")
    ref = Hh.golden_out(g, off)
    Hh.assert_parity(out, ref, f"run(off={off})")
    ridx, _, _, _ = R.route(g["routing_logits"], g["routing_bias"], 8, 4, 8, 2.5)
    assert torch.equal(Hh.sorted_sets(idx), Hh.sorted_sets(ridx))
    loc = ridx[(ridx >= off) & (ridx < off + 32)] - off
    assert torch.equal(counts.cpu().long(), torch.bincount(loc, minlength=32))


def _moe_case(sh, seed, planes=2, device_inputs=True):
    d = W.make_inputs(sh, seed=seed)
    dd = Hh.to_dev(d)
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf,
              inter_planes=planes)
    shared = {k: dd[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale") if k in dd}
    out, idx, w, counts, logits = gemms_b200.moe(dd["x"], dd["router_w"], dd["router_bias"], dd["w13"],
                                                 dd["w13_scale"], dd["w2"], dd["w2_scale"], return_routing=True,
                                                 **shared, **kw)
    gemms_b200.check_device_errors(tag="moe")
    # routing parity at the reference boundary: identical fp32 logits in
    lg = logits.cpu()
    ref_logits = R.router_logits(d["x"], d["router_w"])
    torch.testing.assert_close(lg, ref_logits, rtol=1e-4, atol=1e-5 * float(ref_logits.abs().max()))
    ref = R.moe_layer(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                      d.get("shared_w13"), d.get("shared_w13_scale"), d.get("shared_w2"), d.get("shared_w2_scale"),
                      n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, rsf=sh.rsf, logits=lg)
    ridx, _, _, _ = R.route(lg, d["router_bias"], sh.n_group, sh.topk_group, sh.top_k, sh.rsf)
    assert torch.equal(Hh.sorted_sets(idx), Hh.sorted_sets(ridx))
    assert torch.equal(counts.cpu().long(), torch.bincount(ridx.reshape(-1), minlength=sh.E))
    return out, ref


def test_moe_c0():
    out, ref = _moe_case(W.CONFIGS["c0"], seed=0)
    m = Hh.assert_parity(out, ref, "c0")
    print("c0 parity", m)


def test_moe_c0_three_planes():
    out, ref = _moe_case(W.CONFIGS["c0"], seed=1, planes=3)
    m = Hh.assert_parity(out, ref, "c0 planes=3")
    assert m["mae_rms"] < 2e-4


@pytest.mark.parametrize("T", [1, 3, 130, 300])
def test_moe_c0_ragged_T_with_shared(T):
    sh = W.CONFIGS["c0"].replace(T=T, shared=True)
    out, ref = _moe_case(sh, seed=T)
    Hh.assert_parity(out, ref, f"c0 T={T} shared")


def test_run_expert_slice_without_hits():
    """Local expert slice that no token routes to: output is exactly zero."""
    g = torch.Generator().manual_seed(9)
    T, H, I, E = 16, 256, 128, 32
    logits = torch.full((T, E), -8.0)
    logits[:, :8] = torch.randn(T, 8, generator=g) + 4  # everyone picks experts 0..7
    bias = torch.zeros(E)
    hs = torch.randn(T, H, generator=g).to(torch.float8_e4m3fn)
    hss = torch.ones(H // 128, T)
    w13 = torch.randn(8, 2 * I, H, generator=g).to(torch.float8_e4m3fn)
    w2 = torch.randn(8, H, I, generator=g).to(torch.float8_e4m3fn)
    s13 = torch.full((8, 2 * I // 128, H // 128), 1e-3)
    s2 = torch.full((8, H // 128, I // 128), 1e-3)
    out = gemms_b200.run(logits.cuda(), bias.cuda(), hs.cuda(), hss.cuda(), w13.cuda(), s13.cuda(), w2.cuda(),
                         s2.cuda(), 24, 2.5, n_group=4, topk_group=2, top_k=4)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0
    ref = R.run_local(logits, bias, hs, hss, w13, s13, w2, s2, 0, 2.5, n_group=4, topk_group=2, top_k=4)
    out0 = gemms_b200.run(logits.cuda(), bias.cuda(), hs.cuda(), hss.cuda(), w13.cuda(), s13.cuda(), w2.cuda(),
                          s2.cuda(), 0, 2.5, n_group=4, topk_group=2, top_k=4)
    Hh.assert_parity(out0, ref, "slice 0")


def test_shape_errors_raise():
    x = torch.zeros(4, 7168, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(AssertionError):  # reference-style assertion semantics
        gemms_b200.run(torch.zeros(4, 256, device="cuda"), torch.zeros(256, device="cuda"),
                       x.to(torch.float8_e4m3fn), torch.ones(55, 4, device="cuda"),
                       torch.zeros(32, 4096, 7168, device="cuda", dtype=torch.float8_e4m3fn),
                       torch.ones(32, 32, 56, device="cuda"),
                       torch.zeros(32, 7168, 2048, device="cuda", dtype=torch.float8_e4m3fn),
                       torch.ones(32, 56, 16, device="cuda"), 0, 2.5)


def _cpu_weights_for(d_dev, experts):
    """CPU copies of only the experts the sampled tokens use (others left unset)."""
    E = d_dev["w13"].shape[0]
    out = {}
    for k in ("w13", "w13_scale", "w2", "w2_scale"):
        t = torch.empty(d_dev[k].shape, dtype=d_dev[k].dtype)
        for e in experts:
            t[e] = d_dev[k][e].cpu()
        out[k] = t
    return out


def _full_layer(sh, d, **extra):
    return gemms_b200.moe(
        d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
        shared_w13=d["shared_w13"], shared_w13_scale=d["shared_w13_scale"], shared_w2=d["shared_w2"],
        shared_w2_scale=d["shared_w2_scale"], n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k,
        routed_scaling_factor=sh.rsf, return_routing=True, **extra)


def _check_routing(sh, idx, counts, lg, bias):
    """Top-k sets of every token and per-expert counts equal the oracle's on
    the same fp32 logits, with the reference's torch sigmoid and with the
    correctly rounded one; on failure the message gives the decision margins
    of the tokens that differ."""
    got = Hh.sorted_sets(idx)
    ridx, _, _, _ = R.route(lg, bias, sh.n_group, sh.topk_group, sh.top_k, sh.rsf)
    eidx, _, _, sb = R.route(lg, bias, sh.n_group, sh.topk_group, sh.top_k, sh.rsf, exact_exp=True)
    dt = (got != Hh.sorted_sets(ridx)).any(1)
    de = (got != Hh.sorted_sets(eidx)).any(1)
    if dt.any() or de.any():
        eg, gg = R.routing_margins(sb, eidx, sh.n_group, sh.topk_group)
        bad = torch.nonzero(dt | de).squeeze(1)[:8].tolist()
        detail = [(t, float(eg[t]), float(gg[t]), Hh.sorted_sets(idx)[t].tolist(), Hh.sorted_sets(eidx)[t].tolist())
                  for t in bad]
        raise AssertionError(f"{int(dt.sum())} tokens differ from the torch-exp oracle and {int(de.sum())} from the "
                             f"exact-exp oracle (of {sh.T}); min margins expert {float(eg.min()):.3e} group "
                             f"{float(gg.min()):.3e}; first (token, expert gap, group gap, gpu, oracle): {detail}")
    assert torch.equal(counts.cpu().long(), torch.bincount(ridx.reshape(-1), minlength=sh.E))
    assert int(counts.sum()) == sh.T * sh.top_k
    return ridx


@pytest.mark.slow
def test_moe_c1_all_rows():
    """Config c1 (T=4096, full V3 + shared expert): routing of all tokens exact
    and every one of the 4096 output rows within the parity bar (the oracle
    runs the whole layer on the host cores)."""
    sh = W.CONFIGS["c1"]
    d = W.make_inputs(sh, seed=0, device="cuda")
    out, idx, w, counts, logits = _full_layer(sh, d)
    gemms_b200.check_device_errors(tag="moe")
    lg = logits.cpu()
    cpu = {k: v.cpu() for k, v in d.items()}
    _check_routing(sh, idx, counts, lg, cpu["router_bias"])
    ref = R.moe_layer(cpu["x"], cpu["router_w"], cpu["router_bias"], cpu["w13"], cpu["w13_scale"], cpu["w2"],
                      cpu["w2_scale"], cpu["shared_w13"], cpu["shared_w13_scale"], cpu["shared_w2"],
                      cpu["shared_w2_scale"], n_group=8, topk_group=4, top_k=8, rsf=2.5, logits=lg)
    Hh.assert_parity(out, ref, "c1 all 4096 rows")
    assert torch.isfinite(out.float()).all()


@pytest.mark.slow
@pytest.mark.parametrize("T", [1, 8, 32, 128])
def test_moe_decode_full_size(T):
    """Config c2 (decode, full V3 + shared expert): every token checked against
    the oracle.  At T=1/8 almost every expert gets 0 or 1 rows (nearly empty M
    tiles); at T=32/128 tiles start to fill."""
    sh = W.CONFIGS["c2"].replace(T=T)
    d = W.make_inputs(sh, seed=7, device="cuda")
    out, idx, w, counts, logits = _full_layer(sh, d)
    gemms_b200.check_device_errors(tag="moe decode")
    lg = logits.cpu()
    bias = d["router_bias"].cpu()
    ridx = _check_routing(sh, idx, counts, lg, bias)
    experts = sorted(set(ridx.reshape(-1).tolist()))
    cw = _cpu_weights_for(d, experts)
    ref = R.moe_layer(d["x"].cpu(), d["router_w"].cpu(), bias, cw["w13"], cw["w13_scale"], cw["w2"],
                      cw["w2_scale"], d["shared_w13"].cpu(), d["shared_w13_scale"].cpu(), d["shared_w2"].cpu(),
                      d["shared_w2_scale"].cpu(), n_group=8, topk_group=4, top_k=8, rsf=2.5, logits=lg)
    Hh.assert_parity(out, ref, f"c2 T={T}")


@pytest.mark.slow
def test_moe_c4_skewed_routing():
    """Config c4's skewed routing (router bias calibrated so expert popularity
    follows Zipf(1.2), hottest experts in groups 0-1) on one GPU with all 256
    experts and T=16384: routing sets and counts exact; output rows of tokens
    sampled across the M-tile boundaries of the two hottest experts (thousands
    of rows each, tens of 128-row tiles, a ragged tail tile) within the bar."""
    sh = W.CONFIGS["c4"]
    d = W.make_inputs(sh, seed=3, device="cuda")

    def route_fn(lg, b):
        return gemms_b200.route(lg, b, n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k,
                                routed_scaling_factor=sh.rsf, counts=False)[0]

    bias, frac = W.zipf_bias(sh, route_fn, router_w=d["router_w"], s=1.2, seed=0, hot_ranks=2, world=8,
                             device="cuda")
    d["router_bias"] = bias
    out, idx, w, counts, logits = _full_layer(sh, d)
    gemms_b200.check_device_errors(tag="moe c4")
    lg = logits.cpu()
    cbias = bias.cpu()
    ridx = _check_routing(sh, idx, counts, lg, cbias)
    c = counts.cpu().long()
    hot = torch.argsort(c, descending=True)[:2].tolist()
    print("c4 hottest experts", hot, "rows", [int(c[e]) for e in hot], "share of top expert",
          float(c.max()) / float(c.sum()))
    assert int(c[hot[0]]) > 4 * 128  # several M tiles
    rows = set()
    for e in hot:
        toks = torch.nonzero((ridx == e).any(1)).squeeze(1)  # token order = row order within the expert
        n = toks.numel()
        for pos in (0, 1, 127, 128, 129, 255, 256, n // 2, n - 129, n - 128, n - 2, n - 1):
            if 0 <= pos < n:
                rows.add(int(toks[pos]))
    g = torch.Generator().manual_seed(0)
    rows |= set(torch.randint(0, sh.T, (6,), generator=g).tolist())
    rows = sorted(rows)
    experts = sorted(set(ridx[rows].reshape(-1).tolist()))
    cw = _cpu_weights_for(d, experts)
    ref = R.moe_layer(d["x"].cpu(), d["router_w"].cpu(), cbias, cw["w13"], cw["w13_scale"], cw["w2"],
                      cw["w2_scale"], d["shared_w13"].cpu(), d["shared_w13_scale"].cpu(), d["shared_w2"].cpu(),
                      d["shared_w2_scale"].cpu(), n_group=8, topk_group=4, top_k=8, rsf=2.5, logits=lg,
                      tokens=rows)
    Hh.assert_parity(out, ref, f"c4 skewed, {len(rows)} sampled rows", rows=rows)


def test_gemm_cta_bound_keeps_results():
    """gemms_set_gemm_ctas: the persistent GEMMs stride their work units over
    however many CTAs they get; a small grid gives the same layer output (up to
    the order of the fp32 combine atomics)."""
    from gemms_b200 import _lib
    L = _lib.load()
    sh = W.CONFIGS["c0"].replace(shared=True)
    d = Hh.to_dev(W.make_inputs(sh, seed=4))
    args = (d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"])
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf,
              **{k: d[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")})
    full = gemms_b200.moe(*args, **kw).float()
    assert L.gemms_set_gemm_ctas(-1) == -8  # GEMMS_ERR_ARG
    prev = L.gemms_set_gemm_ctas(5)
    try:
        small = gemms_b200.moe(*args, **kw).float()
        torch.cuda.synchronize()
    finally:
        assert L.gemms_set_gemm_ctas(prev) == 5
    gemms_b200.check_device_errors(tag="cta bound")
    assert (small - full).norm() <= 1e-3 * full.norm()


def test_concurrent_streams_do_not_share_scratch():
    """Layers launched on two streams at once (each with its own inputs) give
    what they give when run one after the other."""
    sh = W.CONFIGS["c0"].replace(shared=True)
    d = Hh.to_dev(W.make_inputs(sh, seed=9))
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf,
              **{k: d[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")})
    wts = (d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"])
    xs = [d["x"], (d["x"].float() * -0.5).to(torch.bfloat16)]
    serial = [gemms_b200.moe(x, *wts, **kw).float() for x in xs]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [None, None]
    for _ in range(3):
        for i, st in enumerate(streams):
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                outs[i] = gemms_b200.moe(xs[i], *wts, **kw)
        torch.cuda.synchronize()
        for i in range(2):
            o = outs[i].float()
            assert (o - serial[i]).norm() <= 1e-3 * serial[i].norm(), f"stream {i}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_second_device_in_one_process():
    """One process, two GPUs: the layer on cuda:1 tensors while cuda:0 is the
    current device runs on cuda:1 (kernels go to the tensors' device) and
    matches the same layer on cuda:0 (each device gets the GEMMs' shared-memory
    opt-in)."""
    sh = W.CONFIGS["c0"].replace(shared=True)
    cpu = W.make_inputs(sh, seed=6)
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf)
    outs = []
    for dev in ("cuda:0", "cuda:1"):
        d = Hh.to_dev(cpu, dev)
        torch.cuda.set_device(0)
        out = gemms_b200.moe(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                             d["w2_scale"], shared_w13=d["shared_w13"], shared_w13_scale=d["shared_w13_scale"],
                             shared_w2=d["shared_w2"], shared_w2_scale=d["shared_w2_scale"], **kw)
        assert out.device == torch.device(dev)
        torch.cuda.synchronize(dev)
        outs.append(out.float().cpu())
    assert (outs[1] - outs[0]).norm() <= 1e-3 * outs[0].norm()
