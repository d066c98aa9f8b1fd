"""GPU: decode-sized batches (T <= 2) run the expert GEMMs on the CUDA cores
(csrc/decode.cu).  Every token is checked against the oracle, and the output
is compared with the tensor-core path on the same inputs
(``gemms_set_decode_max_t(0)``); the deterministic combine and the residual
path go through the same kernels."""
import pytest
import torch

import gemms_b200
from gemms_b200 import _lib
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


def _cpu_weights_for(d_dev, experts):
    out = {}
    for k in ("w13", "w13_scale", "w2", "w2_scale"):
        t = torch.empty(d_dev[k].shape, dtype=d_dev[k].dtype)
        for e in experts:
            t[e] = d_dev[k][e].cpu()
        out[k] = t
    return out


@pytest.fixture()
def decode_limit():
    L = _lib.load()
    prev = L.gemms_set_decode_max_t(4)
    yield L
    L.gemms_set_decode_max_t(prev)


@pytest.mark.parametrize("T", [1, 2, 3])
def test_decode_path_matches_oracle_and_tensor_path(decode_limit, T):
    L = decode_limit
    sh = W.CONFIGS["c2"].replace(T=T)
    d = W.make_inputs(sh, seed=20 + T, device="cuda")
    out, idx, w, counts, logits = _layer(sh, d, return_routing=True)
    det = _layer(sh, d, deterministic=True)
    det2 = _layer(sh, d, deterministic=True)
    gemms_b200.check_device_errors(tag="moe decode path")
    L.gemms_set_decode_max_t(0)
    tc = _layer(sh, d)
    gemms_b200.check_device_errors(tag="moe tensor path")
    lg = logits.cpu()
    ridx, _, _, _ = R.route(lg, d["router_bias"].cpu(), sh.n_group, sh.topk_group, sh.top_k, sh.rsf)
    assert torch.equal(Hh.sorted_sets(idx), Hh.sorted_sets(ridx))
    cw = _cpu_weights_for(d, sorted(set(ridx.reshape(-1).tolist())))
    ref = R.moe_layer(d["x"].cpu(), d["router_w"].cpu(), d["router_bias"].cpu(), cw["w13"], cw["w13_scale"],
                      cw["w2"], cw["w2_scale"], d["shared_w13"].cpu(), d["shared_w13_scale"].cpu(),
                      d["shared_w2"].cpu(), d["shared_w2_scale"].cpu(), n_group=8, topk_group=4, top_k=8, rsf=2.5,
                      logits=lg)
    Hh.assert_parity(out, ref, f"decode path T={T}")
    Hh.assert_parity(tc, ref, f"tensor path T={T}")
    Hh.assert_parity(det, ref, f"decode path, deterministic, T={T}")
    assert torch.equal(det, det2)
    # the decode path keeps the SwiGLU output in fp32 (the tensor path uses two
    # e4m3 planes), so it sits closer to the fp32 oracle
    m_dec, m_tc = R.compare(out.cpu(), ref), R.compare(tc.cpu(), ref)
    print(f"T={T}: decode path {m_dec}\n      tensor path {m_tc}")
    assert m_dec["mae_rms"] <= m_tc["mae_rms"] * 1.5 + 1e-5


def test_decode_path_small_geometry_and_residual(decode_limit):
    """c0 geometry (H=2048, I=768, E=32) with a residual, T=1..3 in a row
    (T=3 past the CUDA-core limit: the tensor cores take it)."""
    sh0 = W.CONFIGS["c0"].replace(shared=True)
    for T in (1, 2, 3):
        sh = sh0.replace(T=T)
        d = W.make_inputs(sh, seed=40 + T, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(T)
        res = torch.randn((T, sh.H), generator=g, device="cuda").to(torch.bfloat16)
        out, idx, w, counts, logits = _layer(sh, d, return_routing=True, residual=res)
        gemms_b200.check_device_errors(tag="moe decode path c0")
        cpu = {k: v.cpu() for k, v in d.items()}
        ref = R.moe_layer(cpu["x"], cpu["router_w"], cpu["router_bias"], cpu["w13"], cpu["w13_scale"], cpu["w2"],
                          cpu["w2_scale"], cpu["shared_w13"], cpu["shared_w13_scale"], cpu["shared_w2"],
                          cpu["shared_w2_scale"], n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k,
                          rsf=sh.rsf, logits=logits.cpu(), return_fp32=True)
        ref = (ref + res.cpu().float()).to(torch.bfloat16)
        Hh.assert_parity(out, ref, f"decode path c0 T={T} + residual")


def test_run_single_token_fp8_input_matches_reference_golden(decode_limit):
    """run() (FP8 input + given logits) one token at a time: the CUDA-core
    GEMM1 then reads the e4m3 rows and [H/128, T] scales of the input itself;
    each row must match the reference's own output for that token."""
    g = Hh.load_golden()
    d = {k: v.cuda() for k, v in Hh.golden_weights(g).items() if isinstance(v, torch.Tensor)}
    T = g["routing_logits"].shape[0]
    rows = []
    for t in range(T):
        rows.append(gemms_b200.run(g["routing_logits"][t:t + 1].contiguous().cuda(), g["routing_bias"].cuda(),
                                   g["hidden_states"][t:t + 1].contiguous().cuda(),
                                   g["hidden_states_scale"][:, t:t + 1].contiguous().cuda(), d["w13"],
                                   d["w13_scale"], d["w2"], d["w2_scale"], 96, 2.5))
    gemms_b200.check_device_errors(tag="run(T=1)")
    Hh.assert_parity(torch.cat(rows), Hh.golden_out(g, 96), "run(off=96), each token alone")
