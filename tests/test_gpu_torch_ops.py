"""GPU: the layer as PyTorch dispatcher operators (torch.ops.gemms_b200.moe /
run, csrc/torch_ops.cpp) calls the same C ABI as gemms_b200.moe / run: same
routing, results equal to the ctypes path up to the order of the fp32
combine atomics, and the Meta kernels give the output shape."""
import pytest
import torch

import gemms_b200
from gemms_b200 import workloads as W
from oracle import reference_moe as R
from tests import helpers as Hh

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _ops():
    gemms_b200.load_torch_ops()


def test_torch_op_moe_matches_python_operator():
    sh = W.CONFIGS["c0"].replace(T=96, shared=True)
    d = Hh.to_dev(W.make_inputs(sh, seed=31))
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf)
    shared = [d[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")]
    ref = gemms_b200.moe(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                         d["w2_scale"], shared_w13=shared[0], shared_w13_scale=shared[1], shared_w2=shared[2],
                         shared_w2_scale=shared[3], **kw)
    got = torch.ops.gemms_b200.moe(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                                   d["w2_scale"], *shared, sh.n_group, sh.topk_group, sh.top_k, sh.rsf, 2)
    torch.cuda.synchronize()
    assert got.dtype == torch.bfloat16 and got.shape == ref.shape
    m = R.compare(got.cpu(), ref.cpu())
    assert m["mae_rms"] <= 1e-4 and m["max_rel"] <= 1e-2, m


def test_torch_op_run_matches_reference_golden():
    g = Hh.load_golden()
    w = {k: v.cuda() for k, v in Hh.golden_weights(g).items() if isinstance(v, torch.Tensor)}
    out = torch.ops.gemms_b200.run(g["routing_logits"].cuda(), g["routing_bias"].cuda(), g["hidden_states"].cuda(),
                                   g["hidden_states_scale"].cuda(), w["w13"], w["w13_scale"], w["w2"],
                                   w["w2_scale"], 96, 2.5)
    torch.cuda.synchronize()
    Hh.assert_parity(out, Hh.golden_out(g, 96), "torch.ops.gemms_b200.run(off=96)")

