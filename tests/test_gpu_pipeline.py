"""GPU: MoePipeline (host-to-host, copies overlapped) gives the outputs of moe().

The combine accumulates expert contributions with fp32 atomics, so two runs may
differ in the last bf16 bit of a few elements; the comparison is normwise."""
import pytest
import torch

import gemms_b200
from gemms_b200 import workloads as W
from tests import helpers as Hh

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("slots", [1, 2, 3])
def test_pipeline_matches_moe(slots):
    sh = W.CONFIGS["c0"]
    d = Hh.to_dev(W.make_inputs(sh, seed=11))
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf)
    g = torch.Generator().manual_seed(5)
    xs = [(torch.randn(sh.T, sh.H, generator=g) * (1 + i)).to(torch.bfloat16).pin_memory() for i in range(5)]
    ys = [torch.empty(sh.T, sh.H, dtype=torch.bfloat16).pin_memory() for _ in range(5)]
    pipe = gemms_b200.MoePipeline(d, slots=slots, **kw)
    pipe.run(xs, ys)
    gemms_b200.check_device_errors(tag="pipeline")
    shared = {k: d[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale") if k in d}
    for i in range(5):
        ref = gemms_b200.moe(xs[i].cuda(), d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                             d["w2_scale"], **shared, **kw)
        y, r = ys[i].float(), ref.cpu().float()
        err = (y - r).norm() / r.norm()
        assert err < 1e-3, f"batch {i}: normwise diff {err:.3e}"
        assert (y - r).abs().max() <= 2 ** -6 * r.abs().max(), f"batch {i}"


def test_pipeline_length_mismatch():
    sh = W.CONFIGS["c0"]
    d = Hh.to_dev(W.make_inputs(sh, seed=1))
    with pytest.raises(ValueError):
        gemms_b200.MoePipeline(d).run([torch.empty(1)], [])
