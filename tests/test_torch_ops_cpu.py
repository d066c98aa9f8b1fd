"""CPU: torch.ops.gemms_b200.{moe, run} are registered by the extension built
over the C ABI; their Meta kernels give output shapes, and CPU tensors are
rejected (there is no CPU kernel: the product has no CPU path)."""
import pytest
import torch

import gemms_b200
from gemms_b200 import workloads as W


@pytest.fixture(scope="module", autouse=True)
def _ops():
    gemms_b200.load_torch_ops()


def test_ops_registered_with_reference_signature():
    schema = str(torch.ops.gemms_b200.run.default._schema)
    names = ["routing_logits", "routing_bias", "hidden_states", "hidden_states_scale", "gemm1_weights",
             "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale", "local_expert_offset",
             "routed_scaling_factor"]
    pos = [schema.index(n) for n in names]
    assert pos == sorted(pos), schema  # the reference run()'s argument order (flashinfer_baseline.py:5-16)
    assert torch.ops.gemms_b200.moe.default._schema.name == "gemms_b200::moe"


def test_meta_shapes():
    sh = W.CONFIGS["c0"].replace(T=5)
    d = W.make_inputs(sh, seed=1)
    meta = {k: v.to("meta") for k, v in d.items()}
    out = torch.ops.gemms_b200.moe(meta["x"], meta["router_w"], meta["router_bias"], meta["w13"],
                                   meta["w13_scale"], meta["w2"], meta["w2_scale"])
    assert out.shape == (5, sh.H) and out.dtype == torch.bfloat16 and out.device.type == "meta"
    hs = torch.empty((5, sh.H), dtype=torch.float8_e4m3fn, device="meta")
    out = torch.ops.gemms_b200.run(torch.empty((5, sh.E), device="meta"), meta["router_bias"], hs,
                                   torch.empty((sh.H // 128, 5), device="meta"), meta["w13"], meta["w13_scale"],
                                   meta["w2"], meta["w2_scale"], 0, 2.5)
    assert out.shape == (5, sh.H) and out.dtype == torch.bfloat16


def test_cpu_tensors_rejected():
    sh = W.CONFIGS["c0"].replace(T=5)
    d = W.make_inputs(sh, seed=1)
    with pytest.raises((RuntimeError, NotImplementedError)):
        torch.ops.gemms_b200.moe(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"],
                                 d["w2_scale"])
