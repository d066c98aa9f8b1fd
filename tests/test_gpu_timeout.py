"""GPU: a device-side wait that runs out ends the kernel with an error status.

The reference spins without a bound (persistent_kernel2.cu:747-757,
blackwell.h mbar_wait): a lost copy hangs the GPU.  Here every pipeline wait of
the grouped GEMMs is bounded.  The test hook ``gemms_test_inject_stall`` makes
CTA 0's TMA producer withhold one stage entirely (no expect_tx, no loads, so
nothing is left in flight) and shortens the wait limit to ~1 ms of SM cycles.
The MMA thread's wait for that stage then expires: the kernel sets the MMA-wait
bit of the device error word, drains what it issued, frees its tensor memory
and returns.  The stream completes within seconds, the host reads
GEMMS_ERR_TIMEOUT, and the next normal call is clean and matches the oracle.
"""
import time

import pytest
import torch

import gemms_b200
from gemms_b200 import _lib
from gemms_b200 import workloads as W
from oracle import reference_moe as R
from tests import helpers as Hh

pytestmark = pytest.mark.gpu

WAIT_BITS = _lib.FLAG_PRODUCER_WAIT | _lib.FLAG_MMA_WAIT | _lib.FLAG_EPILOGUE_WAIT
SHORT_LIMIT_CYCLES = 2_000_000  # ~1 ms at 2 GHz


def _case():
    sh = W.CONFIGS["c0"].replace(shared=True)
    d = W.make_inputs(sh, seed=5)
    dd = Hh.to_dev(d)
    kw = dict(n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, routed_scaling_factor=sh.rsf,
              **{k: dd[k] for k in ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")})

    def call():
        return gemms_b200.moe(dd["x"], dd["router_w"], dd["router_bias"], dd["w13"], dd["w13_scale"], dd["w2"],
                              dd["w2_scale"], return_routing=True, **kw)
    return sh, d, call


@pytest.mark.parametrize("gemm", [1, 2])
def test_expired_wait_reports_timeout_then_recovers(gemm):
    sh, d, call = _case()
    L = _lib.load()
    call()
    torch.cuda.synchronize()
    gemms_b200.check_device_errors(tag="moe")  # clean before the stall

    assert L.gemms_test_inject_stall(gemm, 3, SHORT_LIMIT_CYCLES) == 0
    try:
        t0 = time.monotonic()
        call()
        torch.cuda.synchronize()
        elapsed = time.monotonic() - t0
    finally:
        assert L.gemms_test_inject_stall(0, 0, 0) == 0
    assert elapsed < 10.0, f"stalled layer took {elapsed:.1f} s"
    with pytest.raises(gemms_b200.GemmsError) as ei:
        gemms_b200.check_device_errors(tag="moe")
    assert ei.value.code == _lib.GEMMS_ERR_TIMEOUT
    flags = ei.value.flags
    print(f"GEMM{gemm} stalled: {elapsed * 1e3:.0f} ms, error word 0x{flags:x}")
    assert flags & _lib.FLAG_MMA_WAIT, f"error word 0x{flags:x}"
    assert flags & ~WAIT_BITS == 0, f"error word 0x{flags:x}"
    # the check cleared the word; the next call is clean and correct
    out, idx, w, counts, logits = call()
    torch.cuda.synchronize()
    gemms_b200.check_device_errors(tag="moe")
    ref = R.moe_layer(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                      d["shared_w13"], d["shared_w13_scale"], d["shared_w2"], d["shared_w2_scale"],
                      n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k, rsf=sh.rsf, logits=logits.cpu())
    m = Hh.assert_parity(out, ref, f"after GEMM{gemm} timeout")
    print("recovered parity", m)

