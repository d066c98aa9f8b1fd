"""GPU: gemms_moe_fwd_noalloc, the layer forward for callers that cannot
allocate device memory (plugin hosts that hand over a stream but no
allocator, runtimes that forbid allocations once serving starts).  Its scratch
is a fixed 16 MiB array inside the library, so it only takes decode-sized
batches.  Checked through the C ABI against gemms_moe_fwd (caller workspace)
on the same inputs, on two calls in a row.

Collected last on purpose (file name): if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes

import pytest
import torch

import gemms_b200
from gemms_b200 import _lib
from gemms_b200 import workloads as W
from gemms_b200._lib import GemmsMoeArgs, GemmsMoeShape
from oracle import reference_moe as R

pytestmark = pytest.mark.gpu

GEMMS_ERR_CAPACITY = -9
MAX_REL, MAE_RMS = 2e-2, 1e-3  # the layer parity bar used by every test


def _entry_points():
    L = _lib.load()
    return L, L.gemms_moe_fwd, L.gemms_moe_fwd_noalloc


def _make_args(sh, d, logits, out, idx):
    shape = GemmsMoeShape(T=sh.T, H=sh.H, I=sh.I, E=sh.E, E_local=sh.E, local_expert_offset=0,
                          n_group=sh.n_group, topk_group=sh.topk_group, top_k=sh.top_k,
                          has_shared=int(sh.shared), input_mode=_lib.GEMMS_INPUT_BF16, bias_bf16=0,
                          inter_planes=2, routed_scaling_factor=sh.rsf)
    a = GemmsMoeArgs()
    a.shape = shape
    a.routing_logits = logits.data_ptr()
    a.routing_bias = d["router_bias"].data_ptr()
    a.hidden_bf16 = d["x"].data_ptr()
    a.w13, a.w13_scale = d["w13"].data_ptr(), d["w13_scale"].data_ptr()
    a.w2, a.w2_scale = d["w2"].data_ptr(), d["w2_scale"].data_ptr()
    if sh.shared:
        a.shared_w13, a.shared_w13_scale = d["shared_w13"].data_ptr(), d["shared_w13_scale"].data_ptr()
        a.shared_w2, a.shared_w2_scale = d["shared_w2"].data_ptr(), d["shared_w2_scale"].data_ptr()
    a.out = out.data_ptr()
    a.topk_idx_out = idx.data_ptr()
    return shape, a


@pytest.mark.parametrize("cfg,T", [("c0", 64), ("c2", 8)])
def test_noalloc_matches_workspace_entry_point(cfg, T):
    sh = W.CONFIGS[cfg].replace(T=T, shared=True)
    d = W.make_inputs(sh, seed=21, device="cuda")
    logits = gemms_b200.router_logits(d["x"], d["router_w"])
    L, fwd, noalloc = _entry_points()
    stream = torch.cuda.current_stream().cuda_stream

    ref = torch.empty((sh.T, sh.H), dtype=torch.bfloat16, device="cuda")
    ref_idx = torch.empty((sh.T, sh.top_k), dtype=torch.int32, device="cuda")
    shape, a = _make_args(sh, d, logits, ref, ref_idx)
    nbytes = L.gemms_moe_workspace_size(ctypes.byref(shape))
    assert 0 < nbytes <= (16 << 20)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device="cuda")
    ws_ptr = ws.data_ptr() + ((-ws.data_ptr()) % 256)
    assert fwd(ctypes.byref(a), ws_ptr, nbytes, stream) == 0

    for call in range(2):
        out = torch.full((sh.T, sh.H), float("nan"), dtype=torch.bfloat16, device="cuda")
        idx = torch.full((sh.T, sh.top_k), -1, dtype=torch.int32, device="cuda")
        _, b = _make_args(sh, d, logits, out, idx)
        rc = noalloc(ctypes.byref(b), stream)
        assert rc == 0, f"call {call}: {_lib.strerror(rc)}"
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx), f"call {call}: routing differs from gemms_moe_fwd"
        m = R.compare(out.cpu(), ref.cpu())
        assert m["max_rel"] <= MAX_REL and m["mae_rms"] <= MAE_RMS, f"call {call}: {m}"
    flags = ctypes.c_int32(-1)
    assert L.gemms_moe_check_noalloc(stream, ctypes.byref(flags)) == 0
    assert flags.value == 0


def test_noalloc_reports_an_expired_device_wait():
    """A device-side wait that runs out inside a no-alloc call (forced with the
    test hook) is reported by gemms_moe_check_noalloc, which also clears it;
    the next call is clean and matches the workspace entry point."""
    sh = W.CONFIGS["c0"].replace(T=16, shared=True)
    d = W.make_inputs(sh, seed=22, device="cuda")
    logits = gemms_b200.router_logits(d["x"], d["router_w"])
    L, fwd, noalloc = _entry_points()
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty((sh.T, sh.H), dtype=torch.bfloat16, device="cuda")
    ref_idx = torch.empty((sh.T, sh.top_k), dtype=torch.int32, device="cuda")
    shape, a = _make_args(sh, d, logits, ref, ref_idx)
    nbytes = L.gemms_moe_workspace_size(ctypes.byref(shape))
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device="cuda")
    assert fwd(ctypes.byref(a), ws.data_ptr() + ((-ws.data_ptr()) % 256), nbytes, stream) == 0

    out = torch.empty((sh.T, sh.H), dtype=torch.bfloat16, device="cuda")
    idx = torch.empty((sh.T, sh.top_k), dtype=torch.int32, device="cuda")
    _, b = _make_args(sh, d, logits, out, idx)
    assert L.gemms_test_inject_stall(1, 2, 2_000_000) == 0
    try:
        assert noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize()
    finally:
        assert L.gemms_test_inject_stall(0, 0, 0) == 0
    flags = ctypes.c_int32(0)
    assert L.gemms_moe_check_noalloc(stream, ctypes.byref(flags)) == _lib.GEMMS_ERR_TIMEOUT
    assert flags.value & _lib.FLAG_MMA_WAIT, hex(flags.value)
    assert L.gemms_moe_check_noalloc(stream, ctypes.byref(flags)) == 0 and flags.value == 0  # cleared

    assert noalloc(ctypes.byref(b), stream) == 0
    assert L.gemms_moe_check_noalloc(stream, ctypes.byref(flags)) == 0 and flags.value == 0
    assert torch.equal(idx, ref_idx)
    m = R.compare(out.cpu(), ref.cpu())
    assert m["max_rel"] <= MAX_REL and m["mae_rms"] <= MAE_RMS, m


def test_noalloc_rejects_batches_beyond_its_scratch():
    sh = W.CONFIGS["c2"].replace(T=128, shared=True)  # needs ~16.2 MiB of scratch
    d = W.make_inputs(sh, seed=3, device="cuda", experts=1)
    # Only one expert's weights exist: the call must refuse before it launches
    # anything that would read them.
    logits = torch.zeros((sh.T, sh.E), device="cuda")
    out = torch.zeros((sh.T, sh.H), dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros((sh.T, sh.top_k), dtype=torch.int32, device="cuda")
    L, fwd, noalloc = _entry_points()
    shape, a = _make_args(sh, d, logits, out, idx)
    assert L.gemms_moe_workspace_size(ctypes.byref(shape)) > (16 << 20)
    rc = noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == GEMMS_ERR_CAPACITY, _lib.strerror(rc)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0
