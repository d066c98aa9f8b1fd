"""CPU, world_size 2 (gloo): expert-parallel host logic of gemms_b200.ep.

The device side is replaced by CPU stand-ins (tests/ep_fakes.py) that follow
the C ABI's contracts with the oracle's arithmetic; the exchange itself (count
all-to-all, split sizes, dispatch and combine all-to-alls, or the
device-driven exchange's regions, barriers and plan; the combine mapping) is
the product code.  The 2-rank result must equal the single-process oracle over
all tokens.  A second test makes one rank leave before the first collective:
the remaining rank must raise within its process-group timeout, not hang.
"""
import math
import os
import socket
import tempfile
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gemms_b200 import ep as EP
from gemms_b200 import workloads as W
from oracle import reference_moe as R

SHAPE = W.CONFIGS["c0"].replace(T=48, shared=True)  # E=32, 4 groups / top-2 groups / top-4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs():
    return W.make_inputs(SHAPE, seed=4)


def _ep_worker(rank, world, port, outdir, exchange="nccl"):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from tests.ep_fakes import CpuEpKernels

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    d = _inputs()
    T = SHAPE.T // world
    El = SHAPE.E // world
    sl = slice(rank * T, (rank + 1) * T)
    el = slice(rank * El, (rank + 1) * El)
    K = CpuEpKernels(SHAPE.n_group, SHAPE.topk_group, SHAPE.top_k)
    out = EP.moe_ep(d["x"][sl], d["router_w"], d["router_bias"], d["w13"][el], d["w13_scale"][el], d["w2"][el],
                    d["w2_scale"][el], shared_w13=d["shared_w13"], shared_w13_scale=d["shared_w13_scale"],
                    shared_w2=d["shared_w2"], shared_w2_scale=d["shared_w2_scale"], n_group=SHAPE.n_group,
                    topk_group=SHAPE.topk_group, top_k=SHAPE.top_k, routed_scaling_factor=SHAPE.rsf,
                    group=dist.group.WORLD, kernels=K, exchange=exchange)
    torch.save(out, os.path.join(outdir, f"out{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("exchange,world", [("nccl", 2), ("peer", 2), ("nccl", 4), ("peer", 4)])
def test_ep_ranks_match_single_process_oracle(exchange, world):
    """Both exchange modes: the all-to-alls with host split sizes, and the
    device-driven exchange (rows pulled from the senders' regions, result
    rows read from the computing rank's region, offsets planned from the
    counts in the region headers)."""
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_ep_worker, args=(world, _free_port(), tmp, exchange), nprocs=world, join=True)
        got = torch.cat([torch.load(os.path.join(tmp, f"out{r}.pt")) for r in range(world)])
    d = _inputs()
    ref = R.moe_layer(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                      d["shared_w13"], d["shared_w13_scale"], d["shared_w2"], d["shared_w2_scale"],
                      n_group=SHAPE.n_group, topk_group=SHAPE.topk_group, top_k=SHAPE.top_k, rsf=SHAPE.rsf)
    m = R.compare(got, ref)
    # Same fp32 arithmetic except the combine rows, which travel as fp16 with
    # an exact power-of-two scale (2^-11 relative): that flips a few bf16
    # output roundings (~1e-4 of RMS here).  A misrouted row would cost
    # errors of the order of the output itself.
    assert m["mae_rms"] < 3e-4 and m["max_rel"] < 1e-2, m


def _ragged_worker(rank, world, port, outdir):
    """Ranks hold different token counts (ragged split of the 48 tokens) and
    pass the same max_tokens_per_rank, as the device-driven exchange requires."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from tests.ep_fakes import CpuEpKernels

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    d = _inputs()
    bounds = [0, 7, 30, 41, SHAPE.T] if world == 4 else [0, 31, SHAPE.T]
    sl = slice(bounds[rank], bounds[rank + 1])
    El = SHAPE.E // world
    el = slice(rank * El, (rank + 1) * El)
    K = CpuEpKernels(SHAPE.n_group, SHAPE.topk_group, SHAPE.top_k)
    kw = dict(shared_w13=d["shared_w13"], shared_w13_scale=d["shared_w13_scale"], shared_w2=d["shared_w2"],
              shared_w2_scale=d["shared_w2_scale"], n_group=SHAPE.n_group, topk_group=SHAPE.topk_group,
              top_k=SHAPE.top_k, routed_scaling_factor=SHAPE.rsf, group=dist.group.WORLD, kernels=K,
              exchange="peer")
    wts = (d["w13"][el], d["w13_scale"][el], d["w2"][el], d["w2_scale"][el])
    out = EP.moe_ep(d["x"][sl], d["router_w"], d["router_bias"], *wts, max_tokens_per_rank=SHAPE.T, **kw)
    torch.save(out, os.path.join(outdir, f"out{rank}.pt"))
    # more tokens than the stated capacity: refused on the host before any collective
    err = ""
    try:
        EP.moe_ep(d["x"][sl], d["router_w"], d["router_bias"], *wts, max_tokens_per_rank=0, **kw)
    except ValueError as e:
        err = str(e)
    with open(os.path.join(outdir, f"err{rank}.txt"), "w") as f:
        f.write(err)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_exchange_ragged_ranks_with_capacity(world):
    """Ragged token counts per rank under one max_tokens_per_rank: the plan
    (receive order, offsets in the senders' regions, combine offsets) still
    matches the single-process oracle; a rank past the capacity raises."""
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_ragged_worker, args=(world, _free_port(), tmp), nprocs=world, join=True)
        got = torch.cat([torch.load(os.path.join(tmp, f"out{r}.pt")) for r in range(world)])
        errs = [open(os.path.join(tmp, f"err{r}.txt")).read() for r in range(world)]
    d = _inputs()
    ref = R.moe_layer(d["x"], d["router_w"], d["router_bias"], d["w13"], d["w13_scale"], d["w2"], d["w2_scale"],
                      d["shared_w13"], d["shared_w13_scale"], d["shared_w2"], d["shared_w2_scale"],
                      n_group=SHAPE.n_group, topk_group=SHAPE.topk_group, top_k=SHAPE.top_k, rsf=SHAPE.rsf)
    m = R.compare(got, ref)
    assert m["mae_rms"] < 3e-4 and m["max_rel"] < 1e-2, m
    assert all("max_tokens_per_rank" in e for e in errs), errs


def test_pack_back_round_trip():
    """Packed combine rows: exact power-of-two scale, fp16 rounding only, edge rows."""
    from tests.ep_fakes import CpuEpKernels
    g = torch.Generator().manual_seed(0)
    rows = torch.randn(6, 256, generator=g) * torch.tensor([1e-30, 1e-3, 1.0, 3e4, 1e8, 0.0]).unsqueeze(1)
    K = CpuEpKernels(1, 1, 1)
    packed = K.pack_back(rows)
    assert packed.shape == (6, 2 * 256 + 16)
    for r in range(6):
        back = K.unpack_back(packed[r], 256)
        amax = float(rows[r].abs().max())
        scale = float(packed[r, 512:516].view(torch.float32)[0])
        if amax == 0:
            assert scale == 1.0 and torch.equal(back, rows[r])
            continue
        assert 2 ** 14 <= amax / scale < 2 ** 15          # power of two chosen from the row max
        assert scale == 2.0 ** round(math.log2(scale))
        err = (back - rows[r]).abs().max() / amax
        assert err <= 2 ** -11, (r, err)


def _leaver_worker(rank, world, port, outdir, exchange="nccl", leave="before_layer"):
    import sys
    import time
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from tests.ep_fakes import CpuEpKernels

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1 and leave == "before_layer":
        return  # leaves between steps: never joins the layer's collectives
    d = _inputs()
    T, El = SHAPE.T // world, SHAPE.E // world

    class Leaving(CpuEpKernels):
        def pack_back(self, rows, out=None):
            # rank 1 leaves after the dispatch, before its rows go back
            if rank == 1:
                os._exit(0)
            return super().pack_back(rows, out)

        def pack_back_dev(self, rows, info, reg):
            if rank == 1:
                os._exit(0)
            return super().pack_back_dev(rows, info, reg)

    K = (Leaving if leave == "before_combine" else CpuEpKernels)(SHAPE.n_group, SHAPE.topk_group, SHAPE.top_k)
    sl, el = slice(rank * T, (rank + 1) * T), slice(rank * El, (rank + 1) * El)
    t0 = time.time()
    status = "no-error"
    try:
        EP.moe_ep(d["x"][sl], d["router_w"], d["router_bias"], d["w13"][el], d["w13_scale"][el], d["w2"][el],
                  d["w2_scale"][el], n_group=SHAPE.n_group, topk_group=SHAPE.topk_group, top_k=SHAPE.top_k,
                  routed_scaling_factor=SHAPE.rsf, group=dist.group.WORLD, kernels=K, exchange=exchange)
    except RuntimeError as e:  # gloo: timeout or connection closed by the departed peer
        status = f"error after {time.time() - t0:.1f}s: {type(e).__name__}"
    if rank == 0:
        with open(os.path.join(outdir, "status.txt"), "w") as f:
            f.write(status)


@pytest.mark.parametrize("exchange,leave", [("nccl", "before_layer"), ("nccl", "before_combine"),
                                            ("peer", "before_layer"), ("peer", "before_combine")])
def test_ep_rank_that_leaves_is_detected(exchange, leave):
    """A rank that is gone (before the layer, or after the dispatch and before
    its rows go back) makes the other rank's next collective (the count
    exchange, the combine all-to-all, or the peer mode's barriers) fail within
    the process group's timeout instead of waiting for ever."""
    world = 2
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_leaver_worker, args=(world, _free_port(), tmp, exchange, leave), nprocs=world, join=True)
        status = open(os.path.join(tmp, "status.txt")).read()
    assert status.startswith("error after"), status
    secs = float(status.split()[2].rstrip("s:"))
    assert secs < 30, status
