"""Host-to-host serving loop for the MoE layer with copies overlapped.

A caller that holds its activations in host memory (a serving process, a
pipeline stage fed over the network) pays two PCIe copies per batch: x in and
y out (58.7 MB each at T=4096, H=7168 bf16).  :class:`MoePipeline` overlaps
them with the layer itself: while batch i computes on the compute stream,
batch i+1 is copied in on a copy-in stream and batch i-1 is copied out on a
copy-out stream, with two device slots per direction.  Every batch still makes
the full round trip host -> device -> host; only the waiting is hidden.
"""
from __future__ import annotations

import torch

from . import ops

_SHARED = ("shared_w13", "shared_w13_scale", "shared_w2", "shared_w2_scale")


class MoePipeline:
    """Runs ``ops.moe`` (or, with ``ep_group``, the expert-parallel layer) on
    a sequence of pinned host batches, writing pinned host outputs.

    ``weights`` holds router_w, router_bias, w13, w13_scale, w2, w2_scale and
    optionally the shared expert's four tensors; ``moe_kwargs`` go to
    ``ops.moe`` unchanged (and win over the dict's shared-expert entries)."""

    def __init__(self, weights: dict, *, device=None, slots: int = 2, **moe_kwargs):
        self.w = weights
        self.kw = moe_kwargs
        self.dev = torch.device(device) if device is not None else weights["w13"].device
        self.slots = slots
        self.s_in = torch.cuda.Stream(self.dev)
        self.s_out = torch.cuda.Stream(self.dev)
        self.x_dev = [None] * slots
        self.ev_in = [torch.cuda.Event() for _ in range(slots)]
        self.ev_done = [torch.cuda.Event() for _ in range(slots)]
        self.ev_out = [torch.cuda.Event() for _ in range(slots)]
        self.used = [False] * slots

    def _layer(self, x):
        w = self.w
        kw = {k: w[k] for k in _SHARED if k in w}
        kw.update(self.kw)
        return ops.moe(x, w["router_w"], w["router_bias"], w["w13"], w["w13_scale"], w["w2"], w["w2_scale"], **kw)

    @torch.no_grad()
    def run(self, host_x: list[torch.Tensor], host_y: list[torch.Tensor]) -> None:
        """host_x[i] (pinned bf16 [T, H]) -> host_y[i] (pinned bf16 [T, H]) for every i.

        Returns when every output has been written.
        """
        if len(host_x) != len(host_y):
            raise ValueError("host_x and host_y must have the same length")
        with torch.cuda.device(self.dev):
            self._run(host_x, host_y)

    def _run(self, host_x, host_y):
        compute = torch.cuda.current_stream(self.dev)
        for i, (xh, yh) in enumerate(zip(host_x, host_y)):
            k = i % self.slots
            # copy in: the slot's previous output copy must be done before its
            # input buffer is reused
            with torch.cuda.stream(self.s_in):
                if self.used[k]:
                    self.s_in.wait_event(self.ev_done[k])
                if self.x_dev[k] is None or self.x_dev[k].shape != xh.shape:
                    self.x_dev[k] = torch.empty(xh.shape, dtype=xh.dtype, device=self.dev)
                self.x_dev[k].copy_(xh, non_blocking=True)
                self.ev_in[k].record(self.s_in)
            compute.wait_event(self.ev_in[k])
            y = self._layer(self.x_dev[k])
            self.ev_done[k].record(compute)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(self.ev_done[k])
                yh.copy_(y, non_blocking=True)
                y.record_stream(self.s_out)
                self.ev_out[k].record(self.s_out)
            self.used[k] = True
        self.s_out.synchronize()


class MoeGraph:
    """One ``ops.moe`` call for a fixed token count captured in a CUDA graph.

    Decode batches (a few tokens) spend most of the layer's time launching its
    ~10 kernels; a graph replays them with one launch.  The layer has no host
    synchronisation and keeps its workspace per stream, so it captures as is.
    ``__call__(x)`` copies x into the graph's static input, replays, and
    returns the graph's static output (overwritten by the next replay: copy it
    if it must outlive that).  Weights (``weights`` dict as for
    :class:`MoePipeline`) must stay at the same addresses while the graph is
    used."""

    def __init__(self, weights: dict, T: int, *, device=None, **moe_kwargs):
        self.w = weights
        self.kw = moe_kwargs
        self.dev = torch.device(device) if device is not None else weights["w13"].device
        H = weights["w13"].shape[2]
        self.x = torch.zeros((T, H), dtype=torch.bfloat16, device=self.dev)
        with torch.cuda.device(self.dev):
            # one eager call first: library load, shared-memory opt-in and
            # other one-time set-up must not happen inside the capture
            self._layer()
            torch.cuda.synchronize(self.dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.y = self._layer()

    def _layer(self):
        w = self.w
        kw = {k: w[k] for k in _SHARED if k in w}
        kw.update(self.kw)
        return ops.moe(self.x, w["router_w"], w["router_bias"], w["w13"], w["w13_scale"], w["w2"], w["w2_scale"],
                       **kw)

    @torch.no_grad()
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape != self.x.shape:
            raise ValueError(f"MoeGraph was captured for x of shape {tuple(self.x.shape)}, got {tuple(x.shape)}")
        self.x.copy_(x)
        self.graph.replay()
        return self.y
