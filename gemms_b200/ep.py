"""Expert-parallel MoE layer over torch.distributed (NCCL on B200).

The reference has no distributed code; its only hook is ``local_expert_offset``
(``flashinfer_baseline.py:132-138``): one call computes the experts
``[offset, offset + E_local)``.  Here rank ``r`` of ``W`` owns experts
``[r*E/W, (r+1)*E/W)`` and ``T_r`` tokens; router weights, bias and the shared
expert are replicated.  One layer forward on every rank:

1. router GEMM + CUDA router over the rank's own tokens;
2. dispatch plan: each token goes once to every rank holding any of its top-k
   experts (group-limited routing bounds this at ``topk_group`` ranks when
   groups align with ranks, e.g. EP8 of DeepSeek-V3), rows grouped by
   destination in token order, quantised per 1x128 and packed with the ids and
   weights of the experts on the destination;
3. the exchange of the packed rows, in one of two modes:

   * ``"nccl"``: an ``all_gather`` of each rank's per-destination counts, one
     host read of the count matrix (split sizes), and ``all_to_all_single``
     of the rows; the shared expert runs on the first half of the rank's own
     tokens meanwhile;
   * ``"peer"`` (device-driven, no host synchronisation): each rank writes its
     counts and rows into its own exchange region, a symmetric allocation that
     every rank can address over NVLink; after one barrier each rank's pull
     kernel reads all ranks' counts and copies the rows sent to it straight
     from the senders' regions.  Buffers are sized by capacities
     (``max_tokens_per_rank``), so nothing about the counts is needed on the
     host and the whole layer can be captured in a CUDA graph;

4. grouped GEMMs over the received rows, each row's result pre-reduced over its
   local experts in fp32;
5. the rows go back as fp16 with a per-row power-of-two scale (exact
   scaling, half the bytes of fp32): ``"nccl"`` sends them with
   ``all_to_all_single`` while the shared expert runs on the second half of
   the tokens; ``"peer"`` leaves them in the exchange region of the rank that
   computed them and, after a second barrier, the token's own rank reads them
   from there.  A deterministic gather-sum per token plus the shared expert,
   cast to bf16, ends the layer.

Every rank issues the same collectives in the same order.  The device work
goes through a ``kernels`` object: :class:`CudaEpKernels` (the C ABI) by
default; tests pass CPU stand-ins to exercise the exchange logic on gloo ranks.
"""
from __future__ import annotations

import contextlib
import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib

BLOCK = 128


def row_bytes(H: int, top_k: int) -> int:
    """Bytes of one packed dispatch row (``gemms_ep_row_bytes``)."""
    raw = H + 4 * (H // BLOCK) + 8 * top_k
    return (raw + 15) // 16 * 16


def back_row_bytes(H: int) -> int:
    """Bytes of one packed combine row (``gemms_ep_back_row_bytes``): fp16 [H] + fp32 2^e."""
    return (2 * H + 4 + 15) // 16 * 16


class _Region:
    """A rank's exchange region and the local buffers that go with it: ``hdr``
    (int32 [2, world] counts), ``send`` (packed send rows), ``back`` (packed
    combine rows), ``bases`` / ``back_bases`` (every rank's address of its
    region / of its combine rows), ``recv`` and ``info`` (this rank's received
    rows and exchange plan), ``send_cap`` / ``recv_cap`` (rows)."""


class CudaEpKernels:
    """Device side of expert parallelism through ``include/gemms_moe.h``."""

    def __init__(self):
        self.L = _lib.load()
        self._ws = {}
        self._symm = {}

    @staticmethod
    def _stream() -> int:
        return torch.cuda.current_stream().cuda_stream

    def _workspace(self, dev, nbytes: int, tag: str) -> torch.Tensor:
        key = (dev.index, torch.cuda.current_stream(dev).cuda_stream, tag)  # per stream: no sharing across streams
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes + 256:
            ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            self._ws[key] = ws
        off = (-ws.data_ptr()) % 256
        return ws[off:off + nbytes]

    @contextlib.contextmanager
    def comm_overlap(self):
        """While active, the persistent grouped GEMMs leave ``GEMMS_EP_COMM_SMS``
        (default 32) SMs free for the all-to-all running on NCCL's stream; a
        GEMM given every SM would hold them until it finishes and the
        collective would wait for it."""
        reserve = int(os.environ.get("GEMMS_EP_COMM_SMS", "32"))
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        prev = self.L.gemms_set_gemm_ctas(max(1, sms - reserve) if reserve > 0 else 0)
        try:
            yield
        finally:
            self.L.gemms_set_gemm_ctas(max(prev, 0))

    def router_logits(self, x, router_w):
        from .ops import router_logits
        return router_logits(x, router_w)

    def route(self, logits, bias, n_group, topk_group, top_k, rsf):
        from .ops import route
        idx, w, _ = route(logits, bias, n_group=n_group, topk_group=topk_group, top_k=top_k,
                          routed_scaling_factor=rsf, counts=False)
        return idx, w

    def dispatch(self, idx, w, x, world: int, E_local: int, region=None):
        """Packed send rows and counts; into ``region``'s header and send rows
        (device-driven exchange) when given."""
        T, H = x.shape
        k = idx.shape[1]
        dev = x.device
        rb = row_bytes(H, k)
        if region is not None:
            send_counts, send_buf = region.hdr, region.send
        else:
            send_counts = torch.empty((2, world), dtype=torch.int32, device=dev)  # rows, pairs per destination
            send_buf = torch.empty((max(T * min(world, k), 1), rb), dtype=torch.uint8, device=dev)
        send_row_of = torch.empty((T, world), dtype=torch.int32, device=dev)
        xq = torch.empty((T, H), dtype=torch.float8_e4m3fn, device=dev)
        xq_scale = torch.empty((H // BLOCK, T), dtype=torch.float32, device=dev)
        _lib.check(self.L.gemms_ep_dispatch(idx.data_ptr(), w.data_ptr(), x.data_ptr(), T, H, k, world, E_local,
                                            send_counts.data_ptr(), send_row_of.data_ptr(), send_buf.data_ptr(),
                                            xq.data_ptr(), xq_scale.data_ptr(), self._stream()),
                   "gemms_ep_dispatch")
        return send_counts, send_row_of, send_buf, xq, xq_scale

    def expert_ffn(self, recv_buf, R: int, P: int, H: int, I: int, top_k: int, E_local: int, offset: int,
                   planes: int, w13, w13_scale, w2, w2_scale):
        """Received rows -> fp32 [R, H]; P = (row, local expert) pairs they name."""
        dev = w13.device
        out = torch.empty((max(R, 1), H), dtype=torch.float32, device=dev)
        nbytes = self.L.gemms_ep_ffn_workspace_size(R, P, H, I, E_local, top_k, planes)
        if nbytes == 0:
            raise ValueError("unsupported expert-parallel FFN geometry")
        ws = self._workspace(dev, nbytes, "ep_ffn")
        _lib.check(self.L.gemms_ep_expert_ffn(recv_buf.data_ptr(), R, P, H, I, top_k, E_local, offset, planes,
                                              w13.data_ptr(), w13_scale.data_ptr(), w2.data_ptr(),
                                              w2_scale.data_ptr(), out.data_ptr(), ws.data_ptr(), nbytes,
                                              self._stream()), "gemms_ep_expert_ffn")
        return out[:R]

    def shared_ffn(self, xq, xq_scale, sw13, sw13_scale, sw2, sw2_scale, planes: int, acc, t0: int = 0):
        """acc[t0 : t0 + n] (fp32) += shared expert of the n token-major quantised
        rows ``xq`` [n, H] with scales ``xq_scale`` [H/128, n]."""
        T, H = xq.shape
        I = sw2.shape[1]
        dev = xq.device
        if T == 0:
            return
        xq_scale = xq_scale.contiguous()
        counts = torch.full((1,), T, dtype=torch.int32, device=dev)
        dest = torch.arange(t0, t0 + T, dtype=torch.int32, device=dev)
        wts = torch.ones((T,), dtype=torch.float32, device=dev)
        nbytes = self.L.gemms_expert_ffn_workspace_size(T, H, I, 1, planes)
        ws = self._workspace(dev, nbytes, "shared_ffn")
        _lib.check(self.L.gemms_expert_ffn(xq.data_ptr(), xq_scale.data_ptr(), T, counts.data_ptr(), dest.data_ptr(),
                                           wts.data_ptr(), H, I, 1, planes, sw13.data_ptr(), sw13_scale.data_ptr(),
                                           sw2.data_ptr(), sw2_scale.data_ptr(), acc.data_ptr(), ws.data_ptr(),
                                           nbytes, self._stream()), "gemms_expert_ffn(shared)")
        self._keep = getattr(self, "_keep", ())[-4:] + (counts, dest, wts, xq_scale)  # alive until consumed

    def pack_back(self, rows, out=None):
        """fp32 [R, H] -> packed combine rows uint8 [R, back_row_bytes(H)] (into
        the front of the flat uint8 buffer ``out`` when given)."""
        R, H = rows.shape
        if out is None:
            packed = torch.empty((max(R, 1), back_row_bytes(H)), dtype=torch.uint8, device=rows.device)
        else:
            if out.numel() < R * back_row_bytes(H):
                raise ValueError("pack_back: output buffer too small")
            packed = out[:max(R, 1) * back_row_bytes(H)].view(max(R, 1), back_row_bytes(H))
        _lib.check(self.L.gemms_ep_pack_back(rows.data_ptr(), R, H, packed.data_ptr(), self._stream()),
                   "gemms_ep_pack_back")
        return packed[:R]

    # ---- device-driven exchange (exchange="peer") ------------------------
    def exchange_region(self, group, send_cap: int, recv_cap: int, H: int, top_k: int):
        """This rank's exchange region (a symmetric allocation: the header of
        counts, ``send_cap`` packed send rows, ``recv_cap`` packed combine rows)
        with every rank's address of it, and the local receive buffers.

        Collective when it (re)allocates: every rank must pass the same
        capacities (they follow from ``max_tokens_per_rank``).  One region
        per group serves every call: a rank rewrites its send rows only after
        the combine barrier of the previous call, which no rank passes before
        it has pulled its rows, and its combine rows only after the dispatch
        barrier of this call, which no rank passes before it has finished the
        previous combine."""
        import torch.distributed._symmetric_memory as symm_mem
        g = group if group is not None else dist.group.WORLD
        world = dist.get_world_size(g)
        rb, rbb = row_bytes(H, top_k), back_row_bytes(H)
        send_bytes = self.L.gemms_ep_region_bytes(send_cap, H, top_k)
        if send_bytes == 0:
            raise ValueError("unsupported expert-parallel exchange geometry")
        back_off = -(-send_bytes // 256) * 256
        need = back_off + max(recv_cap, 1) * rbb
        key = (g.group_name, H, top_k)
        st = self._symm.get(key)
        if st is None or st.nbytes < need or st.send_cap < send_cap or st.recv_cap < recv_cap:
            if st is not None:  # peers may still read the old region: barrier, then drain before freeing
                self.peer_barrier(g, st)
                torch.cuda.current_stream().synchronize()
            nbytes = -(-need * 5 // 4 // (1 << 20)) * (1 << 20)  # 25% headroom, whole MiB
            dev = torch.device("cuda", torch.cuda.current_device())
            buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=dev)
            hdl = symm_mem.rendezvous(buf, g)
            st = _Region()
            st.buf, st.hdl, st.nbytes = buf, hdl, nbytes
            st.bases = [int(p) for p in hdl.buffer_ptrs]
            st.world, st.rb, st.rbb, st.back_off = world, rb, rbb, back_off
            st.send_cap = (back_off - 256) // rb          # >= send_cap
            st.recv_cap = (nbytes - back_off) // rbb      # >= recv_cap (the headroom lands here)
            st.hdr = buf[:8 * world].view(torch.int32).view(2, world)
            st.send = buf[256:256 + st.send_cap * rb].view(st.send_cap, rb)
            st.back = buf[back_off:back_off + st.recv_cap * rbb]
            st.back_bases = [b + back_off for b in st.bases]
            st.recv = torch.empty((max(st.recv_cap, 1), rb), dtype=torch.uint8, device=dev)
            st.info = torch.zeros(128, dtype=torch.int32, device=dev)
            st.tok = torch.zeros(1, dtype=torch.int32, device=dev)
            self._symm[key] = st
        return st

    def peer_barrier(self, group, region):
        """Every rank's writes before this point (on its current stream) are
        complete before any rank's work after it: a one-element NCCL
        all-reduce, ordered on each rank's stream after the writes."""
        dist.all_reduce(region.tok, group=group)

    def pull(self, region, rank: int, world: int, H: int, top_k: int):
        """Rows sent to this rank -> region.recv [recv_cap, row_bytes] and the
        exchange plan region.info (``gemms_ep_pull``)."""
        bases = (ctypes.c_void_p * world)(*region.bases)
        _lib.check(self.L.gemms_ep_pull(bases, rank, world, H, top_k, region.send_cap, region.recv_cap,
                                        region.recv.data_ptr(), region.info.data_ptr(), self._stream()),
                   "gemms_ep_pull")
        return region.recv, region.info

    def expert_ffn_dev(self, recv_buf, info, R_cap: int, P_cap: int, H: int, I: int, top_k: int, E_local: int,
                       offset: int, planes: int, w13, w13_scale, w2, w2_scale):
        """As expert_ffn over the first info[0] of R_cap received rows (count
        read on the device) -> fp32 [R_cap, H]."""
        dev = w13.device
        key = (dev.index, torch.cuda.current_stream(dev).cuda_stream, "ep_rows")
        out = self._ws.get(key)
        if out is None or out.shape[0] < max(R_cap, 1) or out.shape[1] != H:
            out = torch.empty((max(R_cap, 1), H), dtype=torch.float32, device=dev)
            self._ws[key] = out
        nbytes = self.L.gemms_ep_ffn_workspace_size(R_cap, P_cap, H, I, E_local, top_k, planes)
        if nbytes == 0:
            raise ValueError("unsupported expert-parallel FFN geometry")
        ws = self._workspace(dev, nbytes, "ep_ffn")
        _lib.check(self.L.gemms_ep_expert_ffn_dev(recv_buf.data_ptr(), R_cap, info.data_ptr(), P_cap, H, I, top_k,
                                                  E_local, offset, planes, w13.data_ptr(), w13_scale.data_ptr(),
                                                  w2.data_ptr(), w2_scale.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                                  nbytes, self._stream()), "gemms_ep_expert_ffn_dev")
        self._ffn_ws = ws
        return out[:max(R_cap, 1)]

    def pack_back_dev(self, rows, info, region):
        """The first info[0] result rows -> packed combine rows in region.back."""
        R_cap, H = rows.shape
        _lib.check(self.L.gemms_ep_pack_back_dev(rows.data_ptr(), min(R_cap, region.recv_cap), info.data_ptr(), H,
                                                 region.back.data_ptr(), self._stream()), "gemms_ep_pack_back_dev")

    def combine_peer(self, acc, region, info, send_row_of, world: int):
        """out bf16 [T, H] = acc + this rank's combine rows read in place from
        every destination's region (``gemms_ep_combine_peer``)."""
        T, H = acc.shape
        out = torch.empty((T, H), dtype=torch.bfloat16, device=acc.device)
        bases = (ctypes.c_void_p * world)(*region.back_bases)
        _lib.check(self.L.gemms_ep_combine_peer(acc.data_ptr(), bases, info.data_ptr(), send_row_of.data_ptr(), T, H,
                                                world, region.recv_cap, out.data_ptr(), self._stream()),
                   "gemms_ep_combine_peer")
        return out

    def side_stream(self):
        """A second stream of the current device (cached), for work that
        overlaps the exchange."""
        dev = torch.cuda.current_device()
        key = ("side", dev)
        st = self._ws.get(key)
        if st is None:
            st = torch.cuda.Stream(device=dev)
            self._ws[key] = st
        return st

    def gather_add_peer(self, acc, region, info, send_row_of, world: int):
        """acc fp32 [T, H] += this rank's combine rows read from every
        destination's region, with atomics (``gemms_ep_gather_add_peer``)."""
        T, H = acc.shape
        bases = (ctypes.c_void_p * world)(*region.back_bases)
        _lib.check(self.L.gemms_ep_gather_add_peer(acc.data_ptr(), bases, info.data_ptr(), send_row_of.data_ptr(), T,
                                                   H, world, region.recv_cap, self._stream()),
                   "gemms_ep_gather_add_peer")

    def to_bf16(self, acc):
        out = torch.empty(acc.shape, dtype=torch.bfloat16, device=acc.device)
        _lib.check(self.L.gemms_f32_to_bf16(acc.data_ptr(), out.data_ptr(), acc.numel(), self._stream()),
                   "gemms_f32_to_bf16")
        return out

    def exchange_flags(self, region) -> int:
        """info[2] of the last pull (reads the device: synchronises)."""
        return int(region.info[2].item())

    def combine(self, acc, back, send_row_of, world: int):
        T, H = acc.shape
        out = torch.empty((T, H), dtype=torch.bfloat16, device=acc.device)
        _lib.check(self.L.gemms_ep_combine(acc.data_ptr(), back.data_ptr() if back.numel() else None,
                                           send_row_of.data_ptr(), T, H, world, out.data_ptr(), self._stream()),
                   "gemms_ep_combine")
        return out


_default_kernels = None


def _cuda_kernels() -> CudaEpKernels:
    global _default_kernels
    if _default_kernels is None:
        _default_kernels = CudaEpKernels()
    return _default_kernels


@torch.no_grad()
def moe_ep(x, router_w, router_bias, w13, w13_scale, w2, w2_scale, *, shared_w13=None, shared_w13_scale=None,
           shared_w2=None, shared_w2_scale=None, n_group=8, topk_group=4, top_k=8, routed_scaling_factor=2.5,
           inter_planes=2, logits=None, group=None, kernels=None, timeline=None, exchange=None,
           max_tokens_per_rank=None):
    """Expert-parallel layer forward on this rank's tokens ``x`` [T_r, H].

    ``w13``/``w2`` (and scales) hold this rank's ``E/W`` experts; the rank's
    first global expert is ``rank * E/W``.  ``timeline`` (a list) receives
    ``(phase, torch.cuda.Event)`` pairs recorded on the current stream at the
    phase boundaries, for per-phase device timing, and the counts
    ``("recv_rows", R)``, ``("pair_rows", P)`` (grouped-GEMM rows: received
    rows times the local experts each names) and ``("experts_hit", n)``
    (read from the device after the last phase).

    ``exchange`` (default: ``GEMMS_EP_EXCHANGE``, else ``"nccl"``) picks how
    rows travel: ``"nccl"`` (count exchange read on the host, then
    ``all_to_all_single`` both ways) or ``"peer"`` (device-driven over
    symmetric memory, no host synchronisation; every rank must pass the same
    ``T_r``, or the same ``max_tokens_per_rank`` >= its ``T_r``, which sizes
    the exchange buffers).
    """
    def mark(name):
        if timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            timeline.append((name, ev))

    mark("start")
    exchange = exchange or os.environ.get("GEMMS_EP_EXCHANGE", "nccl")
    if exchange not in ("nccl", "peer"):
        raise ValueError(f"exchange must be 'nccl' or 'peer', not {exchange!r}")
    K = kernels if kernels is not None else _cuda_kernels()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    E = router_w.shape[0]
    E_local = w13.shape[0]
    if E_local * world != E:
        raise ValueError(f"each rank must hold E/world experts: E={E}, world={world}, local={E_local}")
    T, H = x.shape
    I = w13.shape[1] // 2
    T_cap = T if max_tokens_per_rank is None else int(max_tokens_per_rank)
    if T > T_cap:
        raise ValueError(f"{T} tokens on this rank exceed max_tokens_per_rank={T_cap}")
    if logits is None:
        logits = K.router_logits(x, router_w)
    idx, wts = K.route(logits, router_bias, n_group, topk_group, top_k, routed_scaling_factor)
    mark("router")
    shared = (shared_w13, shared_w13_scale, shared_w2, shared_w2_scale)
    if exchange == "peer":
        return _moe_ep_peer(K, x, idx, wts, w13, w13_scale, w2, w2_scale, shared, group, world, rank, E_local, T_cap,
                            H, I, top_k, inter_planes, mark, timeline)

    send_counts, send_row_of, send_buf, xq, xq_scale = K.dispatch(idx, wts, x, world, E_local)
    mark("pack")
    # count matrices on every rank: m[src][dst] rows and mp[src][dst] routed
    # pairs -- this rank's send and receive counts and the size of its grouped rows
    gathered = [torch.empty_like(send_counts) for _ in range(world)]
    dist.all_gather(gathered, send_counts, group=group)
    both = torch.stack(gathered).cpu().tolist()  # the one host synchronisation of this mode
    m = [b[0] for b in both]
    sc = [int(v) for v in m[rank]]
    rc = [int(m[src][rank]) for src in range(world)]
    S, R = sum(sc), sum(rc)
    P = sum(int(b[1][rank]) for b in both)
    mark("count_exchange")
    rb = send_buf.shape[1]
    recv_buf = torch.empty((R, rb), dtype=torch.uint8, device=send_buf.device)
    work = dist.all_to_all_single(recv_buf, send_buf[:S].contiguous(), rc, sc, group=group, async_op=True)

    acc = torch.zeros((T, H), dtype=torch.float32, device=x.device)
    # the shared expert is split so that its halves hide the two all-to-alls
    T1 = T // 2
    if shared_w13 is not None:  # first half of the tokens overlaps the dispatch all-to-all
        with K.comm_overlap():
            K.shared_ffn(xq[:T1], xq_scale[:, :T1], *shared, inter_planes, acc, 0)
    mark("shared_ffn")
    work.wait()
    mark("dispatch_wait")
    stats = _recv_stats(recv_buf, R, H, top_k, rank, E_local) if timeline is not None else None
    out_rows = K.expert_ffn(recv_buf, R, P, H, I, top_k, E_local, rank * E_local, inter_planes,
                            w13, w13_scale, w2, w2_scale)
    mark("expert_ffn")
    packed = K.pack_back(out_rows)
    mark("pack_back")
    back = torch.empty((S, packed.shape[1]), dtype=torch.uint8, device=x.device)
    work = dist.all_to_all_single(back, packed.contiguous(), sc, rc, group=group, async_op=True)
    if shared_w13 is not None:  # second half of the tokens overlaps the combine all-to-all
        with K.comm_overlap():
            K.shared_ffn(xq[T1:], xq_scale[:, T1:], *shared, inter_planes, acc, T1)
    mark("shared_ffn_2")
    work.wait()
    mark("combine_a2a")
    out = K.combine(acc, back, send_row_of, world)
    mark("gather")
    _timeline_stats(timeline, stats)
    return out


def _moe_ep_peer(K, x, idx, wts, w13, w13_scale, w2, w2_scale, shared, group, world, rank, E_local, T_cap, H, I,
                 top_k, inter_planes, mark, timeline):
    """exchange="peer": the layer after routing with the device-driven
    exchange.  Two barriers per call (after the dispatch, after the result
    rows are packed) and no host read of any count: buffers are sized by
    capacities (received rows <= world * T_cap, grouped pairs <= received
    rows * min(top_k, E_local)); counts beyond them raise the plan's flag
    and nothing is copied (``exchange_flags``)."""
    T = x.shape[0]
    send_cap = max(T_cap * min(world, top_k), 1)
    recv_cap = max(T_cap * world, 1)
    P_cap = recv_cap * min(top_k, E_local)
    reg = K.exchange_region(group, send_cap, recv_cap, H, top_k)
    send_counts, send_row_of, _, xq, xq_scale = K.dispatch(idx, wts, x, world, E_local, region=reg)
    acc = torch.zeros((T, H), dtype=torch.float32, device=x.device)
    mark("pack")
    # The shared expert needs only this rank's tokens: optionally it runs on a
    # side stream beside the barriers, the pull and the routed experts (its
    # GEMMs leave GEMMS_EP_COMM_SMS SMs to the pull and NCCL), and the combine
    # waits for it.
    combine_overlap = shared[0] is not None and _combine_overlap()
    side = K.side_stream() if shared[0] is not None and (_peer_overlap() or combine_overlap) else None
    if side is None:
        combine_overlap = False
    done_shared = None
    if side is not None and not combine_overlap:
        ready = torch.cuda.Event()
        ready.record()
        side.wait_event(ready)
        with torch.cuda.stream(side):
            for t in (xq, xq_scale, acc):
                t.record_stream(side)
            with K.comm_overlap():
                K.shared_ffn(xq, xq_scale, *shared, inter_planes, acc, 0)
            done_shared = torch.cuda.Event()
            done_shared.record()
    K.peer_barrier(group, reg)  # every rank's counts and send rows are written
    mark("publish_rows")
    recv_buf, info = K.pull(reg, rank, world, H, top_k)
    mark("pull")
    if shared[0] is not None and side is None:
        K.shared_ffn(xq, xq_scale, *shared, inter_planes, acc, 0)
        mark("shared_ffn")
    stats = _recv_stats(recv_buf, info, H, top_k, rank, E_local) if timeline is not None else None
    out_rows = K.expert_ffn_dev(recv_buf, info, reg.recv_cap, P_cap, H, I, top_k, E_local, rank * E_local,
                                inter_planes, w13, w13_scale, w2, w2_scale)
    mark("expert_ffn")
    K.pack_back_dev(out_rows, info, reg)
    mark("pack_back")
    K.peer_barrier(group, reg)  # every rank's combine rows are written
    mark("publish")
    if combine_overlap:
        # the NVLink-bound gather (side stream) beside the compute-bound shared
        # expert (this stream, GEMMs bounded to leave SMs to the gather); both
        # add into acc, then one cast
        main = torch.cuda.current_stream()
        ready = torch.cuda.Event()
        ready.record()
        with K.comm_overlap():
            K.shared_ffn(xq, xq_scale, *shared, inter_planes, acc, 0)
        side.wait_event(ready)
        with torch.cuda.stream(side):
            for t in (acc, send_row_of):
                t.record_stream(side)
            K.gather_add_peer(acc, reg, info, send_row_of, world)
            gathered = torch.cuda.Event()
            gathered.record()
        main.wait_event(gathered)
        mark("shared_and_gather")
        out = K.to_bf16(acc)
        mark("cast")
        _timeline_stats(timeline, stats)
        return out
    if done_shared is not None:
        torch.cuda.current_stream().wait_event(done_shared)
        mark("shared_wait")
    out = K.combine_peer(acc, reg, info, send_row_of, world)
    mark("gather")
    _timeline_stats(timeline, stats)
    return out


def _combine_overlap() -> bool:
    """GEMMS_EP_COMBINE_OVERLAP=1 (exchange="peer"): the shared expert runs
    after the second barrier beside the gather of the result rows.  Off by
    default: at N=2 (c3, one box) the two together took 1.64-1.71 ms against
    1.14 + 0.43 ms in sequence, plus a 0.12 ms cast, because the gather's
    NVLink reads and the shared GEMMs slow each other down."""
    return os.environ.get("GEMMS_EP_COMBINE_OVERLAP", "0") == "1"


def _peer_overlap() -> bool:
    """GEMMS_EP_PEER_OVERLAP=1 runs the shared expert on a side stream beside
    the exchange (exchange="peer").  Off by default: at N=2 (c3) the shared
    GEMMs only took SMs from the routed experts' GEMMs (14.45 vs 14.37 ms per
    step), since the exchange itself leaves little idle time to fill."""
    return os.environ.get("GEMMS_EP_PEER_OVERLAP", "0") == "1"


def _recv_stats(recv_buf, R, H, top_k, rank, E_local):
    """Received rows, grouped-GEMM rows (one per received row and local expert
    it names) and local experts hit, as device tensors (no synchronisation;
    read after the timed phases).  R is an int or the exchange plan (info[0])."""
    n = recv_buf.shape[0]
    if n == 0:
        return None
    off = H + 4 * (H // BLOCK)
    ids = recv_buf[:, off:off + 4 * top_k].contiguous().view(torch.int32)
    R_t = R[0] if torch.is_tensor(R) else torch.tensor(R, device=recv_buf.device)
    live = (torch.arange(n, device=recv_buf.device) < R_t).unsqueeze(1)
    le = ids.to(torch.int64) - rank * E_local
    valid = live & (ids >= 0) & (le >= 0) & (le < E_local)
    slot = torch.where(valid, le, torch.full_like(le, E_local)).flatten()
    per_expert = torch.zeros(E_local + 1, dtype=torch.int64, device=ids.device)
    per_expert.scatter_add_(0, slot, torch.ones_like(slot))
    return R_t, valid.sum(), per_expert[:E_local]


def _timeline_stats(timeline, stats):
    if timeline is None:
        return
    R, pairs, per_expert = (0, 0, None) if stats is None else (int(stats[0]), int(stats[1]), stats[2])
    timeline.append(("recv_rows", R))
    timeline.append(("pair_rows", pairs))
    timeline.append(("experts_hit", 0 if per_expert is None else int((per_expert > 0).sum())))
