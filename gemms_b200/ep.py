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
3. count exchange (``all_gather`` of each rank's per-destination row counts,
   then one host read of the count matrix) and the dispatch
   ``all_to_all_single`` of packed rows -- the shared expert runs on the first
   half of the rank's own tokens meanwhile (all of them with the peer
   combine);
4. grouped GEMMs over the received rows, each row's result pre-reduced over its
   local experts in fp32;
5. the rows go back as fp16 with a per-row power-of-two scale (exact
   scaling, half the bytes of fp32), ``all_to_all_single`` while the shared
   expert runs on the second half of the tokens, and a deterministic
   gather-sum per token plus the shared expert, cast to bf16.  With the peer
   combine (``combine="peer"``) the packed rows instead stay in a symmetric
   buffer on the rank that computed them and, after one barrier, the gather
   reads them from there over NVLink.

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

    def dispatch(self, idx, w, x, world: int, E_local: int):
        T, H = x.shape
        k = idx.shape[1]
        dev = x.device
        rb = row_bytes(H, k)
        send_counts = torch.empty((2, world), dtype=torch.int32, device=dev)  # rows, pairs per destination
        send_row_of = torch.empty((T, world), dtype=torch.int32, device=dev)
        send_buf = torch.empty((max(T * min(world, k), 1), rb), dtype=torch.uint8, device=dev)
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

    # ---- peer-memory combine (GEMMS_EP_COMBINE=peer) --------------------
    def peer_buffers(self, group, cap_rows: int, H: int):
        """This rank's half of a double-buffered symmetric allocation for packed
        combine rows and every rank's address of it (peer pointers, mapped into
        this process).  Calls alternate between the two buffers: a rank writes
        buffer i % 2 only after the barrier of call i - 1, which every rank
        passes only once it has finished reading buffer (i - 2) % 2.  Grows
        (collectively: ``cap_rows`` is the same on every rank) when needed."""
        import torch.distributed._symmetric_memory as symm_mem
        g = group if group is not None else dist.group.WORLD
        rbb = back_row_bytes(H)
        need = max(cap_rows, 1) * rbb
        st = self._symm.get(g.group_name)
        if st is None or st["bytes"] < need:
            if st is not None:  # peers may still read the old buffers: barrier, then drain before freeing
                self.peer_publish(g, None, None)
                torch.cuda.current_stream().synchronize()
            nbytes = -(-need * 5 // 4 // (1 << 20)) * (1 << 20)  # 25% headroom, whole MiB
            dev = torch.device("cuda", torch.cuda.current_device())
            bufs, ptrs, hdls = [], [], []
            for _ in range(2):
                b = symm_mem.empty(nbytes, dtype=torch.uint8, device=dev)
                h = symm_mem.rendezvous(b, g)
                bufs.append(b)
                hdls.append(h)
                ptrs.append([int(p) for p in h.buffer_ptrs])
            st = {"bytes": nbytes, "bufs": bufs, "ptrs": ptrs, "hdls": hdls, "parity": 0}
            self._symm[g.group_name] = st
        i = st["parity"]
        st["parity"] ^= 1
        return st["bufs"][i], st["ptrs"][i]

    def peer_publish(self, group, local, peers):
        """Barrier: every rank's writes of its buffer are complete (a one-element
        NCCL all-reduce, ordered after them on each rank's stream)."""
        tok = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", torch.cuda.current_device()))
        dist.all_reduce(tok, group=group)
        return peers

    def combine_rows(self, acc, peers, row_add, send_row_of, world: int):
        """out bf16 [T, H] = acc + the packed rows read in place from each
        destination's buffer (``gemms_ep_combine_rows``)."""
        T, H = acc.shape
        out = torch.empty((T, H), dtype=torch.bfloat16, device=acc.device)
        bases = (ctypes.c_void_p * world)(*peers)
        adds = (ctypes.c_int32 * world)(*row_add)
        _lib.check(self.L.gemms_ep_combine_rows(acc.data_ptr(), bases, adds, send_row_of.data_ptr(), T, H, world,
                                                out.data_ptr(), self._stream()), "gemms_ep_combine_rows")
        return out

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
           inter_planes=2, logits=None, group=None, kernels=None, timeline=None, combine=None):
    """Expert-parallel layer forward on this rank's tokens ``x`` [T_r, H].

    ``w13``/``w2`` (and scales) hold this rank's ``E/W`` experts; the rank's
    first global expert is ``rank * E/W``.  ``timeline`` (a list) receives
    ``(phase, torch.cuda.Event)`` pairs recorded on the current stream at the
    phase boundaries, for per-phase device timing, and the counts
    ``("recv_rows", R)``, ``("pair_rows", P)`` (grouped-GEMM rows: received
    rows times the local experts each names) and ``("experts_hit", n)``.

    ``combine`` (default: ``GEMMS_EP_COMBINE``, else ``"nccl"``) picks how the
    result rows come back: ``"nccl"`` sends them with ``all_to_all_single``;
    ``"peer"`` leaves them in a symmetric (NVLink-mapped) buffer on the rank
    that computed them and the combine kernel of the token's own rank reads
    them from there, after one barrier.
    """
    def mark(name):
        if timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            timeline.append((name, ev))

    mark("start")
    combine = combine or os.environ.get("GEMMS_EP_COMBINE", "nccl")
    if combine not in ("nccl", "peer"):
        raise ValueError(f"combine must be 'nccl' or 'peer', not {combine!r}")
    K = kernels if kernels is not None else _cuda_kernels()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    E = router_w.shape[0]
    E_local = w13.shape[0]
    if E_local * world != E:
        raise ValueError(f"each rank must hold E/world experts: E={E}, world={world}, local={E_local}")
    T, H = x.shape
    I = w13.shape[1] // 2
    if logits is None:
        logits = K.router_logits(x, router_w)
    idx, wts = K.route(logits, router_bias, n_group, topk_group, top_k, routed_scaling_factor)
    mark("router")
    send_counts, send_row_of, send_buf, xq, xq_scale = K.dispatch(idx, wts, x, world, E_local)
    mark("pack")

    # count matrices on every rank: m[src][dst] rows and mp[src][dst] routed
    # pairs -- this rank's send and receive counts, the size of its grouped
    # rows, and (peer combine) where its rows sit in each destination's order
    gathered = [torch.empty_like(send_counts) for _ in range(world)]
    dist.all_gather(gathered, send_counts, group=group)
    both = torch.stack(gathered).cpu().tolist()  # the one host synchronisation of the layer
    m = [b[0] for b in both]
    sc = [int(v) for v in m[rank]]
    rc = [int(m[src][rank]) for src in range(world)]
    S, R = sum(sc), sum(rc)
    P = sum(int(b[1][rank]) for b in both)
    mark("count_exchange")
    if timeline is not None:
        timeline.append(("recv_rows", R))
    rb = send_buf.shape[1]
    recv_buf = torch.empty((R, rb), dtype=torch.uint8, device=send_buf.device)
    work = dist.all_to_all_single(recv_buf, send_buf[:S].contiguous(), rc, sc, group=group, async_op=True)

    acc = torch.zeros((T, H), dtype=torch.float32, device=x.device)
    # With the all-to-all combine the shared expert is split so that its second
    # half hides that collective; the peer combine has no collective to hide.
    T1 = T // 2 if combine == "nccl" else T
    shared = (shared_w13, shared_w13_scale, shared_w2, shared_w2_scale)
    if shared_w13 is not None:  # first half of the tokens overlaps the dispatch all-to-all
        with K.comm_overlap():
            K.shared_ffn(xq[:T1], xq_scale[:, :T1], *shared, inter_planes, acc, 0)
    mark("shared_ffn")
    work.wait()
    mark("dispatch_wait")
    stats = None
    if timeline is not None and R > 0:
        # grouped-GEMM rows (one per received row and local expert it names)
        # and local experts hit, for a roofline byte count; counted on the
        # device now, read on the host after the last mark
        off = H + 4 * (H // BLOCK)
        ids = recv_buf[:R, off:off + 4 * top_k].contiguous().view(torch.int32)
        le = ids.to(torch.int64) - rank * E_local
        valid = (ids >= 0) & (le >= 0) & (le < E_local)
        slot = torch.where(valid, le, torch.full_like(le, E_local)).flatten()  # no host sync (unlike masks)
        per_expert = torch.zeros(E_local + 1, dtype=torch.int64, device=ids.device)
        per_expert.scatter_add_(0, slot, torch.ones_like(slot))
        stats = (valid.sum(), per_expert[:E_local])

    out_rows = K.expert_ffn(recv_buf, R, P, H, I, top_k, E_local, rank * E_local, inter_planes,
                            w13, w13_scale, w2, w2_scale)
    mark("expert_ffn")
    if combine == "peer":
        send_off = [sum(sc[:d]) for d in range(world)]
        row_add = [sum(int(m[src][d]) for src in range(rank)) - send_off[d] for d in range(world)]
        cap = max(sum(int(m[src][d]) for src in range(world)) for d in range(world))
        local, peers = K.peer_buffers(group, cap, H)
        K.pack_back(out_rows, out=local)
        mark("pack_back")
        peers = K.peer_publish(group, local, peers)
        mark("publish")
        out = K.combine_rows(acc, peers, row_add, send_row_of, world)
        mark("gather")
        _timeline_stats(timeline, stats)
        return out
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


def _timeline_stats(timeline, stats):
    if timeline is None:
        return
    pairs, per_expert = (0, None) if stats is None else (int(stats[0]), stats[1])
    timeline.append(("pair_rows", pairs))
    timeline.append(("experts_hit", 0 if per_expert is None else int((per_expert > 0).sum())))
