"""CPU stand-ins for the device side of expert parallelism (test-only).

They follow the contracts of ``include/gemms_moe.h`` (packed row layout,
destination grouping in token order, fp32 pre-reduced rows, deterministic
combine) with the oracle's fp32 arithmetic, so that ``gemms_b200.ep.moe_ep``'s
host logic -- count exchange, split sizes, the two all-to-alls and the
combine mapping -- runs on gloo ranks without a GPU.
"""
from __future__ import annotations

import contextlib
import math

import torch

from gemms_b200 import ep as EP
from oracle import reference_moe as R

BLOCK = 128


class CpuEpKernels:
    def __init__(self, n_group, topk_group, top_k):
        self.ng, self.tg, self.k = n_group, topk_group, top_k

    def comm_overlap(self):
        return contextlib.nullcontext()

    def router_logits(self, x, router_w):
        return R.router_logits(x, router_w)

    def route(self, logits, bias, n_group, topk_group, top_k, rsf):
        idx, dense, _, _ = R.route(logits, bias, n_group, topk_group, top_k, rsf)
        return idx.to(torch.int32), torch.gather(dense, 1, idx)

    def dispatch(self, idx, w, x, world, E_local):
        T, H = x.shape
        k = idx.shape[1]
        rb = EP.row_bytes(H, k)
        KB = H // BLOCK
        xq, xq_scale = R.quantize_1x128(x)
        dests = (idx.long() // E_local)
        send_row_of = torch.full((T, world), -1, dtype=torch.int32)
        rows = []
        counts = torch.zeros((2, world), dtype=torch.int32)  # rows, routed pairs per destination
        for d in range(world):
            for t in range(T):
                if bool((dests[t] == d).any()):
                    send_row_of[t, d] = len(rows)
                    rows.append((t, d))
                    counts[0, d] += 1
                    counts[1, d] += int((dests[t] == d).sum())
        buf = torch.zeros((max(len(rows), 1), rb), dtype=torch.uint8)
        for r, (t, d) in enumerate(rows):
            buf[r, :H] = xq[t].view(torch.uint8)
            buf[r, H:H + 4 * KB] = xq_scale[:, t].contiguous().view(torch.uint8)
            here = dests[t] == d
            ids = torch.where(here, idx[t].long(), torch.full_like(idx[t].long(), -1)).to(torch.int32)
            ws = torch.where(here, w[t], torch.zeros_like(w[t])).to(torch.float32)
            buf[r, H + 4 * KB:H + 4 * KB + 4 * k] = ids.view(torch.uint8)
            buf[r, H + 4 * KB + 4 * k:H + 4 * KB + 8 * k] = ws.view(torch.uint8)
        return counts, send_row_of, buf, xq, xq_scale

    def expert_ffn(self, recv_buf, Rn, P, H, I, top_k, E_local, offset, planes, w13, w13_scale, w2, w2_scale):
        KB = H // BLOCK
        out = torch.zeros((Rn, H), dtype=torch.float32)
        if Rn == 0:
            return out
        xq = recv_buf[:Rn, :H].contiguous().view(torch.float8_e4m3fn)
        sc = recv_buf[:Rn, H:H + 4 * KB].contiguous().view(torch.float32)          # [R, KB]
        ids = recv_buf[:Rn, H + 4 * KB:H + 4 * KB + 4 * top_k].contiguous().view(torch.int32)
        ws = recv_buf[:Rn, H + 4 * KB + 4 * top_k:H + 4 * KB + 8 * top_k].contiguous().view(torch.float32)
        A = R.dequant_hidden(xq, sc.t().contiguous())
        for le in range(E_local):
            sel = (ids == offset + le)
            rows = sel.any(1).nonzero().squeeze(1)
            if rows.numel() == 0:
                continue
            W13 = R.dequant_weight(w13[le], w13_scale[le])
            W2 = R.dequant_weight(w2[le], w2_scale[le])
            G1 = A[rows] @ W13.t()
            C = (G1[:, I:] / (1.0 + torch.exp(-G1[:, I:]))) * G1[:, :I]
            O = C @ W2.t()
            wt = (ws[rows] * sel[rows]).sum(1)
            out.index_add_(0, rows, O * wt.unsqueeze(1))
        return out

    def shared_ffn(self, xq, xq_scale, sw13, sw13_scale, sw2, sw2_scale, planes, acc, t0=0):
        n = xq.shape[0]
        if n:
            acc[t0:t0 + n] += R.shared_expert(R.dequant_hidden(xq, xq_scale.contiguous()), sw13, sw13_scale, sw2,
                                              sw2_scale)

    def pack_back(self, rows, out=None):
        """Packed combine rows: fp16 of value / 2^e, then fp32 2^e (``gemms_ep_pack_back``)."""
        Rn, H = rows.shape
        if out is None:
            packed = torch.zeros((Rn, EP.back_row_bytes(H)), dtype=torch.uint8)
        else:
            packed = out[:Rn * EP.back_row_bytes(H)].view(Rn, EP.back_row_bytes(H))
        for r in range(Rn):
            amax = float(rows[r].abs().max()) if H else 0.0
            e = 0
            if amax > 0 and amax != float("inf") and amax == amax:
                e = math.frexp(amax)[1] - 15
            packed[r, :2 * H] = torch.ldexp(rows[r], torch.tensor(-float(e))).to(torch.float16).view(torch.uint8)
            packed[r, 2 * H:2 * H + 4] = torch.tensor([math.ldexp(1.0, e)], dtype=torch.float32).view(torch.uint8)
        return packed

    # peer combine: each rank's buffer stands for its symmetric allocation; the
    # "barrier" hands every rank a copy of all buffers (gloo all_gather), and
    # the combine reads rows from them with the offsets moe_ep computed.
    def peer_buffers(self, group, cap_rows, H):
        local = torch.zeros(max(cap_rows, 1) * EP.back_row_bytes(H), dtype=torch.uint8)
        return local, None

    def peer_publish(self, group, local, peers):
        import torch.distributed as dist
        bufs = [torch.empty_like(local) for _ in range(dist.get_world_size(group))]
        dist.all_gather(bufs, local, group=group)
        return bufs

    def combine_rows(self, acc, peers, row_add, send_row_of, world):
        out = acc.clone()
        H = acc.shape[1]
        rbb = EP.back_row_bytes(H)
        for t in range(acc.shape[0]):
            for d in range(world):
                r = int(send_row_of[t, d])
                if r >= 0:
                    row = peers[d].view(-1, rbb)[r + row_add[d]]
                    out[t] += self.unpack_back(row, H)
        return out.to(torch.bfloat16)

    @staticmethod
    def unpack_back(packed_row, H):
        vals = packed_row[:2 * H].contiguous().view(torch.float16).to(torch.float32)
        scale = packed_row[2 * H:2 * H + 4].contiguous().view(torch.float32)[0]
        return vals * scale

    def combine(self, acc, back, send_row_of, world):
        out = acc.clone()
        H = acc.shape[1]
        for t in range(acc.shape[0]):
            for d in range(world):
                r = int(send_row_of[t, d])
                if r >= 0:
                    out[t] += self.unpack_back(back[r], H)
        return out.to(torch.bfloat16)
