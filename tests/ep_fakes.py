"""CPU stand-ins for the device side of expert parallelism (test-only).

They follow the contracts of ``include/gemms_moe.h`` (packed row layout,
destination grouping in token order, fp32 pre-reduced rows, deterministic
combine, the device-driven exchange's region layout and plan) with the
oracle's fp32 arithmetic, so that ``gemms_b200.ep.moe_ep``'s host logic --
count exchange, split sizes, the two all-to-alls, the exchange regions and
barriers, the combine mapping -- runs on gloo ranks without a GPU.
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

    def dispatch(self, idx, w, x, world, E_local, region=None):
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
        if region is not None:  # the exchange region's header and send rows
            region.hdr.copy_(counts)
            region.send.zero_()
            region.send[:len(rows)] = buf[:len(rows)]
            buf = region.send
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

    # device-driven exchange: each rank's region is a set of CPU tensors; the
    # barrier hands every rank copies of all regions (gloo all_gather), which
    # stand for the peer mappings the pull and the combine read.
    def exchange_region(self, group, send_cap, recv_cap, H, top_k):
        import torch.distributed as dist

        class Region:
            pass
        world = dist.get_world_size(group)
        reg = Region()
        reg.world, reg.send_cap, reg.recv_cap = world, send_cap, recv_cap
        reg.rb, reg.rbb = EP.row_bytes(H, top_k), EP.back_row_bytes(H)
        reg.hdr = torch.zeros((2, world), dtype=torch.int32)
        reg.send = torch.zeros((send_cap, reg.rb), dtype=torch.uint8)
        reg.back = torch.zeros(recv_cap * reg.rbb, dtype=torch.uint8)
        return reg

    def peer_barrier(self, group, reg):
        import torch.distributed as dist
        world = dist.get_world_size(group)
        reg.peer_hdr = [torch.empty_like(reg.hdr) for _ in range(world)]
        reg.peer_send = [torch.empty_like(reg.send) for _ in range(world)]
        reg.peer_back = [torch.empty_like(reg.back) for _ in range(world)]
        dist.all_gather(reg.peer_hdr, reg.hdr, group=group)
        dist.all_gather(reg.peer_send, reg.send, group=group)
        dist.all_gather(reg.peer_back, reg.back, group=group)

    def pull(self, reg, rank, world, H, top_k):
        """The plan of gemms_ep_pull (info layout of include/gemms_moe.h) and the copy."""
        m = [reg.peer_hdr[s][0].tolist() for s in range(world)]
        mp = [reg.peer_hdr[s][1].tolist() for s in range(world)]
        to_me = [m[s][rank] for s in range(world)]
        total = sum(to_me)
        flags = 1 if total > reg.recv_cap else 0
        if any(sum(m[s]) > reg.send_cap or min(m[s]) < 0 for s in range(world)):
            flags |= 2
        info = torch.zeros(128, dtype=torch.int32)
        R = 0 if flags else total
        info[0], info[1], info[2] = R, (0 if flags else sum(mp[s][rank] for s in range(world))), flags
        start = 0
        recv = torch.zeros((reg.recv_cap, reg.rb), dtype=torch.uint8)
        for s in range(world):
            info[8 + s] = start
            info[48 + s] = sum(m[s][:rank])
            info[88 + s] = sum(m[q][s] for q in range(rank)) - sum(m[rank][:s])
            if not flags:
                o = int(info[48 + s])
                recv[start:start + to_me[s]] = reg.peer_send[s][o:o + to_me[s]]
            start += to_me[s]
        info[8 + world] = total
        return recv, info

    def expert_ffn_dev(self, recv_buf, info, R_cap, P_cap, H, I, top_k, E_local, offset, planes, w13, w13_scale,
                       w2, w2_scale):
        Rn = int(info[0])
        out = torch.zeros((R_cap, H), dtype=torch.float32)
        out[:Rn] = self.expert_ffn(recv_buf[:Rn], Rn, int(info[1]), H, I, top_k, E_local, offset, planes, w13,
                                   w13_scale, w2, w2_scale)
        return out

    def pack_back_dev(self, rows, info, reg):
        self.pack_back(rows[:int(info[0])], out=reg.back)

    def combine_peer(self, acc, reg, info, send_row_of, world):
        out = acc.clone()
        H = acc.shape[1]
        for t in range(acc.shape[0]):
            for d in range(world):
                r = int(send_row_of[t, d])
                if r >= 0:
                    row = reg.peer_back[d].view(-1, reg.rbb)[r + int(info[88 + d])]
                    out[t] += self.unpack_back(row, H)
        return out.to(torch.bfloat16)

    def exchange_flags(self, reg):
        return 0

    def side_stream(self):
        return None  # CPU: the shared expert runs in order

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
