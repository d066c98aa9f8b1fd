"""GPU: the per-1x128 e4m3 activation quantisation is byte-exact against the
oracle's quantize_1x128 (same IEEE division for the scale and the quotient,
same round-to-nearest-even saturating conversion): through the token-major
quantiser (gemms_quantize_1x128) and through the expert-parallel dispatch
(gemms_ep_dispatch), whose packed send rows carry the same bytes and scales."""
import pytest
import torch

import gemms_b200
from gemms_b200 import ep as EP
from gemms_b200 import workloads as W
from oracle import reference_moe as R

pytestmark = pytest.mark.gpu


def _inputs(T, H, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g)
    # blocks of very different magnitudes, an all-zero block, values that
    # quantise to exactly +-448, subnormal e4m3 outputs
    x[:, :128] *= 1e-3
    if H >= 512:
        x[0, 128:256] = 0
        x[min(1, T - 1), 256:384] = torch.linspace(-1, 1, 128)
        x[min(2, T - 1), 384:512] *= 1e4
    else:
        x[0, 128:256] = 0
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("T,H", [(1, 7168), (33, 7168), (4096, 7168), (64, 2048), (5, 256)])
def test_quantize_bytes_match_oracle(T, H):
    x = _inputs(T, H, T + H)
    q, sc = gemms_b200.quantize_1x128(x.cuda())
    torch.cuda.synchronize()
    rq, rsc = R.quantize_1x128(x)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(sc.cpu(), rsc)


def test_ep_dispatch_rows_match_oracle_bytes():
    sh = W.CONFIGS["c1"].replace(T=37)
    x = _inputs(sh.T, sh.H, 5)
    d = W.make_inputs(sh, seed=2, with_weights=False)
    logits = R.router_logits(x, d["router_w"])
    idx, w = EP.CudaEpKernels().route(logits.cuda(), d["router_bias"].cuda(), sh.n_group, sh.topk_group,
                                      sh.top_k, sh.rsf)
    world = 4
    counts, row_of, buf, xq, xs = EP.CudaEpKernels().dispatch(idx, w, x.cuda(), world, sh.E // world)
    torch.cuda.synchronize()
    rq, rsc = R.quantize_1x128(x)
    assert torch.equal(xq.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(xs.cpu(), rsc)
    buf, row_of = buf.cpu(), row_of.cpu()
    H = sh.H
    for t in range(sh.T):
        for dst in range(world):
            r = int(row_of[t, dst])
            if r < 0:
                continue
            row = buf[r]
            assert torch.equal(row[:H], rq[t].view(torch.uint8)), (t, dst)
            assert torch.equal(row[H:H + 4 * (H // 128)].view(torch.float32), rsc[:, t]), (t, dst)


@pytest.mark.parametrize("T", [33, 300])
def test_permute_grouped_rows_match_oracle_bytes(T):
    """The grouped activation rows GEMM1 reads come from permute_kernel, which
    quantises each token's row per 1x128 (bf16 input) and writes it once per
    routed expert and once for the shared expert.  Every copy, and its scale,
    must be byte-identical to the oracle's quantize_1x128 of that token.  Read
    from a gemms_moe_fwd workspace at the offsets gemms_test_workspace_regions
    reports (T=33 routes with the block-per-token router, T=300 with the
    warp-per-token one)."""
    import ctypes

    from gemms_b200._lib import GemmsMoeArgs, GemmsMoeShape

    sh = W.CONFIGS["c0"].replace(T=T, shared=True)
    d = W.make_inputs(sh, seed=17, device="cuda")
    x_cpu = _inputs(T, sh.H, 3 + T)
    x = x_cpu.cuda()
    logits = gemms_b200.router_logits(x, d["router_w"])
    shape = GemmsMoeShape(T=T, H=sh.H, I=sh.I, E=sh.E, E_local=sh.E, local_expert_offset=0, n_group=sh.n_group,
                          topk_group=sh.topk_group, top_k=sh.top_k, has_shared=1,
                          input_mode=_lib_mod().GEMMS_INPUT_BF16, bias_bf16=0, inter_planes=2,
                          routed_scaling_factor=sh.rsf)
    a = GemmsMoeArgs()
    a.shape = shape
    a.routing_logits = logits.data_ptr()
    a.routing_bias = d["router_bias"].data_ptr()
    a.hidden_bf16 = x.data_ptr()
    a.w13, a.w13_scale, a.w2, a.w2_scale = (d[k].data_ptr() for k in ("w13", "w13_scale", "w2", "w2_scale"))
    a.shared_w13, a.shared_w13_scale = d["shared_w13"].data_ptr(), d["shared_w13_scale"].data_ptr()
    a.shared_w2, a.shared_w2_scale = d["shared_w2"].data_ptr(), d["shared_w2_scale"].data_ptr()
    out = torch.empty((T, sh.H), dtype=torch.bfloat16, device="cuda")
    a.out = out.data_ptr()
    L = _lib_mod().load()
    nbytes = L.gemms_moe_workspace_size(ctypes.byref(shape))
    ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device="cuda")
    base = (-ws.data_ptr()) % 256
    ws = ws[base:base + nbytes]
    stream = torch.cuda.current_stream().cuda_stream
    assert L.gemms_moe_fwd(ctypes.byref(a), ws.data_ptr(), nbytes, stream) == 0
    flags = ctypes.c_int32(0)
    assert L.gemms_moe_check(ws.data_ptr(), stream, ctypes.byref(flags)) == 0
    offs = [ctypes.c_size_t(0) for _ in range(4)]
    ld = ctypes.c_int32(0)
    assert L.gemms_test_workspace_regions(ctypes.byref(shape), ctypes.byref(offs[0]), ctypes.byref(offs[1]),
                                          ctypes.byref(ld), ctypes.byref(offs[2]), ctypes.byref(offs[3])) == 0
    rows_off, scale_off, pair_off, groups_off = (o.value for o in offs)
    H, K, n_rows = sh.H, sh.top_k, T * sh.top_k + T
    wsc = ws.cpu()
    rows = wsc[rows_off:rows_off + n_rows * H].view(n_rows, H)
    scales = wsc[scale_off:scale_off + 4 * (H // 128) * ld.value].view(torch.float32).view(H // 128, ld.value)
    pair_row = wsc[pair_off:pair_off + 4 * T * K].view(torch.int32).view(T, K).long()
    first = wsc[groups_off:groups_off + 4 * (sh.E + 2)].view(torch.int32).long()
    rq, rsc = R.quantize_1x128(x_cpu)
    rq = rq.view(torch.uint8)
    assert bool((pair_row >= 0).all()), "every expert is local here"
    tok = torch.arange(T).repeat_interleave(K)
    r = pair_row.reshape(-1)
    assert torch.equal(rows[r], rq[tok]), "routed copies differ from quantize_1x128"
    assert torch.equal(scales[:, r], rsc[:, tok]), "routed copies' scales differ"
    rs = int(first[sh.E]) + torch.arange(T)
    assert torch.equal(rows[rs], rq), "shared-expert rows differ from quantize_1x128"
    assert torch.equal(scales[:, rs], rsc), "shared-expert rows' scales differ"
    assert len(set(r.tolist())) == T * K, "each (token, slot) has its own grouped row"


def _lib_mod():
    from gemms_b200 import _lib
    return _lib
