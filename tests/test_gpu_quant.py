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
