"""CPU oracle for the DeepSeek-V3 FP8 MoE layer -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module.  The product (``gemms_b200``) never calls it and
has no CPU fallback.

This is a parametrised restatement of the reference's PyTorch fp32-dequant
implementation ``run()`` in ``flashinfer_baseline.py:5-169``.  The reference
hard-codes the DeepSeek-V3 geometry (``H=7168, I=2048, E=256, E_local=32``,
``TOP_K=8, N_GROUP=8, TOPK_GROUP=4``; ``flashinfer_baseline.py:33-50``), so
config c0 (H=2048, I=768, E=32, 4 groups, top-4) cannot go through it
unchanged.  Each step below uses the same torch operations in the same order
as the cited reference lines, so at V3 shapes ``run_local`` equals the
reference ``run()`` bit for bit (pinned by ``tests/test_oracle.py`` against
golden outputs the reference itself produced, see ``tests/golden/``).

Two deliberate deviations, neither of which changes a value:
* weights are dequantised one expert at a time inside the expert loop instead
  of all at once (``:81-93``): the elementwise products are identical and host
  memory stays bounded at full V3 shapes;
* an optional ``tokens`` subset evaluates only some output rows (every MoE
  output row depends only on its own token), for full-size spot checks.

Pieces the reference does not have (``moe_layer``): the router GEMM, the
per-1x128 activation quantisation and the shared expert.  Their definitions
here are the build's own and are "parity unpinned" against the reference.
"""
from __future__ import annotations

import numpy as np
import torch

BLOCK = 128
FP8_MAX = 448.0


# --------------------------------------------------------------------------
# dequantisation  (flashinfer_baseline.py:68-93)
# --------------------------------------------------------------------------
def dequant_hidden(hidden_states: torch.Tensor, hidden_states_scale: torch.Tensor) -> torch.Tensor:
    """fp8 [T,H] * scale [H/128,T] (transposed) -> fp32 [T,H]; ``:68-79``."""
    T, H = hidden_states.shape
    A_fp32 = hidden_states.to(torch.float32)
    A_scale = hidden_states_scale.to(torch.float32)          # [H/128, T]
    A_scale_TH = A_scale.permute(1, 0).contiguous()          # [T, H/128]
    A_scale_expanded = (A_scale_TH.unsqueeze(-1).repeat(1, 1, BLOCK).reshape(T, H).contiguous())
    return A_fp32 * A_scale_expanded


def dequant_weight(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp8 [..., R, C] * 128x128 block scale [..., R/128, C/128] -> fp32; ``:81-93``."""
    W = w.to(torch.float32)
    S = s.to(torch.float32)
    S = torch.repeat_interleave(S, BLOCK, dim=-2)
    S = torch.repeat_interleave(S, BLOCK, dim=-1)
    return W * S


# --------------------------------------------------------------------------
# no-aux grouped routing  (flashinfer_baseline.py:95-127)
# --------------------------------------------------------------------------
def sigmoid_exact(logits: torch.Tensor) -> torch.Tensor:
    """1/(1+exp(-x)) with exp correctly rounded to fp32 (exp done in float64).

    The CUDA router computes exactly this.  ``torch.exp`` on CPU (the
    reference's ``:100``) is a vectorised approximation that differs from the
    correctly rounded value by one ulp on ~1% of inputs; tests check that the
    resulting top-k sets agree (an ulp can only matter at an exact near-tie).
    """
    e = torch.from_numpy(np.exp(-logits.to(torch.float64).numpy()).astype(np.float32))
    return 1.0 / (1.0 + e)


def route(routing_logits, routing_bias, n_group, topk_group, top_k, rsf, exact_exp=False):
    """Returns (topk_idx int64 [T,k] unordered, weights fp32 dense [T,E], s, s_with_bias).

    Follows ``flashinfer_baseline.py:96-127`` with the group geometry as
    parameters (the reference fixes ``N_GROUP=8, TOPK_GROUP=4, TOP_K=8`` at
    ``:48-50``).
    """
    logits = routing_logits.to(torch.float32)                       # :96
    bias = routing_bias.to(torch.float32).reshape(-1)               # :97
    T, E = logits.shape
    if exact_exp:
        s = sigmoid_exact(logits)
    else:
        s = 1.0 / (1.0 + torch.exp(-logits))                        # :100
    s_with_bias = s + bias                                          # :101
    group_size = E // n_group                                       # :104
    s_wb_grouped = s_with_bias.view(T, n_group, group_size)         # :105
    top2_vals, _ = torch.topk(s_wb_grouped, k=2, dim=2, largest=True, sorted=False)   # :108
    group_scores = top2_vals.sum(dim=2)                             # :109
    _, group_idx = torch.topk(group_scores, k=topk_group, dim=1, largest=True, sorted=False)  # :112
    group_mask = torch.zeros_like(group_scores)                     # :113
    group_mask.scatter_(1, group_idx, 1.0)                          # :114
    score_mask = group_mask.unsqueeze(2).expand(T, n_group, group_size).reshape(T, E)  # :115
    neg_inf = torch.finfo(torch.float32).min                        # :118
    scores_pruned = s_with_bias.masked_fill(score_mask == 0, neg_inf)  # :119
    _, topk_idx = torch.topk(scores_pruned, k=top_k, dim=1, largest=True, sorted=False)  # :120
    M = torch.zeros_like(s)                                         # :123
    M.scatter_(1, topk_idx, 1.0)                                    # :124
    weights = s * M                                                 # :125
    weights_sum = weights.sum(dim=1, keepdim=True) + 1e-20          # :126
    weights = (weights / weights_sum) * rsf                         # :127
    return topk_idx, weights, s, s_with_bias


def routing_margins(s_with_bias: torch.Tensor, topk_idx: torch.Tensor, n_group: int, topk_group: int):
    """Per-token decision margins (diagnostics for near-ties).

    Returns (expert_gap [T], group_gap [T]): the gap between the smallest kept
    and the largest dropped biased score among kept groups, and between the
    smallest kept and largest dropped group score.  A gap within a couple of
    ulps is a tie that an ulp of sigmoid rounding could flip.
    """
    T, E = s_with_bias.shape
    gs = E // n_group
    grouped = s_with_bias.view(T, n_group, gs)
    gsc = torch.topk(grouped, 2, dim=2).values.sum(2)
    gsorted = torch.sort(gsc, dim=1, descending=True).values
    group_gap = (gsorted[:, topk_group - 1] - gsorted[:, topk_group]) if topk_group < n_group else torch.full((T,), float("inf"))
    kept_g = torch.topk(gsc, topk_group, dim=1).indices
    mask = torch.zeros(T, n_group, dtype=torch.bool)
    mask.scatter_(1, kept_g, True)
    pr = s_with_bias.masked_fill(~mask.repeat_interleave(gs, 1), float("-inf"))
    srt = torch.sort(pr, dim=1, descending=True).values
    k = topk_idx.shape[1]
    expert_gap = srt[:, k - 1] - srt[:, k]
    return expert_gap, group_gap


# --------------------------------------------------------------------------
# run(): one rank's local experts  (flashinfer_baseline.py:5-169)
# --------------------------------------------------------------------------
@torch.no_grad()
def run_local(routing_logits, routing_bias, hidden_states, hidden_states_scale,
              gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
              local_expert_offset, routed_scaling_factor, *, n_group=8, topk_group=4, top_k=8,
              return_fp32=False, tokens=None, exact_exp=False):
    """Parametrised ``flashinfer_baseline.run`` (``:5-169``)."""
    T, H = hidden_states.shape
    E_local, twoI, _ = gemm1_weights.shape
    I = twoI // 2
    E_global = routing_logits.shape[1]
    # shape checks (:57-64)
    assert hidden_states_scale.shape == (H // BLOCK, T)
    assert gemm1_weights.shape == (E_local, 2 * I, H)
    assert gemm1_weights_scale.shape == (E_local, 2 * I // BLOCK, H // BLOCK)
    assert gemm2_weights.shape == (E_local, H, I)
    assert gemm2_weights_scale.shape == (E_local, H // BLOCK, I // BLOCK)
    assert routing_bias.shape[-1] == E_global

    A = dequant_hidden(hidden_states, hidden_states_scale)                      # :68-79
    topk_idx, weights, _, _ = route(routing_logits, routing_bias, n_group, topk_group, top_k,
                                    routed_scaling_factor, exact_exp=exact_exp)  # :95-127
    output = torch.zeros((T, H), dtype=torch.float32)                           # :130
    local_start = int(local_expert_offset)                                      # :132
    tok_mask = None
    if tokens is not None:
        tok_mask = torch.zeros(T, dtype=torch.bool)
        tok_mask[torch.as_tensor(tokens, dtype=torch.long)] = True
    for le in range(E_local):                                                   # :135
        ge = local_start + le
        if ge < 0 or ge >= E_global:
            continue
        sel_mask_per_token = (topk_idx == ge).any(dim=1)                        # :141
        if tok_mask is not None:
            sel_mask_per_token &= tok_mask
        if not sel_mask_per_token.any():
            continue
        token_idx = torch.nonzero(sel_mask_per_token, as_tuple=False).squeeze(1)  # :145
        A_e = A.index_select(0, token_idx)                                      # :149
        W13_e = dequant_weight(gemm1_weights[le], gemm1_weights_scale[le])      # :81-86, :150
        W2_e = dequant_weight(gemm2_weights[le], gemm2_weights_scale[le])       # :88-93, :151
        G1 = A_e.matmul(W13_e.t())                                              # :154
        X1 = G1[:, :I]                                                          # :157
        X2 = G1[:, I:]                                                          # :158
        silu_X2 = X2 / (1.0 + torch.exp(-X2))                                   # :159
        C = silu_X2 * X1                                                        # :160
        O = C.matmul(W2_e.t())                                                  # :163
        w_tok = weights.index_select(0, token_idx)[:, ge]                       # :166
        output.index_add_(0, token_idx, O * w_tok.unsqueeze(1))                 # :167
    return output if return_fp32 else output.to(torch.bfloat16)                # :169


# --------------------------------------------------------------------------
# Full layer (the moe() surface).  Router GEMM, activation quantisation and
# the shared expert are the build's own definitions: parity unpinned.
# --------------------------------------------------------------------------
def router_logits(x: torch.Tensor, router_w: torch.Tensor) -> torch.Tensor:
    """logits = x . router_w^T in fp32 ([T,H] x [E,H] -> [T,E])."""
    return x.to(torch.float32) @ router_w.to(torch.float32).t()


def quantize_1x128(x: torch.Tensor):
    """Per-1x128 e4m3 quantisation: scale = amax/448 (1.0 for an all-zero block),
    q = e4m3_rne(x / scale).  Returns (q [T,H], scale [H/128, T]) in the
    reference's transposed scale layout (``flashinfer_baseline.py:59,72``)."""
    T, H = x.shape
    xf = x.to(torch.float32).reshape(T, H // BLOCK, BLOCK)
    amax = xf.abs().amax(dim=2)
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (xf / scale.unsqueeze(2)).to(torch.float8_e4m3fn).reshape(T, H)
    return q, scale.t().contiguous()


@torch.no_grad()
def shared_expert(A: torch.Tensor, w13, w13_scale, w2, w2_scale, tokens=None) -> torch.Tensor:
    """Dense SwiGLU MLP with the same dequant / GEMM / SwiGLU steps as
    ``flashinfer_baseline.py:81-93, 154-163``, routing weight 1.0."""
    I = w13.shape[0] // 2
    rows = A if tokens is None else A.index_select(0, torch.as_tensor(tokens, dtype=torch.long))
    W13 = dequant_weight(w13, w13_scale)
    W2 = dequant_weight(w2, w2_scale)
    G1 = rows.matmul(W13.t())
    X1, X2 = G1[:, :I], G1[:, I:]
    C = (X2 / (1.0 + torch.exp(-X2))) * X1
    O = C.matmul(W2.t())
    if tokens is None:
        return O
    out = torch.zeros_like(A)
    out.index_copy_(0, torch.as_tensor(tokens, dtype=torch.long), O)
    return out


@torch.no_grad()
def moe_layer(x, router_w, router_bias, w13, w13_scale, w2, w2_scale,
              shared_w13=None, shared_w13_scale=None, shared_w2=None, shared_w2_scale=None, *,
              n_group, topk_group, top_k, rsf, logits=None, tokens=None, chunk=32,
              return_fp32=False, exact_exp=False):
    """Full layer on one device: router GEMM -> 1x128 quant -> ``run_local`` over
    all experts in ``chunk``-expert slices summed in fp32 -> + shared expert ->
    one bf16 cast.  ``logits`` overrides the router GEMM (routing parity is
    judged at the reference's own boundary: identical fp32 logits in)."""
    if logits is None:
        logits = router_logits(x, router_w)
    hs, hs_scale = quantize_1x128(x)
    E = w13.shape[0]
    T, H = x.shape
    out = torch.zeros((T, H), dtype=torch.float32)
    for off in range(0, E, chunk):
        out += run_local(logits, router_bias, hs, hs_scale, w13[off:off + chunk], w13_scale[off:off + chunk],
                         w2[off:off + chunk], w2_scale[off:off + chunk], off, rsf,
                         n_group=n_group, topk_group=topk_group, top_k=top_k,
                         return_fp32=True, tokens=tokens, exact_exp=exact_exp)
    if shared_w13 is not None:
        A = dequant_hidden(hs, hs_scale)
        out += shared_expert(A, shared_w13, shared_w13_scale, shared_w2, shared_w2_scale, tokens=tokens)
    return out if return_fp32 else out.to(torch.bfloat16)


# --------------------------------------------------------------------------
# The steps either side of the layer (no reference code: the reference's
# operator starts from quantised activations).  RMSNorm as the DeepSeek-V3
# decoder defines it: fp32 variance and rsqrt, cast back to the activations'
# dtype, times the weight.  Parity unpinned.
# --------------------------------------------------------------------------
def rmsnorm(h: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """y = weight * bf16(h * rsqrt(mean(h^2) + eps)), rounded to bf16."""
    hs = h.to(torch.float32)
    var = hs.pow(2).mean(-1, keepdim=True)
    hs = hs * torch.rsqrt(var + eps)
    return (weight.to(torch.float32) * hs.to(h.dtype).to(torch.float32)).to(torch.bfloat16)


@torch.no_grad()
def moe_block(h, norm_weight, router_w, router_bias, w13, w13_scale, w2, w2_scale,
              shared_w13=None, shared_w13_scale=None, shared_w2=None, shared_w2_scale=None, *,
              n_group, topk_group, top_k, rsf, eps=1e-6, logits=None, tokens=None):
    """h + moe(rmsnorm(h)) with the residual added to the layer's fp32 result
    and rounded to bf16 once."""
    y = rmsnorm(h, norm_weight, eps)
    out = moe_layer(y, router_w, router_bias, w13, w13_scale, w2, w2_scale, shared_w13, shared_w13_scale,
                    shared_w2, shared_w2_scale, n_group=n_group, topk_group=topk_group, top_k=top_k, rsf=rsf,
                    logits=logits, tokens=tokens, return_fp32=True)
    return (out + h.to(torch.float32)).to(torch.bfloat16)


def compare(out: torch.Tensor, ref: torch.Tensor, rows=None) -> dict:
    """Output parity metrics used by every layer test.

    * ``max_rel`` = max|out-ref| / max|ref| (normwise maximum relative error);
    * ``mae_rms`` = mean|out-ref| / RMS(ref);
    * ``elem_rel`` = max over elements with |ref| >= 1e-2 max|ref| of
      |out-ref| / |ref| (elementwise relative error), and ``elem_rel_10`` the
      same over |ref| >= 1e-1 max|ref|;
    * ``elem_frac`` = the share of elements that ``elem_rel`` covers.

    The bars (tests/helpers.py) are max_rel <= 2e-2 and mae_rms <= 1e-3 (the
    BASELINE north star), elem_rel_10 <= 2e-2 and elem_rel <= 1e-1.  A bf16
    output is only resolved to 2^-8 relative, so an element one rounding step
    off already reads 0.4-0.8% here; elements near 1% of the maximum move by
    a few steps under the fp8 intermediate's rounding (about 4% in a CPU
    emulation of the GPU arithmetic at config c0).
    """
    o = out.to(torch.float64)
    r = ref.to(torch.float64)
    if rows is not None:
        idx = torch.as_tensor(rows, dtype=torch.long)
        o, r = o.index_select(0, idx), r.index_select(0, idx)
    d = (o - r).abs()
    ra = r.abs()
    amax = ra.max().clamp_min(1e-30)
    rms = r.pow(2).mean().sqrt().clamp_min(1e-30)

    def elem(th):
        big = ra >= th * amax
        return float((d[big] / ra[big]).max()) if bool(big.any()) else 0.0

    return {"max_rel": float(d.max() / amax),
            "mae_rms": float(d.mean() / rms),
            "elem_rel": elem(1e-2),
            "elem_rel_10": elem(1e-1),
            "elem_frac": float((ra >= 1e-2 * amax).double().mean()),
            "max_abs": float(d.max()),
            "rms": float(rms)}
