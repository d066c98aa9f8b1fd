"""Operator surface of the B200 MoE layer.

* ``run(...)`` -- drop-in for the reference operator ``run`` in
  ``flashinfer_baseline.py:5-169``: same argument names, order, layouts and
  return value (new bf16 [T, H] holding the weighted sum over the local
  experts ``[local_expert_offset, local_expert_offset + E_local)``).  Shape
  errors raise :class:`ShapeError`, which is both a ``ValueError`` and an
  ``AssertionError`` (the reference asserts, ``:42-64``).
* ``moe(x, router_w, router_bias, w13, w13_scale, w2, w2_scale, ...)`` -- the
  full DeepSeek-V3 layer: router GEMM, per-1x128 activation quantisation,
  routed experts, shared expert, weighted combine.  With ``ep_group`` it runs
  expert-parallel (see :mod:`gemms_b200.ep`).

Both run only on CUDA tensors of an sm_100 device through the C ABI; there is
no CPU fallback.
"""
from __future__ import annotations

import ctypes
import functools

import torch

from . import _lib
from ._lib import GemmsMoeArgs, GemmsMoeShape

BLOCK = 128


class ShapeError(ValueError, AssertionError):
    """Inconsistent or unsupported shapes / dtypes / devices."""


def _req(cond: bool, msg: str) -> None:
    if not cond:
        raise ShapeError(msg)


def _on_tensor_device(fn):
    """Runs the operator with its first CUDA tensor argument's device current,
    so that kernels go to that device's current stream (not to whichever
    device the caller left current, which would be handed another GPU's
    pointers)."""
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        for v in list(args) + list(kwargs.values()):
            if isinstance(v, torch.Tensor) and v.is_cuda:
                with torch.cuda.device(v.device):
                    return fn(*args, **kwargs)
        return fn(*args, **kwargs)
    return wrapper


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_workspaces: dict = {}


def _workspace(device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
    """Per (device, stream, tag) workspace from torch's caching allocator, grown
    on demand.  Keyed by stream so that layers running concurrently on
    different streams never share scratch; a replaced workspace is freed on
    the stream it was allocated on, so the allocator reuses it in stream order."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream, tag)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 256) + 256, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    off = (-ws.data_ptr()) % 256
    return ws[off:off + nbytes] if nbytes else ws[off:off + 1]


def _check_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        _req(t.is_cuda, "gemms_b200 operators take CUDA tensors only (no CPU path)")
        _req(t.is_contiguous(), "tensors must be contiguous")
        dev = t.device if dev is None else dev
        _req(t.device == dev, "all tensors must be on one device")
    return dev


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _call_fwd(shape: GemmsMoeShape, args: GemmsMoeArgs, device: torch.device, tag: str) -> torch.Tensor:
    L = _lib.load()
    nbytes = L.gemms_moe_workspace_size(ctypes.byref(shape))
    if nbytes == 0:
        raise ShapeError("unsupported MoE geometry for the sm_100a kernels "
                         f"(T={shape.T} H={shape.H} I={shape.I} E={shape.E} n_group={shape.n_group} "
                         f"topk_group={shape.topk_group} top_k={shape.top_k})")
    ws = _workspace(device, nbytes, tag)
    args.shape = shape
    _lib.check(L.gemms_moe_fwd(ctypes.byref(args), ws.data_ptr(), nbytes, _stream()), "gemms_moe_fwd")
    return ws


def check_device_errors(ws: torch.Tensor | None = None, tag: str = "moe") -> None:
    """Synchronise and raise if a kernel recorded a device-side timeout."""
    L = _lib.load()
    if ws is None:
        dev = torch.cuda.current_device()
        cached = _workspaces.get((dev, torch.cuda.current_stream(dev).cuda_stream, tag))
        if cached is None:
            return
        ws = cached[(-cached.data_ptr()) % 256:]
    flags = ctypes.c_int32(0)
    rc = L.gemms_moe_check(ws.data_ptr(), _stream(), ctypes.byref(flags))
    if rc != 0:
        raise _lib.GemmsError(rc, "gemms_moe_check", flags.value)


@torch.no_grad()
@_on_tensor_device
def run(routing_logits: torch.Tensor, routing_bias: torch.Tensor, hidden_states: torch.Tensor,
        hidden_states_scale: torch.Tensor, gemm1_weights: torch.Tensor, gemm1_weights_scale: torch.Tensor,
        gemm2_weights: torch.Tensor, gemm2_weights_scale: torch.Tensor, local_expert_offset: int,
        routed_scaling_factor: float, *, n_group: int = 8, topk_group: int = 4, top_k: int = 8,
        inter_planes: int = 2, return_routing: bool = False, deterministic: bool = False):
    """Drop-in for ``flashinfer_baseline.run`` (``:5-16``) on B200.

    The reference fixes n_group=8, topk_group=4, top_k=8 (``:48-50``); they are
    keyword parameters here with those defaults.  ``deterministic=True`` makes
    the combine bit-reproducible (per-token sum of the expert rows in slot
    order instead of fp32 atomics; the reference's ``index_add_`` order,
    ``:166-169``, is also fixed).
    """
    dev = _check_cuda(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                      gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    T, E = routing_logits.shape
    _req(hidden_states.dim() == 2 and hidden_states.shape[0] == T, "hidden_states must be [T, H]")
    H = hidden_states.shape[1]
    _req(gemm1_weights.dim() == 3, "gemm1_weights must be [E_local, 2I, H]")
    E_local, twoI, H1 = gemm1_weights.shape
    I = twoI // 2
    _req(H1 == H and twoI % 2 == 0, "gemm1_weights must be [E_local, 2I, H]")
    _req(H % BLOCK == 0 and I % BLOCK == 0, "H and I must be multiples of 128")
    _req(hidden_states_scale.shape == (H // BLOCK, T), "hidden_states_scale must be [H/128, T]")
    _req(gemm1_weights_scale.shape == (E_local, 2 * I // BLOCK, H // BLOCK), "gemm1_weights_scale shape")
    _req(gemm2_weights.shape == (E_local, H, I), "gemm2_weights must be [E_local, H, I]")
    _req(gemm2_weights_scale.shape == (E_local, H // BLOCK, I // BLOCK), "gemm2_weights_scale shape")
    _req(routing_bias.shape[-1] == E, "routing_bias must have E entries")
    _req(routing_logits.dtype == torch.float32, "routing_logits must be fp32")
    _req(routing_bias.dtype in (torch.float32, torch.bfloat16), "routing_bias must be fp32 or bf16")
    _req(hidden_states.dtype == torch.float8_e4m3fn, "hidden_states must be float8_e4m3fn")
    _req(gemm1_weights.dtype == torch.float8_e4m3fn and gemm2_weights.dtype == torch.float8_e4m3fn,
         "expert weights must be float8_e4m3fn")
    for t in (hidden_states_scale, gemm1_weights_scale, gemm2_weights_scale):
        _req(t.dtype == torch.float32, "scales must be fp32")

    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    shape = GemmsMoeShape(T=T, H=H, I=I, E=E, E_local=E_local, local_expert_offset=int(local_expert_offset),
                          n_group=n_group, topk_group=topk_group, top_k=top_k, has_shared=0,
                          input_mode=_lib.GEMMS_INPUT_FP8, bias_bf16=int(routing_bias.dtype == torch.bfloat16),
                          inter_planes=inter_planes, routed_scaling_factor=float(routed_scaling_factor),
                          deterministic=int(deterministic))
    args = GemmsMoeArgs()
    args.routing_logits = _ptr(routing_logits)
    args.routing_bias = _ptr(routing_bias)
    args.hidden_fp8 = _ptr(hidden_states)
    args.hidden_scale = _ptr(hidden_states_scale)
    args.w13, args.w13_scale = _ptr(gemm1_weights), _ptr(gemm1_weights_scale)
    args.w2, args.w2_scale = _ptr(gemm2_weights), _ptr(gemm2_weights_scale)
    args.out = _ptr(out)
    idx = w = counts = None
    if return_routing:
        idx = torch.empty((T, top_k), dtype=torch.int32, device=dev)
        w = torch.empty((T, top_k), dtype=torch.float32, device=dev)
        counts = torch.empty((max(E_local, 1),), dtype=torch.int32, device=dev)
        args.topk_idx_out, args.topk_w_out, args.expert_counts_out = _ptr(idx), _ptr(w), _ptr(counts)
    _call_fwd(shape, args, dev, "run")
    if return_routing:
        return out, idx, w, counts[:E_local]
    return out


@torch.no_grad()
@_on_tensor_device
def router_logits(x: torch.Tensor, router_w: torch.Tensor) -> torch.Tensor:
    """fp32 logits = x . router_w^T from a bf16 x [T, H] and an fp32 router
    weight [E, H], on the sm_100a router GEMM (``gemms_router_logits``).

    router_w is split into bf16 hi + lo planes (16 significant bits) and both
    products accumulate in fp32 on the tensor cores, so the result tracks an
    fp32 GEMM to ~1e-5 relative; split-K partials are summed in a fixed order.
    """
    dev = _check_cuda(x, router_w)
    _req(x.dim() == 2 and x.dtype == torch.bfloat16, "x must be bf16 [T, H]")
    _req(router_w.dim() == 2 and router_w.dtype == torch.float32 and router_w.shape[1] == x.shape[1],
         "router_w must be fp32 [E, H]")
    T, H = x.shape
    E = router_w.shape[0]
    L = _lib.load()
    nbytes = L.gemms_router_workspace_size(T, H, E)
    if nbytes == 0:
        raise ShapeError(f"unsupported router GEMM shape (T={T} H={H} E={E}; H % 64 == 0, E <= 256)")
    ws = _workspace(dev, nbytes, "router")
    out = torch.empty((T, E), dtype=torch.float32, device=dev)
    _lib.check(L.gemms_router_logits(x.data_ptr(), router_w.data_ptr(), T, H, E, out.data_ptr(), ws.data_ptr(),
                                     nbytes, _stream()), "gemms_router_logits")
    return out


@torch.no_grad()
@_on_tensor_device
def moe(x: torch.Tensor, router_w: torch.Tensor, router_bias: torch.Tensor, w13: torch.Tensor,
        w13_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor, *,
        shared_w13: torch.Tensor | None = None, shared_w13_scale: torch.Tensor | None = None,
        shared_w2: torch.Tensor | None = None, shared_w2_scale: torch.Tensor | None = None,
        n_group: int = 8, topk_group: int = 4, top_k: int = 8, routed_scaling_factor: float = 2.5,
        inter_planes: int = 2, logits: torch.Tensor | None = None, ep_group=None,
        return_routing: bool = False, profile_events=None, residual: torch.Tensor | None = None,
        ep_exchange: str | None = None, max_tokens_per_rank: int | None = None, deterministic: bool = False):
    """DeepSeek-V3 MoE layer forward: bf16 x [T, H] -> bf16 [T, H].

    ``w13`` [E, 2I, H] / ``w2`` [E, H, I] are e4m3 with fp32 128x128 block
    scales; ``router_w`` fp32 [E, H], ``router_bias`` [E].  With ``ep_group``
    (a torch.distributed process group) the weights passed are this rank's
    E/world experts and tokens are exchanged between the ranks:
    ``ep_exchange="nccl"`` (NCCL all-to-all, split sizes read on the host) or
    ``"peer"`` (device-driven over symmetric memory, no host synchronisation;
    every rank passes the same T or ``max_tokens_per_rank``); the default is
    ``GEMMS_EP_EXCHANGE``, else ``"nccl"``.  ``logits`` overrides the router GEMM.  ``profile_events`` (three recorded
    ``torch.cuda.Event``) brackets GEMM1 and GEMM2 for kernel timing.
    ``residual`` (bf16 [T, H]) is added to the layer's fp32 result before the
    single rounding to bf16 (the decoder's residual add, fused).
    ``deterministic=True`` (single GPU) makes the result bit-reproducible run
    to run: each (token, expert) row is stored and the rows are summed per
    token in slot order (k routed experts, then the shared expert) instead of
    added with fp32 atomics, at the cost of writing and reading them once
    (R x H x 4 bytes of workspace, R = T*top_k (+T)).
    """
    if ep_group is not None:
        if residual is not None:
            raise ShapeError("residual is not supported with ep_group")
        if deterministic:
            raise ShapeError("deterministic is not supported with ep_group")
        from . import ep
        return ep.moe_ep(x, router_w, router_bias, w13, w13_scale, w2, w2_scale, shared_w13=shared_w13,
                         shared_w13_scale=shared_w13_scale, shared_w2=shared_w2, shared_w2_scale=shared_w2_scale,
                         n_group=n_group, topk_group=topk_group, top_k=top_k,
                         routed_scaling_factor=routed_scaling_factor, inter_planes=inter_planes,
                         logits=logits, group=ep_group, exchange=ep_exchange,
                         max_tokens_per_rank=max_tokens_per_rank)
    has_shared = shared_w13 is not None
    dev = _check_cuda(x, router_w, router_bias, w13, w13_scale, w2, w2_scale, shared_w13, shared_w13_scale,
                      shared_w2, shared_w2_scale, logits, residual)
    _req(x.dim() == 2 and x.dtype == torch.bfloat16, "x must be bf16 [T, H]")
    T, H = x.shape
    _req(w13.dim() == 3 and w13.shape[2] == H, "w13 must be [E, 2I, H]")
    E, twoI, _ = w13.shape
    I = twoI // 2
    _req(H % BLOCK == 0 and I % BLOCK == 0, "H and I must be multiples of 128")
    _req(router_w.shape == (E, H), "router_w must be [E, H]")
    _req(router_bias.shape[-1] == E, "router_bias must have E entries")
    _req(w13_scale.shape == (E, 2 * I // BLOCK, H // BLOCK), "w13_scale must be [E, 2I/128, H/128]")
    _req(w2.shape == (E, H, I) and w2_scale.shape == (E, H // BLOCK, I // BLOCK), "w2 / w2_scale shapes")
    _req(w13.dtype == torch.float8_e4m3fn and w2.dtype == torch.float8_e4m3fn, "weights must be e4m3")
    if has_shared:
        _req(shared_w13.shape == (2 * I, H) and shared_w2.shape == (H, I), "shared expert shapes")
        _req(shared_w13_scale.shape == (2 * I // BLOCK, H // BLOCK), "shared_w13_scale shape")
        _req(shared_w2_scale.shape == (H // BLOCK, I // BLOCK), "shared_w2_scale shape")
    _req(router_w.dtype == torch.float32, "router_w must be fp32")
    if logits is not None:
        _req(logits.shape == (T, E) and logits.dtype == torch.float32, "logits must be fp32 [T, E]")
    bias = router_bias
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    shape = GemmsMoeShape(T=T, H=H, I=I, E=E, E_local=E, local_expert_offset=0, n_group=n_group,
                          topk_group=topk_group, top_k=top_k, has_shared=int(has_shared),
                          input_mode=_lib.GEMMS_INPUT_BF16, bias_bf16=int(bias.dtype == torch.bfloat16),
                          inter_planes=inter_planes, routed_scaling_factor=float(routed_scaling_factor),
                          deterministic=int(deterministic))
    args = GemmsMoeArgs()
    args.routing_logits = _ptr(logits)  # None: the router GEMM runs inside gemms_moe_fwd
    args.router_w = _ptr(router_w)
    args.routing_bias = _ptr(bias)
    args.hidden_bf16 = _ptr(x)
    args.w13, args.w13_scale, args.w2, args.w2_scale = _ptr(w13), _ptr(w13_scale), _ptr(w2), _ptr(w2_scale)
    if has_shared:
        args.shared_w13, args.shared_w13_scale = _ptr(shared_w13), _ptr(shared_w13_scale)
        args.shared_w2, args.shared_w2_scale = _ptr(shared_w2), _ptr(shared_w2_scale)
    args.out = _ptr(out)
    if residual is not None:
        _req(residual.shape == (T, H) and residual.dtype == torch.bfloat16, "residual must be bf16 [T, H]")
        args.residual = _ptr(residual)
    idx = w = counts = None
    if return_routing:
        idx = torch.empty((T, top_k), dtype=torch.int32, device=dev)
        w = torch.empty((T, top_k), dtype=torch.float32, device=dev)
        counts = torch.empty((E,), dtype=torch.int32, device=dev)
        args.topk_idx_out, args.topk_w_out, args.expert_counts_out = _ptr(idx), _ptr(w), _ptr(counts)
        if logits is None:
            logits = torch.empty((T, E), dtype=torch.float32, device=dev)
            args.logits_out = _ptr(logits)
    ev_arr = None
    if profile_events is not None:
        ev_arr = (ctypes.c_void_p * 3)(*[e.cuda_event for e in profile_events])
        args.profile_events = ctypes.cast(ev_arr, ctypes.c_void_p)
    _call_fwd(shape, args, dev, "moe")
    del ev_arr
    if return_routing:
        return out, idx, w, counts, logits
    return out


@torch.no_grad()
@_on_tensor_device
def quantize_1x128(x: torch.Tensor):
    """Per-1x128 e4m3 quantisation of bf16 x [T, H] on the GPU
    (``gemms_quantize_1x128``): returns (xq float8_e4m3fn [T, H], scale fp32
    [H/128, T]) in the reference's ``hidden_states`` / ``hidden_states_scale``
    layouts, so the pair can be passed to :func:`run`."""
    dev = _check_cuda(x)
    _req(x.dim() == 2 and x.dtype == torch.bfloat16, "x must be bf16 [T, H]")
    T, H = x.shape
    _req(H % BLOCK == 0, "H must be a multiple of 128")
    xq = torch.empty((T, H), dtype=torch.float8_e4m3fn, device=dev)
    sc = torch.empty((H // BLOCK, T), dtype=torch.float32, device=dev)
    L = _lib.load()
    _lib.check(L.gemms_quantize_1x128(x.data_ptr(), T, H, xq.data_ptr(), sc.data_ptr(), _stream()),
               "gemms_quantize_1x128")
    return xq, sc


@torch.no_grad()
@_on_tensor_device
def rmsnorm_quant(h: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """DeepSeek-V3 RMSNorm fused with the per-1x128 quantisation
    (``gemms_rmsnorm_quant``): h bf16 [T, H] -> (y bf16 [T, H], xq e4m3
    [T, H], scale fp32 [H/128, T]), y = weight * bf16(h * rsqrt(mean(h^2) +
    eps)) rounded to bf16 and (xq, scale) its 1x128 quantisation."""
    dev = _check_cuda(h, weight)
    _req(h.dim() == 2 and h.dtype == torch.bfloat16, "h must be bf16 [T, H]")
    T, H = h.shape
    _req(H % BLOCK == 0, "H must be a multiple of 128")
    _req(weight.shape == (H,) and weight.dtype in (torch.bfloat16, torch.float32), "weight must be bf16/fp32 [H]")
    y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    xq = torch.empty((T, H), dtype=torch.float8_e4m3fn, device=dev)
    sc = torch.empty((H // BLOCK, T), dtype=torch.float32, device=dev)
    L = _lib.load()
    _lib.check(L.gemms_rmsnorm_quant(h.data_ptr(), weight.data_ptr(), int(weight.dtype == torch.bfloat16), float(eps),
                                     T, H, y.data_ptr(), xq.data_ptr(), sc.data_ptr(), _stream()),
               "gemms_rmsnorm_quant")
    return y, xq, sc


@torch.no_grad()
@_on_tensor_device
def moe_block(h: torch.Tensor, norm_weight: torch.Tensor, router_w: torch.Tensor, router_bias: torch.Tensor,
              w13: torch.Tensor, w13_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor, *,
              eps: float = 1e-6, shared_w13: torch.Tensor | None = None, shared_w13_scale: torch.Tensor | None = None,
              shared_w2: torch.Tensor | None = None, shared_w2_scale: torch.Tensor | None = None,
              n_group: int = 8, topk_group: int = 4, top_k: int = 8, routed_scaling_factor: float = 2.5,
              inter_planes: int = 2, deterministic: bool = False) -> torch.Tensor:
    """The MoE half of a DeepSeek-V3 decoder layer on the residual stream h
    (bf16 [T, H]): h + moe(rmsnorm(h)).  RMSNorm and the 1x128 quantisation
    run as one kernel whose e4m3 rows feed the experts directly (no second
    quantisation); the router GEMM reads the bf16 normalised rows; the
    residual add is fused into the layer's final cast (one rounding)."""
    dev = _check_cuda(h, norm_weight, router_w, router_bias, w13, w13_scale, w2, w2_scale, shared_w13,
                      shared_w13_scale, shared_w2, shared_w2_scale)
    y, xq, xq_scale = rmsnorm_quant(h, norm_weight, eps)
    logits = router_logits(y, router_w)
    T, H = h.shape
    E, twoI, _ = w13.shape
    I = twoI // 2
    _req(router_w.shape == (E, H) and router_bias.shape[-1] == E, "router_w / router_bias shapes")
    _req(w13.dtype == torch.float8_e4m3fn and w2.dtype == torch.float8_e4m3fn, "weights must be e4m3")
    _req(w2.shape == (E, H, I), "w2 must be [E, H, I]")
    has_shared = shared_w13 is not None
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    shape = GemmsMoeShape(T=T, H=H, I=I, E=E, E_local=E, local_expert_offset=0, n_group=n_group,
                          topk_group=topk_group, top_k=top_k, has_shared=int(has_shared),
                          input_mode=_lib.GEMMS_INPUT_FP8, bias_bf16=int(router_bias.dtype == torch.bfloat16),
                          inter_planes=inter_planes, routed_scaling_factor=float(routed_scaling_factor),
                          deterministic=int(deterministic))
    args = GemmsMoeArgs()
    args.routing_logits = _ptr(logits)
    args.routing_bias = _ptr(router_bias)
    args.hidden_fp8, args.hidden_scale = _ptr(xq), _ptr(xq_scale)
    args.w13, args.w13_scale, args.w2, args.w2_scale = _ptr(w13), _ptr(w13_scale), _ptr(w2), _ptr(w2_scale)
    if has_shared:
        args.shared_w13, args.shared_w13_scale = _ptr(shared_w13), _ptr(shared_w13_scale)
        args.shared_w2, args.shared_w2_scale = _ptr(shared_w2), _ptr(shared_w2_scale)
    args.out = _ptr(out)
    args.residual = _ptr(h)
    _call_fwd(shape, args, dev, "moe_block")
    return out


@torch.no_grad()
@_on_tensor_device
def route(logits: torch.Tensor, bias: torch.Tensor, *, n_group: int, topk_group: int, top_k: int,
          routed_scaling_factor: float = 2.5, counts: bool = True):
    """CUDA router only: returns (topk_idx int32 [T,k], topk_w fp32 [T,k], counts int32 [E])."""
    dev = _check_cuda(logits, bias)
    T, E = logits.shape
    _req(logits.dtype == torch.float32, "logits must be fp32")
    idx = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    w = torch.empty((T, top_k), dtype=torch.float32, device=dev)
    c = torch.zeros((E,), dtype=torch.int32, device=dev) if counts else None
    L = _lib.load()
    _lib.check(L.gemms_route(logits.data_ptr(), bias.data_ptr(), int(bias.dtype == torch.bfloat16), T, E, n_group,
                             topk_group, top_k, float(routed_scaling_factor), idx.data_ptr(), w.data_ptr(),
                             _ptr(c), _stream()), "gemms_route")
    return idx, w, c
