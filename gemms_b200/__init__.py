"""gemms_b200 -- B200-native (sm_100a) DeepSeek-V3 FP8 MoE layer.

Public operators (CUDA tensors only, no CPU fallback):

* :func:`run` -- drop-in for the reference operator ``run`` of
  plops655/GEMMS (``flashinfer_baseline.py:5-169``).
* :func:`moe` -- the full layer ``moe(x, router_w, router_bias, w13, w13_scale,
  w2, w2_scale, ...)``, optionally expert-parallel over a process group.
* :func:`route` -- the group-limited sigmoid top-k router alone.
* :func:`router_logits`, :func:`quantize_1x128` -- the router GEMM and the
  per-1x128 activation quantisation alone.
* :func:`rmsnorm_quant`, :func:`moe_block` -- the steps either side of the
  layer: RMSNorm fused with the quantisation, and h + moe(rmsnorm(h)) with
  the residual add fused into the layer's output cast.
* :class:`MoePipeline` -- host-to-host serving loop with PCIe copies overlapped.
* :class:`MoeGraph` -- one decode-sized layer call captured in a CUDA graph.
* ``torch.ops.gemms_b200.moe`` / ``torch.ops.gemms_b200.run`` -- the same layer
  as PyTorch dispatcher operators (after :func:`load_torch_ops`).
"""
from .ops import (ShapeError, check_device_errors, moe, moe_block, quantize_1x128, rmsnorm_quant, route,  # noqa: F401
                  router_logits, run)
from ._lib import GemmsError, lib_path, load as load_library, load_torch_ops  # noqa: F401
from . import workloads  # noqa: F401
from .pipeline import MoeGraph, MoePipeline  # noqa: F401

__all__ = ["run", "moe", "moe_block", "route", "router_logits", "quantize_1x128", "rmsnorm_quant", "ShapeError", "GemmsError", "check_device_errors",
           "load_library", "load_torch_ops", "lib_path", "workloads", "MoePipeline", "MoeGraph"]
__version__ = "0.1.0"
