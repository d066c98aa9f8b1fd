"""ctypes binding of the C ABI in ``include/gemms_moe.h``.

The shared library is ``gemms_b200/lib/libgemms_b200.so`` (built in-tree by
``gemms_b200.build``).  There is no fallback: if the library cannot be loaded
every operator raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

c_int32 = ctypes.c_int32
c_void_p = ctypes.c_void_p
c_size_t = ctypes.c_size_t
c_float = ctypes.c_float

GEMMS_INPUT_BF16 = 0
GEMMS_INPUT_FP8 = 1

EXPORTS = (
    "gemms_moe_workspace_size",
    "gemms_moe_fwd",
    "gemms_set_decode_max_t",
    "gemms_route",
    "gemms_expert_ffn_workspace_size",
    "gemms_expert_ffn",
    "gemms_moe_check",
    "gemms_strerror",
    "gemms_version",
    "gemms_ep_row_bytes",
    "gemms_ep_dispatch",
    "gemms_ep_ffn_workspace_size",
    "gemms_ep_expert_ffn",
    "gemms_ep_back_row_bytes",
    "gemms_ep_pack_back",
    "gemms_ep_combine",
    "gemms_ep_combine_rows",
    "gemms_ep_region_bytes",
    "gemms_ep_pull",
    "gemms_ep_expert_ffn_dev",
    "gemms_ep_pack_back_dev",
    "gemms_ep_combine_peer",
    "gemms_ep_set_pull_ctas",
    "gemms_ep_gather_add_peer",
    "gemms_f32_to_bf16",
    "gemms_set_gemm_ctas",
    "gemms_moe_fwd_noalloc",
    "gemms_moe_check_noalloc",
    "gemms_test_inject_stall",
    "gemms_test_workspace_regions",
    "gemms_router_workspace_size",
    "gemms_router_logits",
    "gemms_quantize_1x128",
    "gemms_rmsnorm_quant",
)


class GemmsMoeShape(ctypes.Structure):
    _fields_ = [
        ("T", c_int32), ("H", c_int32), ("I", c_int32), ("E", c_int32), ("E_local", c_int32),
        ("local_expert_offset", c_int32), ("n_group", c_int32), ("topk_group", c_int32), ("top_k", c_int32),
        ("has_shared", c_int32), ("input_mode", c_int32), ("bias_bf16", c_int32), ("inter_planes", c_int32),
        ("routed_scaling_factor", c_float), ("deterministic", c_int32),
    ]


class GemmsMoeArgs(ctypes.Structure):
    _fields_ = [
        ("shape", GemmsMoeShape),
        ("routing_logits", c_void_p), ("routing_bias", c_void_p),
        ("hidden_bf16", c_void_p), ("hidden_fp8", c_void_p), ("hidden_scale", c_void_p),
        ("w13", c_void_p), ("w13_scale", c_void_p), ("w2", c_void_p), ("w2_scale", c_void_p),
        ("shared_w13", c_void_p), ("shared_w13_scale", c_void_p), ("shared_w2", c_void_p),
        ("shared_w2_scale", c_void_p),
        ("out", c_void_p), ("topk_idx_out", c_void_p), ("topk_w_out", c_void_p), ("expert_counts_out", c_void_p),
        ("profile_events", c_void_p), ("router_w", c_void_p), ("logits_out", c_void_p), ("residual", c_void_p),
    ]


GEMMS_ERR_TIMEOUT = -5

# Bits of the device error word (GEMMS_FLAG_* in include/gemms_moe.h).
FLAG_PRODUCER_WAIT = 1 << 0
FLAG_MMA_WAIT = 1 << 1
FLAG_EPILOGUE_WAIT = 1 << 2
FLAG_BAD_EXPERT = 1 << 3
FLAG_ROW_OVERFLOW = 1 << 4


class GemmsError(RuntimeError):
    """A GEMMS_ERR_* code returned by the C ABI (``flags``: the device error
    word's bits when the code came from a device-side check)."""

    def __init__(self, code: int, where: str, flags: int = 0):
        self.code = code
        self.flags = flags
        extra = f", device error word 0x{flags:x}" if flags else ""
        super().__init__(f"{where} failed: {strerror(code)} (code {code}{extra})")


_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _build.LIB


def load(auto_build: bool = True) -> ctypes.CDLL:
    """Load (building first if needed and nvcc exists) the shared library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB
        if not os.path.exists(path) and auto_build:
            _build.build()
        if not os.path.exists(path):
            raise ImportError(f"gemms_b200 CUDA library missing: {path} (run `python -m gemms_b200.build`)")
        L = ctypes.CDLL(path)
        L.gemms_moe_workspace_size.argtypes = [ctypes.POINTER(GemmsMoeShape)]
        L.gemms_moe_workspace_size.restype = c_size_t
        L.gemms_moe_fwd.argtypes = [ctypes.POINTER(GemmsMoeArgs), c_void_p, c_size_t, c_void_p]
        L.gemms_moe_fwd.restype = c_int32
        L.gemms_route.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float,
                                  c_void_p, c_void_p, c_void_p, c_void_p]
        L.gemms_route.restype = c_int32
        L.gemms_expert_ffn_workspace_size.argtypes = [c_int32, c_int32, c_int32, c_int32, c_int32]
        L.gemms_expert_ffn_workspace_size.restype = c_size_t
        L.gemms_expert_ffn.argtypes = [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                       c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_size_t, c_void_p]
        L.gemms_expert_ffn.restype = c_int32
        L.gemms_moe_check.argtypes = [c_void_p, c_void_p, ctypes.POINTER(c_int32)]
        L.gemms_moe_check.restype = c_int32
        L.gemms_strerror.argtypes = [c_int32]
        L.gemms_strerror.restype = ctypes.c_char_p
        L.gemms_version.argtypes = []
        L.gemms_version.restype = ctypes.c_char_p
        L.gemms_ep_row_bytes.argtypes = [c_int32, c_int32]
        L.gemms_ep_row_bytes.restype = c_size_t
        L.gemms_ep_dispatch.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32,
                                        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
        L.gemms_ep_dispatch.restype = c_int32
        L.gemms_ep_ffn_workspace_size.argtypes = [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32]
        L.gemms_ep_ffn_workspace_size.restype = c_size_t
        L.gemms_ep_expert_ffn.argtypes = [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
                                          c_int32,
                                          c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                          c_void_p]
        L.gemms_ep_expert_ffn.restype = c_int32
        L.gemms_set_decode_max_t.argtypes = [c_int32]
        L.gemms_set_decode_max_t.restype = c_int32
        L.gemms_set_gemm_ctas.argtypes = [c_int32]
        L.gemms_set_gemm_ctas.restype = c_int32
        L.gemms_ep_back_row_bytes.argtypes = [c_int32]
        L.gemms_ep_back_row_bytes.restype = c_size_t
        L.gemms_ep_pack_back.argtypes = [c_void_p, c_int32, c_int32, c_void_p, c_void_p]
        L.gemms_ep_pack_back.restype = c_int32
        L.gemms_ep_combine.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p]
        L.gemms_ep_combine_rows.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                            c_void_p, c_void_p]
        L.gemms_ep_combine_rows.restype = c_int32
        L.gemms_ep_combine.restype = c_int32
        L.gemms_ep_region_bytes.argtypes = [c_int32, c_int32, c_int32]
        L.gemms_ep_region_bytes.restype = c_size_t
        L.gemms_ep_pull.argtypes = [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p,
                                    c_void_p, c_void_p]
        L.gemms_ep_pull.restype = c_int32
        L.gemms_ep_expert_ffn_dev.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                              c_int32, c_int32, c_int32,
                                              c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                              c_void_p]
        L.gemms_ep_expert_ffn_dev.restype = c_int32
        L.gemms_ep_pack_back_dev.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_void_p]
        L.gemms_ep_pack_back_dev.restype = c_int32
        L.gemms_ep_combine_peer.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                            c_int32, c_void_p, c_void_p]
        L.gemms_ep_combine_peer.restype = c_int32
        L.gemms_ep_gather_add_peer.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                               c_int32, c_void_p]
        L.gemms_ep_gather_add_peer.restype = c_int32
        L.gemms_f32_to_bf16.argtypes = [c_void_p, c_void_p, c_size_t, c_void_p]
        L.gemms_f32_to_bf16.restype = c_int32
        L.gemms_ep_set_pull_ctas.argtypes = [c_int32]
        L.gemms_ep_set_pull_ctas.restype = c_int32
        L.gemms_moe_fwd_noalloc.argtypes = [ctypes.POINTER(GemmsMoeArgs), c_void_p]
        L.gemms_moe_fwd_noalloc.restype = c_int32
        L.gemms_moe_check_noalloc.argtypes = [c_void_p, ctypes.POINTER(c_int32)]
        L.gemms_moe_check_noalloc.restype = c_int32
        L.gemms_test_inject_stall.argtypes = [c_int32, c_int32, ctypes.c_int64]
        L.gemms_test_inject_stall.restype = c_int32
        L.gemms_test_workspace_regions.argtypes = [ctypes.POINTER(GemmsMoeShape), ctypes.POINTER(c_size_t),
                                                   ctypes.POINTER(c_size_t), ctypes.POINTER(c_int32),
                                                   ctypes.POINTER(c_size_t), ctypes.POINTER(c_size_t)]
        L.gemms_test_workspace_regions.restype = c_int32
        L.gemms_router_workspace_size.argtypes = [c_int32, c_int32, c_int32]
        L.gemms_router_workspace_size.restype = c_size_t
        L.gemms_router_logits.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p,
                                          c_size_t, c_void_p]
        L.gemms_router_logits.restype = c_int32
        L.gemms_quantize_1x128.argtypes = [c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p]
        L.gemms_quantize_1x128.restype = c_int32
        L.gemms_rmsnorm_quant.argtypes = [c_void_p, c_void_p, c_int32, c_float, c_int32, c_int32, c_void_p, c_void_p,
                                          c_void_p, c_void_p]
        L.gemms_rmsnorm_quant.restype = c_int32
        _lib = L
        return L


_torch_ops_loaded = False


def load_torch_ops(auto_build: bool = True) -> None:
    """Registers ``torch.ops.gemms_b200.moe`` and ``torch.ops.gemms_b200.run``
    (``gemms_b200/lib/libgemms_torch.so``, PyTorch dispatcher operators over
    the same C ABI).  The C-ABI library is loaded first, so both share one
    copy of it."""
    global _torch_ops_loaded
    if _torch_ops_loaded:
        return
    load(auto_build)
    path = _build.TORCH_LIB
    if not os.path.exists(path) and auto_build:
        _build.build_torch_ops()
    if not os.path.exists(path):
        raise ImportError(f"gemms_b200 torch operator library missing: {path} (run `python -m gemms_b200.build`)")
    import torch
    torch.ops.load_library(path)
    _torch_ops_loaded = True


def strerror(code: int) -> str:
    try:
        return load(auto_build=False).gemms_strerror(code).decode()
    except Exception:  # library itself unavailable
        return f"error {code}"


def check(code: int, where: str) -> None:
    if code != 0:
        raise GemmsError(code, where)
