"""CPU: the C-ABI library loads and exports every symbol include/gemms_moe.h declares."""
import ctypes
import os
import re

import pytest

import gemms_b200
from gemms_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")


def declared_symbols():
    syms = set()
    for fn in os.listdir(HEADER):
        if fn.endswith(".h"):
            txt = open(os.path.join(HEADER, fn)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            syms |= set(re.findall(r"\b(gemms_[a-z0-9_]+)\s*\(", txt))
    return syms


def test_library_loads_and_exports_all_symbols():
    L = gemms_b200.load_library()
    syms = declared_symbols()
    assert "gemms_moe_fwd" in syms and len(syms) >= 8
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/ but not exported"
    assert set(_lib.EXPORTS) <= syms


def test_version_and_strerror():
    L = gemms_b200.load_library()
    assert b"sm_100a" in L.gemms_version()
    for code in range(0, -10, -1):
        assert L.gemms_strerror(code)
    assert L.gemms_strerror(-99) == b"unknown error"


def test_workspace_size_and_shape_rejection():
    L = gemms_b200.load_library()
    s = _lib.GemmsMoeShape(T=4096, H=7168, I=2048, E=256, E_local=256, n_group=8, topk_group=4, top_k=8,
                           has_shared=1, input_mode=0, inter_planes=2, routed_scaling_factor=2.5)
    n = L.gemms_moe_workspace_size(ctypes.byref(s))
    assert 200e6 < n < 700e6
    bad = _lib.GemmsMoeShape(**{f: getattr(s, f) for f, _ in _lib.GemmsMoeShape._fields_})
    bad.n_group = 7  # 256 % 7 != 0
    assert L.gemms_moe_workspace_size(ctypes.byref(bad)) == 0
    bad.n_group = 8
    bad.top_k = 17
    assert L.gemms_moe_workspace_size(ctypes.byref(bad)) == 0
    assert L.gemms_expert_ffn_workspace_size(1024, 7168, 2048, 32, 2) > 0
    assert L.gemms_expert_ffn_workspace_size(1024, 7000, 2048, 32, 2) == 0


def test_fwd_rejects_null_args_without_gpu():
    L = gemms_b200.load_library()
    assert L.gemms_moe_fwd(None, None, 0, None) == -8  # GEMMS_ERR_ARG


def test_operators_refuse_cpu_tensors():
    import torch
    x = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(gemms_b200.ShapeError):
        gemms_b200.moe(x, torch.zeros(8, 256), torch.zeros(8), torch.zeros(8, 256, 256).to(torch.float8_e4m3fn),
                       torch.ones(8, 2, 2), torch.zeros(8, 256, 128).to(torch.float8_e4m3fn), torch.ones(8, 2, 1),
                       n_group=4, topk_group=2, top_k=2)


def test_header_compiles_as_c_and_links(tmp_path):
    """include/gemms_moe.h is a C header: a C99 program that includes it links
    against the library and calls the host-only entry points (no GPU needed)."""
    import shutil
    import subprocess
    from gemms_b200 import build as B
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = tmp_path / "abi.c"
    src.write_text(r"""
#include <stdio.h>
#include <string.h>
#include "gemms_moe.h"
int main(void) {
  GemmsMoeShape s;
  memset(&s, 0, sizeof s);
  s.T = 4096; s.H = 7168; s.I = 2048; s.E = 256; s.E_local = 256; s.n_group = 8; s.topk_group = 4;
  s.top_k = 8; s.has_shared = 1; s.input_mode = GEMMS_INPUT_BF16; s.inter_planes = 2;
  s.routed_scaling_factor = 2.5f;
  size_t n = gemms_moe_workspace_size(&s);
  s.H = 7000;  /* not a multiple of 128: rejected */
  size_t bad = gemms_moe_workspace_size(&s);
  printf("%zu %zu %d\n%s\n", n, bad, gemms_moe_fwd(NULL, NULL, 0, NULL), gemms_version());
  return (n > 0 && bad == 0) ? 0 : 1;
}
""")
    exe = tmp_path / "abi"
    libdir = os.path.dirname(B.LIB)
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(root, "include"), str(src), "-o",
                        str(exe), "-L", libdir, "-lgemms_b200", "-Wl,-rpath," + libdir], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    n, bad, rc = out.stdout.splitlines()[0].split()
    assert int(n) > 0 and int(bad) == 0 and int(rc) == -8  # GEMMS_ERR_ARG for NULL args


def test_new_entry_points_validate_arguments_without_gpu():
    """Argument checks of the expert-parallel combine entry points and the GEMM
    grid bound run on the host, before any CUDA call."""
    L = _lib.load()
    ERR_SHAPE, ERR_ARG = -1, -8  # GEMMS_ERR_SHAPE, GEMMS_ERR_ARG
    assert L.gemms_ep_back_row_bytes(7168) == 2 * 7168 + 16
    assert L.gemms_ep_back_row_bytes(0) == 0
    assert L.gemms_ep_pack_back(None, 0, 7168, None, None) == 0            # nothing to pack
    assert L.gemms_ep_pack_back(None, 4, 7168, None, None) == ERR_ARG
    assert L.gemms_ep_pack_back(None, 4, 7166, None, None) == ERR_SHAPE
    bases = (ctypes.c_void_p * 2)(None, None)
    adds = (ctypes.c_int32 * 2)(0, 0)
    assert L.gemms_ep_combine_rows(None, bases, adds, None, 4, 7168, 2, None, None) == ERR_ARG
    assert L.gemms_ep_combine_rows(None, bases, adds, None, 4, 7168, 33, None, None) == ERR_SHAPE
    assert L.gemms_set_gemm_ctas(-1) == ERR_ARG
    prev = L.gemms_set_gemm_ctas(7)
    assert L.gemms_set_gemm_ctas(prev) == 7
    # device-driven exchange: region size = 256-byte count header + send rows
    rb = L.gemms_ep_row_bytes(7168, 8)
    assert L.gemms_ep_region_bytes(100, 7168, 8) == 256 + 100 * rb
    assert L.gemms_ep_region_bytes(-1, 7168, 8) == 0 and L.gemms_ep_region_bytes(1, 7100, 8) == 0
    info = ctypes.c_void_p(64)  # never dereferenced: every call below fails its host checks
    assert L.gemms_ep_pull(bases, 0, 2, 7168, 8, 10, 10, None, info, None) == ERR_ARG    # NULL region addresses
    assert L.gemms_ep_pull(bases, 2, 2, 7168, 8, 10, 10, None, info, None) == ERR_SHAPE  # rank >= world
    assert L.gemms_ep_pull(bases, 0, 33, 7168, 8, 10, 10, None, info, None) == ERR_SHAPE
    assert L.gemms_ep_pull(None, 0, 2, 7168, 8, 10, 10, None, None, None) == ERR_ARG
    assert L.gemms_ep_pack_back_dev(None, 4, None, 7168, None, None) == ERR_ARG
    assert L.gemms_ep_pack_back_dev(None, 0, None, 7168, None, None) == 0
    assert L.gemms_ep_combine_peer(None, bases, None, None, 4, 7168, 2, 8, None, None) == ERR_ARG
    assert L.gemms_ep_combine_peer(None, bases, info, None, 4, 7168, 33, 8, None, None) == ERR_SHAPE
    assert L.gemms_ep_combine_peer(None, bases, info, None, 4, 7168, 2, 0, None, None) == ERR_SHAPE
    assert L.gemms_ep_expert_ffn_dev(None, 4, None, 32, 7168, 2048, 8, 32, 0, 2, None, None, None, None, None,
                                     None, 0, None) == ERR_ARG
    assert L.gemms_ep_gather_add_peer(None, bases, info, None, 4, 7168, 2, 8, None) == ERR_ARG
    assert L.gemms_ep_gather_add_peer(None, bases, info, None, 4, 7168, 2, 0, None) == ERR_SHAPE
    assert L.gemms_f32_to_bf16(None, None, 6, None) == ERR_SHAPE
    assert L.gemms_f32_to_bf16(None, None, 0, None) == 0
    assert L.gemms_f32_to_bf16(None, None, 8, None) == ERR_ARG
    assert L.gemms_ep_set_pull_ctas(-1) == ERR_ARG
    prev = L.gemms_ep_set_pull_ctas(16)
    assert L.gemms_ep_set_pull_ctas(prev) == 16


def test_stall_hook_rejects_bad_arguments():
    """gemms_test_inject_stall validates its arguments on the host."""
    L = gemms_b200.load_library()
    assert L.gemms_test_inject_stall(3, 0, 0) == -8
    assert L.gemms_test_inject_stall(1, -1, 0) == -8
    assert L.gemms_test_inject_stall(1, 0, -5) == -8
    assert L.gemms_test_inject_stall(0, 0, 0) == 0


def test_noalloc_check_rejects_null_flags():
    L = gemms_b200.load_library()
    assert L.gemms_moe_check_noalloc(None, None) == -8
