"""The C ABI library loads without a GPU and exports what include/spider_b200.h declares.

No compute call is made here: only argument validation paths that return
before touching a device.
"""
import ctypes as C
import os
import re

import pytest
import torch

from spider_web_moe_b200 import _lib as L

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "spider_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"SB_API\s+[\w\s\*]+?\b(sb_\w+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    syms = declared_symbols()
    assert len(syms) >= 15
    assert set(syms) == set(L.SIGNATURES), set(syms) ^ set(L.SIGNATURES)


def test_library_loads_and_exports_every_symbol():
    lib = L.load()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert b"sm_100a" in lib.sb_version()
    assert lib.sb_capabilities() & 1
    assert lib.sb_error_string(L.SB_ERR_WORKSPACE).decode().startswith("workspace")


def test_argument_validation_without_device():
    lib = L.load()
    # null pointers / bad sizes are rejected before any launch (reference code 1)
    assert lib.sb_router(None, L.SB_BF16, 4, 64, None, None, 4, 2, None, None, None, None) == L.SB_ERR_ARG
    assert lib.sb_router(None, L.SB_BF16, 0, 63, None, None, 4, 2, None, None, None, None) == L.SB_ERR_ARG
    assert lib.sb_group(None, None, 4, 2, 0, 0, None, None, None, None, None, None, 0, None) == L.SB_ERR_ARG
    assert lib.sb_grouped_gemm(None, None) == L.SB_ERR_ARG
    a = L.GemmArgs()
    assert lib.sb_grouped_gemm(C.byref(a), None) == L.SB_ERR_ARG
    d = L.BlockDims(hidden=60, num_experts=4, top_k=2, edges_per_expert=2, ffn=128, num_loops=2)
    assert lib.sb_block_workspace_bytes(C.byref(d)) == 0  # hidden not a multiple of 8
    d.hidden = 64
    d.top_k = 5  # routing needs top_k <= num_experts: rejected before any launch
    wts = L.BlockWeights()
    assert lib.sb_block_forward(C.byref(d), C.byref(wts), None, None, None, 4, 0, 1, None, 0, None, None) == L.SB_ERR_ARG
    d.top_k = 2
    d.max_tokens = 64
    assert lib.sb_block_workspace_bytes(C.byref(d)) > 0
    # workspace too small is reported, not written
    assert lib.sb_group_workspace_bytes(10, 2, 4) > 0


def test_workspace_grows_with_tokens():
    lib = L.load()
    d = L.BlockDims(hidden=1024, num_experts=16, top_k=2, edges_per_expert=2, ffn=2048, num_loops=6,
                    act_dtype=L.SB_BF16, wfmt=L.SB_W_BF16, max_tokens=64)
    small = lib.sb_block_workspace_bytes(C.byref(d))
    d.max_tokens = 8192
    big = lib.sb_block_workspace_bytes(C.byref(d))
    assert big > small > 0


def test_product_path_refuses_cpu_tensors():
    from spider_web_moe_b200.config import ModelConfig
    from spider_web_moe_b200.layer import SpiderMoELayer
    from spider_web_moe_b200.sparse_experts import sparse_expert_delta

    cfg = ModelConfig(hidden_size=64, num_heads=4, num_experts=4, top_k=2, edges_per_expert=2, num_loops=2,
                      expert_ffn_size=128)
    layer = SpiderMoELayer(cfg)
    h = torch.randn(1, 4, 64)
    with pytest.raises(RuntimeError):
        layer(h, h, 0)
    with pytest.raises(RuntimeError):
        sparse_expert_delta(h, torch.zeros(1, 4, 2, dtype=torch.long), torch.ones(1, 4, 2),
                            torch.zeros(4, 8, 64), torch.zeros(4, 8), torch.zeros(4, 64, 8), torch.zeros(4, 64), 4, 2)
    from spider_web_moe_b200 import forge_ep
    with pytest.raises(RuntimeError):
        forge_ep.build_dispatch_plan(torch.zeros(1, 4, 2, dtype=torch.long), torch.ones(1, 4, 2), num_experts=4)
    with pytest.raises(RuntimeError):
        forge_ep.ForgeEP().run_dispatched_ffn(h, torch.zeros(1, 4, 2, dtype=torch.long), torch.ones(1, 4, 2),
                                              w_up=torch.zeros(4, 8, 64), b_up=torch.zeros(4, 8),
                                              w_down=torch.zeros(4, 64, 8), b_down=torch.zeros(4, 64), num_experts=4)


def test_header_is_plain_c():
    """The header compiles as C99 on its own: a cgo / C caller can include it."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("no gcc")
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-x", "c", HEADER],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_new_entry_points_validate_without_device():
    lib = L.load()
    d = L.BlockDims(hidden=64, num_experts=8, top_k=2, edges_per_expert=2, ffn=64, num_loops=2,
                    act_dtype=L.SB_F32, wfmt=L.SB_W_F32, max_tokens=16)
    wts = L.BlockWeights()
    assert lib.sb_loop_stats_workspace_bytes(C.byref(d), 16) > 0
    assert lib.sb_loop_stats(C.byref(d), C.byref(wts), 0, None, None, None, 4, None, None, None, None, None, None,
                             0, None) == L.SB_ERR_ARG
    # confidence without h_out is rejected
    assert lib.sb_active_set_step(L.SB_F32, 4, 1, 63, None, None, None, None, None, 0.5, None, None, None, None,
                                  None, None, None, None) == L.SB_ERR_ARG
    assert lib.sb_active_set_step(L.SB_F32, 4, 1, 64, None, None, None, None, None, 0.5, None, None, None, None,
                                  None, None, None, None) == L.SB_ERR_ARG
    assert lib.sb_lumen_workspace_bytes(16, 64, 4, 16) > 0
    assert lib.sb_lumen_workspace_bytes(16, 64, 0, 16) == 0
    lw = L.LumenWeights()
    assert lib.sb_lumen_forward(L.SB_F32, 0, 4, 64, 33, 16, C.byref(lw), None, None, None, None, None, None, None,
                                0, None) == L.SB_ERR_ARG   # more than 32 slots
    assert lib.sb_active_experts(None, None, 4, 2, 8, None, None) == L.SB_ERR_ARG
    assert lib.sb_remap_routes(None, None, 4, 2, None, 8, None, None, None) == L.SB_ERR_ARG
