"""ctypes binding of libspider_b200.so (the C ABI declared in include/spider_b200.h).

Loading fails loudly: there is no CPU fallback behind this package.  The
library is looked up in-tree (``spider_web_moe_b200/lib``), or at the path in
``SPIDER_B200_LIB``.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

SB_OK = 0
SB_ERR_ARG = 1
SB_ERR_INDEX = 2
SB_ERR_UNSUPPORTED = 3
SB_ERR_NO_DEVICE = 4
SB_ERR_WORKSPACE = 5
SB_ERR_DEVICE_STATUS = 6

# device status word bits (SB_DEVERR_* in include/spider_b200.h)
SB_DEVERR_TMA_WAIT, SB_DEVERR_MMA_WAIT, SB_DEVERR_CONV_WAIT, SB_DEVERR_EPI_WAIT = 1, 2, 4, 8
SB_DEVERR_BAD_INDEX, SB_DEVERR_DRAIN, SB_DEVERR_PEER_WAIT = 16, 32, 64

SB_F32, SB_BF16 = 0, 1
SB_W_F32, SB_W_BF16, SB_W_FP8, SB_W_INT4 = 0, 1, 2, 3
SB_ACT_GELU, SB_ACT_SWIGLU = 0, 1
SB_EPI_LINEAR, SB_EPI_GELU, SB_EPI_SWIGLU, SB_EPI_SWIGLU_IL = 0, 1, 2, 3
SB_ENGINE_AUTO, SB_ENGINE_SIMT, SB_ENGINE_TCGEN05 = 0, 1, 2
SB_GROUP_POSITIVE_ONLY = 1

ENGINES = {"auto": SB_ENGINE_AUTO, "simt": SB_ENGINE_SIMT, "tcgen05": SB_ENGINE_TCGEN05}

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
f32 = C.c_float
sz = C.c_size_t


class GemmArgs(C.Structure):
    _fields_ = [
        ("engine", i32), ("wfmt", i32), ("act_dtype", i32), ("epilogue", i32),
        ("num_groups", i32), ("m_rows", i32), ("k", i32), ("group_size", i32),
        ("a_group_rows", i64), ("lda", i64), ("a_rows_total", i64),
        ("a", vp), ("a_scale", vp), ("a_gate", vp), ("a_gate_scale", vp),
        ("bias", vp), ("bias_gate", vp), ("bias_group_stride", i64),
        ("x", vp), ("ldx", i64), ("x_row_index", vp), ("x_rows", i32), ("max_rows", i32), ("rows_hint", i32),
        ("group_rows_bound", i32),
        ("offsets", vp), ("row_scale", vp), ("out", vp), ("ldo", i64),
        ("splits", i32), ("split_stride", i64), ("status", vp),
    ]


class BlockDims(C.Structure):
    _fields_ = [
        ("hidden", i32), ("num_experts", i32), ("top_k", i32), ("edges_per_expert", i32),
        ("ffn", i32), ("num_loops", i32), ("act_dtype", i32), ("wfmt", i32),
        ("activation", i32), ("group_size", i32), ("engine", i32), ("max_tokens", i32),
        ("residual_scale", f32), ("reinject", f32), ("ln_eps", f32),
    ]


class BlockWeights(C.Structure):
    _fields_ = [
        ("router_w", vp), ("loop_bias", vp), ("gen_w", vp), ("gen_bias", vp), ("edge_w", vp),
        ("w_up", vp), ("s_up", vp), ("b_up", vp),
        ("w_gate", vp), ("s_gate", vp), ("b_gate", vp),
        ("w_down", vp), ("s_down", vp), ("b_down", vp),
        ("ln_w", vp), ("ln_b", vp), ("route_w", vp),
    ]


class LumenWeights(C.Structure):
    _fields_ = [
        ("wqv", vp), ("qv_bias", vp), ("w_o", vp), ("gate_w", vp), ("gate_b", vp), ("ln_w", vp), ("ln_b", vp),
        ("ln_eps", C.c_float),
    ]


class BlockTaps(C.Structure):
    _fields_ = [
        ("top_idx", vp), ("top_w", vp), ("edge_idx", vp), ("edge_w", vp), ("messages", vp),
        ("delta", vp), ("ffn_offsets", vp), ("ffn_rows", vp), ("ffn_weights", vp),
    ]


# name -> (restype, argtypes); every symbol the header declares.
SIGNATURES = {
    "sb_capabilities": (i32, []),
    "sb_version": (C.c_char_p, []),
    "sb_error_string": (C.c_char_p, [i32]),
    "sb_router": (i32, [vp, i32, i32, i32, vp, vp, i32, i32, vp, vp, vp, vp]),
    "sb_group_workspace_bytes": (sz, [i32, i32, i32]),
    "sb_group": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, sz, vp]),
    "sb_group_noalloc": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]),
    "sb_gather_rows": (i32, [vp, i32, i32, vp, vp, i32, i32, vp, vp]),
    "sb_grouped_gemm": (i32, [C.POINTER(GemmArgs), vp]),
    "sb_edge_topm": (i32, [vp, i64, i32, i32, vp, vp, i32, i32, vp, vp, vp]),
    "sb_combine_rows": (i32, [vp, i64, i32, i64, vp, i32, i32, i32, vp, vp, i32, vp, i32, vp]),
    "sb_combine_ln": (i32, [vp, i64, i32, i64, vp, i32, vp, vp, vp, i32, i32, i32, vp, vp,
                            f32, f32, f32, vp, vp, vp]),
    "sb_block_workspace_bytes": (sz, [C.POINTER(BlockDims)]),
    "sb_block_forward": (i32, [C.POINTER(BlockDims), C.POINTER(BlockWeights), vp, vp, vp, i32, i32,
                               i32, vp, sz, C.POINTER(BlockTaps), vp]),
    "sb_loop_stats_workspace_bytes": (sz, [C.POINTER(BlockDims), i32]),
    "sb_loop_stats": (i32, [C.POINTER(BlockDims), C.POINTER(BlockWeights), i32, vp, vp, vp, i32, vp, vp, vp, vp,
                            vp, vp, sz, vp]),
    "sb_active_set_step": (i32, [i32, i32, i32, i32, vp, vp, vp, vp, vp, f32, vp, vp, vp, vp, vp, vp, vp, vp]),
    "sb_lumen_workspace_bytes": (sz, [i32, i32, i32, i32]),
    "sb_lumen_forward": (i32, [i32, i32, i32, i32, i32, i32, C.POINTER(LumenWeights), vp, vp, vp, vp, vp, vp, vp,
                               sz, vp]),
    "sb_active_experts": (i32, [vp, vp, i32, i32, i32, vp, vp]),
    "sb_remap_routes": (i32, [vp, vp, i32, i32, vp, i32, vp, vp, vp]),
    "sb_expert_delta_workspace_bytes": (sz, [C.POINTER(BlockDims), i32]),
    "sb_expert_delta": (i32, [C.POINTER(BlockDims), C.POINTER(BlockWeights), vp, vp, vp, i32, i32,
                              i32, vp, vp, sz, vp]),
    "sb_block_route": (i32, [C.POINTER(BlockDims), C.POINTER(BlockWeights), vp, i32, i32, vp, vp, vp, vp, vp, sz,
                             vp]),
    "sb_ep_row_pitch": (sz, [i32, i32, i32]),
    "sb_ep_pack_workspace_bytes": (sz, [i32, i32, i32]),
    "sb_ep_pack": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, sz, vp]),
    "sb_expert_rows_workspace_bytes": (sz, [C.POINTER(BlockDims), i32]),
    "sb_expert_rows": (i32, [C.POINTER(BlockDims), C.POINTER(BlockWeights), vp, i64, i32, i32, vp, vp, sz, vp]),
    "sb_status_offset": (sz, []),
    "sb_num_stages": (i32, []),
    "sb_stage_name": (C.c_char_p, [i32]),
    "sb_stage_timing": (i32, [i32]),
    "sb_stage_timing_read": (i32, [C.POINTER(C.c_double), C.POINTER(i32), i32]),
    "sb_kernel_launches": (C.c_ulonglong, []),
    "sb_ep_peer_region_bytes": (sz, [i32, i32, i64, i32]),
    "sb_ep_peer_create": (i32, [i32, i32, i64, i32, C.POINTER(vp), vp]),
    "sb_ep_peer_map": (i32, [vp, C.POINTER(vp)]),
    "sb_ep_peer_unmap": (i32, [vp]),
    "sb_ep_peer_destroy": (i32, [vp]),
    "sb_ep_dispatch": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, sz, vp]),
    "sb_ep_wait": (i32, [vp, i32, i32, i64, i32, i32, vp, vp]),
    "sb_ep_return": (i32, [vp, i32, i32, i32, i64, i32, vp, vp]),
    "sb_expert_rows_peer": (i32, [C.POINTER(BlockDims), C.POINTER(BlockWeights), vp, vp, i32, i32, i32, i64, i32, vp,
                                  vp, sz, vp]),
    "sb_ep_epilogue_peer": (i32, [vp, i32, i32, i64, vp, i32, vp, vp, i32, i32, i32, vp, vp, f32, f32, f32, vp, vp,
                                  vp]),
}


class SpiderB200Error(RuntimeError):
    def __init__(self, code: int, where: str = ""):
        self.code = code
        msg = error_string(code) if _LIB is not None else str(code)
        super().__init__(f"{where}: spider_b200 error {code} ({msg})")


_LIB = None


def lib_path() -> str:
    return os.environ.get("SPIDER_B200_LIB") or _build.lib_path()


def load(build_if_missing: bool = False):
    """Load the library once; raise if it is absent (no silent fallback)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = lib_path()
    if not os.path.exists(path):
        if build_if_missing:
            _build.build()
        else:
            raise RuntimeError(
                f"libspider_b200.so not found at {path}; run `python -m spider_web_moe_b200.build`")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def error_string(code: int) -> str:
    return load().sb_error_string(int(code)).decode()


def check(rc: int, where: str = "") -> None:
    if rc != SB_OK:
        raise SpiderB200Error(rc, where)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    if t is None:
        return None
    return t.data_ptr()
