"""ctypes wrapper of the reference's scalar C++ sub-step library -- TEST INFRASTRUCTURE ONLY.

``oracle/Makefile`` compiles the reference's own sources
(kernels/scalar/scalar.cpp, scalar_phase1_{1,2,3}.cpp, kernels/src/dispatch.cpp)
into ``oracle/_ref/libspider_ref_scalar.so``.  The tests use it to check the
oracle's sub-steps against code the reference ships:

* spider_router_f32 (scalar.cpp:7-34): softmax, repeated arg-max top-k, renormalise;
* spider_edge_topk_f32 (scalar_phase1_2.cpp:11-47): top-M + softmax per source;
* spider_edge_project_f32 (scalar_phase1_1.cpp:17-32): W_edge[e] . h for all e;
* spider_graph_message_passing_dynamic_f32 (scalar_phase1_2.cpp:49-72): the
  dynamic-graph message sum the PyTorch block computes;
* spider_loop_epilogue_f32 (scalar.cpp:75-92): h + a*delta + b*x0 then LayerNorm.

(The library's expert FFN uses tanh-GELU and its static-CSR graph differs from
the PyTorch block, so those two entry points are not used as checkers.)
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libspider_ref_scalar.so")

_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(LIB_PATH)
        fp, ip = C.POINTER(C.c_float), C.POINTER(C.c_int32)
        _lib.spider_router_f32.argtypes = [fp, fp, C.c_int, C.c_int, C.c_int, C.c_int, fp, ip]
        _lib.spider_edge_topk_f32.argtypes = [fp, C.c_int, C.c_int, C.c_int, ip, fp]
        _lib.spider_edge_project_f32.argtypes = [fp, C.c_int, C.c_int, C.c_int, fp, fp]
        _lib.spider_graph_message_passing_dynamic_f32.argtypes = [fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                                                  C.c_int, ip, fp, ip, fp]
        _lib.spider_loop_epilogue_f32.argtypes = [fp, fp, fp, C.c_int, C.c_int, C.c_float, C.c_float, fp, fp,
                                                  C.c_float, fp]
        for f in ("spider_router_f32", "spider_edge_topk_f32", "spider_edge_project_f32",
                  "spider_graph_message_passing_dynamic_f32", "spider_loop_epilogue_f32"):
            getattr(_lib, f).restype = C.c_int
    return _lib


def _f(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(C.POINTER(C.c_float))


def _i(a):
    a = np.ascontiguousarray(a, dtype=np.int32)
    return a, a.ctypes.data_as(C.POINTER(C.c_int32))


def router(logits, bias_table, loop_idx, k):
    b, e = logits.shape
    lg, plg = _f(logits)
    bt, pbt = _f(bias_table)
    w, pw = _f(np.zeros((b, k)))
    idx, pidx = _i(np.zeros((b, k)))
    rc = lib().spider_router_f32(plg, pbt, b, e, k, loop_idx, pw, pidx)
    return rc, w, idx


def edge_topk(edge_logits, m):
    b, e, _ = edge_logits.shape
    lg, plg = _f(edge_logits)
    idx, pidx = _i(np.zeros((b, e, m)))
    w, pw = _f(np.zeros((b, e, m)))
    rc = lib().spider_edge_topk_f32(plg, b, e, m, pidx, pw)
    return rc, idx, w


def edge_project(hidden, w_edge):
    b, h = hidden.shape
    e = w_edge.shape[0]
    hh, ph = _f(hidden)
    ww, pw = _f(w_edge)
    out, po = _f(np.zeros((b, e, h)))
    rc = lib().spider_edge_project_f32(ph, b, h, e, pw, po)
    return rc, out


def message_passing_dynamic(projected, edge_idx, edge_w, assign):
    b, e, h = projected.shape
    k = assign.shape[1]
    m = edge_idx.shape[2]
    pr, ppr = _f(projected)
    ei, pei = _i(edge_idx)
    ew, pew = _f(edge_w)
    asg, pasg = _i(assign)
    out, po = _f(np.zeros((b, h)))
    rc = lib().spider_graph_message_passing_dynamic_f32(ppr, b, h, e, k, m, pei, pew, pasg, po)
    return rc, out


def loop_epilogue(h, delta, x0, alpha, beta, gamma, ln_b, eps):
    b, hid = h.shape
    a1, p1 = _f(h)
    a2, p2 = _f(delta)
    a3, p3 = _f(x0)
    g, pg = _f(gamma)
    lb, plb = _f(ln_b)
    out, po = _f(np.zeros((b, hid)))
    rc = lib().spider_loop_epilogue_f32(p1, p2, p3, b, hid, alpha, beta, pg, plb, eps, po)
    return rc, out
