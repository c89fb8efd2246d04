"""Token dispatch / combine with the reference Forge EP API (spider_infer/forge/ep/).

Drop-in for ``build_dispatch_plan``, ``dispatch_tokens``, ``combine_tokens``,
``combine_across_ranks``, ``dispatch_expert_ffn`` (dispatch.py:56-186) and the
``ForgeEP`` / ``DeepEPStyleDispatcher`` front end (api.py:21-130), on CUDA
tensors:

* the plan is built on the device by ``sb_group`` (experts ascending, each
  expert's token positions ascending, weights of repeated slots summed in slot
  order, tokens with summed weight <= 0 dropped -- the reference's
  ``tw = sum_k w_k [idx_k == e]; active = tw > 0``), and kept in packed form
  (``offsets``, ``rows``, ``row_weights``) next to the per-expert
  ``ExpertAssignment`` views of the reference;
* ``dispatch_tokens`` gathers an assignment's rows with ``sb_gather_rows``;
* ``dispatch_expert_ffn`` without an ``expert_fn`` is the fused path of
  ``sparse_expert_delta`` (device plan, grouped GEMMs, deterministic combine)
  followed by the cross-rank SUM; with an ``expert_fn`` it loops over the
  device plan's assignments as the reference does.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from . import _lib as L
from .expert_parallel import all_reduce_sum_, ep_enabled, get_rank_world, owns_expert
from .sparse_experts import sparse_expert_delta

LAST_EP_DISPATCH_BACKEND = "not_run"


@dataclass
class ExpertAssignment:
    expert_id: int
    token_index: torch.Tensor  # [n] int64 flat positions
    weights: torch.Tensor      # [n] routing weights for this expert


@dataclass
class DispatchPlan:
    """Per-step dispatch layout (reference fields plus the packed device form)."""

    batch: int
    seq: int
    hidden: int
    top_k: int
    num_experts: int
    assignments: list[ExpertAssignment] = field(default_factory=list)
    local_expert_ids: list[int] = field(default_factory=list)
    offsets: torch.Tensor | None = None      # [E+1] int32: expert e's rows are offsets[e]:offsets[e+1]
    rows: torch.Tensor | None = None         # [P] int32 token positions, expert-major
    row_weights: torch.Tensor | None = None  # [P] fp32 summed routing weights

    def tokens_for(self, expert_id: int) -> ExpertAssignment | None:
        for a in self.assignments:
            if a.expert_id == expert_id:
                return a
        return None


def _stream(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _device_plan(flat_idx: torch.Tensor, flat_w: torch.Tensor, num_experts: int):
    """sb_group over [N, K] routing -> (offsets int32 [E+1], rows int32 [P], weights fp32 [P])."""
    lib = L.load()
    dev = flat_idx.device
    n, k = flat_idx.shape
    idx = flat_idx.to(torch.int32).contiguous()
    w = flat_w.to(torch.float32).contiguous()
    cap = n * k
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    rows = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    slots = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    pw = torch.empty(max(cap, 1), dtype=torch.float32, device=dev)
    inv = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    ws = torch.empty(lib.sb_group_workspace_bytes(n, k, num_experts), dtype=torch.uint8, device=dev)
    L.check(lib.sb_group(idx.data_ptr(), w.data_ptr(), n, k, num_experts, L.SB_GROUP_POSITIVE_ONLY,
                         offsets.data_ptr(), rows.data_ptr(), slots.data_ptr(), pw.data_ptr(), inv.data_ptr(),
                         ws.data_ptr(), ws.numel(), _stream(idx)), "sb_group")
    return offsets, rows, pw


def build_dispatch_plan(top_indices: torch.Tensor, top_weights: torch.Tensor, *, num_experts: int,
                        local_only: bool = True) -> DispatchPlan:
    """Packed assignments from router outputs; top_indices / top_weights [B,T,K] or [N,K]."""
    global LAST_EP_DISPATCH_BACKEND
    if top_indices.ndim == 3:
        b, t, k = top_indices.shape
    elif top_indices.ndim == 2:
        n, k = top_indices.shape
        b, t = n, 1
    else:
        raise ValueError("top_indices must be [B,T,K] or [N,K]")
    if not top_indices.is_cuda:
        raise RuntimeError("spider_b200 build_dispatch_plan runs on CUDA tensors only")
    flat_idx = top_indices.reshape(-1, k)
    flat_w = top_weights.reshape(-1, k)
    rank, world = get_rank_world()
    if local_only and ep_enabled():
        local_ids = [e for e in range(num_experts) if owns_expert(e, rank, world)]
    else:
        local_ids = list(range(num_experts))
    offsets, rows, pw = _device_plan(flat_idx, flat_w, num_experts)
    host_off = offsets.cpu().tolist()
    assignments = []
    wdtype = top_weights.dtype
    for eid in local_ids:
        lo, hi = host_off[eid], host_off[eid + 1]
        if hi > lo:
            assignments.append(ExpertAssignment(expert_id=int(eid), token_index=rows[lo:hi].long(),
                                                weights=pw[lo:hi].to(wdtype)))
    LAST_EP_DISPATCH_BACKEND = "dispatch_plan_b200"
    return DispatchPlan(batch=b, seq=t, hidden=0, top_k=k, num_experts=num_experts, assignments=assignments,
                        local_expert_ids=local_ids, offsets=offsets, rows=rows[:host_off[-1]],
                        row_weights=pw[:host_off[-1]])


def dispatch_tokens(messages: torch.Tensor, assignment: ExpertAssignment) -> torch.Tensor:
    """Gather one expert's packed tokens; messages [B,T,H] or [N,H] (fp32 or bf16)."""
    flat = messages.reshape(-1, messages.shape[-1]).contiguous()
    n = assignment.token_index.numel()
    hdim = flat.shape[-1]
    out = torch.empty(n, hdim, dtype=flat.dtype, device=flat.device)
    if n == 0:
        return out
    if flat.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("dispatch_tokens takes fp32 or bf16 messages")
    lib = L.load()
    rows = assignment.token_index.to(torch.int32).contiguous()
    off = torch.tensor([0, n], dtype=torch.int32, device=flat.device)
    dt = L.SB_F32 if flat.dtype == torch.float32 else L.SB_BF16
    L.check(lib.sb_gather_rows(flat.data_ptr(), dt, hdim, rows.data_ptr(), off.data_ptr(), 1, n, out.data_ptr(),
                               _stream(flat)), "sb_gather_rows")
    return out


def combine_tokens(delta_flat: torch.Tensor, assignment: ExpertAssignment, expert_out: torch.Tensor) -> None:
    """Scatter-add weighted expert outputs into the flat delta (in place)."""
    weighted = expert_out * assignment.weights.unsqueeze(-1).to(expert_out.dtype)
    delta_flat.index_add_(0, assignment.token_index, weighted)


def combine_across_ranks(delta: torch.Tensor) -> torch.Tensor:
    """Cross-rank SUM of the delta (NCCL all-reduce when expert parallel is active)."""
    if ep_enabled():
        all_reduce_sum_(delta)
    return delta


@torch.no_grad()
def dispatch_expert_ffn(messages: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor, *,
                        w_up: torch.Tensor, b_up: torch.Tensor, w_down: torch.Tensor, b_down: torch.Tensor,
                        num_experts: int, expert_fn: Callable | None = None) -> torch.Tensor:
    """dispatch -> local expert FFN (Linear, erf-GELU, Linear) -> combine (+ cross-rank).

    w_up [E,U,H], b_up [E,U], w_down [E,H,U], b_down [E,H], messages [B,T,H] -> delta [B,T,H].
    """
    global LAST_EP_DISPATCH_BACKEND
    if not messages.is_cuda:
        raise RuntimeError("spider_b200 dispatch_expert_ffn runs on CUDA tensors only")
    b, t, h = messages.shape
    k = top_indices.shape[-1]
    if expert_fn is None:
        delta = sparse_expert_delta(messages, top_indices, top_weights, w_up, b_up, w_down, b_down,
                                    num_experts, k, expert_parallel=True)
        LAST_EP_DISPATCH_BACKEND = "dispatch_ffn_b200"
        return delta
    plan = build_dispatch_plan(top_indices, top_weights, num_experts=num_experts, local_only=True)
    plan.hidden = h
    delta_flat = messages.reshape(-1, h).new_zeros(b * t, h)
    for asg in plan.assignments:
        out = expert_fn(asg.expert_id, dispatch_tokens(messages, asg))
        combine_tokens(delta_flat, asg, out)
    delta = delta_flat.view(b, t, h)
    combine_across_ranks(delta)
    LAST_EP_DISPATCH_BACKEND = "dispatch_ffn_b200_expert_fn"
    return delta


def get_last_ep_dispatch_backend() -> str:
    return LAST_EP_DISPATCH_BACKEND


class ForgeEP:
    """Token dispatch + combine across expert-parallel ranks (api.py:21-126).

    ``config`` needs ``ep_enabled`` (and optionally ``ep_async``); ``backend``
    anything with a ``value`` (the reference passes its ForgeConfig,
    ForgeDevice and ForgeBackend)."""

    def __init__(self, config: Any = None, device: Any = None, backend: Any = None):
        self.config = config
        self.device = device
        self.backend = backend
        self.calls = 0
        self._impl = "dispatch_combine_b200"

    def enabled(self) -> bool:
        return bool(getattr(self.config, "ep_enabled", True)) and ep_enabled()

    def rank_world(self) -> tuple[int, int]:
        return get_rank_world()

    def owns(self, expert_id: int) -> bool:
        rank, world = self.rank_world()
        return owns_expert(expert_id, rank, world)

    def combine(self, delta: torch.Tensor) -> torch.Tensor:
        self.calls += 1
        return combine_across_ranks(delta)

    def dispatch_meta(self, top_indices: torch.Tensor, num_experts: int) -> dict:
        self.calls += 1
        plan = build_dispatch_plan(top_indices, torch.ones_like(top_indices, dtype=torch.float32),
                                   num_experts=num_experts, local_only=True)
        rank, world = self.rank_world()
        return {"rank": rank, "world": world, "local_experts": plan.local_expert_ids,
                "assignments": len(plan.assignments), "top_indices_shape": list(top_indices.shape)}

    def dispatch_plan(self, top_indices: torch.Tensor, top_weights: torch.Tensor, num_experts: int) -> DispatchPlan:
        self.calls += 1
        return build_dispatch_plan(top_indices, top_weights, num_experts=num_experts, local_only=True)

    def run_dispatched_ffn(self, messages: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor, *,
                           w_up: torch.Tensor, b_up: torch.Tensor, w_down: torch.Tensor, b_down: torch.Tensor,
                           num_experts: int, expert_fn: Callable | None = None) -> torch.Tensor:
        self.calls += 1
        return dispatch_expert_ffn(messages, top_indices, top_weights, w_up=w_up, b_up=b_up, w_down=w_down,
                                   b_down=b_down, num_experts=num_experts, expert_fn=expert_fn)

    def stats(self) -> dict[str, Any]:
        rank, world = self.rank_world()
        backend = getattr(self.backend, "value", self.backend)
        return {"pillar": "ep", "analogue": "DeepEP", "impl": self._impl, "backend": backend,
                "last_kernel": get_last_ep_dispatch_backend(), "calls": self.calls,
                "dist_initialized": ep_enabled(), "rank": rank, "world": world,
                "async": bool(getattr(self.config, "ep_async", False)), "forge_version_target": "0.4"}


class DeepEPStyleDispatcher(ForgeEP):
    """Named alias for the DeepEP role (api.py:129-131)."""
