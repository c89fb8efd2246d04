"""Drop-in ``sparse_expert_delta`` (reference: spider_moe/sparse_experts.py:11-68).

Same signature and result: for every expert a token selected (weights of
repeated slots summed, tokens with summed weight <= 0 skipped), ``delta +=
tw * (W_down gelu(W_up x + b_up) + b_down)``, experts restricted to this
rank's (``e % world == rank``) and the delta summed across ranks when expert
parallel is active.  The work runs in libspider_b200 (device grouping, grouped
GEMMs, deterministic combine) on CUDA tensors; fp32 inputs use the CUDA-core
engine, bf16 inputs the tcgen05 engine.
"""
from __future__ import annotations

import torch

from .config import ModelConfig
from .engine import BlockEngine
from .expert_parallel import all_reduce_sum_, ep_enabled, get_rank_world

# Packed engines of recently used weight sets.  An entry keeps the weight
# tensors themselves and is reused only for those same tensor objects at the
# same in-place version: a freed and reallocated tensor can come back at the
# same address with version 0, so addresses alone would hand out an engine
# packed from the old weights.
_CACHE: dict = {}
_CACHE_MAX = 8


def _engine_for(w_up, b_up, w_down, b_down, num_experts, top_k, act_dtype, device) -> BlockEngine:
    tensors = (w_up, b_up, w_down, b_down)
    key = (tuple(t.data_ptr() for t in tensors), tuple(w_up.shape), int(num_experts), int(top_k), act_dtype,
           str(device))
    versions = tuple(int(t._version) for t in tensors)
    hit = _CACHE.get(key)
    if hit is not None:
        held, held_versions, eng = hit
        if all(a is b for a, b in zip(held, tensors)) and held_versions == versions:
            return eng
        del _CACHE[key]
    e, u, h = w_up.shape
    cfg = ModelConfig(hidden_size=h, num_heads=1, num_experts=num_experts, top_k=top_k, edges_per_expert=1,
                      num_loops=1, expert_ffn_size=u, loop_embed_size=8)
    state = {}
    for i in range(e):
        state[f"experts.{i}.0.weight"] = w_up[i]
        state[f"experts.{i}.0.bias"] = b_up[i]
        state[f"experts.{i}.2.weight"] = w_down[i]
        state[f"experts.{i}.2.bias"] = b_down[i]
    eng = BlockEngine(cfg, state, device, act_dtype=act_dtype, max_tokens=1)
    if len(_CACHE) >= _CACHE_MAX:
        _CACHE.pop(next(iter(_CACHE)))  # oldest entry
    _CACHE[key] = (tensors, versions, eng)
    return eng


def sparse_expert_delta(messages, top_indices, top_weights, w_up, b_up, w_down, b_down,
                        num_experts: int, top_k: int, expert_parallel: bool = True) -> torch.Tensor:
    """messages [B,T,H], top_indices/top_weights [B,T,K], w_up [E,U,H], b_up [E,U],
    w_down [E,H,U], b_down [E,H] -> delta [B,T,H] (messages dtype)."""
    if not messages.is_cuda:
        raise RuntimeError("spider_b200 sparse_expert_delta runs on CUDA tensors only")
    act = torch.float32 if messages.dtype == torch.float32 else torch.bfloat16
    eng = _engine_for(w_up, b_up, w_down, b_down, num_experts, top_k, act, messages.device)
    use_ep = expert_parallel and ep_enabled()
    rank, world = get_rank_world() if use_ep else (0, 1)
    delta = eng.expert_delta(messages, top_indices, top_weights, rank, world)
    if use_ep:
        all_reduce_sum_(delta)
    return delta.to(messages.dtype).view(messages.shape)
