"""Dobu expert offload on the B200 kernels (reference: spider_moe/expert_store.py).

``ExpertChunkStore`` keeps the reference's constructor, ``sparse_delta``,
``release_gpu``, ``stats`` and its LRU accounting (hits / misses / loads,
``max_gpu_experts`` resident experts, 0 = stream every expert), with a device
layout of its own:

* every expert's weights sit in pinned host memory in the activation dtype the
  kernels read (bf16 or fp32), so a load is one asynchronous host-to-device copy
  per tensor straight into a device slot;
* the device holds ``max(max_gpu_experts, 1)`` slots, stacked like the block's
  expert weights ([slots, U, H] up, [slots, H, U] down), so the grouped expert
  FFN (``sb_expert_delta``) runs over slots;
* per call, ``sb_active_experts`` finds the experts some token's summed routing
  weight is positive for (the ones the reference materialises, in ascending
  order), the host replays the reference's LRU over them, and the experts are
  computed in waves of at most ``slots``: load the misses of the wave,
  ``sb_remap_routes`` rewrites the routing onto slots (others weight 0), one
  ``sb_expert_delta`` call over the slots, accumulate.

The one host synchronisation per call (reading the active-expert flags) stands
for the reference's ``flat_idx.unique().tolist()``.
"""
from __future__ import annotations

import ctypes as C
from collections import OrderedDict

import torch
from torch import nn

from . import _lib as L


def _act_code(dtype: torch.dtype) -> int:
    return L.SB_F32 if dtype == torch.float32 else L.SB_BF16


class ExpertChunkStore:
    """Host-resident expert catalogue with a small device working set."""

    def __init__(self, experts: nn.ModuleList, *, storage_device="cpu", compute_device=None,
                 max_gpu_experts: int = 4, pin_memory: bool = True):
        self.storage_device = torch.device(storage_device)
        self.compute_device = torch.device(compute_device) if compute_device is not None else (
            torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu"))
        self.max_gpu_experts = max(0, int(max_gpu_experts))
        self.pin_memory = bool(pin_memory) and self.storage_device.type == "cpu" and torch.cuda.is_available()
        # fp32 master copies (the reference's chunks), one dict per expert
        self._master = []
        for ex in experts:
            up, down = ex[0], ex[2]
            self._master.append({k: v.detach().to(self.storage_device, torch.float32).contiguous()
                                 for k, v in (("w_up", up.weight), ("b_up", up.bias), ("w_down", down.weight),
                                              ("b_down", down.bias))})
        self.num_experts = len(self._master)
        self.ffn, self.hidden = self._master[0]["w_up"].shape
        self._staged = {}   # dtype -> list of pinned host chunks in that dtype
        self._pool = None   # device slots
        self._lru: OrderedDict[int, int] = OrderedDict()   # expert -> slot
        self.hits = self.misses = self.loads = 0

    def __len__(self) -> int:
        return self.num_experts

    # ------------------------------------------------------------------ storage
    def _host_chunks(self, dtype):
        if dtype not in self._staged:
            chunks = []
            for m in self._master:
                c = {"w_up": m["w_up"].to(dtype), "w_down": m["w_down"].to(dtype), "b_up": m["b_up"],
                     "b_down": m["b_down"]}
                if self.pin_memory:
                    c = {k: v.pin_memory() for k, v in c.items()}
                chunks.append(c)
            self._staged[dtype] = chunks
        return self._staged[dtype]

    def _slots(self) -> int:
        return max(self.max_gpu_experts, 1)

    def _ensure_pool(self, device, dtype):
        if self._pool is not None and self._pool["device"] == device and self._pool["dtype"] == dtype:
            return self._pool
        S, U, H = self._slots(), self.ffn, self.hidden
        f32 = dict(device=device, dtype=torch.float32)
        pool = {"device": device, "dtype": dtype,
                "w_up": torch.empty(S, U, H, device=device, dtype=dtype), "b_up": torch.zeros(S, U, **f32),
                "w_down": torch.empty(S, H, U, device=device, dtype=dtype), "b_down": torch.zeros(S, H, **f32),
                "slot_of": torch.full((self.num_experts,), -1, device=device, dtype=torch.int32),
                "active": torch.zeros(self.num_experts, device=device, dtype=torch.int32)}
        pool["weights"] = L.BlockWeights(w_up=pool["w_up"].data_ptr(), b_up=pool["b_up"].data_ptr(),
                                         w_down=pool["w_down"].data_ptr(), b_down=pool["b_down"].data_ptr())
        self._pool = pool
        self._lru.clear()
        return pool

    def _load(self, pool, expert_id: int, slot: int) -> None:
        c = self._host_chunks(pool["dtype"])[expert_id]
        for k in ("w_up", "b_up", "w_down", "b_down"):
            pool[k][slot].copy_(c[k], non_blocking=True)
        self.loads += 1

    # ------------------------------------------------------------------ residency (reference LRU)
    def _materialise(self, pool, expert_id: int, wave: dict) -> None:
        """expert_store.py:101-115: hit -> most recent; miss -> load, insert,
        evict the least recent beyond max_gpu_experts (0: stream, keep none)."""
        if expert_id in self._lru:
            self.hits += 1
            self._lru.move_to_end(expert_id)
            wave[expert_id] = self._lru[expert_id]
            return
        self.misses += 1
        if self.max_gpu_experts == 0:
            slot = 0
        else:
            used = set(self._lru.values())
            slot = next((s for s in range(self._slots()) if s not in used), None)
            if slot is None:  # full: the least recent leaves (never one of this wave, which is at most slots long)
                _, slot = self._lru.popitem(last=False)
            self._lru[expert_id] = slot
        self._load(pool, expert_id, slot)
        wave[expert_id] = slot

    def release_gpu(self) -> None:
        """Drop the device working set (experts stay in host memory)."""
        self._lru.clear()
        self._pool = None
        if self.compute_device.type == "cuda":
            torch.cuda.empty_cache()

    # ------------------------------------------------------------------ compute
    @torch.no_grad()
    def sparse_delta(self, messages: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor,
                     top_k: int) -> torch.Tensor:
        """sum_k w_k * FFN_{e_k}(messages) over the routed experts, with expert
        weights brought in from host memory (expert_store.py:117-166); in the
        messages' dtype, as the reference returns it."""
        return self.sparse_delta_f32(messages, top_indices, top_weights, top_k).to(messages.dtype)

    @torch.no_grad()
    def sparse_delta_f32(self, messages: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor,
                         top_k: int) -> torch.Tensor:
        """sparse_delta with the fp32 sum the block's LayerNorm epilogue reads."""
        if not messages.is_cuda:
            raise RuntimeError("spider_b200 ExpertChunkStore computes on CUDA tensors only")
        lib = L.load()
        self.compute_device = messages.device
        H = messages.shape[-1]
        lead = messages.shape[:-1]
        n = messages.numel() // H
        dtype = messages.dtype if messages.dtype in (torch.float32, torch.bfloat16) else torch.float32
        pool = self._ensure_pool(messages.device, dtype)
        stream = torch.cuda.current_stream(messages.device).cuda_stream
        msgs = messages.reshape(n, H).to(dtype).contiguous()
        idx = top_indices.reshape(n, top_k).to(torch.int32).contiguous()
        w = top_weights.reshape(n, top_k).to(torch.float32).contiguous()
        L.check(lib.sb_active_experts(idx.data_ptr(), w.data_ptr(), n, top_k, self.num_experts,
                                      pool["active"].data_ptr(), stream), "sb_active_experts")
        used = pool["active"].nonzero().view(-1).tolist()   # ascending, as unique() orders them
        delta = torch.zeros(n, H, device=messages.device, dtype=torch.float32)
        if not used:
            return delta.view(*lead, H)
        S = self._slots()
        dims = L.BlockDims(hidden=H, num_experts=S, top_k=top_k, edges_per_expert=1, ffn=self.ffn, num_loops=1,
                           act_dtype=_act_code(dtype), wfmt=L.SB_W_F32 if dtype == torch.float32 else L.SB_W_BF16,
                           activation=L.SB_ACT_GELU, group_size=0, engine=L.ENGINES["auto"], max_tokens=n,
                           residual_scale=0.5, reinject=0.1, ln_eps=1e-5)
        idx_s = torch.empty_like(idx)
        w_s = torch.empty_like(w)
        ws_bytes = lib.sb_expert_delta_workspace_bytes(C.byref(dims), n)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=messages.device)
        part = torch.empty(n, H, device=messages.device, dtype=torch.float32)
        slot_map = torch.full((self.num_experts,), -1, dtype=torch.int32)
        for w0 in range(0, len(used), S):
            wave = {}
            for e in used[w0:w0 + S]:
                self._materialise(pool, e, wave)
            slot_map.fill_(-1)
            for e, s in wave.items():
                slot_map[e] = s
            pool["slot_of"].copy_(slot_map, non_blocking=False)
            L.check(lib.sb_remap_routes(idx.data_ptr(), w.data_ptr(), n, top_k, pool["slot_of"].data_ptr(),
                                        self.num_experts, idx_s.data_ptr(), w_s.data_ptr(), stream),
                    "sb_remap_routes")
            L.check(lib.sb_expert_delta(C.byref(dims), C.byref(pool["weights"]), msgs.data_ptr(), idx_s.data_ptr(),
                                        w_s.data_ptr(), n, 0, 1, part.data_ptr(), ws.data_ptr(), ws_bytes, stream),
                    "sb_expert_delta")
            delta += part
        return delta.view(*lead, H)

    def stats(self) -> dict:
        nbytes = lambda c: sum(v.numel() * v.element_size() for v in c.values())  # noqa: E731
        storage = sum(nbytes(c) for c in self._master)
        hot = sum(nbytes(self._master[e]) for e in self._lru)
        return {
            "num_experts": self.num_experts,
            "gpu_hot_experts": list(self._lru.keys()),
            "max_gpu_experts": self.max_gpu_experts,
            "storage_device": str(self.storage_device),
            "compute_device": str(self.compute_device),
            "storage_bytes": storage,
            "gpu_working_set_bytes": hot,
            "hits": self.hits,
            "misses": self.misses,
            "loads": self.loads,
            "top_dobu_lru": self.max_gpu_experts,
            "policy": "dobu_residency",
        }
