"""Lumen global workspace on the B200 kernels (reference: spider_moe/lumen.py).

``LumenWorkspace`` keeps the reference's constructor, parameter names
(``write_q``, ``write_v``, ``slot_to_h``, ``gate``, ``norm``, ``slot_bias``,
optional ``j_lens``), ``forward(h, *, return_state=False, j_lens=False)``,
``read_j_space`` and ``stats``; ``LumenState`` has the reference's fields.
The forward runs ``sb_lumen_forward`` (two one-group GEMMs and two
warp-per-token kernels); the slot tensor ``slots = w (x) values`` is only
formed when the state is asked for.  CUDA tensors only: there is no CPU path.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Any

import torch
from torch import nn

from . import _lib as L


@dataclass
class LumenState:
    """Workspace contents after a write cycle (lumen.py:27-34)."""

    slots: torch.Tensor          # [B, T, S, D]
    slot_weights: torch.Tensor   # [B, T, S]
    broadcast: torch.Tensor      # [B, T, H]
    j_logits: torch.Tensor | None = None  # [B, T, V]


def _act_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return L.SB_F32
    if dtype == torch.bfloat16:
        return L.SB_BF16
    raise TypeError(f"Lumen activations must be float32 or bfloat16, got {dtype}")


class LumenWorkspace(nn.Module):
    """Low-rank global workspace with competitive write + broadcast (lumen.py:37-79)."""

    def __init__(self, hidden_size: int, num_slots: int = 8, slot_dim: int | None = None,
                 vocab_size: int | None = None, dropout: float = 0.0):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_slots = int(num_slots)
        self.slot_dim = int(slot_dim or max(32, hidden_size // 4))
        self.vocab_size = vocab_size
        self.write_q = nn.Linear(hidden_size, self.num_slots, bias=False)
        self.write_v = nn.Linear(hidden_size, self.slot_dim, bias=False)
        self.slot_to_h = nn.Linear(self.slot_dim, hidden_size, bias=False)
        self.gate = nn.Linear(hidden_size + hidden_size, 1)
        self.norm = nn.LayerNorm(hidden_size)
        self.drop = nn.Dropout(dropout)
        self.j_lens: nn.Linear | None = None
        if vocab_size is not None and vocab_size > 0:
            self.j_lens = nn.Linear(self.slot_dim, vocab_size, bias=False)
        self.slot_bias = nn.Parameter(torch.zeros(self.num_slots))
        self.engine_name = "auto"
        self._packed = None
        self._packed_key = None

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        self._packed = None
        # a model-level state dict carries the J-lens head SpiderWebLM attaches
        # (model.py:365-371): take it on rather than reject the key
        key = prefix + "j_lens.weight"
        if self.j_lens is None and key in state_dict:
            v = state_dict[key]
            self.j_lens = nn.Linear(v.shape[1], v.shape[0], bias=False).to(self.write_q.weight.device)
        return super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def invalidate(self) -> None:
        """Drop the packed device copies (call after changing parameters in place)."""
        self._packed = None

    def _pack(self, device, dtype):
        key = (str(device), dtype)
        if self._packed is None or self._packed_key != key:
            f32 = torch.float32
            g = lambda t: t.detach().to(device)  # noqa: E731
            t = {
                "wqv": torch.cat([g(self.write_q.weight), g(self.write_v.weight)], 0).to(dtype).contiguous(),
                "qv_bias": torch.cat([g(self.slot_bias).to(f32), torch.zeros(self.slot_dim, device=device)]).contiguous(),
                "w_o": g(self.slot_to_h.weight).to(dtype).contiguous(),
                "gate_w": g(self.gate.weight).reshape(-1).to(f32).contiguous(),
                "gate_b": g(self.gate.bias).reshape(1).to(f32).contiguous(),
                "ln_w": g(self.norm.weight).to(f32).contiguous(),
                "ln_b": g(self.norm.bias).to(f32).contiguous(),
            }
            w = L.LumenWeights(wqv=t["wqv"].data_ptr(), qv_bias=t["qv_bias"].data_ptr(), w_o=t["w_o"].data_ptr(),
                               gate_w=t["gate_w"].data_ptr(), gate_b=t["gate_b"].data_ptr(),
                               ln_w=t["ln_w"].data_ptr(), ln_b=t["ln_b"].data_ptr(), ln_eps=float(self.norm.eps))
            self._packed = (t, w, {})
            self._packed_key = key
        return self._packed

    def forward(self, h: torch.Tensor, *, return_state: bool = False, j_lens: bool = False):
        """Write ``h`` [B, T, H] into the workspace and broadcast back (lumen.py:81-123)."""
        if not h.is_cuda:
            raise RuntimeError("spider_b200 LumenWorkspace runs on CUDA tensors only")
        if self.training and self.drop.p > 0:
            raise NotImplementedError("Lumen dropout in training mode is not on the B200 path")
        lib = L.load()
        H, S, D = self.hidden_size, self.num_slots, self.slot_dim
        dtype = h.dtype if h.dtype in (torch.float32, torch.bfloat16) else torch.float32
        n = h.numel() // H
        h2 = h.reshape(n, H).to(dtype).contiguous()
        _, w, cache = self._pack(h.device, dtype)
        want = return_state or j_lens
        out = torch.empty_like(h2)
        f32 = dict(dtype=torch.float32, device=h.device)
        sw = torch.empty(n, S, **f32) if want else None
        vals = torch.empty(n, D, **f32) if want else None
        bc = torch.empty(n, H, **f32) if want else None
        nbytes = lib.sb_lumen_workspace_bytes(n, H, S, D)
        ws = cache.get("ws")
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=h.device)
            cache["ws"] = ws
        ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        rc = lib.sb_lumen_forward(_act_code(dtype), L.ENGINES[self.engine_name], n, H, S, D, C.byref(w), h2.data_ptr(),
                                  out.data_ptr(), ptr(sw), ptr(vals), ptr(bc), None, ws.data_ptr(), ws.numel(),
                                  torch.cuda.current_stream(h.device).cuda_stream)
        L.check(rc, "sb_lumen_forward")
        out = out.view(h.shape).to(h.dtype)
        if not want:
            return out
        lead = h.shape[:-1]
        slots = (sw.unsqueeze(-1) * vals.unsqueeze(-2)).view(*lead, S, D).to(h.dtype)
        j_logits = None
        if j_lens and self.j_lens is not None:
            j_logits = self.j_lens(slots.mean(dim=-2))
        state = LumenState(slots=slots, slot_weights=sw.view(*lead, S).to(h.dtype),
                           broadcast=bc.view(*lead, H).to(h.dtype), j_logits=j_logits)
        if return_state:
            return out, state
        return out

    def read_j_space(self, state: LumenState, top_k: int = 5) -> list:
        """Top-k vocab ids per token from the J-lens readout (lumen.py:125-130)."""
        if state.j_logits is None:
            return []
        _, idx = torch.topk(state.j_logits, k=min(top_k, state.j_logits.shape[-1]), dim=-1)
        return idx.tolist()

    def stats(self) -> dict[str, Any]:
        return {
            "name": "Lumen",
            "analogue": "global_workspace_j_space",
            "num_slots": self.num_slots,
            "slot_dim": self.slot_dim,
            "j_lens": self.j_lens is not None,
        }
