"""Drop-in ``SpiderMoELayer`` running on the B200 kernels.

Same constructor, parameter names (so ``load_state_dict`` of a reference
checkpoint works unchanged), ``forward(h, x0, loop_idx, return_stats=False)``
signature and ``quantize_experts(group_size)`` / ``dequantize_experts()`` as
the reference module (spider_moe/model.py:163-349).  The forward pass runs in
libspider_b200 on CUDA tensors; CPU tensors raise (there is no CPU path).

Expert parallel (reference semantics, spider_moe/expert_parallel.py:1-37):
when ``torch.distributed`` is initialised with more than one rank and
``cfg.expert_parallel`` is true, every rank holds all tokens, computes its own
experts (``e % world == rank``) and the delta is summed across ranks before
the LayerNorm epilogue, so every rank returns the same output.  The
token-sharded all-to-all variant lives in ``spider_web_moe_b200.ep``.
"""
from __future__ import annotations

import torch
from torch import nn

from . import expert_parallel as ep_helpers
from .config import from_any
from .engine import BlockEngine
from .dobu import ExpertChunkStore
from .lumen import LumenWorkspace
from .quant import Int4Tensor, quantize_fp8_per_channel, quantize_int4


class SpiderMoELayer(nn.Module):
    """Shared recurrent layer: token router + per-loop sparse graph + expert FFNs."""

    def __init__(self, cfg):
        super().__init__()
        cfg = from_any(cfg)
        self.cfg = cfg
        h, e = cfg.hidden_size, cfg.num_experts
        self.num_experts, self.top_k = e, cfg.top_k
        self.top_dobu = int(getattr(cfg, "offload_max_gpu_experts", 4))
        self.edges_per_expert = cfg.edges_per_expert
        self.router = nn.Linear(h, e, bias=False)
        self.loop_bias = nn.Parameter(torch.zeros(cfg.num_loops, e))
        self.loop_embedding = nn.Embedding(cfg.num_loops, cfg.loop_embed_size)
        self.edge_generator = nn.Linear(h + cfg.loop_embed_size, e * e)
        self.edge_value = nn.ModuleList([nn.Linear(h, h, bias=False) for _ in range(e)])
        self.experts = nn.ModuleList([
            nn.Sequential(nn.Linear(h, cfg.expert_ffn_size), nn.GELU(), nn.Linear(cfg.expert_ffn_size, h))
            for _ in range(e)
        ])
        self.norm = nn.LayerNorm(h)
        self.exit_head = nn.Linear(h, 1)
        # Lumen global workspace after the LayerNorm (model.py:202-210)
        self.lumen: LumenWorkspace | None = None
        if bool(getattr(cfg, "use_lumen", False)):
            self.lumen = LumenWorkspace(h, num_slots=int(getattr(cfg, "lumen_slots", 8)),
                                        slot_dim=(int(getattr(cfg, "lumen_slot_dim", 0)) or None), vocab_size=None)
        if cfg.expert_activation == "swiglu":
            self.expert_gates = nn.ModuleList([nn.Linear(h, cfg.expert_ffn_size) for _ in range(e)])
        self.residual_scale = cfg.residual_scale
        self.reinject_weight = cfg.re_inject_weight
        self.expert_parallel = bool(getattr(cfg, "expert_parallel", True))
        # Dobu offload (model.py:185-199): experts stay in host memory, a few
        # in device slots; the store is built at the first forward
        self.offload_experts = bool(getattr(cfg, "offload_experts", False))
        self._expert_store: ExpertChunkStore | None = None
        self.engine_name = "auto"
        self._int4_w_up: Int4Tensor | None = None
        self._int4_w_down: Int4Tensor | None = None
        self._int4_w_gate: Int4Tensor | None = None
        self._fp8 = None
        self._engine: BlockEngine | None = None
        self._engine_key = None

    @classmethod
    def from_spiderw(cls, path, device="cuda", **cfg_overrides) -> "SpiderMoELayer":
        """The block stored in a .spiderw bundle (docs/NATIVE_WEIGHT_FORMAT.md of
        the reference); the format keeps no biases, so they load as zeros."""
        from .spiderw import block_state_dict, load_spiderw, model_config

        bundle = load_spiderw(path)
        layer = cls(model_config(bundle.meta, **cfg_overrides)).to(device)
        layer.load_state_dict(block_state_dict(bundle, device), strict=False)
        return layer.eval()

    # ------------------------------------------------------------------ weight formats
    @torch.no_grad()
    def quantize_experts(self, group_size: int = 64) -> None:
        """Pack expert up/down weights to group-wise INT4 (reference: model.py:218-231)."""
        stack = lambda j: torch.stack([ex[j].weight.detach() for ex in self.experts], dim=0)  # noqa: E731
        self._int4_w_up = quantize_int4(stack(0), group_size=group_size)
        self._int4_w_down = quantize_int4(stack(2), group_size=group_size)
        if hasattr(self, "expert_gates"):
            self._int4_w_gate = quantize_int4(torch.stack([g.weight.detach() for g in self.expert_gates]),
                                              group_size=group_size)
        self._fp8 = None
        self.invalidate()

    @torch.no_grad()
    def quantize_experts_fp8(self) -> None:
        """e4m3 expert weights with one fp32 scale per output channel (absmax/448)."""
        stack = lambda j: torch.stack([ex[j].weight.detach() for ex in self.experts], dim=0)  # noqa: E731
        up = quantize_fp8_per_channel(stack(0))
        down = quantize_fp8_per_channel(stack(2))
        self._fp8 = {"up": (up.q, up.scale), "down": (down.q, down.scale)}
        if hasattr(self, "expert_gates"):
            gt = quantize_fp8_per_channel(torch.stack([g.weight.detach() for g in self.expert_gates]))
            self._fp8["gate"] = (gt.q, gt.scale)
        self._int4_w_up = self._int4_w_down = self._int4_w_gate = None
        self.invalidate()

    def dequantize_experts(self) -> None:
        """Clear quantised expert buffers and use the nn.Linear weights again."""
        self._int4_w_up = self._int4_w_down = self._int4_w_gate = None
        self._fp8 = None
        self.invalidate()

    def invalidate(self) -> None:
        """Drop packed device weights (call after changing parameters in place)."""
        self._engine = None
        self._engine_key = None

    def _load_from_state_dict(self, *args, **kwargs):
        self.invalidate()
        return super()._load_from_state_dict(*args, **kwargs)

    def engine(self, device, act_dtype, n_tokens: int) -> BlockEngine:
        key = (str(device), act_dtype, self.engine_name)
        if self._engine is None or self._engine_key != key:
            int4 = None
            if self._int4_w_up is not None:
                int4 = {"up": self._int4_w_up, "down": self._int4_w_down}
                if self._int4_w_gate is not None:
                    int4["gate"] = self._int4_w_gate
            state = self.state_dict()
            if self.offload_experts:  # dense parts only: the experts come from the store
                state = {k: v for k, v in state.items() if not k.startswith(("experts.", "expert_gates."))}
                int4 = None
            self._engine = BlockEngine(self.cfg, state, device, act_dtype=act_dtype,
                                       max_tokens=max(n_tokens, 1), engine=self.engine_name,
                                       int4=int4, fp8=self._fp8)
            self._engine_key = key
        return self._engine

    # ------------------------------------------------------------------ forward
    def forward(self, h, x0, loop_idx, return_stats=False):
        """One loop of the block (model.py:240-317) on CUDA tensors [B, T, H]."""
        if not h.is_cuda:
            raise RuntimeError("spider_b200 SpiderMoELayer runs on CUDA tensors only")
        n = h.numel() // h.shape[-1]
        eng = self.engine(h.device, h.dtype if h.dtype in (torch.float32, torch.bfloat16) else torch.float32, n)
        use_ep = self.expert_parallel and ep_helpers.ep_enabled()
        if self.offload_experts:
            out, taps = self._forward_offload(eng, h, x0, loop_idx)
        elif not use_ep and not return_stats:
            out = eng.forward(h, x0, loop_idx, loop_idx + 1).to(h.dtype)
            return self.lumen(out) if self.lumen is not None else out
        elif not use_ep:
            taps = eng.make_taps(n)
            out = eng.forward(h, x0, loop_idx, loop_idx + 1, taps=taps).to(h.dtype)
        else:
            out, taps = self._forward_ep(eng, h, x0, loop_idx)
        lumen_state = None
        if self.lumen is not None:
            if return_stats:
                out, lumen_state = self.lumen(out, return_state=True)
            else:
                out = self.lumen(out)
        if not return_stats:
            return out
        stats = self._stats(eng, h, out, loop_idx, taps)
        if lumen_state is not None:  # model.py:346-348
            stats["lumen_slot_weights"] = lumen_state.slot_weights
            stats["lumen_broadcast_norm"] = lumen_state.broadcast.float().norm(dim=-1).to(lumen_state.broadcast.dtype)
        return out, stats

    def expert_store(self, device) -> ExpertChunkStore:
        if self._expert_store is None:
            self._expert_store = ExpertChunkStore(self.experts, storage_device="cpu", compute_device=device,
                                                  max_gpu_experts=self.top_dobu)
        return self._expert_store

    def _forward_offload(self, eng, h, x0, loop_idx):
        """The block with offloaded experts (model.py:294-297): routing and
        messages on the device (sb_block_route), the delta from the Dobu store,
        the LayerNorm epilogue (sb_combine_ln).  Returns (out, routing taps)."""
        if self.expert_parallel and ep_helpers.ep_enabled():
            raise NotImplementedError("expert offload with reference expert parallelism")
        n, H = h.numel() // h.shape[-1], h.shape[-1]
        msgs, top_idx, top_w = eng.route(h, loop_idx)
        delta = self.expert_store(h.device).sparse_delta_f32(msgs, top_idx, top_w, self.top_k)
        inv = torch.arange(n, dtype=torch.int32, device=h.device).view(n, 1)
        out = eng.epilogue(delta, inv, h, x0).to(h.dtype)
        return out, {"top_idx": top_idx, "top_w": top_w}

    def _forward_ep(self, eng, h, x0, loop_idx):
        """Reference expert-parallel semantics (sparse_experts.py:38-43,66-67):
        every rank routes all tokens and computes their messages
        (sb_block_route), runs only its own experts (sb_expert_delta with
        e % world == rank), SUM-all-reduces the delta, and applies the LayerNorm
        epilogue (sb_combine_ln).  Returns (out, routing taps for the stats)."""
        rank, world = ep_helpers.get_rank_world()
        n = h.numel() // h.shape[-1]
        msgs, top_idx, top_w = eng.route(h, loop_idx)
        delta = eng.expert_delta(msgs, top_idx, top_w, rank, world)
        ep_helpers.all_reduce_sum_(delta)
        inv = torch.arange(n, dtype=torch.int32, device=h.device).view(n, 1)
        out = eng.epilogue(delta, inv, h, x0).to(h.dtype)
        return out, {"top_idx": top_idx, "top_w": top_w}

    def run_loops(self, h, x0, loop_begin: int = 0, loop_end: int | None = None):
        """All loops [loop_begin, loop_end) in one library call (model.py:445-448)."""
        n = h.numel() // h.shape[-1]
        eng = self.engine(h.device, h.dtype, n)
        if self.offload_experts:  # the store's residency decisions run per loop on the host
            for loop_idx in range(loop_begin, self.cfg.num_loops if loop_end is None else loop_end):
                h = self(h, x0, loop_idx)
            return h
        if self.lumen is None:
            return eng.forward(h, x0, loop_begin, loop_end)
        loop_end = self.cfg.num_loops if loop_end is None else loop_end
        for loop_idx in range(loop_begin, loop_end):  # Lumen after every loop's LayerNorm
            h = self.lumen(eng.forward(h, x0, loop_idx, loop_idx + 1))
        return h

    def run_recurrent_decode(self, h, x0, early_exit: bool = True, threshold: float | None = None):
        """SpiderWebLM._run_recurrent_decode (model.py:450-473) on this block:
        with early_exit, batch rows whose exit confidence passes the threshold
        (cfg.early_exit_threshold by default) stop looping; the active set is
        kept and compacted on the device (sb_active_set_step)."""
        if not early_exit:
            return self.run_recurrent_full(h, x0)
        thr = self.cfg.early_exit_threshold if threshold is None else float(threshold)
        n = h.numel() // h.shape[-1]
        eng = self.engine(h.device, h.dtype if h.dtype in (torch.float32, torch.bfloat16) else torch.float32, n)
        loop_fn = None
        if self.lumen is not None:
            def loop_fn(hc, xc, loop_idx, out):
                out.copy_(self.lumen(eng.forward(hc, xc, loop_idx, loop_idx + 1)).reshape(out.shape))
        if (self.expert_parallel and ep_helpers.ep_enabled()) or self.offload_experts:
            # the module's own loop (Lumen included); under expert parallelism
            # every rank holds the same rows, so the active sets agree and each
            # loop's all-reduce has the same shape everywhere
            def loop_fn(hc, xc, loop_idx, out):
                out.copy_(self(hc, xc, loop_idx).reshape(out.shape))
        out, _ = eng.run_recurrent_decode(h, x0, thr, self.exit_head.weight, self.exit_head.bias, loop_fn=loop_fn)
        return out.view(h.shape).to(h.dtype)

    def run_recurrent_full(self, h, x0):
        """SpiderWebLM._run_recurrent_full (model.py:445-448): all loops in one
        library call, or loop by loop under the reference's expert parallelism."""
        if self.expert_parallel and ep_helpers.ep_enabled():
            for loop_idx in range(self.cfg.num_loops):
                h = self(h, x0, loop_idx)
            return h
        return self.run_loops(h, x0).to(h.dtype)

    def _stats(self, eng, h, out, loop_idx, taps):
        """The stats dict of model.py:327-343 (sb_loop_stats): router
        probabilities [B, T, E], expert / edge load, both auxiliary losses and
        the exit-head confidence [B, T] of the loop's output."""
        st = eng.loop_stats(h, out, loop_idx, top_idx=taps["top_idx"], exit_w=self.exit_head.weight,
                            exit_b=self.exit_head.bias)
        lead = h.shape[:-1]
        return {"router_probs": st["router_probs"].view(*lead, self.num_experts),
                "expert_load": st["expert_load"], "edge_load": st["edge_load"],
                "aux_loss": st["aux_loss"], "edge_loss": st["edge_loss"],
                "confidence": st["confidence"].view(lead)}
