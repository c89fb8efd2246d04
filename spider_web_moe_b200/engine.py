"""Device-side state of one recurrent Spider-MoE block and the calls into the C ABI.

``BlockEngine`` packs a block's parameters (reference state-dict names,
spider_moe/model.py:165-216) into the layouts the kernels read, owns the
workspace, and runs loops of the block through ``sb_block_forward``.  Packed
layouts in HBM:

* routing weights ``[E + E*E, H]``: the router rows followed by the hidden
  part of the edge generator's rows (one tensor, so a large batch computes
  every router and edge logit in one GEMM), and edge values ``[E, H, H]`` --
  all in the activation dtype, row-major, i.e. each weight row is one K-major
  MMA operand row;
* per-loop edge-generator bias ``[L, E*E]`` fp32: the generator bias plus the
  loop-embedding columns applied to ``loop_embedding[l]``, folded once at
  packing time (the loop embedding is constant per loop, model.py:260-263);
* experts ``w_up [E, U, H]`` / ``w_down [E, H, U]`` in bf16, fp8 (+ fp32
  scale per output row) or packed int4 (+ bf16 scale per row and group of
  the reduction dim), biases fp32.
"""
from __future__ import annotations

import copy
import ctypes as C
import os

import torch

from . import _lib as L
from .config import ModelConfig, from_any
from .quant import Int4Tensor, dequantize_int4, quantize_fp8_per_channel, quantize_int4


def _act_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return L.SB_F32
    if dtype == torch.bfloat16:
        return L.SB_BF16
    raise TypeError(f"activation dtype {dtype} not supported (float32 or bfloat16)")


def _stream_ptr(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def stacked(sd: dict, fmt: str, e: int) -> torch.Tensor:
    return torch.stack([sd[fmt.format(i)] for i in range(e)])


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[E, U, ...] gate and up rows (weights, their per-row scales or biases) ->
    [E, 2U, ...] with, for every block b of 64 features, the 64 gate rows then
    the 64 up rows: the layout SB_EPI_SWIGLU_IL reads."""
    e, u = up.shape[:2]
    rest = up.shape[2:]
    g = gate.reshape(e, u // 64, 1, 64, *rest)
    v = up.reshape(e, u // 64, 1, 64, *rest)
    return torch.cat([g, v], dim=2).reshape(e, 2 * u, *rest).contiguous()


def split_gate_up(packed: torch.Tensor, which: str) -> torch.Tensor:
    """Inverse of interleave_gate_up for one half: "gate" or "up" rows [E, U, ...]."""
    e, u2 = packed.shape[:2]
    rest = packed.shape[2:]
    half = packed.reshape(e, u2 // 128, 2, 64, *rest)[:, :, 0 if which == "gate" else 1]
    return half.reshape(e, u2 // 2, *rest)


class BlockEngine:
    """Packed weights + workspace for one block on one device."""

    def __init__(self, cfg, state: dict, device, act_dtype=torch.bfloat16, max_tokens: int = 64,
                 weight_format: str | None = None, engine: str = "auto",
                 int4: dict | None = None, fp8: dict | None = None, resident_bf16: bool = False):
        self.cfg = from_any(cfg)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("BlockEngine runs on CUDA devices only (no CPU path)")
        self.lib = L.load()
        self.act_dtype = act_dtype
        cfg = self.cfg
        H, E, U, Lp = cfg.hidden_size, cfg.num_experts, cfg.expert_ffn_size, cfg.num_loops
        fmt = weight_format or cfg.expert_weight_format
        if int4 is not None:
            fmt = "int4"
        elif fp8 is not None:
            fmt = "fp8"
        if fmt == "native":
            fmt = "f32" if act_dtype == torch.float32 else "bf16"
        if fmt == "f32" and act_dtype != torch.float32:
            raise ValueError("fp32 expert weights need fp32 activations")
        self.weight_format = fmt
        dev, dt = self.device, act_dtype
        f32 = torch.float32
        g = lambda k: state[k].detach().to(dev)  # noqa: E731
        self.t = {}
        t = self.t
        if "router.weight" in state:  # experts-only engines (sparse_expert_delta) skip the dense parts
            t["loop_bias"] = g("loop_bias").to(f32).contiguous()
            gen_full = g("edge_generator.weight").to(f32)
            t["route_w"] = torch.cat([g("router.weight").to(dt), gen_full[:, :H].to(dt)]).contiguous()
            emb = g("loop_embedding.weight").to(f32)                  # [L, Le]
            t["gen_bias"] = (g("edge_generator.bias").to(f32).unsqueeze(0)
                             + emb @ gen_full[:, H:].t()).contiguous()  # [L, E*E]
            del gen_full
            t["edge_w"] = stacked(state, "edge_value.{}.weight", E).to(dev, dt).contiguous()
            t["ln_w"] = g("norm.weight").to(f32).contiguous()
            t["ln_b"] = g("norm.bias").to(f32).contiguous()
        swiglu = cfg.expert_activation == "swiglu"
        self.group_size = 0
        has_experts = "experts.0.0.weight" in state or int4 is not None or fp8 is not None
        if has_experts:  # dense-only engines (routing of an expert-parallel rank) skip the experts
            t["b_up"] = stacked(state, "experts.{}.0.bias", E).to(dev, f32).contiguous()
            t["b_down"] = stacked(state, "experts.{}.2.bias", E).to(dev, f32).contiguous()
            if swiglu:
                t["b_gate"] = stacked(state, "expert_gates.{}.bias", E).to(dev, f32).contiguous()
        names = ([("up", "experts.{}.0.weight")] + ([("gate", "expert_gates.{}.weight")] if swiglu else [])
                 + [("down", "experts.{}.2.weight")]) if has_experts else []
        for short, key in names:
            if fmt in ("f32", "bf16"):
                t["w_" + short] = stacked(state, key, E).to(dev, f32 if fmt == "f32" else torch.bfloat16).contiguous()
            elif fmt == "fp8":
                if fp8 is not None and short in fp8:
                    q, s = fp8[short]
                else:
                    q8 = quantize_fp8_per_channel(stacked(state, key, E).to(dev, f32))
                    q, s = q8.q, q8.scale
                t["w_" + short] = q.to(dev).view(torch.uint8).contiguous()
                t["s_" + short] = s.to(dev, f32).contiguous()
            elif fmt == "int4":
                if int4 is not None and short in int4:
                    qt: Int4Tensor = int4[short]
                else:
                    gs = cfg.moe_int4_group_size
                    qt = quantize_int4(stacked(state, key, E).to(dev, f32), gs)
                self.group_size = qt.group_size
                t["w_" + short] = qt.packed.to(dev).contiguous()
                t["s_" + short] = qt.device_scales().to(dev).contiguous()
            else:
                raise ValueError(f"unknown weight format {fmt}")
        if resident_bf16 and fmt in ("fp8", "int4") and names:
            # The quantised experts held as bf16 with the same values the GEMMs'
            # conversion makes: e4m3 exactly (the per-row scale stays, applied to
            # the accumulator), int4 as bf16(q * s).  For callers whose every
            # call is prefill-sized (an expert-parallel owner), so the tensor-core
            # schedules of bf16 weights apply without a conversion per call.
            for short, _ in names:
                q = t["w_" + short]
                if fmt == "fp8":
                    t["w_" + short] = q.view(torch.float8_e4m3fn).to(torch.bfloat16).contiguous()
                else:  # q * (bf16 group scale) in fp32 is exact; one rounding to bf16
                    sc = t.pop("s_" + short)
                    shape = (*q.shape[:-1], q.shape[-1] * 2)
                    t["w_" + short] = dequantize_int4(q, sc, shape, self.group_size, torch.bfloat16).contiguous()
            fmt = "bf16"
        self.swiglu = swiglu and has_experts
        if self.swiglu:
            # SwiGLU: gate and up rows interleaved in blocks of 64 in one tensor
            # ([E, 2U, ...]; SB_EPI_SWIGLU_IL), so one MMA operand covers both
            if U % 64:
                raise ValueError("SwiGLU experts need expert_ffn_size divisible by 64")
            for k in ("w", "s", "b"):
                if k + "_gate" in t:
                    t[k + "_up"] = interleave_gate_up(t.pop(k + "_gate"), t[k + "_up"])
        wcode = {"f32": L.SB_W_F32, "bf16": L.SB_W_BF16, "fp8": L.SB_W_FP8, "int4": L.SB_W_INT4}[fmt]
        self.dims = L.BlockDims(
            hidden=H, num_experts=E, top_k=cfg.top_k, edges_per_expert=cfg.edges_per_expert, ffn=U,
            num_loops=Lp, act_dtype=_act_code(dt), wfmt=wcode,
            activation=L.SB_ACT_SWIGLU if swiglu else L.SB_ACT_GELU, group_size=self.group_size,
            engine=L.ENGINES[engine], max_tokens=int(max_tokens),
            residual_scale=float(cfg.residual_scale), reinject=float(cfg.re_inject_weight), ln_eps=1e-5)
        p = lambda k: t[k].data_ptr() if k in t else None  # noqa: E731
        rw = t.get("route_w")
        gen_ptr = rw[E:].data_ptr() if rw is not None else None
        self.weights = L.BlockWeights(
            router_w=p("route_w"), loop_bias=p("loop_bias"), gen_w=gen_ptr, gen_bias=p("gen_bias"),
            route_w=p("route_w"),
            edge_w=p("edge_w"), w_up=p("w_up"), s_up=p("s_up"), b_up=p("b_up"), w_gate=p("w_gate"),
            s_gate=p("s_gate"), b_gate=p("b_gate"), w_down=p("w_down"), s_down=p("s_down"),
            b_down=p("b_down"), ln_w=p("ln_w"), ln_b=p("ln_b"))
        self.workspace = None
        self._ensure_workspace(int(max_tokens))

    @classmethod
    def from_spiderw(cls, path, device, act_dtype=torch.bfloat16, max_tokens: int = 64, **kwargs) -> "BlockEngine":
        """Engine for the block of a .spiderw bundle: sections go to the device
        once and are packed there (spiderw.block_state_dict)."""
        from .spiderw import block_state_dict, load_spiderw, model_config

        bundle = load_spiderw(path)
        cfg = model_config(bundle.meta)
        return cls(cfg, block_state_dict(bundle, device), device, act_dtype=act_dtype, max_tokens=max_tokens,
                   **kwargs)

    # ------------------------------------------------------------------ workspace
    def _ensure_workspace(self, n_tokens: int):
        if self.workspace is not None and n_tokens <= self.dims.max_tokens:
            return
        self.dims.max_tokens = max(int(n_tokens), int(self.dims.max_tokens))
        nbytes = self.lib.sb_block_workspace_bytes(C.byref(self.dims))
        if nbytes == 0:
            raise L.SpiderB200Error(L.SB_ERR_ARG, "sb_block_workspace_bytes")
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)

    def weight_bytes(self) -> int:
        return sum(v.numel() * v.element_size() for v in self.t.values())

    def twin(self) -> "BlockEngine":
        """An engine on the same packed weights with workspaces of its own, so
        that work for two independent token batches can be in flight on two
        streams at once (the micro-batches of an expert-parallel step)."""
        t = copy.copy(self)
        t.dims = L.BlockDims.from_buffer_copy(self.dims)
        t.workspace = None
        for k in ("_epws", "_dws"):  # per-engine scratch, made on first use
            t.__dict__.pop(k, None)
        t._ensure_workspace(int(self.dims.max_tokens))
        return t

    def expert_tensors(self, short: str):
        """(weights, scales or None, biases) of one expert projection ("up",
        "gate" or "down") in the [E, rows, ...] layout of the reference's
        stacked Linear weights, as stored on the device (views; SwiGLU's
        interleaved gate/up tensor is split back into its halves)."""
        t = self.t
        if self.swiglu and short in ("up", "gate"):
            s = t.get("s_up")
            return (split_gate_up(t["w_up"], short), None if s is None else split_gate_up(s, short),
                    split_gate_up(t["b_up"], short))
        return t["w_" + short], t.get("s_" + short), t["b_" + short]

    def status(self) -> int:
        """Device status word (non-zero: a bounded wait ran out); synchronises."""
        off = self.lib.sb_status_offset()
        return int(self.workspace[off:off + 4].view(torch.int32).item())

    def check_status(self):
        s = self.status()
        if s:
            raise L.SpiderB200Error(L.SB_ERR_DEVICE_STATUS, f"device status 0x{s:x}")

    # ------------------------------------------------------------------ calls
    def forward(self, h: torch.Tensor, x0: torch.Tensor, loop_begin: int = 0, loop_end: int | None = None,
                out: torch.Tensor | None = None, taps: dict | None = None, stream=None) -> torch.Tensor:
        """Run loops [loop_begin, loop_end) on h (shape [..., H]); x0 is the block input."""
        H = self.cfg.hidden_size
        loop_end = self.cfg.num_loops if loop_end is None else loop_end
        if h.device != self.device or x0.device != self.device:
            raise RuntimeError("inputs must live on the engine's CUDA device")
        n = h.numel() // H
        self._ensure_workspace(n)
        h2 = h.reshape(n, H)
        if h2.dtype != self.act_dtype or not h2.is_contiguous():
            h2 = h2.to(self.act_dtype).contiguous()
        x2 = x0.reshape(n, H)
        if x2.dtype != self.act_dtype or not x2.is_contiguous():
            x2 = x2.to(self.act_dtype).contiguous()
        if out is None:
            out = torch.empty((n, H), dtype=self.act_dtype, device=self.device)
        ctaps = None
        if taps is not None:
            ctaps = L.BlockTaps(**{k: (v.data_ptr() if v is not None else None) for k, v in taps.items()})
        rc = self.lib.sb_block_forward(C.byref(self.dims), C.byref(self.weights), h2.data_ptr(), x2.data_ptr(),
                                       out.data_ptr(), n, int(loop_begin), int(loop_end),
                                       self.workspace.data_ptr(), self.workspace.numel(),
                                       C.byref(ctaps) if ctaps is not None else None, _stream_ptr(stream))
        L.check(rc, "sb_block_forward")
        if os.environ.get("SPIDER_B200_CHECK"):
            self.check_status()
        return out.view(h.shape)

    def route(self, h: torch.Tensor, loop_idx: int, stream=None):
        """Router + edge graph + messages of one loop (sb_block_route): returns
        (messages [n, H] act dtype, top_idx [n, K] int32, top_w [n, K] fp32)."""
        H, K = self.cfg.hidden_size, self.cfg.top_k
        n = h.numel() // H
        self._ensure_workspace(n)
        h2 = h.reshape(n, H)
        if h2.dtype != self.act_dtype or not h2.is_contiguous():
            h2 = h2.to(self.act_dtype).contiguous()
        msgs = torch.empty((n, H), dtype=self.act_dtype, device=self.device)
        top_idx = torch.empty((n, K), dtype=torch.int32, device=self.device)
        top_w = torch.empty((n, K), dtype=torch.float32, device=self.device)
        rc = self.lib.sb_block_route(C.byref(self.dims), C.byref(self.weights), h2.data_ptr(), n, int(loop_idx),
                                     msgs.data_ptr(), None, top_idx.data_ptr(), top_w.data_ptr(),
                                     self.workspace.data_ptr(), self.workspace.numel(), _stream_ptr(stream))
        L.check(rc, "sb_block_route")
        return msgs, top_idx, top_w

    def epilogue(self, rows: torch.Tensor, inv: torch.Tensor, h: torch.Tensor, x0: torch.Tensor, stream=None):
        """h_out = LayerNorm(h + a*delta + b*x0) with delta[t] = sum of rows[inv[t, k]] (sb_combine_ln)."""
        H = self.cfg.hidden_size
        n = h.numel() // H
        slots = inv.shape[-1]
        h2 = h.reshape(n, H).to(self.act_dtype).contiguous()
        x2 = x0.reshape(n, H).to(self.act_dtype).contiguous()
        out = torch.empty((n, H), dtype=self.act_dtype, device=self.device)
        rc = self.lib.sb_combine_ln(rows.data_ptr(), H, 1, 0, inv.data_ptr(), slots, None, h2.data_ptr(),
                                    x2.data_ptr(), self.dims.act_dtype, n, H, self.t["ln_w"].data_ptr(),
                                    self.t["ln_b"].data_ptr(), self.dims.residual_scale, self.dims.reinject,
                                    self.dims.ln_eps, out.data_ptr(), None, _stream_ptr(stream))
        L.check(rc, "sb_combine_ln")
        return out.view(h.shape)

    def ep_pack(self, top_idx, top_w, msgs, world: int, cap: int, stream=None):
        """Packed per-owner send rows for the all-to-all (sb_ep_pack): a uint8
        tensor [world, cap, pitch] and the return positions [n, K]."""
        H, K, E = self.cfg.hidden_size, self.cfg.top_k, self.cfg.num_experts
        n = msgs.shape[0]
        pitch = self.lib.sb_ep_row_pitch(H, self.dims.act_dtype, K)
        send = torch.empty((world, cap, pitch), dtype=torch.uint8, device=self.device)
        ret_pos = torch.empty((n, K), dtype=torch.int32, device=self.device)
        nbytes = self.lib.sb_ep_pack_workspace_bytes(n, K, world)
        ws = self._ep_ws(nbytes)
        rc = self.lib.sb_ep_pack(top_idx.data_ptr(), top_w.data_ptr(), msgs.data_ptr(), self.dims.act_dtype, n, H,
                                 K, E, world, cap, send.data_ptr(), ret_pos.data_ptr(), ws.data_ptr(), ws.numel(),
                                 _stream_ptr(stream))
        L.check(rc, "sb_ep_pack")
        return send, ret_pos

    def ep_dispatch(self, top_idx, top_w, msgs, world: int, rank: int, cap: int, regions: torch.Tensor,
                    stream=None) -> torch.Tensor:
        """sb_ep_dispatch: the packed rows go straight into the owners' exchange
        regions (`regions`: int64 device tensor of the mapped region pointers);
        returns the return positions [n, K]."""
        H, K, E = self.cfg.hidden_size, self.cfg.top_k, self.cfg.num_experts
        n = msgs.shape[0]
        ret_pos = torch.empty((n, K), dtype=torch.int32, device=self.device)
        ws = self._ep_ws(self.lib.sb_ep_pack_workspace_bytes(n, K, world))
        rc = self.lib.sb_ep_dispatch(top_idx.data_ptr(), top_w.data_ptr(), msgs.data_ptr(), self.dims.act_dtype, n, H,
                                     K, E, world, rank, cap, regions.data_ptr(), ret_pos.data_ptr(), ws.data_ptr(),
                                     ws.numel(), _stream_ptr(stream))
        L.check(rc, "sb_ep_dispatch")
        return ret_pos

    def expert_rows_peer(self, xch, expected_pairs: int, status_ptr: int, stream=None):
        """Owner side of the peer transport (sb_expert_rows_peer): waits for the
        ranks' rows in this rank's region, runs the local experts on them and
        writes the results into the sources' regions."""
        r = xch.world * xch.cap
        ws = self._delta_ws(self.lib.sb_expert_rows_workspace_bytes(C.byref(self.dims), r))
        rc = self.lib.sb_expert_rows_peer(C.byref(self.dims), C.byref(self.weights), xch.region, xch.regions.data_ptr(),
                                          xch.world, xch.rank, xch.cap, xch.pitch, int(expected_pairs), status_ptr,
                                          ws.data_ptr(), ws.numel(), _stream_ptr(stream))
        L.check(rc, "sb_expert_rows_peer")

    def ep_epilogue_peer(self, xch, ret_pos: torch.Tensor, h: torch.Tensor, x0: torch.Tensor, stream=None):
        """Source side of the peer transport (sb_ep_epilogue_peer): waits for the
        owners' returned rows, then the delta + LayerNorm epilogue."""
        H = self.cfg.hidden_size
        n = h.numel() // H
        h2 = h.reshape(n, H).to(self.act_dtype).contiguous()
        x2 = x0.reshape(n, H).to(self.act_dtype).contiguous()
        out = torch.empty((n, H), dtype=self.act_dtype, device=self.device)
        rc = self.lib.sb_ep_epilogue_peer(xch.region, xch.world, xch.cap, xch.pitch, ret_pos.data_ptr(),
                                          ret_pos.shape[-1], h2.data_ptr(), x2.data_ptr(), self.dims.act_dtype, n, H,
                                          self.t["ln_w"].data_ptr(), self.t["ln_b"].data_ptr(), self.dims.residual_scale,
                                          self.dims.reinject, self.dims.ln_eps, out.data_ptr(), self.status_ptr(),
                                          _stream_ptr(stream))
        L.check(rc, "sb_ep_epilogue_peer")
        return out.view(h.shape)

    def status_ptr(self) -> int:
        """Device address of the status word (kernels outside the block record there)."""
        return self.workspace.data_ptr() + self.lib.sb_status_offset()

    def expert_rows(self, rows: torch.Tensor, out: torch.Tensor | None = None, expected_pairs: int = 0,
                    stream=None) -> torch.Tensor:
        """Owner side: packed rows [R, pitch] (uint8) -> fp32 [R, H] weighted sums of this
        engine's (local) experts (sb_expert_rows)."""
        H = self.cfg.hidden_size
        r, pitch = rows.shape[0], rows.shape[-1]
        if out is None:
            out = torch.empty((r, H), dtype=torch.float32, device=self.device)
        nbytes = self.lib.sb_expert_rows_workspace_bytes(C.byref(self.dims), r)
        ws = self._delta_ws(nbytes)
        rc = self.lib.sb_expert_rows(C.byref(self.dims), C.byref(self.weights), rows.data_ptr(), pitch, r,
                                     int(expected_pairs), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                     _stream_ptr(stream))
        L.check(rc, "sb_expert_rows")
        return out

    def _ep_ws(self, nbytes: int) -> torch.Tensor:
        ws = getattr(self, "_epws", None)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._epws = ws
        return ws

    def make_taps(self, n: int) -> dict:
        cfg = self.cfg
        K, M, E, H = cfg.top_k, cfg.edges_per_expert, cfg.num_experts, cfg.hidden_size
        z = lambda *s, dt=torch.float32: torch.zeros(*s, dtype=dt, device=self.device)  # noqa: E731
        return dict(top_idx=z(n, K, dt=torch.int32), top_w=z(n, K), edge_idx=z(n, K, M, dt=torch.int32),
                    edge_w=z(n, K, M), messages=z(n, H), delta=z(n, H),
                    ffn_offsets=z(E + 1, dt=torch.int32), ffn_rows=z(n * K, dt=torch.int32),
                    ffn_weights=z(n * K))

    def expert_delta(self, messages: torch.Tensor, top_idx: torch.Tensor, top_w: torch.Tensor,
                     rank: int = 0, world: int = 1, stream=None) -> torch.Tensor:
        """sparse_expert_delta for this rank's experts (e % world == rank), fp32 [n, H]."""
        H, K = self.cfg.hidden_size, self.cfg.top_k
        n = messages.numel() // H
        m2 = messages.reshape(n, H)
        if m2.dtype != self.act_dtype or not m2.is_contiguous():
            m2 = m2.to(self.act_dtype).contiguous()
        idx = top_idx.reshape(n, K).to(torch.int32).contiguous()
        w = top_w.reshape(n, K).to(torch.float32).contiguous()
        delta = torch.empty((n, H), dtype=torch.float32, device=self.device)
        nbytes = self.lib.sb_expert_delta_workspace_bytes(C.byref(self.dims), n)
        ws = self._delta_ws(nbytes)
        rc = self.lib.sb_expert_delta(C.byref(self.dims), C.byref(self.weights), m2.data_ptr(), idx.data_ptr(),
                                      w.data_ptr(), n, int(rank), int(world), delta.data_ptr(), ws.data_ptr(),
                                      ws.numel(), _stream_ptr(stream))
        L.check(rc, "sb_expert_delta")
        return delta

    def run_recurrent_decode(self, h: torch.Tensor, x0: torch.Tensor, threshold: float, exit_w: torch.Tensor,
                             exit_b: torch.Tensor, stream=None, loop_fn=None, trace: list | None = None):
        """Early-exit decode over all loops (SpiderWebLM._run_recurrent_decode,
        model.py:450-473): h, x0 [B, T, H].  Each loop runs the block on the
        compact rows still active, then sb_active_set_step scatters them back,
        computes the exit confidence and compacts the next loop's inputs on the
        device; the host reads only the new count (as ActiveSet.n_active does).
        ``loop_fn(h, x0, loop_idx, out)`` replaces the block call (the module's
        expert-parallel forward uses it); ``trace`` collects, per loop, host
        copies of the active batch rows, their inputs, outputs and exit
        confidences (dict keys rows, h_in, h_new, conf).  Returns (h [B, T, H],
        loops run)."""
        H = self.cfg.hidden_size
        B = h.shape[0]
        P = h[0].numel() // H if B else 1
        dt = self.act_dtype
        h_full = h.detach().to(self.device, dt).contiguous().clone()
        if B == 0:
            return h_full.to(h.dtype), 0
        self._ensure_workspace(B * P)
        hc = [h_full.clone(), torch.empty_like(h_full)]
        xc = [x0.detach().to(self.device, dt).contiguous().clone(), torch.empty_like(h_full)]
        idx = [torch.arange(B, dtype=torch.int32, device=self.device),
               torch.empty(B, dtype=torch.int32, device=self.device)]
        h_new = torch.empty(B * P, H, dtype=dt, device=self.device)
        flags = torch.empty(B, dtype=torch.int32, device=self.device)
        n_next = torch.zeros(1, dtype=torch.int32, device=self.device)
        conf = torch.empty(B, dtype=torch.float32, device=self.device) if trace is not None else None
        ew = exit_w.detach().reshape(H).to(self.device, torch.float32).contiguous()
        eb = exit_b.detach().reshape(1).to(self.device, torch.float32).contiguous()
        n, cur, loops = B, 0, 0
        for l in range(self.cfg.num_loops):
            if n == 0:
                break
            out = h_new[: n * P]
            if loop_fn is None:
                self.forward(hc[cur][:n], xc[cur][:n], l, l + 1, out=out, stream=stream)
            else:
                loop_fn(hc[cur][:n], xc[cur][:n], l, out)
            nxt = cur ^ 1
            rc = self.lib.sb_active_set_step(self.dims.act_dtype, n, P, H, out.data_ptr(), xc[cur].data_ptr(),
                                             idx[cur].data_ptr(), ew.data_ptr(), eb.data_ptr(), float(threshold),
                                             h_full.data_ptr(), idx[nxt].data_ptr(), hc[nxt].data_ptr(),
                                             xc[nxt].data_ptr(), n_next.data_ptr(), flags.data_ptr(),
                                             conf.data_ptr() if conf is not None else None, _stream_ptr(stream))
            L.check(rc, "sb_active_set_step")
            if trace is not None:
                trace.append(dict(rows=idx[cur][:n].cpu(), h_in=hc[cur][:n].cpu(), h_new=out.view(n, *h.shape[1:]).cpu(),
                                  conf=conf[:n].cpu()))
            if stream is not None:
                stream.synchronize()
            n = int(n_next.item())
            cur = nxt
            loops += 1
        return h_full.to(h.dtype), loops

    def loop_stats(self, h: torch.Tensor, h_out: torch.Tensor | None, loop_idx: int,
                   top_idx: torch.Tensor | None = None, exit_w: torch.Tensor | None = None,
                   exit_b: torch.Tensor | None = None, stream=None) -> dict:
        """return_stats=True statistics of loop loop_idx (sb_loop_stats,
        model.py:327-343): h is the loop's input, h_out its output, top_idx
        [n, K] int32 its routing (None: recomputed).  Returns the reference's
        keys; confidence is None without exit-head weights."""
        cfg = self.cfg
        H, E = cfg.hidden_size, cfg.num_experts
        n = h.numel() // H
        act = lambda t: t.reshape(n, H).to(self.act_dtype).contiguous()  # noqa: E731
        h2 = act(h)
        conf = None
        hp = ew = eb = None
        if exit_w is not None and h_out is not None:
            ho = act(h_out)
            ew = exit_w.detach().reshape(H).to(self.device, torch.float32).contiguous()
            eb = exit_b.detach().reshape(1).to(self.device, torch.float32).contiguous()
            conf = torch.empty(n, dtype=torch.float32, device=self.device)
            hp = ho.data_ptr()
        ti = None
        if top_idx is not None:
            ti = top_idx.reshape(n, cfg.top_k).to(self.device, torch.int32).contiguous()
        probs = torch.empty(n, E, dtype=torch.float32, device=self.device)
        stats = torch.empty(3 * E + 2, dtype=torch.float32, device=self.device)
        nbytes = self.lib.sb_loop_stats_workspace_bytes(C.byref(self.dims), n)
        if nbytes == 0:
            raise L.SpiderB200Error(L.SB_ERR_ARG, "sb_loop_stats_workspace_bytes")
        ws = self._delta_ws(nbytes)
        rc = self.lib.sb_loop_stats(C.byref(self.dims), C.byref(self.weights), int(loop_idx), h2.data_ptr(), hp,
                                    ti.data_ptr() if ti is not None else None, n,
                                    ew.data_ptr() if ew is not None else None, eb.data_ptr() if eb is not None else None,
                                    probs.data_ptr(), conf.data_ptr() if conf is not None else None, stats.data_ptr(),
                                    ws.data_ptr(), ws.numel(), _stream_ptr(stream))
        L.check(rc, "sb_loop_stats")
        return {"router_probs": probs, "expert_load": stats[:E], "edge_load": stats[E:2 * E],
                "edge_importance": stats[2 * E:3 * E], "aux_loss": stats[3 * E], "edge_loss": stats[3 * E + 1],
                "confidence": conf}

    def _delta_ws(self, nbytes: int) -> torch.Tensor:
        ws = getattr(self, "_dws", None)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._dws = ws
        return ws


class CapturedBlock:
    """All loops of a block for a fixed token count, captured in one CUDA graph."""

    def __init__(self, engine: BlockEngine, n_tokens: int, loop_begin: int = 0, loop_end: int | None = None,
                 x0_is_h: bool = False):
        """x0_is_h: the block input is also x0 (the whole recurrent stack from
        its input), so one buffer serves both and a step copies one tensor in."""
        self.engine = engine
        H = engine.cfg.hidden_size
        dev, dt = engine.device, engine.act_dtype
        engine._ensure_workspace(n_tokens)
        self.h = torch.zeros(n_tokens, H, dtype=dt, device=dev)
        self.x0 = self.h if x0_is_h else torch.zeros(n_tokens, H, dtype=dt, device=dev)
        self.out = torch.zeros(n_tokens, H, dtype=dt, device=dev)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            engine.forward(self.h, self.x0, loop_begin, loop_end, out=self.out)  # warm-up (lazy init)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        lib = L.load()
        before = lib.sb_kernel_launches()
        with torch.cuda.graph(self.graph):
            engine.forward(self.h, self.x0, loop_begin, loop_end, out=self.out)
        self.kernels_per_replay = int(lib.sb_kernel_launches() - before)

    def __call__(self, h=None, x0=None):
        if h is not None:
            self.h.copy_(h.reshape(self.h.shape))
        if x0 is not None and self.x0 is not self.h:
            self.x0.copy_(x0.reshape(self.x0.shape))
        self.graph.replay()
        return self.out


class HostPipeline:
    """Block steps from and to pinned host memory with the copies off the
    critical path: two captured graphs on two buffer sets, the input of step
    s + 1 copied in (one stream) and the output of step s - 1 copied out
    (another stream) while step s runs, events ordering each buffer's reuse.
    Every step still moves its own input in and its output out."""

    def __init__(self, engine: BlockEngine, n_tokens: int, loop_begin: int = 0, loop_end: int | None = None,
                 x0_is_h: bool = False):
        dev = engine.device
        self.x0_is_h = x0_is_h
        self.blocks = [CapturedBlock(engine, n_tokens, loop_begin, loop_end, x0_is_h=x0_is_h) for _ in range(2)]
        self.kernels_per_replay = self.blocks[0].kernels_per_replay
        self.h2d = torch.cuda.Stream(device=dev)
        self.d2h = torch.cuda.Stream(device=dev)
        ev = lambda: [torch.cuda.Event(), torch.cuda.Event()]  # noqa: E731
        self.ev_in, self.ev_done, self.ev_out = ev(), ev(), ev()
        self.device = dev

    def run(self, h_hosts, out_hosts, x0_hosts=None) -> None:
        """Steps s = 0.. : out_hosts[s] <- block(h_hosts[s], x0_hosts[s]) (x0 = h
        when the pipeline was built with x0_is_h).  Host tensors should be
        pinned; returns once every step is enqueued (synchronise to read)."""
        if len(out_hosts) < len(h_hosts) or (not self.x0_is_h and (x0_hosts is None or len(x0_hosts) < len(h_hosts))):
            raise ValueError("HostPipeline.run needs an output (and, without x0_is_h, an x0) per input step")
        compute = torch.cuda.current_stream(self.device)
        self.h2d.wait_stream(compute)
        self.d2h.wait_stream(compute)
        for s, h_host in enumerate(h_hosts):
            b = s & 1
            blk = self.blocks[b]
            with torch.cuda.stream(self.h2d):
                if s >= 2:
                    self.h2d.wait_event(self.ev_done[b])  # step s - 2 no longer reads this input
                blk.h.copy_(h_host.reshape(blk.h.shape), non_blocking=True)
                if not self.x0_is_h:
                    blk.x0.copy_(x0_hosts[s].reshape(blk.x0.shape), non_blocking=True)
                self.ev_in[b].record(self.h2d)
            compute.wait_event(self.ev_in[b])
            if s >= 2:
                compute.wait_event(self.ev_out[b])  # step s - 2's output has left this buffer
            blk.graph.replay()
            self.ev_done[b].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.ev_done[b])
                out_hosts[s].copy_(blk.out.reshape(out_hosts[s].shape), non_blocking=True)
                self.ev_out[b].record(self.d2h)
        compute.wait_stream(self.h2d)
        compute.wait_stream(self.d2h)
