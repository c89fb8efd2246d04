"""CPU oracle for the recurrent Spider-MoE block -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The B200 package never imports anything under ``oracle/``.

It restates, in plain fp32 PyTorch on the CPU, the algorithm of the reference
block ``SpiderMoELayer.forward`` (spider_moe/model.py:240-317), its sparse
expert FFN (spider_moe/sparse_experts.py:11-68), the dispatch plan
(spider_infer/forge/ep/dispatch.py:56-115) and the quantisation formats
(spider_moe/quant.py:30-169).  Every function cites the lines it follows.

Pinning: ``tests/test_oracle_golden.py`` checks this restatement against
fixtures captured from the reference itself (``tests/golden/make_golden.py``
imports the reference package and records its intermediates) and against the
known-answer tests of the reference's own test suites; ``oracle/ref_scalar.py``
additionally runs the reference's scalar C++ sub-step library built from its
sources by ``oracle/Makefile``.

Two restatement choices, both exact in real arithmetic:

* messages are formed from the per-(token, destination) coefficient
  ``c[n,d] = sum_{src in topK(n)} sum_m w[n,src,m] [dst(n,src,m) = d]`` and only
  the destinations with a coefficient are transformed; the reference transforms
  all E destinations and multiplies the inactive ones by zero
  (spider_moe/model.py:271-288);
* the expert FFN visits experts in ascending id exactly as the reference does.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

FP8_E4M3_MAX = 448.0  # spider_moe/quant.py:13


# ---------------------------------------------------------------------------
# parameters
# ---------------------------------------------------------------------------

@dataclass
class BlockParams:
    """Stacked fp32 views of a SpiderMoELayer state dict (names of model.py:165-216)."""
    router_w: torch.Tensor      # [E, H]            router.weight
    loop_bias: torch.Tensor     # [L, E]            loop_bias
    loop_emb: torch.Tensor      # [L, Le]           loop_embedding.weight
    gen_w: torch.Tensor         # [E*E, H+Le]       edge_generator.weight
    gen_b: torch.Tensor         # [E*E]             edge_generator.bias
    edge_w: torch.Tensor        # [E, H, H]         edge_value.{i}.weight
    w_up: torch.Tensor          # [E, U, H]         experts.{i}.0.weight
    b_up: torch.Tensor          # [E, U]            experts.{i}.0.bias
    w_down: torch.Tensor        # [E, H, U]         experts.{i}.2.weight
    b_down: torch.Tensor        # [E, H]            experts.{i}.2.bias
    ln_w: torch.Tensor          # [H]               norm.weight
    ln_b: torch.Tensor          # [H]               norm.bias
    w_gate: torch.Tensor | None = None  # [E, U, H]  SwiGLU gate (B200 extra mode)
    b_gate: torch.Tensor | None = None  # [E, U]
    lumen: dict | None = None           # lumen.* parameters (model.py:202-210) when use_lumen

    @property
    def num_experts(self):
        return self.router_w.shape[0]


def params_from_state_dict(sd: dict, num_experts: int) -> BlockParams:
    f = lambda t: t.detach().float().cpu()  # noqa: E731
    e = num_experts
    gates = [k for k in sd if k.startswith("expert_gates.")]
    return BlockParams(
        router_w=f(sd["router.weight"]),
        loop_bias=f(sd["loop_bias"]),
        loop_emb=f(sd["loop_embedding.weight"]),
        gen_w=f(sd["edge_generator.weight"]),
        gen_b=f(sd["edge_generator.bias"]),
        edge_w=torch.stack([f(sd[f"edge_value.{i}.weight"]) for i in range(e)]),
        w_up=torch.stack([f(sd[f"experts.{i}.0.weight"]) for i in range(e)]),
        b_up=torch.stack([f(sd[f"experts.{i}.0.bias"]) for i in range(e)]),
        w_down=torch.stack([f(sd[f"experts.{i}.2.weight"]) for i in range(e)]),
        b_down=torch.stack([f(sd[f"experts.{i}.2.bias"]) for i in range(e)]),
        ln_w=f(sd["norm.weight"]),
        ln_b=f(sd["norm.bias"]),
        w_gate=torch.stack([f(sd[f"expert_gates.{i}.weight"]) for i in range(e)]) if gates else None,
        b_gate=torch.stack([f(sd[f"expert_gates.{i}.bias"]) for i in range(e)]) if gates else None,
        lumen={k[len("lumen."):]: f(v) for k, v in sd.items() if k.startswith("lumen.")} or None,
    )


# ---------------------------------------------------------------------------
# the block, step by step
# ---------------------------------------------------------------------------

def router(h: torch.Tensor, router_w: torch.Tensor, bias_l: torch.Tensor, top_k: int):
    """spider_moe/model.py:254-258: logits + loop bias, fp32 softmax, top-k of the
    probabilities (sorted descending), renormalised with a 1e-9 floor.

    h: [N, H] fp32.  Returns (top_w [N,K] fp32, top_idx [N,K] int64, probs [N,E]).
    """
    logits = F.linear(h, router_w) + bias_l.view(1, -1)
    probs = logits.float().softmax(dim=-1)
    top_w, top_idx = probs.topk(top_k, dim=-1)
    top_w = top_w / top_w.sum(dim=-1, keepdim=True).clamp_min(1e-9)
    return top_w, top_idx, probs


def edge_graph(h: torch.Tensor, emb_l: torch.Tensor, gen_w: torch.Tensor, gen_b: torch.Tensor,
               num_experts: int, edges: int):
    """spider_moe/model.py:260-266: edge logits from [h || loop_emb] through the
    edge generator, viewed [N, E_src, E_dst]; top-M over destinations (sorted
    descending) and an fp32 softmax over the M selected logits.

    Returns (edge_idx [N,E,M] int64, edge_w [N,E,M] fp32, edge_logits [N,E,E]).
    """
    n = h.shape[0]
    e = num_experts
    feat = torch.cat([h, emb_l.view(1, -1).expand(n, -1)], dim=-1)
    logits = F.linear(feat, gen_w, gen_b).view(n, e, e)
    vals, idx = logits.topk(edges, dim=-1)
    return idx, vals.float().softmax(dim=-1), logits


def destination_coefficients(top_idx: torch.Tensor, edge_idx: torch.Tensor,
                             edge_w: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Per-(token, destination) weight of the message sum of model.py:274-288.

    The source mask is binary (``scatter_`` of 1.0, model.py:277-278), so source
    ``s`` contributes ``edge_w[n, s, m]`` to destination ``edge_idx[n, s, m]``
    when ``s`` is one of the token's router top-k.  Returns c [N, E] fp32.
    """
    n, k = top_idx.shape
    m = edge_idx.shape[-1]
    src_active = torch.zeros(n, num_experts)
    src_active.scatter_(-1, top_idx, 1.0)
    w = edge_w * src_active.unsqueeze(-1)                      # [N, E, M]
    c = torch.zeros(n, num_experts)
    c.scatter_add_(-1, edge_idx.reshape(n, -1), w.reshape(n, -1))
    return c


def messages_from_coefficients(h: torch.Tensor, edge_weights: torch.Tensor,
                               coef: torch.Tensor) -> torch.Tensor:
    """messages[n] = sum_d c[n,d] * (W_edge[d] @ h[n])  (model.py:271-288)."""
    out = torch.zeros_like(h)
    for d in range(edge_weights.shape[0]):
        rows = (coef[:, d] != 0).nonzero(as_tuple=False).flatten()
        if rows.numel() == 0:
            continue
        out[rows] += coef[rows, d].unsqueeze(-1) * F.linear(h[rows], edge_weights[d])
    return out


def messages_dense(h: torch.Tensor, edge_weights: torch.Tensor, top_idx: torch.Tensor,
                   edge_idx: torch.Tensor, edge_w: torch.Tensor) -> torch.Tensor:
    """model.py:271-288 as the reference computes it: every token through all E
    destination transforms, gather of the selected ones, binary source mask,
    weighted sum.  (Used as the timed CPU reference; same result as the sparse form.)"""
    n, width = h.shape
    e, m = edge_idx.shape[1], edge_idx.shape[2]
    transformed = torch.einsum("nh,eoh->neo", h, edge_weights)            # [N, E, H]
    src_active = torch.zeros(n, e)
    src_active.scatter_(-1, top_idx, 1.0)
    gathered = torch.gather(transformed, 1, edge_idx.reshape(n, e * m, 1).expand(n, e * m, width))
    w = edge_w * src_active.unsqueeze(-1)
    return (gathered.view(n, e, m, width) * w.unsqueeze(-1)).sum(dim=(1, 2))


def dispatch_plan(top_idx: torch.Tensor, top_w: torch.Tensor, num_experts: int,
                  local_experts=None):
    """spider_infer/forge/ep/dispatch.py:56-115: experts in ascending id; for
    each, ``tw = sum_k w_k [idx_k == e]``; the expert's tokens are the ascending
    positions with ``tw > 0`` and their weights ``tw[pos]``.

    Returns a list of (expert_id, positions int64[n_e], weights fp32[n_e]).
    """
    flat_idx = top_idx.reshape(-1, top_idx.shape[-1])
    flat_w = top_w.reshape(-1, top_w.shape[-1]).float()
    ids = range(num_experts) if local_experts is None else local_experts
    plan = []
    for eid in ids:
        tw = torch.zeros(flat_idx.shape[0])
        for slot in range(flat_idx.shape[1]):
            tw = tw + flat_w[:, slot] * (flat_idx[:, slot] == eid).float()
        active = tw > 0
        if not active.any():
            continue
        pos = active.nonzero(as_tuple=False).flatten()
        plan.append((int(eid), pos, tw[pos]))
    return plan


def plan_offsets(plan, num_experts: int):
    """Flatten a dispatch plan into (offsets [E+1], tokens [P], weights [P])."""
    counts = torch.zeros(num_experts, dtype=torch.int64)
    toks, ws = [], []
    for eid, pos, w in plan:
        counts[eid] = pos.numel()
        toks.append(pos)
        ws.append(w)
    offsets = torch.zeros(num_experts + 1, dtype=torch.int64)
    offsets[1:] = counts.cumsum(0)
    tok = torch.cat(toks) if toks else torch.zeros(0, dtype=torch.int64)
    w = torch.cat(ws) if ws else torch.zeros(0)
    return offsets, tok, w


def expert_ffn(x: torch.Tensor, w_up, b_up, w_down, b_down, activation="gelu",
               w_gate=None, b_gate=None) -> torch.Tensor:
    """One expert: sparse_experts.py:59-62 (Linear -> erf-GELU -> Linear).

    ``activation="swiglu"`` is the B200 extra mode
    ``down(silu(gate(x) + b_gate) * (up(x) + b_up)) + b_down``.
    """
    up = F.linear(x, w_up, b_up)
    if activation == "gelu":
        act = F.gelu(up)
    elif activation == "swiglu":
        act = F.silu(F.linear(x, w_gate, b_gate)) * up
    else:
        raise ValueError(activation)
    return F.linear(act, w_down, b_down)


def expert_delta(messages: torch.Tensor, top_idx: torch.Tensor, top_w: torch.Tensor,
                 w_up, b_up, w_down, b_down, num_experts: int, local_experts=None,
                 activation="gelu", w_gate=None, b_gate=None) -> torch.Tensor:
    """spider_experts.sparse_expert_delta (sparse_experts.py:11-68) without the
    cross-rank all-reduce: ``delta[active] += ffn_e(x[active]) * tw[active]``
    for each local expert in ascending id."""
    width = messages.shape[-1]
    flat = messages.reshape(-1, width).float()
    delta = torch.zeros_like(flat)
    for eid, pos, tw in dispatch_plan(top_idx, top_w, num_experts, local_experts):
        y = expert_ffn(flat[pos], w_up[eid], b_up[eid], w_down[eid], b_down[eid], activation,
                       None if w_gate is None else w_gate[eid],
                       None if b_gate is None else b_gate[eid])
        delta[pos] = delta[pos] + y * tw.unsqueeze(-1)
    return delta.view(messages.shape)


def block_epilogue(h, delta, x0, ln_w, ln_b, residual_scale=0.5, reinject=0.1, eps=1e-5):
    """spider_moe/model.py:317: LayerNorm(h + a*delta + b*x0) (nn.LayerNorm, eps 1e-5)."""
    u = h + residual_scale * delta + reinject * x0
    return F.layer_norm(u, (u.shape[-1],), ln_w, ln_b, eps)


def lumen_forward(h: torch.Tensor, lp: dict, eps: float = 1e-5, j_lens: bool = False):
    """LumenWorkspace.forward (spider_moe/lumen.py:81-123) in fp32, dropout off.

    lp holds the module's parameters by their names under ``lumen.``
    (slot_bias, write_q.weight, write_v.weight, slot_to_h.weight, gate.weight,
    gate.bias, norm.weight, norm.bias, optional j_lens.weight).  Returns
    (out, state dict with slots, slot_weights, broadcast, j_logits)."""
    h = h.float()
    w = (F.linear(h, lp["write_q.weight"]) + lp["slot_bias"]).softmax(dim=-1)   # competition over slots
    values = F.linear(h, lp["write_v.weight"])
    slots = torch.einsum("...s,...d->...sd", w, values)                        # every token writes every slot
    mixed = torch.einsum("...s,...sd->...d", w, slots)                         # read back with the same weights
    raw = F.linear(mixed, lp["slot_to_h.weight"])
    gate = torch.sigmoid(F.linear(torch.cat([h, raw], dim=-1), lp["gate.weight"], lp["gate.bias"]))
    broadcast = gate * raw
    out = F.layer_norm(h + broadcast, (h.shape[-1],), lp["norm.weight"], lp["norm.bias"], eps)
    j_logits = None
    if j_lens and "j_lens.weight" in lp:
        j_logits = F.linear(slots.mean(dim=-2), lp["j_lens.weight"])
    return out, dict(slots=slots, slot_weights=w, broadcast=broadcast, j_logits=j_logits)


def block_forward(p: BlockParams, h: torch.Tensor, x0: torch.Tensor, loop_idx: int, cfg,
                  activation: str | None = None, local_experts=None, dense: bool = False) -> dict:
    """One SpiderMoELayer.forward (model.py:240-317) on fp32 CPU tensors.

    h, x0: [..., H].  Returns every intermediate the parity tests compare.
    """
    shape = h.shape
    hid = h.reshape(-1, shape[-1]).float()
    x0f = x0.reshape(-1, shape[-1]).float()
    e, k, m = cfg.num_experts, cfg.top_k, cfg.edges_per_expert
    act = activation or getattr(cfg, "expert_activation", "gelu")
    top_w, top_idx, probs = router(hid, p.router_w, p.loop_bias[loop_idx], k)
    edge_idx, edge_w, edge_logits = edge_graph(hid, p.loop_emb[loop_idx], p.gen_w, p.gen_b, e, m)
    coef = destination_coefficients(top_idx, edge_idx, edge_w, e)
    if dense:
        msgs = messages_dense(hid, p.edge_w, top_idx, edge_idx, edge_w)
    else:
        msgs = messages_from_coefficients(hid, p.edge_w, coef)
    delta = expert_delta(msgs, top_idx, top_w, p.w_up, p.b_up, p.w_down, p.b_down, e,
                         local_experts, act, p.w_gate, p.b_gate)
    out = block_epilogue(hid, delta, x0f, p.ln_w, p.ln_b, cfg.residual_scale, cfg.re_inject_weight)
    lumen = None
    if p.lumen is not None:  # model.py:318-323
        out, lumen = lumen_forward(out, p.lumen)
    return dict(top_idx=top_idx, top_w=top_w, probs=probs, edge_idx=edge_idx, edge_w=edge_w,
                edge_logits=edge_logits, coef=coef, messages=msgs, delta=delta,
                h_out=out.view(shape), lumen=lumen)


def loop_stats(r: dict, exit_w: torch.Tensor, exit_b: torch.Tensor, num_experts: int) -> dict:
    """Statistics of SpiderMoELayer.forward(..., return_stats=True)
    (model.py:327-343) from one block_forward result ``r``: router / edge load
    histograms over ALL E sources' top-M destinations (model.py:329-330), the
    importance-weighted edge load, both auxiliary losses and the exit-head
    confidence of the loop's output."""
    e = num_experts
    load = torch.bincount(r["top_idx"].reshape(-1), minlength=e).float()
    load = load / load.sum().clamp_min(1.0)
    edge_load = torch.bincount(r["edge_idx"].reshape(-1), minlength=e).float()
    edge_load = edge_load / edge_load.sum().clamp_min(1.0)
    importance = r["edge_w"].new_zeros(e).scatter_add(0, r["edge_idx"].reshape(-1), r["edge_w"].reshape(-1))
    importance = importance / importance.sum().clamp_min(1e-9)
    probs = r["probs"].reshape(-1, e)
    aux = e * torch.sum(load * probs.mean(dim=0))
    edge_aux = e * torch.sum(edge_load * importance)
    out = r["h_out"].reshape(-1, r["h_out"].shape[-1]).float()
    confidence = torch.sigmoid(F.linear(out, exit_w.float().view(1, -1), exit_b.float().view(1))).squeeze(-1)
    st = dict(router_probs=probs, expert_load=load, edge_load=edge_load, edge_importance=importance,
              aux_loss=aux, edge_loss=edge_aux, confidence=confidence)
    if r.get("lumen") is not None:  # model.py:346-348
        st["lumen_slot_weights"] = r["lumen"]["slot_weights"]
        st["lumen_broadcast_norm"] = r["lumen"]["broadcast"].norm(dim=-1)
    return st


def run_recurrent_decode(p: BlockParams, h, x0, cfg, exit_w, exit_b, threshold: float, confidences=None):
    """SpiderWebLM._run_recurrent_decode with early_exit=True (model.py:450-473)
    and the ActiveSet primitives (active_set.py: all_active, drop,
    compact_active, scatter_active): each loop runs the block on the batch rows
    still active, writes their outputs back, and drops the rows whose
    exit-head confidence at position 0 exceeds the threshold.

    h, x0: [B, T, H].  Returns (h [B, T, H], the active row lists per loop);
    ``confidences`` (a list) collects each loop's confidences."""
    h = h.float().clone()
    x0 = x0.float()
    indices = torch.arange(h.shape[0])
    trace = []
    for loop_idx in range(cfg.num_loops):
        if indices.numel() == 0:
            break
        trace.append(indices.clone())
        h_act = h.index_select(0, indices)
        x0_act = x0.index_select(0, indices)
        h_new = block_forward(p, h_act, x0_act, loop_idx, cfg)["h_out"]
        h.index_copy_(0, indices, h_new)
        conf = torch.sigmoid(F.linear(h_new, exit_w.float().view(1, -1), exit_b.float().view(1))).squeeze(-1)
        if conf.ndim > 1:
            conf = conf[:, 0]
        if confidences is not None:
            confidences.append(conf)
        indices = indices[~(conf > threshold)]
    return h, trace


def run_loops(p: BlockParams, h, x0, cfg, activation=None, dense: bool = False):
    """SpiderWebLM._run_recurrent_full (model.py:445-448): L applications."""
    outs = []
    for l in range(cfg.num_loops):
        r = block_forward(p, h, x0, l, cfg, activation, dense=dense)
        outs.append(r)
        h = r["h_out"]
    return h, outs


# ---------------------------------------------------------------------------
# quantisation formats (spider_moe/quant.py)
# ---------------------------------------------------------------------------

def quantize_int4(weight: torch.Tensor, group_size: int = 64):
    """quant.py:89-117: symmetric per-group INT4 along the last dim, scale =
    amax/7 (floor 1e-8), q = round(w/s) clamped to [-8, 7], two values per
    byte with the even index in the low nibble.  Returns (packed u8, scales fp32)."""
    *lead, n = weight.shape
    if n % 2:
        raise ValueError("last dimension must be even for INT4 packing")
    g = group_size if (group_size > 0 and n % group_size == 0) else n
    w = weight.detach().float().reshape(-1, n)
    wg = w.view(w.shape[0], n // g, g)
    scales = wg.abs().amax(dim=-1).clamp_min(1e-8) / 7.0
    q = torch.round(wg / scales.unsqueeze(-1)).clamp(-8, 7).to(torch.int8).view(w.shape[0], n)
    packed = ((q[:, 0::2] & 0x0F).to(torch.uint8) | ((q[:, 1::2] & 0x0F).to(torch.uint8) << 4))
    return packed.view(*lead, n // 2).contiguous(), scales.view(*lead, n // g).contiguous()


def dequantize_int4(packed: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    """quant.py:120-143: unpack nibbles (two's complement), multiply by the group
    scale in fp32."""
    *lead, half = packed.shape
    n = half * 2
    flat = packed.reshape(-1, half)
    lo = (flat & 0x0F).to(torch.int16)
    hi = ((flat >> 4) & 0x0F).to(torch.int16)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    q = torch.stack([lo, hi], dim=-1).reshape(flat.shape[0], n).float()
    g = group_size
    w = q.view(q.shape[0], n // g, g) * scales.reshape(q.shape[0], n // g, 1).float()
    return w.view(*lead, n)


def quantize_fp8_per_channel(w: torch.Tensor):
    """Per-output-channel e4m3 via quant.py:146-158 with scale[out] = amax/448
    (floor 1e-12).  Returns (q float8_e4m3fn [..., out, in], scale fp32 [..., out])."""
    s = (w.detach().float().abs().amax(dim=-1) / FP8_E4M3_MAX).clamp_min(1e-12)
    q = (w.float() / s.unsqueeze(-1).clamp_min(1e-12)).to(torch.float8_e4m3fn)
    return q, s


def dequantize_fp8_per_channel(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """quant.py:161-169: (fp32(q) * scale) in fp32."""
    return q.float() * s.float().unsqueeze(-1)


# ---------------------------------------------------------------------------
# tie detection for the bit-exact index comparisons
# ---------------------------------------------------------------------------

def topk_margin(values: torch.Tensor, k: int) -> torch.Tensor:
    """Gap, along the last dim, between the k-th and (k+1)-th largest value and
    between consecutive selected values (smallest of these gaps).  A gap at
    fp32 rounding level means the index order is not defined by the math."""
    srt = values.sort(dim=-1, descending=True).values
    kk = min(k + 1, srt.shape[-1])
    gaps = srt[..., : kk - 1] - srt[..., 1:kk]
    if gaps.shape[-1] == 0:
        return torch.full(values.shape[:-1], math.inf)
    return gaps.min(dim=-1).values


def relative_error(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |a-b| / max |b| per row, worst row (relative to each row's max-norm)."""
    a = a.float().reshape(-1, a.shape[-1])
    b = b.float().reshape(-1, b.shape[-1])
    den = b.abs().amax(dim=-1).clamp_min(1e-30)
    return float(((a - b).abs().amax(dim=-1) / den).max()) if a.numel() else 0.0
