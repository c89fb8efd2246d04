"""Seeded synthetic parameters and inputs for the Spider-MoE block.

The reference publishes no checkpoints or datasets for this block, so every
measurement and parity case uses seeded synthetic data:

* every weight and bias ~ N(0, 0.02) drawn from one ``torch.Generator`` in
  ``named_parameters()`` order (the order of spider_moe/model.py:165-216, which
  this package's module reproduces), LayerNorm weights 1 and biases 0 (the
  block's and Lumen's);
* ``loop_bias`` zero, or a Zipf(s) bias per expert (the reference has no Zipf
  option; its own ``loop_bias[num_loops, E]`` parameter, added to the router
  logits at spider_moe/model.py:255, is the hook);
* hidden states ~ N(0, 1) and ``x0 = h``.
"""
from __future__ import annotations

import math

import torch


def _is_layer_norm(name: str) -> bool:
    """The block's LayerNorm and Lumen's (weight 1, bias 0)."""
    return name.startswith("norm.") or name.startswith("lumen.norm.")


def block_param_shapes(cfg) -> list:
    """(name, shape) of every SpiderMoELayer parameter in named_parameters() order
    (spider_moe/model.py:165-216; SwiGLU gates, a B200 extra, come last)."""
    h, e, u = cfg.hidden_size, cfg.num_experts, cfg.expert_ffn_size
    lp, le = cfg.num_loops, cfg.loop_embed_size
    out = [("loop_bias", (lp, e)), ("router.weight", (e, h)), ("loop_embedding.weight", (lp, le)),
           ("edge_generator.weight", (e * e, h + le)), ("edge_generator.bias", (e * e,))]
    out += [(f"edge_value.{i}.weight", (h, h)) for i in range(e)]
    for i in range(e):
        out += [(f"experts.{i}.0.weight", (u, h)), (f"experts.{i}.0.bias", (u,)),
                (f"experts.{i}.2.weight", (h, u)), (f"experts.{i}.2.bias", (h,))]
    out += [("norm.weight", (h,)), ("norm.bias", (h,)), ("exit_head.weight", (1, h)), ("exit_head.bias", (1,))]
    if getattr(cfg, "use_lumen", False):  # LumenWorkspace (lumen.py:62-79): own parameter first
        s = int(getattr(cfg, "lumen_slots", 8))
        d = int(getattr(cfg, "lumen_slot_dim", 0) or max(32, h // 4))
        out += [("lumen.slot_bias", (s,)), ("lumen.write_q.weight", (s, h)), ("lumen.write_v.weight", (d, h)),
                ("lumen.slot_to_h.weight", (h, d)), ("lumen.gate.weight", (1, 2 * h)), ("lumen.gate.bias", (1,)),
                ("lumen.norm.weight", (h,)), ("lumen.norm.bias", (h,))]
    if getattr(cfg, "expert_activation", "gelu") == "swiglu":
        for i in range(e):
            out += [(f"expert_gates.{i}.weight", (u, h)), (f"expert_gates.{i}.bias", (u,))]
    return out


def synthetic_state_dict(cfg, seed: int = 0, device="cpu", std: float = 0.02, zipf: float | None = None,
                         zipf_seed: int = 0, round_bf16: bool = False) -> dict:
    """fp32 parameters drawn in named_parameters() order from one generator on `device`.

    With device="cpu" this draws exactly what ``init_block_params_`` writes into
    a module of the same config.
    """
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(int(seed))
    sd = {}
    for name, shape in block_param_shapes(cfg):
        if _is_layer_norm(name):
            t = torch.full(shape, 1.0 if name.endswith("weight") else 0.0, device=dev)
        elif name == "loop_bias":
            t = torch.zeros(shape, device=dev)
            if zipf is not None:
                t.copy_(zipf_loop_bias(shape[0], shape[1], zipf, zipf_seed))
        else:
            t = torch.empty(shape, dtype=torch.float32, device=dev).normal_(0.0, std, generator=g)
        if round_bf16:
            t = t.to(torch.bfloat16).float()
        sd[name] = t
    return sd


def init_block_params_(module: torch.nn.Module, seed: int = 0, std: float = 0.02,
                       zipf: float | None = None, zipf_seed: int = 0) -> None:
    """Overwrite every parameter of a SpiderMoELayer-shaped module in place."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    with torch.no_grad():
        for name, p in module.named_parameters():
            if _is_layer_norm(name):
                p.fill_(1.0 if name.endswith("weight") else 0.0)
                continue
            if name == "loop_bias":
                p.zero_()
                continue
            t = torch.empty(p.shape, dtype=torch.float32).normal_(0.0, std, generator=g)
            p.copy_(t.to(p.dtype))
        if zipf is not None:
            e = module.loop_bias.shape[1]
            module.loop_bias.copy_(zipf_loop_bias(module.loop_bias.shape[0], e, zipf, zipf_seed))


def zipf_loop_bias(num_loops: int, num_experts: int, s: float = 1.1, seed: int = 0) -> torch.Tensor:
    """``bias[l, perm[e]] = ln(p_e)`` with ``p_e = (e+1)^-s / sum_j (j+1)^-s``."""
    ranks = torch.arange(1, num_experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    logp = (p / p.sum()).log().float()
    perm = torch.randperm(num_experts, generator=torch.Generator().manual_seed(int(seed)))
    row = torch.empty(num_experts, dtype=torch.float32)
    row[perm] = logp
    return row.unsqueeze(0).expand(num_loops, num_experts).contiguous()


def round_params_to_bf16_(module: torch.nn.Module) -> None:
    """Make every parameter bf16-representable (kept in its storage dtype)."""
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(p.to(torch.bfloat16).to(p.dtype))


def block_inputs(tokens: int, hidden: int, seed: int = 1, device="cpu",
                 dtype=torch.float32):
    """h ~ N(0,1) as [1, tokens, hidden]; x0 = h (the block input)."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    h = torch.randn(1, tokens, hidden, generator=g, dtype=torch.float32)
    if dtype == torch.bfloat16:
        h = h.to(torch.bfloat16)
    else:
        h = h.to(dtype)
    h = h.to(device)
    return h, h.clone()


def per_channel_fp8_scales(w: torch.Tensor) -> torch.Tensor:
    """Per-output-channel scale ``amax(|w|, dim=-1) / 448`` clamped at 1e-12, fp32 [..., out]."""
    return (w.detach().float().abs().amax(dim=-1) / 448.0).clamp_min(1e-12)


def zipf_expected_share(num_experts: int, s: float = 1.1):
    ranks = [math.pow(e + 1, -s) for e in range(num_experts)]
    z = sum(ranks)
    return [r / z for r in ranks]
