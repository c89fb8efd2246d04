"""CPU restatement of the reference's full SpiderWebLM forward -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` import this module.  It stands in for the reference model class
on machines without the reference package, so that the ``spider_b200``
backend can be swapped into a whole model (prelude, recurrent loops, coda,
tied LM head) and its logits compared with the logits the reference itself
produced (``tests/golden/cfg1_model.pt``, written by
``tests/golden/make_golden.py`` from ``spider_moe.model.SpiderWebLM``).

It follows the reference's inference forward without early exit or
statistics:

* ``SpiderWebLM.forward`` (spider_moe/model.py:673-701): token embedding
  (model.py:392-403; with ``use_rope`` the position table is not added),
  prelude layers, ``num_loops`` applications of the recurrent block,
  coda layers, ``final_norm`` and the LM head tied to the token embedding
  (model.py:371-372);
* ``TransformerLayer.forward`` (model.py:134-151): pre-LN attention and a GELU
  MLP of width 4H, both residual;
* ``CausalSelfAttention.forward`` (model.py:38-76): one fused ``qkv``
  projection without bias, rotary embedding of q and k, causal scaled
  dot-product attention, output projection without bias;
* rotary tables and rotation (spider_moe/rope.py:8-44, 67-70);
* the recurrent block through ``oracle.spider_oracle.block_forward``.

Parameters are registered under the reference's names and in its order, so
``named_parameters()`` walks them exactly as the reference model does (the
seeded initialisation of the fixture depends on that order).
"""
from __future__ import annotations

import torch
from torch import nn
import torch.nn.functional as F

from . import spider_oracle as O


def rope_tables(head_dim: int, max_seq_len: int, theta: float = 10000.0):
    """rope.py:8-25: cos / sin tables [max_seq_len, head_dim] (frequencies repeated twice)."""
    half = head_dim // 2
    inv_freq = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) / half))
    ang = torch.outer(torch.arange(max_seq_len, dtype=torch.float32), inv_freq)
    full = torch.cat([ang, ang], dim=-1)
    return full.cos(), full.sin()


def rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """rope.py:28-44, 67-70: x * cos + rotate_half(x) * sin on [B, heads, T, D]."""
    t, d = x.shape[2], x.shape[3]
    c = cos[:t].to(x.dtype).view(1, 1, t, d)
    s = sin[:t].to(x.dtype).view(1, 1, t, d)
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return x * c + torch.cat([-x2, x1], dim=-1) * s


class Attention(nn.Module):
    def __init__(self, hidden: int, heads: int):
        super().__init__()
        self.heads, self.head_dim, self.hidden = heads, hidden // heads, hidden
        self.qkv = nn.Linear(hidden, 3 * hidden, bias=False)
        self.proj = nn.Linear(hidden, hidden, bias=False)

    def forward(self, x, cos, sin):
        b, t, _ = x.shape
        q, k, v = (y.view(b, t, self.heads, self.head_dim).transpose(1, 2) for y in self.qkv(x).chunk(3, dim=-1))
        if cos is not None:
            q, k = rotate(q, cos, sin), rotate(k, cos, sin)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.proj(y.transpose(1, 2).contiguous().view(b, t, self.hidden))


class Layer(nn.Module):
    def __init__(self, hidden: int, heads: int):
        super().__init__()
        self.ln1 = nn.LayerNorm(hidden)
        self.attn = Attention(hidden, heads)
        self.ln2 = nn.LayerNorm(hidden)
        self.ffn = nn.Sequential(nn.Linear(hidden, 4 * hidden), nn.GELU(), nn.Linear(4 * hidden, hidden),
                                 nn.Dropout(0.0))

    def forward(self, x, cos, sin):
        x = x + self.attn(self.ln1(x), cos, sin)
        return x + self.ffn(self.ln2(x))


class Block(nn.Module):
    """The recurrent block's parameters under the reference names (model.py:165-216),
    computed by the oracle restatement."""

    def __init__(self, cfg):
        super().__init__()
        h, e = cfg.hidden_size, cfg.num_experts
        self.cfg = cfg
        self.loop_bias = nn.Parameter(torch.zeros(cfg.num_loops, e))
        self.router = nn.Linear(h, e, bias=False)
        self.loop_embedding = nn.Embedding(cfg.num_loops, cfg.loop_embed_size)
        self.edge_generator = nn.Linear(h + cfg.loop_embed_size, e * e)
        self.edge_value = nn.ModuleList([nn.Linear(h, h, bias=False) for _ in range(e)])
        self.experts = nn.ModuleList([nn.Sequential(nn.Linear(h, cfg.expert_ffn_size), nn.GELU(),
                                                    nn.Linear(cfg.expert_ffn_size, h)) for _ in range(e)])
        self.norm = nn.LayerNorm(h)
        self.exit_head = nn.Linear(h, 1)

    def forward(self, h, x0, loop_idx):
        p = O.params_from_state_dict({k: v.detach() for k, v in self.state_dict().items()}, self.cfg.num_experts)
        return O.block_forward(p, h, x0, loop_idx, self.cfg, activation="gelu")["h_out"]


class OracleSpiderWebLM(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        h = cfg.hidden_size
        self.token_embedding = nn.Embedding(cfg.vocab_size, h)
        self.position_embedding = nn.Embedding(cfg.max_seq_len, h)
        self.prelude = nn.ModuleList([Layer(h, cfg.num_heads) for _ in range(cfg.num_prelude_layers)])
        self.recurrent = Block(cfg)
        self.coda = nn.ModuleList([Layer(h, cfg.num_heads) for _ in range(cfg.num_coda_layers)])
        self.final_norm = nn.LayerNorm(h)
        self.lm_head = nn.Linear(h, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.token_embedding.weight  # tied (model.py:371-372)
        self.use_rope = bool(cfg.use_rope)
        cos, sin = rope_tables(h // cfg.num_heads, cfg.max_seq_len, cfg.rope_theta) if self.use_rope else (None, None)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def _embed(self, ids):
        tok = self.token_embedding(ids)
        if self.use_rope:
            return tok
        return tok + self.position_embedding(torch.arange(ids.shape[1], device=ids.device)).unsqueeze(0)

    def _run_recurrent_full(self, h, x0):
        """model.py:445-448."""
        for loop_idx in range(self.cfg.num_loops):
            h = self.recurrent(h, x0, loop_idx)
        return h

    def forward(self, ids):
        """model.py:673-701 (no early exit, no statistics, no loss)."""
        x0 = self._embed(ids)
        h = x0
        for layer in self.prelude:
            h = layer(h, self.rope_cos, self.rope_sin)
        for loop_idx in range(self.cfg.num_loops):
            h = self.recurrent(h, x0, loop_idx)
        for layer in self.coda:
            h = layer(h, self.rope_cos, self.rope_sin)
        return {"logits": self.lm_head(self.final_norm(h)), "loops_used": self.cfg.num_loops}


@torch.no_grad()
def seeded_init_(model: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    """The fixture's initialisation (tests/golden/make_golden.py, cfg1_full_model):
    every parameter in named_parameters() order drawn N(0, std) from one
    generator, then loop_bias zero and every LayerNorm weight 1 / bias 0."""
    g = torch.Generator().manual_seed(seed)
    for name, p in model.named_parameters():
        if name == "recurrent.loop_bias":
            p.zero_()
        else:
            p.copy_(torch.empty(p.shape).normal_(0.0, std, generator=g))
    for mod in model.modules():
        if isinstance(mod, nn.LayerNorm):
            mod.weight.fill_(1.0)
            mod.bias.fill_(0.0)
