"""Shared helpers for the parity tests (test infrastructure)."""
from __future__ import annotations

import os

import torch

from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances (relative to each row's max-norm: max|a-b| / max|b|), as stated
# for this path: fp32 1e-5, bf16 / fp8 2e-2, int4 3e-2.
TOL = {"fp32": 1e-5, "bf16": 2e-2, "fp8": 2e-2, "int4": 3e-2}
# A gap between consecutive sorted candidates below this (relative) is a tie
# at fp32 rounding level: index order there is not defined by the arithmetic.
TIE_REL = 1e-5


def load_golden(name: str) -> dict:
    return torch.load(os.path.join(GOLDEN, name + ".pt"), weights_only=False)


def golden_cfg(fx: dict) -> ModelConfig:
    kw = dict(vocab_size=512, num_heads=4)
    kw.update(fx["cfg"])
    return ModelConfig(**kw).validate()


def golden_state(fx: dict, cfg: ModelConfig) -> dict:
    """Parameters of a fixture: stored, or regenerated from its seed."""
    if "state_dict" in fx:
        return {k: v.float() for k, v in fx["state_dict"].items()}
    sd = synth.synthetic_state_dict(cfg, seed=fx["seed"], device="cpu", zipf=fx["zipf"],
                                    round_bf16=bool(fx["bf16"]))
    return sd


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().float().cpu().reshape(-1, a.shape[-1])
    b = b.detach().float().cpu().reshape(-1, b.shape[-1])
    if a.numel() == 0:
        return 0.0
    den = b.abs().amax(dim=-1).clamp_min(1e-30)
    return float(((a - b).abs().amax(dim=-1) / den).max())


def topk_tie_mask(values: torch.Tensor, k: int) -> torch.Tensor:
    """True where the top-k set / order is within fp32 rounding of a tie."""
    srt = values.float().sort(dim=-1, descending=True).values
    kk = min(k + 1, srt.shape[-1])
    gaps = (srt[..., : kk - 1] - srt[..., 1:kk]).abs()
    scale = srt[..., :kk].abs().amax(dim=-1, keepdim=True).clamp_min(1.0)
    return (gaps < TIE_REL * scale).any(dim=-1)


def compare_indices(got: torch.Tensor, want: torch.Tensor, ties: torch.Tensor) -> tuple[int, int]:
    """Return (mismatching rows outside ties, number of tie rows). Rows = leading dims."""
    got = got.cpu().long().reshape(ties.numel(), -1)
    want = want.cpu().long().reshape(ties.numel(), -1)
    bad = (got != want).any(dim=-1) & ~ties.reshape(-1)
    return int(bad.sum()), int(ties.sum())
