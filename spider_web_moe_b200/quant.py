"""Expert weight formats, identical to the reference's (spider_moe/quant.py).

* int4: symmetric per-group along the last (reduction) dim, scale =
  amax/7 with a 1e-8 floor, ``q = round(w/s)`` clamped to [-8, 7], two values
  per byte with the even index in the low nibble (quant.py:89-117).  The
  device kernels read bf16 group scales, so ``Int4Tensor.device_scales()``
  rounds the fp32 scales to bf16 (the reference dequantises with fp32 scales;
  a model quantised for this backend uses the bf16-rounded scales on both
  sides).
* fp8: e4m3 with one fp32 scale per output row, ``s = amax(|w|)/448`` with a
  1e-12 floor, quantised by ``quantize_fp8_with_scale_tensor(w, s[:, None])``
  (quant.py:146-158) and dequantised as ``fp32(q) * s`` (quant.py:161-169).

The packing is a format that must match the reference byte for byte, so the
steps are the reference's steps (the golden vectors in tests/golden pin it).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

FP8_E4M3_MAX = 448.0


@dataclass
class Int4Tensor:
    """Packed INT4 weights with per-group scales (the reference's container)."""
    packed: torch.Tensor   # uint8 [..., n/2]
    scales: torch.Tensor   # fp32  [..., n/group_size]
    shape: tuple
    group_size: int

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        return dequantize_int4(self.packed, self.scales, self.shape, self.group_size, dtype)

    def device_scales(self) -> torch.Tensor:
        return self.scales.to(torch.bfloat16)


def quantize_int4(weight: torch.Tensor, group_size: int = 64) -> Int4Tensor:
    *lead, n = weight.shape
    if n % 2:
        raise ValueError("last dimension must be even for INT4 packing")
    if group_size <= 0 or n % group_size:
        group_size = n
    w = weight.detach().float().reshape(-1, n)
    wg = w.view(w.shape[0], n // group_size, group_size)
    scales = wg.abs().amax(dim=-1).clamp_min(1e-8) / 7.0
    q = torch.round(wg / scales.unsqueeze(-1)).clamp(-8, 7).to(torch.int8).view(w.shape[0], n)
    even = (q[:, 0::2] & 0x0F).to(torch.uint8)
    odd = (q[:, 1::2] & 0x0F).to(torch.uint8)
    packed = (even | (odd << 4)).view(*lead, n // 2)
    return Int4Tensor(packed.contiguous(), scales.view(*lead, n // group_size).contiguous(),
                      tuple(weight.shape), group_size)


def dequantize_int4(packed, scales, shape, group_size, dtype=None) -> torch.Tensor:
    *lead, half = packed.shape
    n = half * 2
    flat = packed.reshape(-1, half)
    lo = (flat & 0x0F).to(torch.int8)
    hi = ((flat >> 4) & 0x0F).to(torch.int8)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    q = torch.stack([lo, hi], dim=-1).reshape(flat.shape[0], n).float()
    w = (q.view(q.shape[0], n // group_size, group_size)
         * scales.reshape(q.shape[0], n // group_size).unsqueeze(-1).float()).view(*lead, n)
    if dtype is not None:
        w = w.to(dtype)
    return w.view(shape)


@dataclass
class Fp8Tensor:
    """e4m3 weights with one fp32 scale per output row."""
    q: torch.Tensor        # float8_e4m3fn [..., out, in]
    scale: torch.Tensor    # fp32 [..., out]

    def dequantize(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return (self.q.float() * self.scale.float().unsqueeze(-1)).to(dtype)


def quantize_fp8_per_channel(w: torch.Tensor) -> Fp8Tensor:
    s = (w.detach().float().abs().amax(dim=-1) / FP8_E4M3_MAX).clamp_min(1e-12)
    q = (w.detach().float() / s.unsqueeze(-1).clamp_min(1e-12)).to(torch.float8_e4m3fn)
    return Fp8Tensor(q, s)
