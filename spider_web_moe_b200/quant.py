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
* the reference's general fp8 helpers (quant.py:16-69, 146-169):
  ``quantize_fp8`` / ``dequantize_fp8`` with one per-tensor scale (computed as
  amax/448 with a 1e-12 floor when not given), the broadcastable-scale pair
  ``quantize_fp8_with_scale_tensor`` / ``dequantize_fp8_with_scale_tensor``,
  and ``fp8_available`` / ``fp8_dtype`` / ``is_fp8_dtype`` /
  ``compute_fp8_scale``.

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


# ---------------------------------------------------------------------------
# general fp8 helpers of the reference (quant.py:16-69, 146-169)
# ---------------------------------------------------------------------------
_E4M3 = getattr(torch, "float8_e4m3fn", None)


def fp8_available() -> bool:
    return _E4M3 is not None


def fp8_dtype() -> torch.dtype:
    if _E4M3 is None:
        raise RuntimeError("torch.float8_e4m3fn is not available in this PyTorch build")
    return _E4M3


def is_fp8_dtype(dtype: torch.dtype) -> bool:
    return _E4M3 is not None and dtype == _E4M3


def compute_fp8_scale(x: torch.Tensor, eps: float = 1e-12) -> torch.Tensor:
    """One scale for the whole tensor: amax(|x|) / 448, at least eps (0-dim fp32)."""
    return (x.detach().float().abs().amax() / FP8_E4M3_MAX).clamp_min(eps)


def _scalar_scale(scale, device) -> torch.Tensor:
    if isinstance(scale, torch.Tensor):
        return scale.detach().float().reshape(()).to(device)
    return torch.tensor(float(scale), dtype=torch.float32, device=device)


def quantize_fp8(x: torch.Tensor, scale=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(e4m3 tensor, 0-dim fp32 scale): x / scale cast to e4m3, the scale
    computed from x when not given."""
    s = compute_fp8_scale(x) if scale is None else _scalar_scale(scale, x.device)
    return (x.float() / s).to(fp8_dtype()), s


def dequantize_fp8(x: torch.Tensor, scale=None, compute_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """fp32(x) * scale in compute_dtype (a plain cast without a scale)."""
    y = x.to(torch.float32)
    if scale is None:
        return y.to(compute_dtype)
    s = scale.to(device=y.device, dtype=torch.float32) if isinstance(scale, torch.Tensor) else \
        torch.tensor(float(scale), dtype=torch.float32, device=y.device)
    return (y * s).to(compute_dtype)


def _broadcast_scale(scale: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    s = scale.to(device=x.device, dtype=torch.float32)
    while s.ndim < x.ndim:  # trailing singleton dims, so [H] scales rows of [H, D]
        s = s.unsqueeze(-1)
    return s


def quantize_fp8_with_scale_tensor(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """x / scale (broadcast over trailing dims, floored at 1e-12) cast to e4m3."""
    return (x.float() / _broadcast_scale(scale, x).clamp_min(1e-12)).to(fp8_dtype())


def dequantize_fp8_with_scale_tensor(x: torch.Tensor, scale: torch.Tensor,
                                     compute_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """fp32(x) * scale (broadcast over trailing dims) in compute_dtype."""
    return (x.float() * _broadcast_scale(scale, x)).to(compute_dtype)
