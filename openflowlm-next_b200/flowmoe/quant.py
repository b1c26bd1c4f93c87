"""Q4_1 quantisation on the device (torch ops), for building layers from float weights.

Restates the quantiser the reference toolchain uses, ``gguf.quantize(w, Q4_1)`` (PyPI ``gguf`` 0.19.0,
``gguf/quants.py`` class ``Q4_1``, called at ``utilities/q4nx-build/q4nx/gguf_tensor.py:524``): per
32-value block, ``d = (max - min) / 15``, ``q = trunc((x - min) * (1/d) + 0.5)`` clipped to [0, 15],
d and min stored as fp16. Every step is an IEEE f32 operation, so the bytes equal gguf's.
"""
from __future__ import annotations

import torch

BLK = 32


def quantize_q4_1(w: torch.Tensor) -> torch.Tensor:
    """f32 [..., n, k] -> GGUF Q4_1 blocks uint8 [..., n, k/32, 20] (same device)."""
    if w.shape[-1] % BLK:
        raise ValueError("K must be a multiple of 32")
    lead = w.shape[:-1]
    b = w.to(torch.float32).reshape(*lead, w.shape[-1] // BLK, BLK)
    mx = b.amax(-1, keepdim=True)
    mn = b.amin(-1, keepdim=True)
    d = (mx - mn) / 15.0
    inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    q = torch.trunc((b - mn) * inv + 0.5).to(torch.uint8).clamp_(0, 15)
    out = torch.empty(*lead, w.shape[-1] // BLK, 20, dtype=torch.uint8, device=w.device)
    out[..., 0:2] = d.to(torch.float16).view(torch.uint8)
    out[..., 2:4] = mn.to(torch.float16).view(torch.uint8)
    out[..., 4:20] = q[..., :16] | (q[..., 16:] << 4)
    return out


def dequantize_q4_1(blocks: torch.Tensor) -> torch.Tensor:
    """GGUF Q4_1 blocks uint8 [..., n, nb, 20] -> f32 [..., n, nb*32] (exact fp16 scales)."""
    d = blocks[..., 0:2].contiguous().view(torch.float16).to(torch.float32)
    m = blocks[..., 2:4].contiguous().view(torch.float16).to(torch.float32)
    qs = blocks[..., 4:20]
    q = torch.cat([qs & 0xF, qs >> 4], dim=-1).to(torch.float32)
    return (q * d + m).reshape(*blocks.shape[:-2], -1)
