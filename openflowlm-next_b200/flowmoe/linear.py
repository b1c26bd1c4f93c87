"""Dense Q4_1 projection on the tcgen05 GEMM (``fm_q4_gemm``): the prefill projections beside the MoE block.

The reference runs these matrices (attention q/k/v/o, dense FFN weights) as its gemm_q4_prefill design,
open_kernels/designs/gemm_q4_prefill/gemm_q4_prefill.py:1-3: ``Y[N_WEIGHT, T] = W(q4_1)[N_WEIGHT, K] @
X^T[K, T]`` with the weight dequantised on-core. :meth:`Q4Linear.forward` computes the same product with f32
accumulation and returns it token-major, ``y [T, N]`` (the transpose of that device layout).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import call
from .layer import _ptr, _stream, pool_to_q4_1, q4_1_to_tiles


class Q4Linear:
    """``y = bf16(x) @ dequant(W)^T`` for one Q4_1 matrix W [n, k] held in the device tile layout.

    n % 128 == 0 and k % 64 == 0 (the tiles' 128-row bands and 64-wide K slabs)."""

    def __init__(self, tiles: torch.Tensor, n: int, k: int):
        if n <= 0 or n % 128 or k <= 0 or k % 64:
            raise ValueError(f"Q4Linear: n={n} must be a positive multiple of 128 and k={k} of 64")
        if not isinstance(tiles, torch.Tensor) or tiles.dtype != torch.uint8 or not tiles.is_cuda or \
                not tiles.is_contiguous() or tiles.numel() != n * k // 32 * 20:
            raise ValueError(f"Q4Linear: tiles must be a contiguous uint8 GPU tensor of {n * k // 32 * 20} bytes")
        self.tiles, self.n, self.k = tiles, n, k
        self._ws: torch.Tensor | None = None

    @classmethod
    def from_q4_1(cls, blocks, n: int, k: int, device="cuda") -> "Q4Linear":
        """From GGUF Q4_1 blocks uint8 [n, k/32, 20] (numpy or torch)."""
        return cls(q4_1_to_tiles(blocks, n, k, device=device), n, k)

    @classmethod
    def from_pool(cls, pool, n: int, k: int, rs: int = 2, chunk_bytes: int | None = None, device="cuda") -> "Q4Linear":
        """From the reference's pool chunk bytes of the matrix (``pack_q4_1_pool`` / ``pack_q4_pool``)."""
        return cls.from_q4_1(pool_to_q4_1(pool, n, k, rs=rs, chunk_bytes=chunk_bytes, device=device), n, k, device=device)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x [T, k] f32 or bf16 on the weight's device -> y [T, n] f32."""
        if not isinstance(x, torch.Tensor) or x.dim() != 2 or x.shape[1] != self.k or \
                x.dtype not in (torch.float32, torch.bfloat16) or x.device != self.tiles.device:
            raise ValueError(f"Q4Linear.forward: x must be a [T, {self.k}] f32 or bf16 tensor on {self.tiles.device}")
        x = x.contiguous()
        T = x.shape[0]
        if out is None:
            out = torch.empty(T, self.n, dtype=torch.float32, device=x.device)
        elif out.shape != (T, self.n) or out.dtype != torch.float32 or not out.is_contiguous() or out.device != x.device:
            raise ValueError(f"Q4Linear.forward: out must be a contiguous f32 [{T}, {self.n}] tensor on {x.device}")
        dt = _lib.FM_F32 if x.dtype == torch.float32 else _lib.FM_BF16
        need = ctypes.c_size_t()
        call("fm_q4_gemm_workspace_size", self.n, self.k, T, dt, ctypes.byref(need))
        if self._ws is None or self._ws.numel() < need.value:
            self._ws = torch.empty(max(need.value, 256), dtype=torch.uint8, device=x.device)
        call("fm_q4_gemm", self.tiles.data_ptr(), self.n, self.k, x.data_ptr(), dt, T, out.data_ptr(),
             self._ws.data_ptr(), self._ws.numel(), _stream(x.device))
        return out

    __call__ = forward

    def check(self) -> None:
        """Raises if a device wait of the last call gave up (fm_moe_check on this object's workspace)."""
        if self._ws is not None:
            call("fm_moe_check", self._ws.data_ptr(), _stream(self._ws.device))
