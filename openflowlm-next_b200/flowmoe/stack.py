"""A stack of MoE layers with the post-attention RMSNorm and residual between them:
x_{l+1} = x_l + MoE_l(RMSNorm_l(x_l)), the engine's staged_tail -> ffn_block sequence repeated per layer
(src/open_qwen36/core.cpp:4934-4957; open_kernels/model/replica.py:121-143). Attention and the rest of a
transformer block are not part of this path; the stack isolates the MoE half of each layer.

Each layer is one ``fm_moe_layer_norm`` call; ``capture()`` records the whole stack for a fixed token
count into one CUDA graph (the decode loop of config 5), replayed by ``forward``.
"""
from __future__ import annotations

import torch

from .layer import MoELayer


class MoEStack:
    def __init__(self, layers: list[MoELayer], norm_ws: list[torch.Tensor], eps: float = 1e-6):
        if len(layers) != len(norm_ws) or not layers:
            raise ValueError("one RMSNorm weight per layer")
        self.layers = layers
        self.norm_ws = [w.to(layers[0].device, torch.bfloat16).contiguous() for w in norm_ws]
        self.eps = eps
        self.device = layers[0].device
        self._graph = None
        self._bufs = None

    def _run(self, x: torch.Tensor, bufs) -> torch.Tensor:
        cur = x
        for i, (layer, nw) in enumerate(zip(self.layers, self.norm_ws)):
            nxt = bufs[i & 1]
            layer.forward_norm(cur, nw, self.eps, out=nxt)
            cur = nxt
        return cur

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x f32 [T, H] -> the stack's output (a new tensor unless a captured graph is replayed)."""
        if self._graph is not None and x.shape == self._x.shape:
            self._x.copy_(x)
            self._graph.replay()
            return self._y
        bufs = [torch.empty_like(x), torch.empty_like(x)]
        return self._run(x, bufs)

    __call__ = forward

    def capture(self, T: int):
        """Record the whole stack for T tokens into one CUDA graph (workspaces and buffers are allocated
        first, outside the capture)."""
        H = self.layers[0].cfg.hidden
        self._x = torch.zeros(T, H, dtype=torch.float32, device=self.device)
        bufs = [torch.empty_like(self._x), torch.empty_like(self._x)]
        for layer in self.layers:
            layer.workspace(T)
        self._run(self._x, bufs)           # warm-up outside the capture (library state, kernel loading)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._y = self._run(self._x, bufs)
        self._graph, self._bufs = g, bufs
        return self
