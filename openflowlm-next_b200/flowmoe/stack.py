"""A stack of MoE layers with the post-attention RMSNorm and residual between them (e.g. the 48 MoE layers
of a Qwen3.6-MoE-shaped model at a decode batch):
x_{l+1} = x_l + MoE_l(RMSNorm_l(x_l)), the engine's staged_tail -> ffn_block sequence repeated per layer
(src/open_qwen36/core.cpp:4934-4957; open_kernels/model/replica.py:121-143). Attention and the rest of a
transformer block are not part of this path; the stack isolates the MoE half of each layer.

Each layer is one ``fm_moe_layer_norm`` call; ``capture()`` records the whole stack for a fixed token
count into one CUDA graph (a decode loop), replayed by ``forward``. ``flowmoe.profile.StageProfile`` records
per-layer stage times of an eager pass (``forward(x, layer_hook=...)``) as the reference's JSONL profile.
"""
from __future__ import annotations

import ctypes

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

    def _run(self, x: torch.Tensor, bufs, layer_hook=None, t_real=None) -> torch.Tensor:
        cur = x
        for i, (layer, nw) in enumerate(zip(self.layers, self.norm_ws)):
            nxt = bufs[i & 1]
            layer.forward_norm(cur, nw, self.eps, out=nxt, t_real=t_real)
            if layer_hook is not None:
                layer_hook(i)
            cur = nxt
        return cur

    def forward(self, x: torch.Tensor, layer_hook=None, t_real: int | None = None) -> torch.Tensor:
        """x f32 [T, H] -> the stack's output (a new tensor unless a captured graph is replayed).
        ``layer_hook(i)`` (eager passes only) is called after layer i is enqueued; rows past ``t_real`` are
        padding (carried through every layer as they are).

        Given a whole prompt, this is the reference's layer-major prefill schedule for the MoE half of
        each layer (Core::step_gemm_prompt, src/open_qwen36/core.cpp:3734-3846): every token through layer
        l's MoE in one call, then layer l + 1, so each layer's experts stream from HBM once per prompt;
        with the layers' ``fixed_order`` set, the result is bit for bit that of running the prompt in
        blocks."""
        if self._graph is not None and x.shape == self._x.shape and layer_hook is None and t_real is None:
            self._x.copy_(x)
            self._graph.replay()
            return self._y
        bufs = [torch.empty_like(x), torch.empty_like(x)]
        return self._run(x, bufs, layer_hook, t_real)

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


class EPMoEStack:
    """The stack across an expert-parallel group (e.g. 48 layers at a decode batch, experts sharded over the
    node's GPUs). Each rank holds its expert range of every layer and runs its own tokens; a layer is
    ``fm_rmsnorm_bf16`` (xb = RMSNorm_l(x)) then ``fm_ep_peer_layer`` (x <- x + MoE_l(xb) over peer memory).
    All layers share one peer group -- one symmetric buffer, its epochs advancing call by call, since the
    layers have one geometry and run in sequence -- and ``capture()`` records the whole stack into one CUDA
    graph per rank (the exchange synchronises on device flags, so replays need no host step). Every rank
    must make the same calls in the same order."""

    def __init__(self, layers: list[MoELayer], norm_ws: list[torch.Tensor], t_cap: int, group=None, eps: float = 1e-6,
                 timeout_ms: int = 10000):
        from .ep import PeerGroup
        if len(layers) != len(norm_ws) or not layers:
            raise ValueError("one RMSNorm weight per layer")
        geo = {(L.cfg.hidden, L.cfg.n_experts, L.cfg.top_k, L.cfg.ffn, L.cfg.shared_ffn, L.cfg.e_begin, L.cfg.local)
               for L in layers}
        if len(geo) != 1:
            raise ValueError("the layers of one stack share one geometry and expert range")
        self.layers = layers
        self.norm_ws = [w.to(layers[0].device, torch.bfloat16).contiguous() for w in norm_ws]
        self.eps = eps
        self.device = layers[0].device
        self.t_cap = t_cap
        self.peers = PeerGroup(layers[0], t_cap, group, timeout_ms)
        self._graph = None

    def _run(self, x: torch.Tensor, bufs, xb: torch.Tensor) -> torch.Tensor:
        from ._lib import FM_BF16, call
        from .layer import _stream
        T, H = x.shape
        if T > self.t_cap:
            raise ValueError(f"{T} tokens past the group's capacity {self.t_cap}")
        st = _stream(self.device)
        ws = self.peers.ws
        cur = x
        for i, (layer, nw) in enumerate(zip(self.layers, self.norm_ws)):
            nxt = bufs[i & 1]
            call("fm_rmsnorm_bf16", cur.data_ptr(), nw.data_ptr(), self.eps, T, H, xb.data_ptr(), st)
            call("fm_ep_peer_layer", ctypes.byref(layer._L), ctypes.byref(self.peers.g), xb.data_ptr(), FM_BF16,
                 cur.data_ptr(), T, T, nxt.data_ptr(), None, None, ws.data_ptr(), ws.numel(), st)
            cur = nxt
        return cur

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's tokens x f32 [T, H] -> their stack output (the graph's buffer when replayed)."""
        L0 = self.layers[0]
        L0._check_x(x)
        if x.dtype != torch.float32:
            raise ValueError(f"x must be float32, not {x.dtype}")
        if self._graph is not None and x.shape == self._x.shape:
            self._x.copy_(x)
            self._graph.replay()
            return self._y
        bufs = [torch.empty_like(x), torch.empty_like(x)]
        xb = torch.empty(x.shape, dtype=torch.bfloat16, device=self.device)
        return self._run(x, bufs, xb)

    __call__ = forward

    def capture(self, T: int):
        """Record the stack for T tokens of this rank into one CUDA graph (all ranks together)."""
        H = self.layers[0].cfg.hidden
        self._x = torch.zeros(T, H, dtype=torch.float32, device=self.device)
        bufs = [torch.empty_like(self._x), torch.empty_like(self._x)]
        xb = torch.empty(T, H, dtype=torch.bfloat16, device=self.device)
        self._run(self._x, bufs, xb)          # warm-up outside the capture, on every rank
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._y = self._run(self._x, bufs, xb)
        self._graph, self._bufs, self._xb = g, bufs, xb
        return self

    def check(self):
        """Synchronise; raise FM_ETIMEOUT if a peer did not take its step in time (any layer)."""
        from ._lib import call
        from .layer import _stream
        call("fm_moe_check", self.peers.ws.data_ptr(), _stream(self.device))

    def close(self):
        """Release the graph, then the peer group's buffers (collective: every rank)."""
        self._graph = None
        torch.cuda.synchronize(self.device)
        self.peers.close()
