"""Host-memory streaming through an MoE layer: token batches come from pinned host memory and their
outputs go back to pinned host memory, with the copies overlapped with the layer's kernels.

The reference engine stages every MoE block through host memory (xm and the residual synced to the
device, the expert dispatch, the result read back: ``Core::moe_block``, src/open_qwen36/core.cpp:5150-5259,
with the BO syncs at :5207, :5212). Done one batch after another, the two PCIe copies and the kernels of a
batch add up. ``HostPipeline`` keeps ``depth`` device slots and three streams: batch i's host->device copy
runs while batch i-1 computes and batch i-2's result is copied back, so a stream of batches is bound by
the slowest of the three, not their sum. Every batch is still copied in and out in full.

    pipe = HostPipeline(layer, T)
    for x_h, res_h, out_h in batches:          # pinned host tensors
        pipe.submit(x_h, res_h, out_h)
    pipe.synchronize()                         # every out_h holds its result
"""
from __future__ import annotations

import torch

from .layer import MoELayer


class HostPipeline:
    def __init__(self, layer: MoELayer, T: int, depth: int = 2, x_dtype: torch.dtype = torch.bfloat16, call=None):
        """``call(x, res, out, t_real)`` runs the layer on device tensors (default: ``layer.forward``; an
        expert-parallel layer passes its own call, made in the same order on every rank)."""
        if depth < 1:
            raise ValueError("depth must be at least 1")
        self.layer, self.T = layer, T
        self.call = call or (lambda x, res, out, t_real: layer.forward(x, res, t_real=t_real, out=out))
        dev, H = layer.device, layer.cfg.hidden
        self.h2d = torch.cuda.Stream(dev)
        self.comp = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.slots = []
        for _ in range(depth):
            self.slots.append({"x": torch.empty(T, H, dtype=x_dtype, device=dev),
                               "res": torch.empty(T, H, dtype=torch.float32, device=dev),
                               "out": torch.empty(T, H, dtype=torch.float32, device=dev),
                               "loaded": torch.cuda.Event(), "computed": torch.cuda.Event(),
                               "stored": torch.cuda.Event(), "used": False})
        if call is None:
            layer.workspace(T)   # allocated once, outside the stream of batches
        self.n = 0

    @staticmethod
    def _check_host(t: torch.Tensor, name: str, shape, dtype):
        if t.is_cuda or not t.is_pinned() or tuple(t.shape) != shape or t.dtype != dtype or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous pinned host {dtype} tensor of shape {shape}")

    def submit(self, x_host: torch.Tensor, res_host: torch.Tensor, out_host: torch.Tensor, t_real: int | None = None):
        """Enqueues one batch: x_host [T, H] (the slot dtype) and res_host [T, H] f32 in, out_host [T, H] f32
        out; returns at once (out_host is written when the batch's device->host copy completes)."""
        H = self.layer.cfg.hidden
        s = self.slots[self.n % len(self.slots)]
        self._check_host(x_host, "x_host", (self.T, H), s["x"].dtype)
        self._check_host(res_host, "res_host", (self.T, H), torch.float32)
        self._check_host(out_host, "out_host", (self.T, H), torch.float32)
        self.n += 1
        if s["used"]:
            self.h2d.wait_event(s["computed"])   # the slot's inputs were consumed by its previous batch
            self.comp.wait_event(s["stored"])    # and its output was copied back
        with torch.cuda.stream(self.h2d):
            s["x"].copy_(x_host, non_blocking=True)
            s["res"].copy_(res_host, non_blocking=True)
            s["loaded"].record(self.h2d)
        self.comp.wait_event(s["loaded"])
        with torch.cuda.stream(self.comp):
            self.call(s["x"], s["res"], s["out"], t_real)
            s["computed"].record(self.comp)
        self.d2h.wait_event(s["computed"])
        with torch.cuda.stream(self.d2h):
            out_host.copy_(s["out"], non_blocking=True)
            s["stored"].record(self.d2h)
        s["used"] = True

    def wait_on(self, stream: torch.cuda.Stream):
        """Makes the pipeline's streams start after the work already enqueued on ``stream``."""
        for s in (self.h2d, self.comp, self.d2h):
            s.wait_stream(stream)

    def join(self, stream: torch.cuda.Stream):
        """Makes ``stream`` wait for every batch submitted so far (nothing blocks on the host)."""
        for s in (self.h2d, self.comp, self.d2h):
            stream.wait_stream(s)

    def synchronize(self):
        for s in (self.h2d, self.comp, self.d2h):
            s.synchronize()
