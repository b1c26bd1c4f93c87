"""Per-layer stage accounting as JSONL, the reference engine's ``OFLM_OPEN_PROFILE`` records.

The reference writes one ``header`` record per run, then per profiled request one ``request`` record and
one ``layer`` record per layer, with the MoE block's time split as ``moe_prep_ms`` (xm, the router record
and the residual staged for the device), ``moe_patch_ms`` (expert selection: the DMA-offset patch),
``moe_run_ms`` (the expert dispatch) and ``moe_read_ms`` (the result read back)
(src/open_qwen36/core.cpp:592-600, :850-935; fields core.hpp:99-125). Here the same records come from the
library's stage events (``fm_profile``, CUDA events recorded on the launching stream around each stage),
mapped onto those names:

  moe_prep_ms   to_bf16 + router        (x to bf16, logits, softmax top-k, shared gate)
  moe_patch_ms  dispatch + gather       (counts, scan, permutation and the expert-sorted rows: what the
                                         reference's stream patch selects by rewriting DMA offsets)
  moe_run_ms    gate_up + down          (the grouped expert GEMMs / GEMVs)
  moe_read_ms   combine                 (the ordered weighted sum; 0 where the down epilogue adds it)

and each stage also appears under its own name (``router_ms``, ``gate_up_ms`` ...). Reading the events
synchronises the device after every layer: a measurement tool, not for production runs, and like the
library's profiler it is one process-wide record (one host thread at a time).

    with StageProfile("run.jsonl", family="qwen36moe", layers=len(stack.layers)) as prof:
        prof.request("prefill", tokens=T, run=lambda layer_hook: stack.forward(x, layer_hook=layer_hook))

or simply ``StageProfile.from_env()``, which opens the file named by ``OFLM_OPEN_PROFILE`` (None if unset).
"""
from __future__ import annotations

import json
import os
import time

import torch

from . import _lib

_MAP = {"moe_prep_ms": ("to_bf16", "router"), "moe_patch_ms": ("dispatch", "gather"),
        "moe_run_ms": ("gate_up", "down"), "moe_read_ms": ("combine",)}


class StageProfile:
    def __init__(self, path: str, family: str = "qwen36moe", layers: int = 1):
        self.f = open(path, "w")
        self.f.write(json.dumps({"record": "header", "version": 1, "family": family, "layers": layers}) + "\n")
        self.rows: list[dict] = []
        self._t0 = None

    @classmethod
    def from_env(cls, family: str = "qwen36moe", layers: int = 1):
        p = os.environ.get("OFLM_OPEN_PROFILE")
        return cls(p, family, layers) if p else None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self):
        if self.f:
            self.f.close()
            self.f = None

    # ---- one request: the layers run inside, each closed by layer_done
    def begin(self):
        torch.cuda.synchronize()
        _lib.profile(True)
        self.rows = []
        self._t0 = time.perf_counter()

    def layer_done(self, layer: int, kind: str = "moe"):
        """Closes a layer's row: waits for its events and records wall time and stage times."""
        torch.cuda.synchronize()
        st = _lib.profile_read()
        now = time.perf_counter()
        row = {"record": "layer", "kind": kind, "layer": layer, "wall_ms": round((now - self._t0) * 1e3, 3),
               "total_ms": round(sum(st.values()), 3)}
        for name, stages in _MAP.items():
            row[name] = round(sum(st[s] for s in stages), 3)
        for s, v in st.items():
            row[f"{s}_ms"] = round(v, 3)
        self.rows.append(row)
        self._t0 = now

    def end(self, what: str, tokens: int):
        _lib.profile(False)
        total = sum(r["wall_ms"] for r in self.rows)
        self.f.write(json.dumps({"record": "request", "what": what, "tokens": tokens, "total_ms": round(total, 3),
                                 "layer_wall_ms": round(total, 3), "layers": len(self.rows)}) + "\n")
        for r in self.rows:
            self.f.write(json.dumps({**r, "what": what}) + "\n")
        self.f.flush()
        self.rows = []

    def request(self, what: str, tokens: int, run):
        """Profiles one request: ``run(layer_hook)`` runs the layers and calls ``layer_hook(i)`` after
        each (``MoEStack.forward`` takes it as ``layer_hook``); returns run's result."""
        self.begin()
        out = run(self.layer_done)
        self.end(what, tokens)
        return out
