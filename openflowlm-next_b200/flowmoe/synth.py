"""Seeded synthetic layers and tokens of the BASELINE configs, generated on the device.

Expert weights fp32 N(0, 0.02) quantised to GGUF Q4_1 (``quantize_q4_1``, gguf's algorithm); router
weight and shared gate bf16 N(0, 0.02); activations bf16 N(0, 1); residual f32 N(0, 1). The prefill
configs bias the router logits by ln p_{pi(e)} with p_r ~ r^-s (Zipf) and pi a seeded permutation,
so expert loads are skewed. The reference measures on real model weights that are not available
here; these stand in with the stated shapes and distributions.
"""
from __future__ import annotations

import torch

from .layer import MoEConfig, MoELayer
from .quant import quantize_q4_1

C30 = dict(hidden=2048, n_experts=128, top_k=8, ffn=768, shared_ffn=0)    # Qwen3-30B-A3B-shaped (configs 1-3)
C36 = dict(hidden=2048, n_experts=256, top_k=8, ffn=512, shared_ffn=512)  # Qwen3.6-MoE-shaped (configs 4-5)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def synth_blocks(cfg: MoEConfig, seed: int = 0, device="cuda", experts=None):
    """Q4_1 blocks for experts ``experts`` (default: the local range) + router + shared expert."""
    H, F, FS, E = cfg.hidden, cfg.ffn, cfg.shared_ffn, cfg.n_experts
    g = _gen(seed, device)
    wr = (torch.randn(H, E, generator=g, device=device) * 0.02).to(torch.bfloat16)
    sgw = (torch.randn(H, generator=g, device=device) * 0.02).to(torch.bfloat16) if FS else None
    shared = None
    if FS:
        def q(r, c):
            return quantize_q4_1(torch.randn(r, c, generator=g, device=device) * 0.02)
        shared = (q(FS, H), q(FS, H), q(H, FS), sgw)
    ids = range(cfg.e_begin, cfg.e_begin + cfg.local) if experts is None else experts
    gate, up, down = [], [], []
    for e in ids:
        ge = _gen(seed * 1000003 + 7919 * (e + 1), device)     # per expert: independent of the sharding
        gate.append(quantize_q4_1(torch.randn(F, H, generator=ge, device=device) * 0.02))
        up.append(quantize_q4_1(torch.randn(F, H, generator=ge, device=device) * 0.02))
        down.append(quantize_q4_1(torch.randn(H, F, generator=ge, device=device) * 0.02))
    return torch.stack(gate), torch.stack(up), torch.stack(down), wr, shared


def zipf_bias(E: int, s: float = 1.1, seed: int = 0, device="cuda") -> torch.Tensor:
    p = torch.arange(1, E + 1, dtype=torch.float64) ** -s
    p /= p.sum()
    perm = torch.randperm(E, generator=_gen(seed + 17, "cpu"))
    return torch.log(p[perm]).to(torch.float32).to(device)


def synth_layer(cfg: MoEConfig, seed: int = 0, device="cuda", zipf: float | None = None) -> MoELayer:
    gate, up, down, wr, shared = synth_blocks(cfg, seed, device)
    bias = zipf_bias(cfg.n_experts, zipf, seed, device) if zipf else None
    return MoELayer.from_q4_1(cfg, gate, up, down, wr, shared=shared, device=device, router_bias=bias)


def synth_tokens(T: int, H: int, seed: int = 0, device="cuda"):
    g = _gen(seed + 101, device)
    x = torch.randn(T, H, generator=g, device=device).to(torch.bfloat16)
    res = torch.randn(T, H, generator=g, device=device)
    return x, res
