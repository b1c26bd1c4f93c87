"""Seeded synthetic layers and tokens of the benchmarked shapes, generated on the device.

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

C30 = dict(hidden=2048, n_experts=128, top_k=8, ffn=768, shared_ffn=0)    # Qwen3-30B-A3B-shaped MoE layer
C36 = dict(hidden=2048, n_experts=256, top_k=8, ffn=512, shared_ffn=512)  # Qwen3.6-MoE-shaped, shared expert


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


def random_q4_1(rows: int, k: int, gen: torch.Generator, device="cuda") -> torch.Tensor:
    """GGUF Q4_1 blocks uint8[rows, k/32, 20] drawn directly (fp16 d ~ |N(0, 0.0013)|, fp16 m ~ -8 d, random
    nibbles), so values spread like N(0, 0.02) weights quantised, without running the quantiser: for
    benchmarks that only need the bytes (the layer stack's 24 GB of experts)."""
    nb = k // 32
    d = (torch.randn(rows, nb, generator=gen, device=device).abs() * 0.0013 + 1e-4).to(torch.float16)
    m = (-8.0 * d.float() + torch.randn(rows, nb, generator=gen, device=device) * 1e-3).to(torch.float16)
    blocks = torch.empty(rows, nb, 20, dtype=torch.uint8, device=device)
    blocks[:, :, 0:2] = d.view(torch.uint8).view(rows, nb, 2)
    blocks[:, :, 2:4] = m.view(torch.uint8).view(rows, nb, 2)
    blocks[:, :, 4:] = torch.randint(0, 256, (rows, nb, 16), generator=gen, device=device, dtype=torch.uint8)
    return blocks


def synth_stack(cfg: MoEConfig, n_layers: int, seed: int = 0, device="cuda"):
    """n_layers independent seeded layers of geometry cfg (random Q4_1 blocks, bf16 N(0, 0.02) router and
    shared gate) and their RMSNorm weights bf16 1 + N(0, 0.01)."""
    H, F, FS, E = cfg.hidden, cfg.ffn, cfg.shared_ffn, cfg.local
    layers, norms = [], []
    for l in range(n_layers):
        g = _gen(seed * 7919 + l, device)
        gate = random_q4_1(E * F, H, g, device).view(E, F, H // 32, 20)
        up = random_q4_1(E * F, H, g, device).view(E, F, H // 32, 20)
        down = random_q4_1(E * H, F, g, device).view(E, H, F // 32, 20)
        wr = (torch.randn(H, cfg.n_experts, generator=g, device=device) * 0.02).to(torch.bfloat16)
        shared = None
        if FS:
            sgw = (torch.randn(H, generator=g, device=device) * 0.02).to(torch.bfloat16)
            shared = (random_q4_1(FS, H, g, device), random_q4_1(FS, H, g, device), random_q4_1(H, FS, g, device), sgw)
        layers.append(MoELayer.from_q4_1(cfg, gate, up, down, wr, shared=shared, device=device))
        norms.append((1.0 + torch.randn(H, generator=g, device=device) * 0.01).to(torch.bfloat16))
    return layers, norms
