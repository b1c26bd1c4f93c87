"""Seeded synthetic inputs of the BASELINE configs -- TEST INFRASTRUCTURE ONLY.

Expert weights fp32 N(0, 0.02) quantised to GGUF Q4_1 by the oracle's restatement of gguf.quantize;
router weight and shared gate bf16 N(0, 0.02); activations bf16 N(0, 1); residual f32 N(0, 1);
numpy ``default_rng(seed)``. Optional Zipf(s) router bias for the prefill configs: logits +=
ln p_{pi(e)}, p_r ~ r^-s, pi a seeded permutation (the skew form the prefill benchmark uses).
"""
from __future__ import annotations

import numpy as np

from .moe import bf16_round
from .q4_1 import quantize_q4_1, random_q4_1_blocks


def make_case(H=2048, E=128, F=768, FS=0, k=8, T=16, seed=0, zipf=None, weights="blocks"):
    """weights: "blocks" = random GGUF blocks drawn as the reference's q4_1_pack generator draws them
    (fast; the parity tests' default), "normal" = N(0, 0.02) quantised (the BASELINE recipe), or
    None (router-only cases)."""
    rng = np.random.default_rng(seed)
    x = bf16_round(rng.standard_normal((T, H), dtype=np.float32))
    Wr = bf16_round(rng.normal(0, 0.02, (H, E)).astype(np.float32))

    def q(rows, cols, n):
        if weights == "normal":
            return np.stack([quantize_q4_1(rng.normal(0, 0.02, (rows, cols)).astype(np.float32)) for _ in range(n)])
        return np.stack([random_q4_1_blocks(rows, cols, rng) for _ in range(n)])

    if weights is None:
        gate = up = down = None
    else:
        gate, up, down = q(F, H, E), q(F, H, E), q(H, F, E)
    shared = None
    if FS and weights is not None:
        sg, su, sd = q(FS, H, 1)[0], q(FS, H, 1)[0], q(H, FS, 1)[0]
        sgw = bf16_round(rng.normal(0, 0.02, H).astype(np.float32))
        shared = (sg, su, sd, sgw)
    res = rng.standard_normal((T, H)).astype(np.float32)
    bias = None
    if zipf is not None:
        p = np.arange(1, E + 1, dtype=np.float64) ** -zipf
        p /= p.sum()
        bias = np.log(p[rng.permutation(E)]).astype(np.float32)
    return dict(H=H, E=E, F=F, FS=FS, k=k, T=T, x=x, Wr=Wr, gate=gate, up=up, down=down, shared=shared, res=res,
                bias=bias)
