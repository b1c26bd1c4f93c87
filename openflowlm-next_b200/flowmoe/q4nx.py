"""Reads the MoE layers of the reference's ``.q4nx`` weight containers straight into device layers.

The container (the reference's reader: open_kernels/model/q4nx.py:1-20, class ``Q4NX``) is a safetensors
file -- an 8-byte little-endian header length, a JSON header of tensor name -> {dtype, shape,
data_offsets}, then the data. A quantized tensor is ``I8`` [chunks, chunk bytes]; its 5120-byte chunks are
q4_1 tiles of 32 rows x 256 inputs (bf16 d and m per 32-value block, then the nibbles), placed in the
plain raster of the matrix (chunk f covers rows 32*(f // ncol), inputs 256*(f % ncol)) -- the reference's
pool chunk law with a band row split of 1, which ``fm_pool_to_q4_1`` reads on the device. A layer's
routed experts are one tensor, expert-major (``Q4NX.expert_w``: 128 chunks per expert at the
Qwen3.6-MoE shapes). Tensor names (``open_kernels/model/replica.py:121-143``):

    model.layer.{l}.post_attention_layernorm.weight   bf16 [H]
    model.layer.{l}.moe_router.weight                 bf16 [H, E]
    model.layer.{l}.shared_expert_gate.weight         bf16 [H]
    model.layer.{l}.mlp.{gate,up,down}_exps_proj.weight        I8 chunks, experts stacked
    model.layer.{l}.mlp.share_{gate,up,down}_exps_proj.weight  I8 chunks

A 5120-byte tensor whose first chunk's mins are all zero is the signed quantiser's (w = d * int4(q)); it is
read as the reference's packer reads it (open_kernels/recipes/pack.py:583-622): every nibble's bit 3
flipped (two's complement -> offset binary) and min = bf16(-8 d), exact. Containers hold d and m in bf16,
so a layer read from one computes with the NPU pool's numerics. Tensors in other chunk formats (8704-byte
q8, 4736-byte Q4_K) are refused by name: the reference re-quantises those to q4_1 before they reach a
q4_1 kernel, which is a lossy step this importer does not repeat.
"""
from __future__ import annotations

import json
import mmap
import struct

import numpy as np
import torch

from .layer import MoEConfig, MoELayer, pool_to_q4_1

CHUNK_Q4_1 = 5120


def _bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16(f: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(f, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


class Q4nxFile:
    """One container, memory-mapped; nothing is read until a tensor is asked for."""

    def __init__(self, path):
        self.path = str(path)
        self._f = open(self.path, "rb")
        n = struct.unpack("<Q", self._f.read(8))[0]
        self.header = json.loads(self._f.read(n))
        self._base = 8 + n
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.tensors = {k: v for k, v in self.header.items() if k != "__metadata__"}

    def close(self):
        self._mm.close()
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def raw(self, name: str) -> np.ndarray:
        if name not in self.tensors:
            raise KeyError(f"{self.path}: no tensor {name}")
        o0, o1 = self.tensors[name]["data_offsets"]
        if o1 < o0 or self._base + o1 > len(self._mm):
            raise ValueError(f"{self.path}: {name} lies outside the file ({o0}..{o1})")
        return np.frombuffer(self._mm, np.uint8, o1 - o0, self._base + o0)

    def bf16(self, name: str) -> np.ndarray:
        """A bf16 tensor as its uint16 bit patterns, in its shape."""
        t = self.tensors[name]
        if t.get("dtype") != "BF16":
            raise ValueError(f"{name} is {t.get('dtype')}, not BF16")
        return self.raw(name).view(np.uint16).reshape(t["shape"])

    def q4_1_chunks(self, name: str) -> np.ndarray:
        """A quantized tensor's [chunks, 5120] q4_1 bytes (a copy, transcoded when it is the signed form)."""
        t = self.tensors[name]
        cb = t["shape"][-1] if t.get("dtype") == "I8" and t.get("shape") else 0
        if cb != CHUNK_Q4_1:
            raise ValueError(f"{self.path}: {name} holds {cb}-byte chunks; this importer reads {CHUNK_Q4_1}-byte "
                             f"q4_1 chunks (8704 = q8 and 4736 = Q4_K need the reference's lossy re-quantisation)")
        c = self.raw(name).reshape(-1, CHUNK_Q4_1).copy()
        if c.shape[0] and not c[0, 512:1024].any():   # every min of the first chunk exactly zero: signed codes
            d = _bf16_to_f32(np.ascontiguousarray(c[:, :512]).view(np.uint16))
            c[:, 512:1024] = _f32_to_bf16(-8.0 * d).view(np.uint8).reshape(-1, 512)
            c[:, 1024:] ^= 0x88
        return c

    # ---- MoE layers
    def expert_blocks(self, layer: int, F: int, H: int, experts=None, device="cuda"):
        """(gate, up, down) GGUF Q4_1 blocks on the device for the routed experts ``experts`` (default: all):
        gate/up [E, F, H/32, 20], down [E, H, F/32, 20]."""
        per_ud, per_dn = F * H // (32 * 256), H * F // (32 * 256)
        out = []
        for kind, (n, k, per) in (("gate", (F, H, per_ud)), ("up", (F, H, per_ud)), ("down", (H, F, per_dn))):
            c = self.q4_1_chunks(f"model.layer.{layer}.mlp.{kind}_exps_proj.weight")
            if c.shape[0] % per:
                raise ValueError(f"{kind}_exps_proj has {c.shape[0]} chunks, not a whole number of [{n}, {k}] experts")
            ids = range(c.shape[0] // per) if experts is None else experts
            dev = torch.from_numpy(np.ascontiguousarray(c)).to(device)
            out.append(torch.stack([pool_to_q4_1(dev[e * per:(e + 1) * per].reshape(-1), n, k, rs=1,
                                                 chunk_bytes=CHUNK_Q4_1, device=device) for e in ids]))
        return tuple(out)

    def shared_blocks(self, layer: int, F_s: int, H: int, device="cuda"):
        """The shared expert's (gate, up, down) blocks and its gate vector (bf16 bits [H])."""
        blocks = []
        for kind, (n, k) in (("gate", (F_s, H)), ("up", (F_s, H)), ("down", (H, F_s))):
            c = self.q4_1_chunks(f"model.layer.{layer}.mlp.share_{kind}_exps_proj.weight")
            blocks.append(pool_to_q4_1(torch.from_numpy(c).to(device).reshape(-1), n, k, rs=1, chunk_bytes=CHUNK_Q4_1,
                                       device=device))
        sgw = self.bf16(f"model.layer.{layer}.shared_expert_gate.weight")
        return (*blocks, sgw.copy())

    def post_attention_norm(self, layer: int) -> np.ndarray:
        return self.bf16(f"model.layer.{layer}.post_attention_layernorm.weight").copy()

    def moe_layer(self, layer: int, cfg: MoEConfig, device="cuda") -> MoELayer:
        """The layer's MoE block as a device layer for this rank's expert range (cfg.e_begin, cfg.local)."""
        wr = self.bf16(f"model.layer.{layer}.moe_router.weight")
        if tuple(wr.shape) != (cfg.hidden, cfg.n_experts):
            raise ValueError(f"moe_router.weight is {tuple(wr.shape)}, the config wants ({cfg.hidden}, {cfg.n_experts})")
        gate, up, down = self.expert_blocks(layer, cfg.ffn, cfg.hidden, range(cfg.e_begin, cfg.e_begin + cfg.local),
                                            device)
        shared = self.shared_blocks(layer, cfg.shared_ffn, cfg.hidden, device) if cfg.shared_ffn else None
        return MoELayer.from_q4_1(cfg, gate, up, down, wr.copy(), shared=shared, device=device)
