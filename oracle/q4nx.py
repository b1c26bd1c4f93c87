"""Writer of small ``.q4nx`` weight containers -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` and ``tests/golden/make_golden.py`` use it, to build containers that both the reference's
reader (``open_kernels/model/q4nx.py``, class ``Q4NX``) and this repository's importer
(``flowmoe.q4nx``) read. The layout is the one that reader parses (``q4nx.py:1-20``, ``Q4NX.__init__``):
a safetensors file -- an 8-byte little-endian header length, a JSON header of tensor name ->
{dtype, shape, data_offsets}, then the data -- where a quantized tensor is ``I8`` [chunks, 5120] of
q4_1 pool chunks (``q4_1_pack`` chunk format, bf16 d and m) in the plain raster of the matrix: chunk f of
an [out, in] matrix covers rows 32*(f // ncol) and columns 256*(f % ncol) -- ``blocks_to_pool`` with a band
row split of 1. The routed experts of a layer are one tensor, expert-major (``Q4NX.expert_w``); bf16
tensors are plain row-major uint16.
"""
from __future__ import annotations

import json
import struct

import numpy as np

from .q4_1 import blocks_to_pool


def q4nx_matrix(blocks: np.ndarray) -> np.ndarray:
    """GGUF Q4_1 blocks [out, in/32, 20] -> the container's [chunks, 5120] bytes (plain raster)."""
    return blocks_to_pool(blocks, 1).reshape(-1, 5120)


def signed_q4_matrix(blocks: np.ndarray) -> np.ndarray:
    """The same matrix as a container of the signed quantiser writes it (``recipes/pack.py:583-622``,
    ``is_signed_q4`` / ``q4_0_to_q4_1``): codes as two's-complement nibbles (bit 3 of every nibble
    flipped) and every min written as zero. Reading it back -- flip the bits, min = bf16(-8 d) -- gives
    the blocks whose min is -8 d, so the blocks here must have m == -8 d for a round trip."""
    c = q4nx_matrix(blocks).copy()
    c[:, 512:1024] = 0
    c[:, 1024:] ^= 0x88
    return c


def write_q4nx(path, tensors: dict) -> None:
    """tensors: name -> ("I8", uint8 [chunks, chunk_bytes]) or ("BF16", uint16 array)."""
    header, blobs, off = {}, [], 0
    for name, (dtype, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
