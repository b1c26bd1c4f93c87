"""GGUF ingestion: a model file's MoE tensors straight into the device layout.

Replaces the reference's GGUF index reader and expert packers (``open_kernels/gguf_pool/gguf_pool.py``
``read_gguf``; ``src/open_qwen36/pools.cpp`` ``expert_stripes_gguf`` / ``expert_down_gguf``) for this
path. The container follows the public GGUF layout: a header (magic ``GGUF``, version, tensor count,
metadata count), typed metadata key/values, one info record per tensor (name, dims with the innermost
first, type, offset into the data section), and the data section at the next multiple of
``general.alignment`` (32 by default).

The MoE tensors use llama.cpp's names (the map the reference's own test pins,
``src/open_qwen36/gguf_pack_test.cpp:497-507``):
  ``blk.{l}.ffn_{gate,up}_exps.weight``  Q4_1 dims [H, F, E]    -> blocks [E, F, H/32, 20]
  ``blk.{l}.ffn_down_exps.weight``       Q4_1 dims [F, H, E]    -> blocks [E, H, F/32, 20]
  ``blk.{l}.ffn_{gate,up,down}_shexp.weight``  the shared expert (2-D)
  ``blk.{l}.ffn_gate_inp.weight``        router dims [H, E] (E rows of H), F32 / F16 / BF16
  ``blk.{l}.ffn_gate_inp_shexp.weight``  shared-expert gate [H]
  ``blk.{l}.ffn_norm.weight`` or ``blk.{l}.post_attention_norm.weight``  the RMSNorm in front of the MoE
GGUF stores each expert's matrix contiguously (experts outermost), rows of Q4_1 blocks along the input
dimension, which is already this library's block order: the bytes are viewed, not converted, then
repacked on the device.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"GGUF"
# metadata value types
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
T_STRING, T_ARRAY = 8, 9
# tensor types: (name, bytes per block, values per block)
TENSOR_TYPES = {0: ("F32", 4, 1), 1: ("F16", 2, 1), 2: ("Q4_0", 18, 32), 3: ("Q4_1", 20, 32), 8: ("Q8_0", 34, 32),
                30: ("BF16", 2, 1)}


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dims: tuple          # innermost first, as GGUF stores them
    type: int
    offset: int          # absolute byte offset in the file
    nbytes: int

    @property
    def type_name(self) -> str:
        return TENSOR_TYPES.get(self.type, (f"type{self.type}",))[0]


class GGUFFile:
    """The index of a GGUF file (metadata and tensor infos); tensor bytes are memory-mapped on demand."""

    def __init__(self, path):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            head = f.read(24)
            if len(head) < 24 or head[:4] != MAGIC:
                raise ValueError(f"{self.path}: not a GGUF file")
            self.version, n_tensors, n_kv = struct.unpack("<IQQ", head[4:24])
            if self.version < 2:
                raise ValueError(f"{self.path}: GGUF version {self.version} is not supported (2 or later)")
            self.meta = {}
            for _ in range(n_kv):
                key = self._str(f)
                (vt,) = struct.unpack("<I", f.read(4))
                self.meta[key] = self._value(f, vt)
            infos = []
            for _ in range(n_tensors):
                name = self._str(f)
                (nd,) = struct.unpack("<I", f.read(4))
                dims = struct.unpack(f"<{nd}Q", f.read(8 * nd))
                tt, off = struct.unpack("<IQ", f.read(12))
                infos.append((name, dims, tt, off))
            align = int(self.meta.get("general.alignment", 32))
            base = f.tell()
            base += (align - base % align) % align
        self.data_offset = base
        self.tensors = {}
        for name, dims, tt, off in infos:
            n = int(np.prod(dims, dtype=np.int64))
            if tt in TENSOR_TYPES:
                _, bb, bv = TENSOR_TYPES[tt]
                if n % bv:
                    raise ValueError(f"{name}: {n} values is not a whole number of {bv}-value blocks")
                nbytes = n // bv * bb
            else:
                nbytes = -1   # a type this reader does not size (not needed for the MoE path)
            self.tensors[name] = TensorInfo(name, tuple(int(d) for d in dims), tt, base + off, nbytes)

    @staticmethod
    def _str(f) -> str:
        (n,) = struct.unpack("<Q", f.read(8))
        return f.read(n).decode("utf-8")

    def _value(self, f, vt):
        if vt in _SCALAR:
            fmt = _SCALAR[vt]
            return struct.unpack(fmt, f.read(struct.calcsize(fmt)))[0]
        if vt == T_STRING:
            return self._str(f)
        if vt == T_ARRAY:
            et, n = struct.unpack("<IQ", f.read(12))
            return [self._value(f, et) for _ in range(n)]
        raise ValueError(f"{self.path}: unknown metadata value type {vt}")

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes (read-only uint8 memory map)."""
        t = self.tensors[name]
        if t.nbytes < 0:
            raise ValueError(f"{name}: tensor type {t.type} is not supported here")
        return np.memmap(self.path, np.uint8, "r", offset=t.offset, shape=(t.nbytes,))

    def values(self, name: str) -> np.ndarray:
        """An F32 / F16 / BF16 tensor as f32, shape dims reversed (outermost first)."""
        t = self.tensors[name]
        b = np.asarray(self.raw(name))
        if t.type == 0:
            v = b.view(np.float32)
        elif t.type == 1:
            v = b.view(np.float16).astype(np.float32)
        elif t.type == 30:
            v = (b.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            raise ValueError(f"{name}: {t.type_name} is not a float tensor")
        return v.reshape(t.dims[::-1])

    def q4_1_blocks(self, name: str) -> np.ndarray:
        """A Q4_1 tensor as blocks [..., rows, in/32, 20] (dims reversed: experts, rows, blocks)."""
        t = self.tensors[name]
        if t.type != 3:
            raise ValueError(f"{name}: {t.type_name}, expected Q4_1")
        inner = t.dims[0]
        return np.asarray(self.raw(name)).reshape(*t.dims[:0:-1], inner // 32, 20)


def moe_tensors(layer: int) -> dict:
    b = f"blk.{layer}."
    return {"gate": b + "ffn_gate_exps.weight", "up": b + "ffn_up_exps.weight", "down": b + "ffn_down_exps.weight",
            "router": b + "ffn_gate_inp.weight", "sgate": b + "ffn_gate_shexp.weight", "sup": b + "ffn_up_shexp.weight",
            "sdown": b + "ffn_down_shexp.weight", "sgw": b + "ffn_gate_inp_shexp.weight",
            "norm": (b + "post_attention_norm.weight", b + "ffn_norm.weight")}


def read_moe_layer(gg: GGUFFile, layer: int, top_k: int | None = None, experts: range | None = None):
    """The MoE tensors of one layer in the reference's block layout (host numpy):
    dict(cfg=dict(hidden, n_experts, top_k, ffn, shared_ffn), gate, up, down [E_sel, ...], router_w [H, E],
    shared=(gate, up, down, sgw) or None, norm_w [H] or None). ``experts`` selects a contiguous range
    (expert parallelism); the router always covers all experts."""
    n = moe_tensors(layer)
    gate, up, down = (gg.q4_1_blocks(n[k]) for k in ("gate", "up", "down"))
    E, F, nbh, _ = gate.shape
    H = nbh * 32
    if up.shape != gate.shape or down.shape != (E, H, F // 32, 20):
        raise ValueError(f"layer {layer}: expert tensors disagree on (E, F, H) = ({E}, {F}, {H})")
    if experts is not None:
        gate, up, down = gate[experts.start:experts.stop], up[experts.start:experts.stop], down[experts.start:experts.stop]
    router = gg.values(n["router"])                      # [E, H] rows
    if router.shape != (E, H):
        raise ValueError(f"{n['router']}: shape {router.shape}, expected ({E}, {H})")
    shared, FS = None, 0
    if n["sgate"] in gg.tensors:
        sg, su, sd = (gg.q4_1_blocks(n[k]) for k in ("sgate", "sup", "sdown"))
        FS = sg.shape[0]
        shared = (sg, su, sd, gg.values(n["sgw"]).reshape(H))
    norm = next((gg.values(nm).reshape(H) for nm in n["norm"] if nm in gg.tensors), None)
    arch = gg.meta.get("general.architecture", "")
    k = top_k if top_k is not None else int(gg.meta.get(f"{arch}.expert_used_count", 8))
    return dict(cfg=dict(hidden=H, n_experts=E, top_k=k, ffn=F, shared_ffn=FS), gate=gate, up=up, down=down,
                router_w=np.ascontiguousarray(router.T), shared=shared, norm_w=norm)


def load_moe_layer(path_or_file, layer: int, device="cuda", top_k: int | None = None, experts: range | None = None,
                   scales: str = "fp16"):
    """(MoELayer, norm_w or None) for one layer of a GGUF model, weights repacked on the device."""
    import torch

    from .layer import MoEConfig, MoELayer
    gg = path_or_file if isinstance(path_or_file, GGUFFile) else GGUFFile(path_or_file)
    d = read_moe_layer(gg, layer, top_k, experts)
    c = d["cfg"]
    eb, el = (experts.start, experts.stop - experts.start) if experts is not None else (0, None)
    cfg = MoEConfig(c["hidden"], c["n_experts"], c["top_k"], c["ffn"], c["shared_ffn"], eb, el)
    layer_obj = MoELayer.from_q4_1(cfg, np.ascontiguousarray(d["gate"]), np.ascontiguousarray(d["up"]),
                                   np.ascontiguousarray(d["down"]), d["router_w"], shared=d["shared"], device=device,
                                   scales=scales)
    norm = None if d["norm_w"] is None else torch.from_numpy(d["norm_w"].astype(np.float32)).to(device, torch.bfloat16)
    return layer_obj, norm
