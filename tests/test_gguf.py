"""GGUF ingestion (flowmoe.gguf): a small Qwen-MoE-shaped GGUF file written here (the GGUF container layout,
llama.cpp's MoE tensor names and dims), read back into the block layout; where the PyPI ``gguf`` package is
installed, its reader is the cross-check of the index. The GPU test runs the loaded layer against the
oracle on the same blocks."""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

from oracle import cases, moe as OM


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, tensors, meta, align=32):
    """tensors: [(name, dims innermost-first, type, bytes)]; meta: {key: (type, value)}."""
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta))
    kv = b""
    for k, (vt, v) in meta.items():
        kv += _str(k) + struct.pack("<I", vt)
        kv += _str(v) if vt == 8 else struct.pack({4: "<I", 6: "<f"}[vt], v)
    infos, off, blobs = b"", 0, []
    for name, dims, tt, data in tensors:
        infos += _str(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        infos += struct.pack("<IQ", tt, off)
        pad = (align - len(data) % align) % align
        blobs.append(bytes(data) + b"\0" * pad)
        off += len(data) + pad
    body = head + kv + infos
    body += b"\0" * ((align - len(body) % align) % align)
    with open(path, "wb") as f:
        f.write(body + b"".join(blobs))


def _model_file(tmp_path, c, layer=0):
    H, F, FS, E = c["H"], c["F"], c["FS"], c["E"]
    sg, su, sd, sgw = c["shared"]
    norm = OM.bf16_round((1.0 + np.random.default_rng(1).normal(0, 0.01, H)).astype(np.float32))
    b = f"blk.{layer}."
    tensors = [
        (b + "ffn_gate_exps.weight", (H, F, E), 3, c["gate"].tobytes()),
        (b + "ffn_up_exps.weight", (H, F, E), 3, c["up"].tobytes()),
        (b + "ffn_down_exps.weight", (F, H, E), 3, c["down"].tobytes()),
        (b + "ffn_gate_inp.weight", (H, E), 0, np.ascontiguousarray(c["Wr"].T, np.float32).tobytes()),
        (b + "ffn_gate_shexp.weight", (H, FS), 3, sg.tobytes()),
        (b + "ffn_up_shexp.weight", (H, FS), 3, su.tobytes()),
        (b + "ffn_down_shexp.weight", (FS, H), 3, sd.tobytes()),
        (b + "ffn_gate_inp_shexp.weight", (H,), 0, np.asarray(sgw, np.float32).tobytes()),
        (b + "ffn_norm.weight", (H,), 0, norm.tobytes()),
    ]
    meta = {"general.architecture": (8, "qwen3moe"), "qwen3moe.expert_used_count": (4, c["k"]),
            "general.alignment": (4, 32)}
    p = tmp_path / "moe.gguf"
    write_gguf(p, tensors, meta)
    return p, norm


def _case():
    return cases.make_case(H=256, E=8, F=128, FS=128, k=2, T=24, seed=31)


def test_read_moe_layer_blocks(tmp_path):
    from flowmoe.gguf import GGUFFile, read_moe_layer
    c = _case()
    p, norm = _model_file(tmp_path, c)
    gg = GGUFFile(p)
    d = read_moe_layer(gg, 0)
    assert d["cfg"] == dict(hidden=256, n_experts=8, top_k=2, ffn=128, shared_ffn=128)
    for k in ("gate", "up", "down"):
        assert np.array_equal(d[k], c[k])
    assert np.array_equal(d["router_w"], c["Wr"])
    for got, want in zip(d["shared"], c["shared"]):
        assert np.array_equal(np.asarray(got, np.float32) if got.dtype != np.uint8 else got,
                              want if want.dtype == np.uint8 else np.asarray(want, np.float32))
    assert np.array_equal(d["norm_w"], norm)
    sub = read_moe_layer(gg, 0, experts=range(2, 6))
    assert np.array_equal(sub["gate"], c["gate"][2:6])


def test_index_matches_gguf_package(tmp_path):
    gguf = pytest.importorskip("gguf")
    from flowmoe.gguf import GGUFFile
    p, _ = _model_file(tmp_path, _case())
    mine = GGUFFile(p)
    ref = gguf.GGUFReader(str(p))
    assert {t.name for t in ref.tensors} == set(mine.tensors)
    for t in ref.tensors:
        m = mine.tensors[t.name]
        assert int(t.data_offset) == m.offset
        assert tuple(int(x) for x in t.shape) == m.dims
        assert int(t.n_bytes) == m.nbytes


def test_not_gguf_rejected(tmp_path):
    from flowmoe.gguf import GGUFFile
    p = tmp_path / "x.bin"
    p.write_bytes(b"NOPE" + b"\0" * 40)
    with pytest.raises(ValueError, match="not a GGUF"):
        GGUFFile(p)


@pytest.mark.gpu
def test_loaded_layer_matches_oracle(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from flowmoe.gguf import load_moe_layer
    c = _case()
    p, norm = _model_file(tmp_path, c)
    layer, nw = load_moe_layer(p, 0, device="cuda")
    x = torch.from_numpy(c["res"]).cuda()
    out = layer.forward_norm(x, nw).cpu().numpy()
    want = OM.moe_stack_f64(c["res"], [dict(norm_w=norm, Wr=c["Wr"], gate=c["gate"], up=c["up"], down=c["down"],
                                            shared=c["shared"], k=c["k"])])
    assert float(np.abs(out - want).max() / np.abs(want - c["res"]).max()) < 2e-2
