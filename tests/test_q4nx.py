"""The .q4nx importer (flowmoe.q4nx) against the reference's own container reader.

tests/golden/q4nx.npz holds the SHA-256 of every matrix the reference's reader
(open_kernels/model/q4nx.py, Q4NX.expert_w / shared_w / bf16) dequantises from a one-layer container that
the oracle's writer builds from seeded blocks; the shared expert's up matrix is in the signed quantiser's
form (mins written as zero), which both readers transcode. The CPU test rebuilds the container byte for
byte, reads it with this repository's importer and converts its chunks with the oracle's pool inverse;
the GPU test imports the layer onto the device and compares it with a layer built from the same blocks.
"""
import hashlib

import numpy as np
import pytest
import torch

from oracle import moe as OM, q4_1 as OQ, q4nx as OQX


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _container(golden, tmp_path):
    g = golden["q4nx"]
    E, F, H = int(g["E"]), int(g["F"]), int(g["H"])
    rng = np.random.default_rng(int(g["seed"]))
    ex = {k: [OQ.random_q4_1_blocks(F if k != "down" else H, H if k != "down" else F, rng) for _ in range(E)]
          for k in ("gate", "up", "down")}
    sh = {k: OQ.random_q4_1_blocks(F if k != "down" else H, H if k != "down" else F, rng) for k in ("gate", "up", "down")}
    d16 = np.ascontiguousarray(sh["up"][..., 0:2]).view(np.float16)
    sh["up"][..., 2:4] = (OM.bf16_round(d16.astype(np.float32)) * -8).astype(np.float16).view(np.uint8)
    wr = OM.bf16_bits(rng.normal(0, 0.02, (H, 8)).astype(np.float32))
    sgw = OM.bf16_bits(rng.normal(0, 0.02, H).astype(np.float32))
    pln = OM.bf16_bits(1 + rng.normal(0, 0.01, H).astype(np.float32))
    L = "model.layer.0."
    tens = {L + "post_attention_layernorm.weight": ("BF16", pln), L + "moe_router.weight": ("BF16", wr),
            L + "shared_expert_gate.weight": ("BF16", sgw)}
    for k in ("gate", "up", "down"):
        tens[L + f"mlp.{k}_exps_proj.weight"] = ("I8", np.concatenate([OQX.q4nx_matrix(b) for b in ex[k]]))
        tens[L + f"mlp.share_{k}_exps_proj.weight"] = ("I8", OQX.signed_q4_matrix(sh[k]) if k == "up"
                                                       else OQX.q4nx_matrix(sh[k]))
    path = tmp_path / "l0.q4nx"
    OQX.write_q4nx(path, tens)
    assert hashlib.sha256(path.read_bytes()).hexdigest() == str(g["container_sha"])
    return g, E, F, H, path, ex, sh, wr, sgw


def test_q4nx_reads_what_the_reference_reader_reads(golden, tmp_path):
    from flowmoe.q4nx import Q4nxFile
    g, E, F, H, path, ex, sh, wr, sgw = _container(golden, tmp_path)
    per = F * H // (32 * 256)
    with Q4nxFile(path) as f:
        for k in ("gate", "up", "down"):
            n, kk = (H, F) if k == "down" else (F, H)
            c = f.q4_1_chunks(f"model.layer.0.mlp.{k}_exps_proj.weight")
            for e in range(E):
                blocks = OQ.pool_to_blocks(c[e * per:(e + 1) * per].reshape(-1), n, kk, 1)
                assert _sha(OQ.dequant_q4_1(blocks)) == str(g[f"expert_{k}_{e}"]), (k, e)
            c = f.q4_1_chunks(f"model.layer.0.mlp.share_{k}_exps_proj.weight")
            assert _sha(OQ.dequant_q4_1(OQ.pool_to_blocks(c.reshape(-1), n, kk, 1))) == str(g[f"shared_{k}"]), k
        assert _sha(OM.bf16_to_f32(f.bf16("model.layer.0.moe_router.weight"))) == str(g["router"])
        with pytest.raises(KeyError):
            f.raw("model.layer.1.moe_router.weight")


@pytest.mark.gpu
def test_q4nx_layer_on_device(golden, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import flowmoe
    from flowmoe.q4nx import Q4nxFile
    g, E, F, H, path, ex, sh, wr, sgw = _container(golden, tmp_path)
    dev = torch.device("cuda:0")
    cfg = flowmoe.MoEConfig(hidden=H, n_experts=8, top_k=2, ffn=F, shared_ffn=F, e_begin=0, e_local=E)
    narrow = lambda b: OQ.pool_to_blocks(OQX.q4nx_matrix(b).reshape(-1), b.shape[0], b.shape[1] * 32, 1)
    with Q4nxFile(path) as f:
        layer = f.moe_layer(0, cfg, device=dev)
        gate, up, down = f.expert_blocks(0, F, H, device=dev)
    for k, got in (("gate", gate), ("up", up), ("down", down)):
        for e in range(E):
            assert np.array_equal(got[e].cpu().numpy(), narrow(ex[k][e])), (k, e)
    sgu = np.stack([narrow(sh["gate"]), narrow(sh["up"])])
    ref = flowmoe.MoELayer.from_q4_1(cfg, np.stack([narrow(b) for b in ex["gate"]]), np.stack([narrow(b) for b in ex["up"]]),
                                     np.stack([narrow(b) for b in ex["down"]]), wr,
                                     shared=(sgu[0], sgu[1], narrow(sh["down"]), sgw), device=dev)
    for a, b in ((layer.gate_up, ref.gate_up), (layer.down, ref.down), (layer.shared_gate_up, ref.shared_gate_up),
                 (layer.shared_down, ref.shared_down), (layer.router, ref.router)):
        assert torch.equal(a, b)
