"""The JSONL stage record (the reference's OFLM_OPEN_PROFILE: header, request and per-layer rows with the
MoE block split as moe_prep / moe_patch / moe_run / moe_read, src/open_qwen36/core.cpp:850-935) written
from the library's stage events over an eager pass of a small stack, on both kernel paths."""
import json

import numpy as np
import pytest
import torch

from oracle import cases, moe as OM

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [8, 300])
def test_stage_profile_records(tmp_path, T):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import flowmoe
    from flowmoe.profile import StageProfile
    from flowmoe.stack import MoEStack
    dev = torch.device("cuda:0")
    layers, nws = [], []
    rng = np.random.default_rng(T)
    for l in range(2):
        c = cases.make_case(H=256, E=8, F=128, FS=128, k=2, T=T, seed=50 + l)
        cfg = flowmoe.MoEConfig(hidden=256, n_experts=8, top_k=2, ffn=128, shared_ffn=128)
        layers.append(flowmoe.MoELayer.from_q4_1(cfg, c["gate"], c["up"], c["down"], c["Wr"], shared=c["shared"],
                                                 device=dev))
        nws.append(torch.from_numpy(OM.bf16_round((1 + rng.normal(0, 0.01, 256)).astype(np.float32))))
    stack = MoEStack(layers, nws)
    x = torch.from_numpy(c["res"]).to(dev)
    path = tmp_path / "prof.jsonl"
    with StageProfile(str(path), layers=2) as prof:
        y = prof.request("prefill" if T > 128 else "decode", T, lambda hook: stack.forward(x, layer_hook=hook))
    ref = stack.forward(x)
    np.testing.assert_allclose(y.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-5)   # profiling changes nothing
    recs = [json.loads(l) for l in path.read_text().splitlines()]
    assert recs[0] == {"record": "header", "version": 1, "family": "qwen36moe", "layers": 2}
    assert recs[1]["record"] == "request" and recs[1]["tokens"] == T and recs[1]["layers"] == 2
    rows = recs[2:]
    assert [r["layer"] for r in rows] == [0, 1] and all(r["record"] == "layer" for r in rows)
    for r in rows:
        for k in ("moe_prep_ms", "moe_patch_ms", "moe_run_ms", "moe_read_ms", "router_ms", "gate_up_ms", "down_ms"):
            assert k in r and r[k] >= 0
        assert r["moe_run_ms"] > 0 and r["router_ms"] > 0 and r["wall_ms"] >= r["total_ms"] * 0.5
        assert abs(r["moe_run_ms"] - (r["gate_up_ms"] + r["down_ms"])) < 2e-3
