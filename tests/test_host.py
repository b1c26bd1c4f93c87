"""Host-side pieces of flowmoe checked on the CPU: the torch Q4_1 quantiser against gguf's bytes, and the
layer's input checks."""
import numpy as np
import pytest
import torch


def test_torch_quantizer_matches_gguf(golden):
    import flowmoe
    g = golden["q4_1"]
    got = flowmoe.quantize_q4_1(torch.from_numpy(g["gguf_in"])).numpy()
    assert np.array_equal(got.reshape(-1), g["gguf_q4_1"].reshape(-1))


def test_torch_dequant_matches_reference(golden):
    import flowmoe
    g = golden["q4_1"]
    got = flowmoe.dequantize_q4_1(torch.from_numpy(g["blocks"])).numpy()
    assert np.array_equal(got, g["dequant"])


@pytest.mark.parametrize("bad", ["gate", "down", "router", "shared", "sgw", "bias"])
def test_layer_inputs_checked_before_device_work(bad):
    # every size check of MoELayer.from_q4_1 runs on the host first: no device is touched here
    import flowmoe
    from oracle import cases
    c = cases.make_case(H=256, E=4, F=128, FS=128, k=2, T=1, seed=0)
    cfg = flowmoe.MoEConfig(hidden=256, n_experts=4, top_k=2, ffn=128, shared_ffn=128)
    gate, down, wr, shared, bias = c["gate"], c["down"], c["Wr"], c["shared"], np.zeros(4, np.float32)
    if bad == "gate":
        gate = gate[:3]
    elif bad == "down":
        down = down[:, :128]
    elif bad == "router":
        wr = wr.T
    elif bad == "shared":
        shared = (shared[0][:64],) + tuple(shared[1:])
    elif bad == "sgw":
        shared = tuple(shared[:3]) + (shared[3][:100],)
    else:
        bias = np.zeros(5, np.float32)
    with pytest.raises(ValueError):
        flowmoe.MoELayer.from_q4_1(cfg, gate, c["up"], down, wr, shared=shared, device="cpu", router_bias=bias)


@pytest.mark.parametrize("which", ["res_dtype", "out_shape", "idx_dtype", "w_device", "gate_shape"])
def test_buffers_checked_before_the_library_sees_their_pointers(which):
    # a layer object over host tensors (its constructor makes no library call); every wrong buffer must be
    # refused in Python, since the kernels would read or write through the raw pointer
    import flowmoe
    cfg = flowmoe.MoEConfig(hidden=256, n_experts=4, top_k=2, ffn=128, shared_ffn=0)
    dummy = torch.empty(16, dtype=torch.uint8)
    layer = flowmoe.MoELayer(cfg, dummy, dummy, torch.empty(5, 256, dtype=torch.bfloat16))
    T = 3
    x = torch.zeros(T, 256, dtype=torch.bfloat16)
    res, out = torch.zeros(T, 256), torch.zeros(T, 256)
    idx, w, sg = torch.zeros(T, 2, dtype=torch.int32), torch.zeros(T, 2), torch.zeros(T)
    if which == "res_dtype":
        res = res.double()
    elif which == "out_shape":
        out = torch.zeros(T + 1, 256)
    elif which == "idx_dtype":
        idx = idx.long()
    elif which == "w_device":
        w = w.to("meta")
    else:
        sg = torch.zeros(T + 2)
    with pytest.raises(ValueError):
        if which == "gate_shape":
            layer.moe_block(x, res, idx, w, shared_gate=sg)
        else:
            layer.forward(x, res, out=out, idx=idx, w=w)


def test_tile_wrappers_refuse_host_buffers():
    # the tile kernels take raw device pointers: host tensors and short outputs are refused in Python
    import flowmoe
    from flowmoe.layer import narrow_scales
    host = torch.zeros(5120, dtype=torch.uint8)
    with pytest.raises(ValueError):
        flowmoe.tiles_to_q4_1(host, 128, 64)
    with pytest.raises(ValueError):
        narrow_scales(host)
    with pytest.raises(ValueError):
        flowmoe.q4_1_to_tiles(host, 128, 64, device="cpu", out=torch.zeros(100, dtype=torch.uint8))
