"""Host-side pieces of flowmoe checked on the CPU: the torch Q4_1 quantiser against gguf's bytes."""
import numpy as np
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
