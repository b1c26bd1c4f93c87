"""fm_moe_layer_noalloc: the MoE layer for callers that cannot allocate device memory.

A decode loop being captured into a CUDA graph cannot call cudaMalloc, and an engine that plans all of
its device buffers up front has nowhere to put an extra workspace; this entry point takes only inputs
and outputs and keeps its scratch space in a static device array inside the library. The test calls
it through the C ABI twice in a row and checks each result against fm_moe_layer with a caller-owned
workspace, within the parity tolerance the other GPU tests use. The file sorts last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import cases

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import flowmoe
    c = cases.make_case(H=2048, E=16, F=512, FS=512, k=8, T=48, seed=11)
    cfg = flowmoe.MoEConfig(hidden=2048, n_experts=16, top_k=8, ffn=512, shared_ffn=512)
    lay = flowmoe.MoELayer.from_q4_1(cfg, c["gate"], c["up"], c["down"], c["Wr"], shared=c["shared"],
                                     device="cuda:0")
    return c, lay


def _noalloc(lay, x, res, T, t_real, out):
    from flowmoe import _lib
    st = torch.cuda.current_stream().cuda_stream
    return _lib.lib.fm_moe_layer_noalloc(ctypes.byref(lay._L), x.data_ptr(), _lib.FM_BF16, res.data_ptr(), T, t_real,
                                         out.data_ptr(), None, None, st)


def test_noalloc_matches_workspace_entry_point_twice(layer):
    from flowmoe import _lib
    c, lay = layer
    dev = torch.device("cuda:0")
    for call, T in enumerate((48, 40)):          # two calls in a row, the second over fewer tokens
        x = torch.from_numpy(c["x"][:T]).to(dev).to(torch.bfloat16)
        res = torch.from_numpy(c["res"][:T]).to(dev)
        want = lay.forward(x, res).cpu().numpy()
        got = torch.full_like(res, float("nan"))
        assert _noalloc(lay, x, res, T, T - call, got) == _lib.FM_OK, _lib.last_error()
        torch.cuda.synchronize()
        got = got.cpu().numpy()
        if call:   # rows past t_real are carried from res
            want[T - 1] = c["res"][T - 1]
        err = np.abs(got - want).max() / np.abs(want - c["res"][:T]).max()
        assert err < TOL, f"call {call}: max rel err {err:.3e}"


def test_noalloc_rejects_more_tokens_than_the_static_array(layer):
    from flowmoe import _lib
    c, lay = layer
    T = 4096
    x = torch.zeros(T, 2048, dtype=torch.bfloat16, device="cuda:0")
    res = torch.zeros(T, 2048, device="cuda:0")
    out = torch.empty_like(res)
    assert _noalloc(lay, x, res, T, T, out) == _lib.FM_EWORKSPACE
    assert "static" in _lib.last_error()
