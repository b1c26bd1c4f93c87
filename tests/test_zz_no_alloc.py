"""fm_moe_layer_noalloc: the MoE layer for callers that cannot allocate device memory.

An engine that reserves all of its device memory at model load has nowhere to put a per-call workspace,
and a decode loop that must not stall cannot afford the device synchronisation a cudaMalloc may cause;
this entry point takes only inputs and outputs and keeps its scratch space in a static device array
inside the library. The tests call it through the C ABI twice in a row and check each result against
fm_moe_layer with a caller-owned workspace and against the fp64 oracle, within the parity tolerance the
other GPU tests use, on both kernel paths (the decode GEMV, and the tcgen05 path with the tcgen05 router
from 256 tokens), and check that device memory stays where it was across the calls: the first call on a
device only looks the array up (with lazy module loading that is when the driver places the array on the
device, so the first call may lower free memory by at most the array's size) and creates its side
stream; later calls change nothing. The file sorts last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import cases, moe as OM

pytestmark = pytest.mark.gpu

TOL = 2e-2
ARRAY_BYTES = 24 << 20


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda:0")


def _layer(c, dev):
    import flowmoe
    cfg = flowmoe.MoEConfig(hidden=c["H"], n_experts=c["E"], top_k=c["k"], ffn=c["F"], shared_ffn=c["FS"])
    return flowmoe.MoELayer.from_q4_1(cfg, c["gate"], c["up"], c["down"], c["Wr"], shared=c["shared"], device=dev)


def _noalloc(lay, x, res, T, t_real, out, idx, w):
    from flowmoe import _lib
    st = torch.cuda.current_stream().cuda_stream
    return _lib.lib.fm_moe_layer_noalloc(ctypes.byref(lay._L), x.data_ptr(), _lib.FM_BF16, res.data_ptr(), T, t_real,
                                         out.data_ptr(), idx.data_ptr(), w.data_ptr(), st)


def _free():
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]


def _two_calls(c, dev, lay, sizes):
    """Two noalloc calls in a row (sizes = [(T, t_real), ...]), each against fm_moe_layer and the oracle; the
    free device memory after the first call stays the same through the second."""
    from flowmoe import _lib
    k = c["k"]
    runs = []
    for T, t_real in sizes:   # every torch-side buffer (and fm_moe_layer's workspace) exists before the calls
        x = torch.from_numpy(c["x"][:T]).to(dev).to(torch.bfloat16)
        res = torch.from_numpy(c["res"][:T]).to(dev)
        want = lay.forward(x, res, t_real=t_real).cpu().numpy()
        got = torch.full_like(res, float("nan"))
        idx = torch.empty(T, k, dtype=torch.int32, device=dev)
        w = torch.empty(T, k, dtype=torch.float32, device=dev)
        runs.append((T, t_real, x, res, want, got, idx, w))
    free = [_free()]
    for T, t_real, x, res, want, got, idx, w in runs:
        assert _noalloc(lay, x, res, T, t_real, got, idx, w) == _lib.FM_OK, _lib.last_error()
        free.append(_free())
    assert free[0] - free[1] <= ARRAY_BYTES, f"the first call took {free[0] - free[1]} B of device memory"
    assert free[2] == free[1], f"the second call changed free device memory by {free[1] - free[2]} B"
    for call, (T, t_real, x, res, want, got, idx, w) in enumerate(runs):
        got_h, res_h = got.cpu().numpy(), c["res"][:T]
        np.testing.assert_array_equal(got_h[t_real:], res_h[t_real:])   # rows past t_real carry res
        err = np.abs(got_h - want).max() / np.abs(want - res_h).max()
        assert err < TOL, f"call {call}: max rel err {err:.3e} against fm_moe_layer"
        idx_h, w_h = idx.cpu().numpy()[:t_real], w.cpu().numpy()[:t_real]
        ref = OM.moe_block_f64(c["x"][:t_real], res_h[:t_real], idx_h, w_h, c["gate"], c["up"], c["down"],
                               shared=c["shared"])
        err = np.abs(got_h[:t_real] - ref).max() / np.abs(ref - res_h[:t_real]).max()
        assert err < TOL, f"call {call}: max rel err {err:.3e} against the oracle"
        sure = OM.router_margins(c["x"][:t_real], c["Wr"], k) > 1e-3
        _, idx_ref, _ = OM.router_block(c["x"][:t_real], c["Wr"], k)
        np.testing.assert_array_equal(idx_h[sure], idx_ref[sure])


def test_noalloc_decode_path_twice(dev):
    """Decode sizes (the GEMV path): 48 then 40 tokens (the second with a padding row), shared expert on."""
    c = cases.make_case(H=2048, E=16, F=512, FS=512, k=8, T=48, seed=11)
    _two_calls(c, dev, _layer(c, dev), [(48, 48), (40, 39)])


def test_noalloc_prefill_path_twice(dev):
    """Prefill sizes on a narrow layer (the tcgen05 grouped GEMM and, from 256 tokens, the tcgen05 router):
    300 then 260 tokens, shared expert on (its kernels run on the side stream the first call created)."""
    c = cases.make_case(H=256, E=8, F=64, FS=64, k=2, T=300, seed=12)
    _two_calls(c, dev, _layer(c, dev), [(300, 300), (260, 257)])


@pytest.mark.parametrize("T", [1, 32])
def test_noalloc_captured_in_a_graph(dev, T):
    """The use the entry point exists for: after one eager call, the call is captured into a CUDA graph
    (the decode chain's kernels carry the programmatic-dependent-launch attribute into it) and replayed
    on new inputs copied into the captured buffers; every replay matches an eager fm_moe_layer call on
    the same inputs, and replays leave free device memory unchanged."""
    from flowmoe import _lib
    c = cases.make_case(H=2048, E=16, F=512, FS=512, k=8, T=3 * T, seed=14 + T)
    lay = _layer(c, dev)
    x = torch.from_numpy(c["x"][:T]).to(dev).to(torch.bfloat16)
    res = torch.from_numpy(c["res"][:T]).to(dev)
    out = torch.empty_like(res)
    idx = torch.empty(T, 8, dtype=torch.int32, device=dev)
    w = torch.empty(T, 8, device=dev)
    assert _noalloc(lay, x, res, T, T, out, idx, w) == _lib.FM_OK, _lib.last_error()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        assert _noalloc(lay, x, res, T, T, out, idx, w) == _lib.FM_OK, _lib.last_error()
    inputs = []
    for r in range(3):   # the eager references first, so that no torch allocation falls between replays
        xs = torch.from_numpy(c["x"][r * T:(r + 1) * T]).to(dev).to(torch.bfloat16)
        rs = torch.from_numpy(c["res"][r * T:(r + 1) * T]).to(dev)
        inputs.append((xs, rs, lay.forward(xs, rs).cpu().numpy()))
    free = _free()
    for r, (xs, rs, want) in enumerate(inputs):
        x.copy_(xs)
        res.copy_(rs)
        out.fill_(float("nan"))
        g.replay()
        got = out.cpu().numpy()
        err = np.abs(got - want).max() / np.abs(want - c["res"][r * T:(r + 1) * T]).max()
        assert err < TOL, f"replay {r}: max rel err {err:.3e} against fm_moe_layer"
    assert _free() == free, "a replay changed free device memory"
    del g


def test_noalloc_rejects_more_tokens_than_the_static_array(dev):
    from flowmoe import _lib
    c = cases.make_case(H=2048, E=16, F=512, FS=512, k=8, T=4, seed=13)
    lay = _layer(c, dev)
    T = 4096
    x = torch.zeros(T, 2048, dtype=torch.bfloat16, device=dev)
    res = torch.zeros(T, 2048, device=dev)
    out = torch.empty_like(res)
    idx = torch.empty(T, 8, dtype=torch.int32, device=dev)
    w = torch.empty(T, 8, device=dev)
    assert _noalloc(lay, x, res, T, T, out, idx, w) == _lib.FM_EWORKSPACE
    assert "static" in _lib.last_error()
