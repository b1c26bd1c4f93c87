"""The CPU oracle pinned against the reference's own golden vectors (tests/golden/*.npz)."""
import ctypes
import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import moe as OM
from oracle import q4_1 as OQ

ROOT = Path(__file__).resolve().parents[1]


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_generator_matches_reference_bytes(golden):
    blocks = OQ.random_q4_1_blocks(64, 256, np.random.default_rng(0))
    assert np.array_equal(blocks, golden["q4_1"]["blocks"])


def test_dequant_bit_exact(golden):
    g = golden["q4_1"]
    assert np.array_equal(OQ.dequant_q4_1(g["blocks"]), g["dequant"])


def test_quantizer_matches_gguf_bytes(golden):
    g = golden["q4_1"]
    got = OQ.quantize_q4_1(g["gguf_in"])
    assert np.array_equal(got.reshape(-1), g["gguf_q4_1"].reshape(-1))
    assert np.array_equal(OQ.dequant_q4_1(got).reshape(-1), g["gguf_dequant"].reshape(-1))


def test_router_random_case(golden):
    r = golden["router"]
    p, idx, w = OM.router_block(r["rc_xm"], r["rc_Wr"], int(r["rc_topk"]))
    np.testing.assert_allclose(p, r["rc_probs"], rtol=1e-12, atol=1e-15)
    assert np.array_equal(idx, r["rc_idx"])
    np.testing.assert_allclose(w, r["rc_w"], rtol=1e-12)


def test_router_tie_lowest_index(golden):
    r = golden["router"]
    p, idx, w = OM.router_block(r["tie_x"], r["tie_W"], 2)
    assert idx.tolist() == r["tie_idx"].tolist() == [[0, 1]]
    np.testing.assert_allclose(w, r["tie_w"])


def _c1_inputs():
    from oracle.moe import bf16_round
    r2 = np.random.default_rng(0)
    x1 = bf16_round(r2.standard_normal((16, 2048), dtype=np.float32))
    W1 = bf16_round(r2.normal(0, 0.02, (2048, 128)).astype(np.float32))
    return x1, W1


def test_router_config1(golden):
    r = golden["router"]
    x1, W1 = _c1_inputs()
    assert _sha(x1) == str(r["c1_x_sha"]) and _sha(W1) == str(r["c1_W_sha"])
    p, idx, w = OM.router_block(x1, W1, 8)
    assert np.array_equal(idx, r["c1_idx"])
    np.testing.assert_allclose(w, r["c1_w"], rtol=1e-12)


def test_router_topk_past_experts_raises():
    with pytest.raises(ValueError):
        OM.router_block(np.zeros((1, 4)), np.zeros((4, 3)), 4)


def _moe_inputs(g):
    H, E, F, FS = int(g["H"]), int(g["E"]), int(g["F"]), int(g["FS"])
    rng = np.random.default_rng(0)
    gate = [OQ.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    up = [OQ.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    down = [OQ.random_q4_1_blocks(H, F, rng, scale=0.05) for _ in range(E)]
    sg, su, sd = (OQ.random_q4_1_blocks(FS, H, rng), OQ.random_q4_1_blocks(FS, H, rng),
                  OQ.random_q4_1_blocks(H, FS, rng, scale=0.05))
    allb = np.concatenate([b.reshape(-1) for b in gate + up + down + [sg, su, sd]])
    assert _sha(allb) == str(g["blocks_sha"]), "regenerated blocks differ from the reference's"
    return gate, up, down, (sg, su, sd, g["sgw"])


def test_moe_block_matches_replica_fp64(golden):
    g = golden["moe"]
    gate, up, down, shared = _moe_inputs(g)
    xm, top, probs = g["xm"], g["top"], g["probs"]
    w = np.take_along_axis(probs, top, -1)
    w = w / w.sum(-1, keepdims=True)
    out = OM.moe_block_f64(xm, g["xres"], top, w, gate, up, down, shared=shared, engine_rounding=False)
    # replica.moe_decode multiplies f32 matrices (numpy f32 matmuls), the oracle in f64: agree to f32 roundoff
    assert np.abs(out - g["out"]).max() / np.abs(g["out"]).max() < 1e-5
    # the router the block consumed is the oracle's own
    p, idx, w2 = OM.router_block(xm, g["Wr"], 8)
    assert np.array_equal(idx, top)
    # the engine's bf16 rounding points move the result by far less than the parity tolerance
    out_r = OM.moe_block_f64(xm, g["xres"], top, w, gate, up, down, shared=shared)
    assert np.abs(out_r - out).max() / np.abs(out - g["xres"]).max() < 2e-2


def test_dispatch_stable_and_checked():
    idx = np.array([[2, 0], [0, 1], [2, 1]], np.int32)
    counts, offsets, pos, pair = OM.dispatch(idx, 3)
    assert counts.tolist() == [2, 2, 2]
    assert pair.tolist() == [1, 2, 3, 5, 0, 4]
    assert pos.reshape(-1)[pair].tolist() == list(range(6))
    with pytest.raises(ValueError):
        OM.dispatch(np.array([[3]], np.int32), 3)


def test_sampled_rows_equal_whole_block():
    """moe_rows_f64 (the checker of the full-size GPU calls) gives the whole-block oracle's rows exactly,
    shared expert and an expert offset (expert-parallel weights) included."""
    from oracle import cases
    c = cases.make_case(H=256, E=8, F=128, FS=128, k=3, T=20, seed=4)
    _, idx, w = OM.router_block(c["x"], c["Wr"], c["k"])
    whole = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    rows = np.array([17, 0, 5, 11])
    got = OM.moe_rows_f64(rows, c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    np.testing.assert_allclose(got, whole[rows], rtol=0, atol=1e-12)
    keep = np.nonzero((idx >= 2).all(axis=1))[0]   # tokens whose experts are all >= 2
    got2 = OM.moe_rows_f64(keep, c["x"], c["res"], idx, w, c["gate"][2:], c["up"][2:], c["down"][2:],
                           shared=c["shared"], e_begin=2)
    np.testing.assert_allclose(got2, whole[keep], rtol=0, atol=1e-12)


def test_cpu_baseline_matches_fp64():
    rng = np.random.default_rng(3)
    H, E, F, T = 256, 8, 128, 12
    gate = [OQ.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    up = [OQ.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    down = [OQ.random_q4_1_blocks(H, F, rng, scale=0.05) for _ in range(E)]
    Wr = OM.bf16_round(rng.normal(0, 0.2, (H, E)).astype(np.float32))
    x = OM.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    res = rng.standard_normal((T, H)).astype(np.float32)
    layer = OM.MoeLayerF32(Wr, gate, up, down, topk=3)
    out, idx, w = layer.forward(x, res)
    ref = OM.moe_block_f64(x, res, idx, w, gate, up, down)
    assert np.abs(out - ref).max() / np.abs(ref - res).max() < 1e-3


_REF = ROOT / "oracle" / "_ref" / "libref_router.so"


@pytest.mark.skipif(not _REF.exists(), reason="reference router not built (make -C oracle)")
def test_reference_cpp_router_agrees_with_oracle(golden):
    lib = ctypes.CDLL(str(_REF))
    x1, W1 = _c1_inputs()
    T, H = x1.shape
    E, k = W1.shape[1], 8
    probs = np.zeros((T, E), np.float32)
    idx = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    rc = lib.ref_router_block(ctypes.c_size_t(T), ctypes.c_size_t(H), ctypes.c_size_t(E), ctypes.c_size_t(k),
                              P(np.ascontiguousarray(x1)), P(np.ascontiguousarray(W1)), P(probs), P(idx), P(w))
    assert rc == 0
    r = golden["router"]
    assert np.array_equal(idx, r["c1_idx"])
    np.testing.assert_allclose(w, r["c1_w"], rtol=1e-4)


def test_rmsnorm_matches_reference_route(golden):
    """The post-attention RMSNorm (xm of replica.route, reference open_kernels/model/replica.py:121-124)."""
    g = golden["moe"]
    xm = OM.rmsnorm(g["xres"], g["postln"])
    np.testing.assert_array_equal(xm, g["xm"])


def test_dequant_bf16_scales_bit_exact(golden):
    """The q4nx numerics (d, m narrowed to bf16): the reference's dequant_q4_1(scale_dtype=bfloat16)."""
    g = golden["q4_1"]
    assert np.array_equal(OQ.dequant_q4_1(g["blocks"], bf16_scales=True), g["dequant_bf16_scales"])


def test_pool_packers_match_reference_bytes(golden):
    """The oracle's restatement of the reference's two pool packers writes their very bytes
    (q4_1_pack.pack_q4_1_pool: bf16 planes; gguf_pool.pack_q4_pool: f32 planes; rs = 2), and the inverse
    gives back the blocks exactly (f32) or with the bf16-narrowed scales the NPU pool computes with."""
    g = golden["q4_1"]
    b = g["blocks"]
    assert np.array_equal(OQ.blocks_to_pool(b, 2, 5120), g["pool_bf16_rs2"])
    assert np.array_equal(OQ.blocks_to_pool(b, 2, 6144), g["pool_f32_rs2"])
    assert np.array_equal(OQ.pool_to_blocks(g["pool_f32_rs2"], 64, 256, 2, 6144), b)
    b16 = OQ.pool_to_blocks(g["pool_bf16_rs2"], 64, 256, 2, 5120)
    assert np.array_equal(b16[..., 4:], b[..., 4:])
    assert np.array_equal(OQ.dequant_q4_1(b16), g["dequant_bf16_scales"])


def test_ep_stack_case_flips_only_through_bf16_y():
    """The expert-parallel paths carry routed y rows between ranks as bf16, an extra rounding point the
    oracle models with ``y_bf16``. On the two-rank stack case of tests/test_gpu_ep.py that rounding alone
    moves rank 1's output by about 5 % of the stack's update: one token there sits 4e-6 from a top-k tie
    in the third layer and changes an expert. Rank 0 has no such token, and one layer (no compounding)
    stays within the rounding itself."""
    from oracle import cases
    rng = np.random.default_rng(77)
    cs = []
    for l in range(3):
        c = cases.make_case(H=512, E=32, F=256, FS=256, k=8, T=64, seed=400 + l)
        c["norm_w"] = OM.bf16_round((1.0 + rng.normal(0, 0.01, c["H"])).astype(np.float32))
        cs.append(c)
    rel = []
    for lo, hi in ((0, 32), (32, 64)):
        x0 = cs[0]["res"][lo:hi]
        a, b = OM.moe_stack_f64(x0, cs), OM.moe_stack_f64(x0, cs, y_bf16=True)
        rel.append(float(np.abs(a - b).max() / np.abs(a - x0).max()))
    assert rel[0] < 2e-3 and rel[1] > 2e-2, rel
    # one layer: bf16 y rows change the block output by no more than their own rounding
    c = cs[0]
    xm = OM.rmsnorm(c["res"], c["norm_w"])
    _, idx, w = OM.router_block(OM.bf16_round(xm), c["Wr"], c["k"])
    a = OM.moe_block_f64(xm, c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    b = OM.moe_block_f64(xm, c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"], y_bf16=True)
    assert np.abs(a - b).max() <= 2.0 ** -8 * np.abs(a - c["res"]).max()


def _expert_pool_case(golden):
    g = golden["expert_pool"]
    E, F, H = int(g["E"]), int(g["F"]), int(g["H"])
    rng = np.random.default_rng(int(g["seed"]))
    up = [OQ.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    gate = [OQ.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    down = [OQ.random_q4_1_blocks(H, F, rng) for _ in range(E)]
    assert _sha(np.concatenate([b.reshape(-1) for b in up + gate + down])) == str(g["blocks_sha"])
    return g, E, F, H, up, gate, down


def test_expert_pool_matches_reference_bytes(golden):
    """The oracle's restatement of the engine's expert_stripes / expert_down ops (pools.cpp:927-962 over
    recipes/pack.py:498-530) writes the very pool bytes the reference's own packers and chunk orders
    produce for the same seeded experts, and its inverse gives the experts back (bf16 scales)."""
    g, E, F, H, up, gate, down = _expert_pool_case(golden)
    gu, dn = OQ.expert_pool(up, gate, down)
    assert _sha(gu) == str(g["gate_up_sha"]) and _sha(dn) == str(g["down_sha"])
    per = gu.size // E
    for e in range(E):
        st = gu[e * per:(e + 1) * per].reshape(F // 128, 2, -1)
        u_back = OQ.pool_to_blocks(st[:, 0].reshape(-1), F, H, 4)
        assert np.array_equal(OQ.dequant_q4_1(u_back), OQ.dequant_q4_1(up[e], bf16_scales=True))


def test_gemm_oracle_matches_reference_pool_reference(golden):
    """The dense Q4_1 GEMM oracle over the blocks recovered from the reference's pool bytes equals the
    reference's own fp64 pool_reference (designs/gemm_q4_prefill/make_test.py recipe), token by token."""
    g = golden["gemm_q4"]
    n, k = int(g["n"]), int(g["k"])
    blocks = OQ.pool_to_blocks(g["pool"], n, k, int(g["rs"]))
    x = OM.bf16_to_f32(g["x_bf16"])
    y = OM.q4_gemm_f64(x, blocks)
    ref = g["y"]
    assert y.shape == ref.shape == (int(g["T"]), n)
    assert np.abs(y - ref).max() <= 1e-6 * np.abs(ref).max()
