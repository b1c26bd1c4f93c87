"""Parity of the CUDA path (through the C ABI) against the CPU oracle on identical seeded inputs.

Bars: expert ids, counts and permutations bit-exact wherever the router margin
(k-th minus (k+1)-th probability) exceeds 1e-3; block outputs within max relative error 2e-2 of an
fp64 accumulation of the same dequantised weights, measured as max|got - ref| / max|ref - res| (the
expert contribution, so the residual cannot hide an error).
"""
import numpy as np
import pytest
import torch

from oracle import cases, moe as OM, q4_1 as OQ

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda:0")


def _layer(c, dev, path="auto"):
    import flowmoe
    cfg = flowmoe.MoEConfig(hidden=c["H"], n_experts=c["E"], top_k=c["k"], ffn=c["F"], shared_ffn=c["FS"])
    layer = flowmoe.MoELayer.from_q4_1(cfg, c["gate"], c["up"], c["down"], c["Wr"], shared=c["shared"], device=dev,
                                       router_bias=c.get("bias"))
    layer.path = path
    return layer


def _rel(got, ref, res):
    return float(np.abs(got - ref).max() / max(np.abs(ref - res).max(), 1e-30))


def test_tiles_round_trip_bit_exact(dev):
    import flowmoe
    rng = np.random.default_rng(5)
    blocks = OQ.random_q4_1_blocks(256, 512, rng)
    t = flowmoe.q4_1_to_tiles(blocks, 256, 512, dev)
    back = flowmoe.tiles_to_q4_1(t, 256, 512).cpu().numpy()
    assert np.array_equal(back.reshape(blocks.shape), blocks)
    assert not np.array_equal(t.cpu().numpy(), blocks.reshape(-1))   # it is a real permutation


@pytest.mark.parametrize("chunk", [5120, 6144])
def test_pool_import_bit_exact(dev, golden, chunk):
    """The reference's pool bytes (its own packers' output, and the oracle's restatement of them at an
    expert-stripe split rs = 4) -> GGUF blocks on the device, bit for bit the oracle's inverse; the f32
    pool gives back the original blocks, the bf16 pool their bf16-scale twins; the imported blocks then
    tile like any others."""
    import flowmoe
    g = golden["q4_1"]
    pool = g["pool_bf16_rs2" if chunk == 5120 else "pool_f32_rs2"]
    got = flowmoe.pool_to_q4_1(pool, 64, 256, rs=2, device=dev).cpu().numpy()
    assert np.array_equal(got, OQ.pool_to_blocks(pool, 64, 256, 2, chunk))
    blocks = OQ.random_q4_1_blocks(512, 2048, np.random.default_rng(7))
    pool4 = OQ.blocks_to_pool(blocks, 4, chunk)
    got4 = flowmoe.pool_to_q4_1(pool4, 512, 2048, rs=4, device=dev)
    want4 = OQ.pool_to_blocks(pool4, 512, 2048, 4, chunk)
    assert np.array_equal(got4.cpu().numpy(), want4)
    if chunk == 6144:
        assert np.array_equal(want4, blocks)
    t = flowmoe.q4_1_to_tiles(got4, 512, 2048, dev)
    assert np.array_equal(flowmoe.tiles_to_q4_1(t, 512, 2048).cpu().numpy().reshape(want4.shape), want4)


def _check_router(c, probs, idx, w):
    xb = c["x"]
    p_ref, idx_ref, w_ref = OM.router_block(xb, c["Wr"], c["k"])
    margin = OM.router_margins(xb, c["Wr"], c["k"])
    sure = margin > 1e-3
    assert sure.sum() >= 1
    np.testing.assert_array_equal(np.sort(idx[sure], 1), np.sort(idx_ref[sure], 1))
    np.testing.assert_array_equal(idx[sure], idx_ref[sure])
    np.testing.assert_allclose(w, w_ref, rtol=1e-3, atol=1e-5)
    if probs is not None:
        np.testing.assert_allclose(probs, p_ref, rtol=1e-3, atol=1e-6)


@pytest.mark.parametrize("T,E,H", [(16, 128, 2048), (1, 128, 2048), (333, 256, 2048), (64, 8, 256)])
def test_router_topk_parity(dev, T, E, H):
    import flowmoe
    c = cases.make_case(H=H, E=E, F=128, T=T, seed=T, weights=None)
    x = torch.from_numpy(c["x"]).to(dev).to(torch.bfloat16)
    Wr = torch.from_numpy(c["Wr"]).to(dev)
    probs, idx, w = flowmoe.router_block(x, Wr, c["k"])
    _check_router(c, probs.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy())


def test_router_reference_fixture_and_tie(dev, golden):
    import flowmoe
    r = golden["router"]
    x = torch.tensor(r["rc_xm"], dtype=torch.float32, device=dev)
    W = torch.tensor(r["rc_Wr"], dtype=torch.float32, device=dev)
    # the device rounds xm and Wr to bf16 (the reference's NPU router does too); compare with the
    # oracle on the same rounded operands, ids exact where the margin allows
    p, idx, w = flowmoe.router_block(x, W, int(r["rc_topk"]))
    xb, Wb = OM.bf16_round(r["rc_xm"]), OM.bf16_round(r["rc_Wr"])
    p_ref, idx_ref, w_ref = OM.router_block(xb, Wb, int(r["rc_topk"]))
    sure = OM.router_margins(xb, Wb, int(r["rc_topk"])) > 1e-3
    np.testing.assert_array_equal(idx.cpu().numpy()[sure], idx_ref[sure])
    np.testing.assert_allclose(w.cpu().numpy(), w_ref, rtol=1e-3)
    # tie KAT (test_prefill_batch.py:363-369): experts 0, 1, 3 tie -> [0, 1], weights 0.5 / 0.5
    tx = torch.tensor(r["tie_x"], dtype=torch.float32, device=dev)
    tW = torch.tensor(r["tie_W"], dtype=torch.float32, device=dev)
    p, idx, w = flowmoe.router_block(tx, tW, 2)
    assert idx.cpu().tolist() == [[0, 1]]
    np.testing.assert_allclose(w.cpu().numpy(), [[0.5, 0.5]], rtol=1e-6)


@pytest.mark.parametrize("T,E,k", [(16, 128, 8), (4096, 256, 8), (3, 8, 3), (700, 64, 6)])
def test_dispatch_bit_exact(dev, T, E, k):
    import flowmoe
    rng = np.random.default_rng(T)
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    if T > 100:   # skew: a hot expert (duplicates within a token are legal owed-list entries)
        idx[: T // 2, 0] = 3
    cfg = flowmoe.MoEConfig(hidden=256, n_experts=E, top_k=k, ffn=128)
    dummy = torch.zeros(256, dtype=torch.uint8, device=dev)
    layer = flowmoe.MoELayer(cfg, dummy, dummy, torch.zeros(E + 1, 256, dtype=torch.bfloat16, device=dev))
    t_real = T - 1 if T > 3 else T
    counts, offsets, pos, pair = layer.dispatch(torch.from_numpy(idx).to(dev), t_real)
    c_ref, o_ref, pos_ref, pair_ref = OM.dispatch(idx, E, t_real)
    np.testing.assert_array_equal(counts.cpu().numpy(), c_ref)
    np.testing.assert_array_equal(offsets.cpu().numpy(), o_ref)
    np.testing.assert_array_equal(pos.cpu().numpy(), pos_ref[:t_real])
    np.testing.assert_array_equal(pair.cpu().numpy(), pair_ref)


def _run_block(c, dev, t_real=None, path="auto"):
    layer = _layer(c, dev, path)
    x = torch.from_numpy(c["x"]).to(dev).to(torch.bfloat16)
    res = torch.from_numpy(c["res"]).to(dev)
    probs, idx, w = layer.router_block(x)
    sg = layer.shared_gate_buf if c["FS"] else None
    out = layer.moe_block(x, res, idx, w, t_real=t_real, shared_gate=sg)
    return layer, x, res, idx.cpu().numpy(), w.cpu().numpy(), out.cpu().numpy()


@pytest.mark.parametrize("T,path", [(16, "auto"), (1, "auto"), (32, "auto"), (16, "tc"), (1, "tc")])
def test_moe_block_config1(dev, T, path):
    """Config 1 (C30: H 2048, E 128, F 768, top-8, no shared) with its weight recipe (f32 N(0, 0.02)
    quantised to Q4_1), both kernel paths."""
    c = cases.make_case(T=T, seed=0, weights="normal")
    layer, x, res, idx, w, out = _run_block(c, dev, path=path)
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"])
    assert _rel(out, ref, c["res"]) < TOL


@pytest.mark.parametrize("path", ["tc", "gemv"])
def test_moe_block_shared_expert_and_padding(dev, path):
    """C36-shaped (shared expert + sigmoid gate) at small E, with rows past t_real carried."""
    c = cases.make_case(H=2048, E=16, F=512, FS=512, k=8, T=24, seed=1)
    layer, x, res, idx, w, out = _run_block(c, dev, t_real=21, path=path)
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], t_real=21, shared=c["shared"])
    assert _rel(out, ref, c["res"]) < TOL
    np.testing.assert_array_equal(out[21:], c["res"][21:])


@pytest.mark.parametrize("path", ["tc", "gemv"])
def test_moe_block_all_rows_padding(dev, path):
    """t_real = 0: every row is padding and is carried as res exactly (core.cpp:5155), shared expert off."""
    c = cases.make_case(H=2048, E=16, F=512, FS=512, k=8, T=16, seed=3)
    layer, x, res, idx, w, out = _run_block(c, dev, t_real=0, path=path)
    np.testing.assert_array_equal(out, c["res"])


def test_moe_layer_fused_matches_staged(dev):
    c = cases.make_case(H=2048, E=32, F=256, FS=256, k=8, T=40, seed=2)
    layer, x, res, idx, w, out = _run_block(c, dev, path="gemv")   # a fixed summation order: bit-comparable
    fused = layer.forward(x, res).cpu().numpy()
    np.testing.assert_allclose(fused, out, rtol=0, atol=0)


@pytest.mark.parametrize("path", ["tc"])
def test_moe_block_prefill_sized(dev, path):
    """T=512 over several dispatch chunks and several work items per expert (C30 prefill shape, fewer
    experts to keep the oracle fast)."""
    c = cases.make_case(H=2048, E=32, F=768, k=8, T=512, seed=3)
    layer, x, res, idx, w, out = _run_block(c, dev, path=path)
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"])
    assert _rel(out, ref, c["res"]) < TOL


def test_moe_block_skewed_prefill_tc(dev):
    """Zipf-skewed routing (BASELINE config 3's bias): hot experts span many 256-row items, others
    get a handful of rows or none; shared expert on; tcgen05 path."""
    c = cases.make_case(H=2048, E=16, F=256, FS=256, k=4, T=1000, seed=6, zipf=1.1)
    layer, x, res, idx, w, out = _run_block(c, dev, path="tc")
    counts = np.bincount(idx.reshape(-1), minlength=16)
    assert counts.max() > 256 and counts.min() < 256
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    assert _rel(out, ref, c["res"]) < TOL
    # repeated calls: a race between the kernel's roles shows as a wrong item in some calls only
    sg = layer.shared_gate_buf
    ti, tw = torch.from_numpy(idx).to(dev), torch.from_numpy(w).to(dev)
    for _ in range(8):
        again = layer.moe_block(x, res, ti, tw, shared_gate=sg).cpu().numpy()
        assert _rel(again, ref, c["res"]) < TOL


@pytest.mark.parametrize("T", [1, 3, 32])
def test_gemv_decode_c36(dev, T):
    """Decode sizes on the C36 geometry (256 experts, shared expert): the GEMV path, split-K chosen
    by the number of active experts (T=1: 4 chunks, T=32: 1)."""
    c = cases.make_case(H=2048, E=256, F=512, FS=512, k=8, T=T, seed=20 + T)
    layer, x, res, idx, w, out = _run_block(c, dev, path="gemv")
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    assert _rel(out, ref, c["res"]) < TOL


@pytest.mark.parametrize("T", [48, 128])
def test_auto_path_past_32_tokens(dev, T):
    """48 and 128 tokens on the size default: the GEMV path (up to T * k = 1024 pairs, one dispatch CTA)
    without K chunks; 128 x 8 = 1024 pairs is the largest GEMV call; shared expert on."""
    c = cases.make_case(H=2048, E=64, F=512, FS=512, k=8, T=T, seed=40 + T)
    layer, x, res, idx, w, out = _run_block(c, dev, path="auto")
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    assert _rel(out, ref, c["res"]) < TOL


def test_gemv_split_k_small_layer(dev):
    """Few active bands: the GEMV splits K (4 chunks for gate/up, 2 for down) and the last chunk in
    reduces them; shared expert on."""
    c = cases.make_case(H=256, E=8, F=128, FS=128, k=2, T=2, seed=12)
    layer, x, res, idx, w, out = _run_block(c, dev, path="gemv")
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    assert _rel(out, ref, c["res"]) < TOL


def test_gemv_hot_expert_many_rows(dev):
    """All 32 tokens on the same two experts: GEMV items of 16 rows, several per expert."""
    import flowmoe
    c = cases.make_case(H=2048, E=8, F=768, k=2, T=32, seed=9)
    layer = _layer(c, dev, "gemv")
    x = torch.from_numpy(c["x"]).to(dev).to(torch.bfloat16)
    res = torch.from_numpy(c["res"]).to(dev)
    idx = torch.tensor([[3, 5]] * 32, dtype=torch.int32, device=dev)
    w = torch.tensor([[0.75, 0.25]] * 32, dtype=torch.float32, device=dev)
    out = layer.moe_block(x, res, idx, w).cpu().numpy()
    ref = OM.moe_block_f64(c["x"], c["res"], idx.cpu().numpy(), w.cpu().numpy(), c["gate"], c["up"], c["down"])
    assert _rel(out, ref, c["res"]) < TOL


@pytest.mark.parametrize("shared", [False, True])
def test_gemv_every_token_width(dev, shared):
    """Experts with 1, 2, 3, 4, 5, 6 and 11 tokens: GEMV items of every token-column width (1, 2, 4
    and 8 columns, i.e. 8, 4, 2 and 1 Q4_1 blocks per accumulator) and an expert split over two items;
    K split into chunks (few items); with and without the shared expert's 16-token items."""
    c = cases.make_case(H=2048, E=8, F=768, FS=512 if shared else 0, k=2, T=16, seed=31)
    layer = _layer(c, dev, "gemv")
    x = torch.from_numpy(c["x"]).to(dev).to(torch.bfloat16)
    res = torch.from_numpy(c["res"]).to(dev)
    flat = np.repeat(np.arange(7), [1, 2, 3, 4, 5, 6, 11])          # 32 assignments, sorted
    idx_h = np.stack([flat[:16], flat[16:]], axis=1).astype(np.int32)  # token t: entries t and t+16 (distinct)
    rng = np.random.default_rng(5)
    w_h = rng.uniform(0.2, 1.0, (16, 2)).astype(np.float32)
    w_h /= w_h.sum(axis=1, keepdims=True)
    idx, w = torch.from_numpy(idx_h).to(dev), torch.from_numpy(w_h).to(dev)
    sg = None
    if shared:
        layer.router_block(x)
        sg = layer.shared_gate_buf
    out = layer.moe_block(x, res, idx, w, shared_gate=sg).cpu().numpy()
    ref = OM.moe_block_f64(c["x"], c["res"], idx_h, w_h, c["gate"], c["up"], c["down"], shared=c["shared"])
    assert _rel(out, ref, c["res"]) < TOL


@pytest.mark.parametrize("H,F,FS,T,seed", [(2048, 128, 128, 300, 7), (256, 256, 128, 700, 8), (512, 192, 0, 90, 9),
                                          (256, 64, 64, 1400, 10)])
def test_tc_item_splits(dev, H, F, FS, T, seed):
    """The tcgen05 path against the oracle on shapes whose experts are cut into one, two and several
    items of at most 192 rows (equal-sized, the last taking the rest), odd band counts and the shared
    expert's items included."""
    c = cases.make_case(H=H, E=8, F=F, FS=FS, k=2, T=T, seed=seed)
    layer, x, res, idx, w, out = _run_block(c, dev, path="tc")
    counts = np.bincount(idx.reshape(-1), minlength=8)
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    assert _rel(out, ref, c["res"]) < TOL, counts


def test_bad_expert_id_raises(dev):
    import flowmoe
    c = cases.make_case(H=256, E=8, F=128, k=2, T=4, seed=4)
    layer = _layer(c, dev)
    x = torch.from_numpy(c["x"]).to(dev)
    res = torch.from_numpy(c["res"]).to(dev)
    idx = torch.tensor([[0, 1], [2, 9], [3, 4], [5, 6]], dtype=torch.int32, device=dev)
    w = torch.full((4, 2), 0.5, device=dev)
    with pytest.raises(flowmoe._lib.FlowMoeError, match="FM_EINVAL_EXPERT"):
        layer.moe_block(x, res, idx, w)


@pytest.mark.parametrize("T,path", [(5, "auto"), (64, "auto"), (64, "gemv")])
def test_moe_stack_rmsnorm_matches_oracle(dev, T, path):
    """Three layers of x + MoE(RMSNorm(x)) (config 5's stack, small) against the fp64 oracle stack."""
    import flowmoe
    from flowmoe.stack import MoEStack
    rng = np.random.default_rng(T)
    cs, layers, nws = [], [], []
    for l in range(3):
        c = cases.make_case(H=256, E=16, F=128, FS=128, k=4, T=T, seed=100 + l)
        c["norm_w"] = OM.bf16_round((1.0 + rng.normal(0, 0.01, c["H"])).astype(np.float32))
        cs.append(c)
        layers.append(_layer(c, dev, path))
        nws.append(torch.from_numpy(c["norm_w"]))
    x0 = cs[0]["res"]
    got = MoEStack(layers, nws).forward(torch.from_numpy(x0).to(dev)).cpu().numpy()
    want = OM.moe_stack_f64(x0, cs)
    # relative to the total change the stack makes to x
    assert float(np.abs(got - want).max() / np.abs(want - x0).max()) < TOL


def test_bf16_scales_narrowing(dev, golden):
    """q4nx numerics: tiles with narrowed scales map back to exactly the blocks with d, m rounded to bf16,
    and a layer built with scales="bf16" matches the oracle's bf16-scale dequantisation."""
    import flowmoe
    from flowmoe.layer import narrow_scales
    blocks = golden["q4_1"]["blocks"]                       # [64, 256/32, 20]
    rows, k = blocks.shape[0], blocks.shape[1] * 32
    pad = np.concatenate([blocks, blocks])                   # 128 rows: one tile band
    t = flowmoe.q4_1_to_tiles(pad, 2 * rows, k, dev)
    back = flowmoe.tiles_to_q4_1(narrow_scales(t), 2 * rows, k).cpu().numpy().reshape(pad.shape)
    d = np.ascontiguousarray(pad[..., 0:4]).view(np.float16).astype(np.float32)
    want = pad.copy()
    want[..., 0:4] = OQ.bf16_narrow(d).astype(np.float16).view(np.uint8).reshape(want[..., 0:4].shape)
    assert np.array_equal(back, want)
    assert np.array_equal(OQ.dequant_q4_1(back[:rows]), golden["q4_1"]["dequant_bf16_scales"])
    c = cases.make_case(H=256, E=8, F=128, FS=0, k=2, T=40, seed=21)
    cfg = flowmoe.MoEConfig(hidden=c["H"], n_experts=c["E"], top_k=c["k"], ffn=c["F"], shared_ffn=0)
    layer = flowmoe.MoELayer.from_q4_1(cfg, c["gate"], c["up"], c["down"], c["Wr"], device=dev, scales="bf16")
    x = torch.from_numpy(c["x"]).to(dev).to(torch.bfloat16)
    res = torch.from_numpy(c["res"]).to(dev)
    _, idx, w = layer.router_block(x)
    out = layer.moe_block(x, res, idx, w).cpu().numpy()
    narrow = lambda bl: np.stack([flowmoe.tiles_to_q4_1(narrow_scales(flowmoe.q4_1_to_tiles(b, b.shape[0], b.shape[1] * 32, dev)),
                                                        b.shape[0], b.shape[1] * 32).cpu().numpy().reshape(b.shape) for b in bl])
    ref = OM.moe_block_f64(c["x"], c["res"], idx.cpu().numpy(), w.cpu().numpy(), narrow(c["gate"]), narrow(c["up"]),
                           narrow(c["down"]))
    assert _rel(out, ref, c["res"]) < TOL


def test_host_pipeline_matches_direct_calls(dev):
    """flowmoe.HostPipeline (host->device copy, layer, device->host copy on their own streams, two device
    slots): five batches from pinned host memory give the direct calls' results bit for bit, each batch in
    its own host output buffer and in one shared one."""
    import flowmoe
    c = cases.make_case(H=2048, E=16, F=512, FS=512, k=8, T=40, seed=14)
    layer = _layer(c, dev, "gemv")
    T, H = 40, 2048
    rng = np.random.default_rng(1)
    xs = [torch.from_numpy(OM.bf16_round(rng.standard_normal((T, H), dtype=np.float32))).to(torch.bfloat16).pin_memory()
          for _ in range(5)]
    rs = [torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).pin_memory() for _ in range(5)]
    outs = [torch.empty(T, H).pin_memory() for _ in range(5)]
    pipe = flowmoe.HostPipeline(layer, T)
    for x, r, o in zip(xs, rs, outs):
        pipe.submit(x, r, o)
    pipe.synchronize()
    for x, r, o in zip(xs, rs, outs):
        want = layer.forward(x.to(dev), r.to(dev)).cpu()
        assert torch.equal(o, want)
    shared = torch.empty(T, H).pin_memory()
    for x, r in zip(xs, rs):
        pipe.submit(x, r, shared)
    pipe.synchronize()
    assert torch.equal(shared, outs[-1])
    with pytest.raises(ValueError, match="pinned"):
        pipe.submit(xs[0], rs[0], torch.empty(T, H))


def test_expert_pool_import_bit_exact(dev, golden):
    """The reference engine's expert pool regions (expert_stripes / expert_down, pools.cpp:927-962; bytes
    pinned to the reference's own packers by test_expert_pool_matches_reference_bytes) -> per-expert GGUF
    blocks on the device, bit for bit the oracle's inverse (bf16 scales), and a layer built straight from
    the pool equals one built from those blocks."""
    import flowmoe
    g = golden["expert_pool"]
    E, F, H = int(g["E"]), int(g["F"]), int(g["H"])
    rng = np.random.default_rng(int(g["seed"]))
    up = [OQ.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    gate = [OQ.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    down = [OQ.random_q4_1_blocks(H, F, rng) for _ in range(E)]
    gu, dn = OQ.expert_pool(up, gate, down)
    gb, ub, db = flowmoe.experts_from_pool(gu, dn, E, F, H, device=dev)
    per = gu.size // E
    for e in range(E):
        st = gu[e * per:(e + 1) * per].reshape(F // 128, 2, -1)
        assert np.array_equal(ub[e].cpu().numpy(), OQ.pool_to_blocks(st[:, 0].reshape(-1), F, H, 4))
        assert np.array_equal(gb[e].cpu().numpy(), OQ.pool_to_blocks(st[:, 1].reshape(-1), F, H, 4))
        assert np.array_equal(db[e].cpu().numpy(), OQ.pool_to_blocks(dn[e * dn.size // E:(e + 1) * dn.size // E], H, F, 4))
    cfg = flowmoe.MoEConfig(hidden=H, n_experts=E, top_k=1, ffn=F)
    Wr = OM.bf16_round(rng.normal(0, 0.02, (H, E)).astype(np.float32))
    a = flowmoe.MoELayer.from_expert_pool(cfg, gu, dn, Wr, device=dev)
    b = flowmoe.MoELayer.from_q4_1(cfg, gb, ub, db, Wr, device=dev)
    assert torch.equal(a.gate_up, b.gate_up) and torch.equal(a.down, b.down)


def _fixed_run(layer, x, res, t_real=None):
    probs, idx, w = layer.router_block(x)
    sg = layer.shared_gate_buf if layer.cfg.shared_ffn else None
    return layer.moe_block(x, res, idx, w, t_real=t_real, shared_gate=sg).cpu().numpy(), idx.cpu().numpy(), \
        w.cpu().numpy()


@pytest.mark.parametrize("path", ["tc", "gemv"])
def test_fixed_order_matches_oracle(dev, path):
    """FM_FIXED_ORDER on both kernel paths: shared expert, padding rows, against the fp64 oracle."""
    c = cases.make_case(H=2048, E=16, F=512, FS=512, k=8, T=40, seed=11)
    layer = _layer(c, dev, path)
    layer.fixed_order = True
    assert layer.path == path and layer.fixed_order
    x = torch.from_numpy(c["x"]).to(dev).to(torch.bfloat16)
    res = torch.from_numpy(c["res"]).to(dev)
    out, idx, w = _fixed_run(layer, x, res, t_real=37)
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], t_real=37, shared=c["shared"])
    assert _rel(out, ref, c["res"]) < TOL
    np.testing.assert_array_equal(out[37:], c["res"][37:])
    again, _, _ = _fixed_run(layer, x, res, t_real=37)
    np.testing.assert_array_equal(again, out)


@pytest.mark.parametrize("path,T,blocks", [("tc", 600, [128, 200, 16, 256]), ("gemv", 40, [1] * 40),
                                           ("gemv", 96, [32, 7, 57])])
def test_fixed_order_layer_major_equals_block_major(dev, path, T, blocks):
    """A prompt through the layer in one call (layer-major prefill) gives the same bits as the same
    prompt in blocks, and as one token at a time on the GEMV path, once the order is fixed."""
    c = cases.make_case(H=1024, E=32, F=256, FS=256, k=8, T=T, seed=12)
    layer = _layer(c, dev, path)
    layer.fixed_order = True
    x = torch.from_numpy(c["x"]).to(dev).to(torch.bfloat16)
    res = torch.from_numpy(c["res"]).to(dev)
    whole, idx, w = _fixed_run(layer, x, res)
    parts, b0 = [], 0
    for n in blocks:
        parts.append(_fixed_run(layer, x[b0:b0 + n].contiguous(), res[b0:b0 + n].contiguous())[0])
        b0 += n
    assert b0 == T
    np.testing.assert_array_equal(np.concatenate(parts), whole)
    ref = OM.moe_block_f64(c["x"], c["res"], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])
    assert _rel(whole, ref, c["res"]) < TOL


def test_fixed_order_stack_prompt_layer_major(dev):
    """Three layers of the RMSNorm stack over a 300-token prompt in one pass per layer equal the same stack
    run block by block (blocks of 100), bit for bit."""
    from flowmoe.stack import MoEStack
    rng = np.random.default_rng(5)
    layers, nws = [], []
    for l in range(3):
        c = cases.make_case(H=512, E=16, F=256, FS=128, k=4, T=4, seed=200 + l)
        layers.append(_layer(c, dev, "tc"))
        layers[-1].fixed_order = True
        nws.append(torch.from_numpy(OM.bf16_round((1.0 + rng.normal(0, 0.01, 512)).astype(np.float32))))
    st = MoEStack(layers, nws)
    x = torch.from_numpy(rng.normal(0, 1, (300, 512)).astype(np.float32)).to(dev)
    whole = st.forward(x).cpu().numpy()
    blocks = np.concatenate([st.forward(x[i:i + 100].contiguous()).cpu().numpy() for i in range(0, 300, 100)])
    np.testing.assert_array_equal(blocks, whole)


def test_q4_gemm_reference_fixture(dev, golden):
    """The dense Q4_1 projection GEMM on the reference's own gemm_q4_prefill test vectors: its pool bytes
    (pack_q4_1_pool, bf16 scales) imported as they are, its bf16 token rows, against its fp64 pool_reference;
    the reference design's gate is rel_fro <= 5e-3 (designs/gemm_q4_prefill/compare.py)."""
    import flowmoe
    g = golden["gemm_q4"]
    n, k = int(g["n"]), int(g["k"])
    lin = flowmoe.Q4Linear.from_pool(g["pool"], n, k, rs=int(g["rs"]), device=dev)
    x = torch.from_numpy(g["x_bf16"].astype(np.int16)).view(torch.bfloat16).to(dev)
    y = lin.forward(x).cpu().numpy()
    lin.check()
    ref = g["y"]
    assert float(np.linalg.norm(y - ref) / np.linalg.norm(ref)) <= 5e-3
    assert np.abs(y - ref).max() / np.abs(ref).max() < TOL


@pytest.mark.parametrize("N,K,T,f32", [(2560, 2560, 256, False), (256, 512, 300, True), (1024, 2048, 8192, False),
                                       (128, 64, 17, True)])
def test_q4_gemm_matches_oracle(dev, N, K, T, f32):
    """fm_q4_gemm against the fp64 oracle: the reference's qkv projection shape (2560 x 2560, T 256), ragged
    token counts (300, 17: a partial last item), f32 input (rounded to bf16 on the device), and a
    prefill-sized call (T 8192: 32 row chunks per band) checked on a sample of rows."""
    import flowmoe
    rng = np.random.default_rng(N + K + T)
    blocks = OQ.random_q4_1_blocks(N, K, rng)
    lin = flowmoe.Q4Linear.from_q4_1(blocks, N, K, device=dev)
    x = rng.standard_normal((T, K)).astype(np.float32)
    xt = torch.from_numpy(x).to(dev)
    y = lin.forward(xt if f32 else xt.to(torch.bfloat16)).cpu().numpy()
    lin.check()
    rows = np.arange(T) if T <= 512 else np.sort(rng.choice(T, 64, replace=False))
    ref = OM.q4_gemm_f64(x[rows], blocks)
    got = y[rows]
    assert float(np.linalg.norm(got - ref) / np.linalg.norm(ref)) <= 5e-3
    assert np.abs(got - ref).max() / np.abs(ref).max() < TOL
