"""Writes the golden vectors under tests/golden/ by running the REFERENCE's own Python code.

    python tests/golden/make_golden.py --ref /path/to/OpenFlowLM-Next    (or OFLM_REFERENCE=/path ...)

Needs the reference tree (read in place; nothing is copied) and ``gguf`` 0.19.0. The GPU box has
neither, so the fixtures are committed and the tests read only the ``.npz`` files. Each fixture
stores the reference's outputs and, for large inputs that a seeded generator reproduces, a
SHA-256 of the input bytes so a test can prove its regenerated inputs are the very bytes the
reference saw.

Fixtures:
  q4_1.npz    reference ``q4_1_pack.random_q4_1_blocks`` (seed 0) bytes and its ``dequant_q4_1``;
              ``gguf.quantize(.., Q4_1)`` bytes of a seeded f32 matrix and ``gguf.dequantize``;
              the reference pool packers' bytes (``pack_q4_1_pool`` rs=2, ``gguf_pool.pack_q4_pool``).
  router.npz  ``replica_block.random_case(0)`` router inputs/outputs (E=8, topk=3); the tie KAT of
              ``test_prefill_batch.py:363-369``; a config-1 router (T=16, H=2048, E=128, k=8) on
              seeded bf16 inputs.
  moe.npz     ``replica.moe_decode`` (fp64, HF-faithful) over 4 tokens of a small Qwen3.6-shaped
              block (H=2048 as replica.py fixes it, E=16, F=128, shared F=128, top-8) whose Q4_1
              experts come from the reference's block generator (seed 0).
  q4nx.npz    the SHA-256 of what the reference's .q4nx reader (open_kernels/model/q4nx.py) dequantises
              from a one-layer container the oracle writes (2 experts, shared expert with a signed-
              quantiser matrix, router).
  gemm_q4.npz the reference's gemm_q4_prefill test recipe (designs/gemm_q4_prefill/make_test.py:73-97) at a
              small shape (n 256, k 512, T 32): a random_q4_1_blocks weight (seed 0) packed by
              pack_q4_1_pool (rs 2, bf16 scales), T distinct bf16 token rows, and pool_reference (fp64 from
              the pool bytes) per token. ``--only gemm`` writes this fixture alone.
  expert_pool.npz  the SHA-256 of the MoE expert pool regions (gate_up stripes and down slices) the
              engine's pack ops write for 2 seeded experts (F=512, H=256), built from the reference's
              own pack_q4_1_pool, stripe_transpose and down_perm, and of their source blocks.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bf16_vals(a: np.ndarray) -> np.ndarray:
    from ml_dtypes import bfloat16
    return np.asarray(a, np.float32).astype(bfloat16).astype(np.float32)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("OFLM_REFERENCE"),
                    help="the reference tree (required; default: $OFLM_REFERENCE)")
    ap.add_argument("--only", default=None, help="write one fixture only (gemm)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref (or OFLM_REFERENCE) must name the reference tree")
    ref = Path(a.ref)
    sys.path[:0] = [str(ref / "open_kernels"), str(ref / "open_kernels" / "model"), str(ref)]
    import gguf
    import q4_1_pack as QP                       # open_kernels/q4_1_pack.py
    from open_kernels.gguf_pool import gguf_pool as GP   # open_kernels/gguf_pool/gguf_pool.py
    import replica_block as RB                   # open_kernels/model/replica_block.py
    import replica as RP                         # open_kernels/model/replica.py
    from ml_dtypes import bfloat16

    # ---- gemm_q4: the reference's dense prefill GEMM recipe
    rng = np.random.default_rng(0)
    gn, gk, gT = 256, 512, 32
    gpool = QP.pack_q4_1_pool(QP.random_q4_1_blocks(gn, gk, rng), 2)
    gx = [rng.standard_normal(gk).astype(np.float32).astype(bfloat16) for _ in range(gT)]
    gy = np.stack([QP.pool_reference(gpool, gx[t].astype(np.float32), gn, gk, rs=2) for t in range(gT)])
    np.savez_compressed(HERE / "gemm_q4.npz", n=gn, k=gk, T=gT, rs=2, pool=gpool,
                        x_bf16=np.stack(gx).view(np.uint16), y=gy.astype(np.float32))
    if a.only == "gemm":
        print(f"wrote {HERE / 'gemm_q4.npz'} ({(HERE / 'gemm_q4.npz').stat().st_size} B)")
        return 0

    # ---- q4_1
    rng = np.random.default_rng(0)
    blocks = QP.random_q4_1_blocks(64, 256, rng)
    deq = QP.dequant_q4_1(blocks)
    deq_bf16s = QP.dequant_q4_1(blocks, bfloat16)
    pool_bf16 = QP.pack_q4_1_pool(blocks, 2)
    pool_f32 = GP.pack_q4_pool(blocks, 2, "Q4_1")
    wq = np.random.default_rng(1).normal(0, 0.02, (32, 256)).astype(np.float32)
    wq[0, :32] = 0.0                               # a constant block (d == 0)
    gq = gguf.quantize(wq, gguf.GGMLQuantizationType.Q4_1)
    gdq = gguf.dequantize(gq, gguf.GGMLQuantizationType.Q4_1)
    np.savez_compressed(HERE / "q4_1.npz", blocks=blocks, dequant=deq, dequant_bf16_scales=deq_bf16s,
                        pool_bf16_rs2=pool_bf16, pool_f32_rs2=pool_f32, gguf_in=wq,
                        gguf_q4_1=np.asarray(gq, np.uint8), gguf_dequant=np.asarray(gdq, np.float32))

    # ---- router
    case = RB.random_case(0)
    p, idx, w = RB.router_block(case["xm"], case["Wr"], case["topk"])
    tie_x = np.array([[1.0, 0.0]])
    tie_W = np.array([[0.5, 0.5, 0.2, 0.5], [0.0, 0.0, 0.0, 0.0]])
    tp, tidx, tw = RB.router_block(tie_x, tie_W, 2)
    r2 = np.random.default_rng(0)
    x1 = bf16_vals(r2.standard_normal((16, 2048), dtype=np.float32))
    W1 = bf16_vals(r2.normal(0, 0.02, (2048, 128)).astype(np.float32))
    p1, idx1, w1 = RB.router_block(x1.astype(np.float64), W1.astype(np.float64), 8)
    np.savez_compressed(HERE / "router.npz",
                        rc_xm=case["xm"], rc_Wr=case["Wr"], rc_topk=case["topk"], rc_probs=p, rc_idx=idx, rc_w=w,
                        tie_x=tie_x, tie_W=tie_W, tie_probs=tp, tie_idx=tidx, tie_w=tw,
                        c1_x_sha=sha(x1), c1_W_sha=sha(W1), c1_probs=p1, c1_idx=idx1, c1_w=w1)

    # ---- moe_decode over 4 tokens
    H, E, F, FS, T = 2048, 16, 128, 128, 4
    rng = np.random.default_rng(0)
    gate = [QP.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    up = [QP.random_q4_1_blocks(F, H, rng) for _ in range(E)]
    down = [QP.random_q4_1_blocks(H, F, rng, scale=0.05) for _ in range(E)]
    sg, su, sd = (QP.random_q4_1_blocks(FS, H, rng), QP.random_q4_1_blocks(FS, H, rng),
                  QP.random_q4_1_blocks(H, FS, rng, scale=0.05))
    postln = bf16_vals(1 + rng.normal(0, 0.01, H).astype(np.float32))
    Wr = bf16_vals(rng.normal(0, 0.02, (H, E)).astype(np.float32))
    sgw = bf16_vals(rng.normal(0, 0.02, H).astype(np.float32))
    xres = rng.standard_normal((T, H)).astype(np.float32)

    class Model:
        """The accessors replica.moe_decode reads, over the seeded blocks above."""
        def bf16(self, name):
            return {"model.layer.0.post_attention_layernorm.weight": postln,
                    "model.layer.0.moe_router.weight": Wr,
                    "model.layer.0.shared_expert_gate.weight": sgw}[name]

        def expert_w(self, layer, kind, e):
            return QP.dequant_q4_1({"gate": gate, "up": up, "down": down}[kind][e])

        def shared_w(self, layer, kind):
            return QP.dequant_q4_1({"gate": sg, "up": su, "down": sd}[kind])

    m = Model()
    outs, xms, tops, probs = [], [], [], []
    for t in range(T):
        xm, pt, top = RP.route(m, 0, xres[t].astype(np.float64))
        outs.append(RP.moe_decode(m, 0, xres[t].astype(np.float64)))
        xms.append(xm)
        tops.append(top)
        probs.append(pt)
    allb = np.concatenate([b.reshape(-1) for b in gate + up + down + [sg, su, sd]])
    np.savez_compressed(HERE / "moe.npz", H=H, E=E, F=F, FS=FS, T=T, blocks_sha=sha(allb),
                        postln=postln, Wr=Wr, sgw=sgw, xres=xres, xm=np.array(xms, np.float32),
                        top=np.array(tops, np.int32), probs=np.array(probs), out=np.array(outs))
    # ---- the MoE expert pool regions the engine packs (pools.cpp:927-962 expert_stripes / expert_down over
    # recipes/pack.py's stripe_transpose and down_perm), built from the reference's own functions: the
    # container's plain chunk raster of each matrix (chunk (row block, k-tile) at rb * ncol + kt, which is
    # pack_q4_1_pool with a row split of 1), then the ops' chunk orders and the [up_k | gate_k] interleave
    from open_kernels.recipes import pack as RPK
    Ep, Fp, Hp = 2, 512, 256
    rng = np.random.default_rng(7)
    pu = [QP.random_q4_1_blocks(Fp, Hp, rng) for _ in range(Ep)]
    pg = [QP.random_q4_1_blocks(Fp, Hp, rng) for _ in range(Ep)]
    pd = [QP.random_q4_1_blocks(Hp, Fp, rng) for _ in range(Ep)]
    CHB = QP.CH
    ns, ncol = Fp // 128, Hp // 256
    tp = RPK.stripe_transpose(Hp)
    gu_pool, dn_pool = [], []
    for e in range(Ep):
        fu = QP.pack_q4_1_pool(pu[e], 1).reshape(-1, CHB)
        fg = QP.pack_q4_1_pool(pg[e], 1).reshape(-1, CHB)
        for k in range(ns):
            for f in (fu, fg):   # [up_k | gate_k]
                stripe = f[k * 4 * ncol:(k + 1) * 4 * ncol]
                gu_pool.append(stripe[tp].reshape(-1))
        fd = QP.pack_q4_1_pool(pd[e], 1).reshape(-1, CHB)
        dn_pool.append(fd[RPK.down_perm(fd.shape[0])].reshape(-1))
    gu_pool, dn_pool = np.concatenate(gu_pool), np.concatenate(dn_pool)
    np.savez_compressed(HERE / "expert_pool.npz", E=Ep, F=Fp, H=Hp, seed=7,
                        blocks_sha=sha(np.concatenate([b.reshape(-1) for b in pu + pg + pd])),
                        gate_up_sha=sha(gu_pool), down_sha=sha(dn_pool),
                        gate_up_bytes=gu_pool.size, down_bytes=dn_pool.size)
    # ---- a one-layer .q4nx container (2 routed experts of F 512 at H 2048, shared expert, router, gate,
    # post-attention norm) written by the oracle's writer and read back by the reference's own reader
    # (open_kernels/model/q4nx.py, Q4NX): the SHA-256 of every matrix that reader dequantises. The shared
    # expert's up matrix is stored by the signed quantiser (mins written as zero), which the reader
    # transcodes (recipes/pack.py is_signed_q4 / q4_0_to_q4_1).
    import tempfile
    import q4nx as RQ                             # open_kernels/model/q4nx.py
    sys.path.insert(0, str(HERE.parents[1]))
    from oracle import q4nx as OQX
    rng = np.random.default_rng(11)
    Ex, Fx, Hx = 2, 512, 2048
    ex = {k: [QP.random_q4_1_blocks(Fx if k != "down" else Hx, Hx if k != "down" else Fx, rng) for _ in range(Ex)]
          for k in ("gate", "up", "down")}
    sh = {k: QP.random_q4_1_blocks(Fx if k != "down" else Hx, Hx if k != "down" else Fx, rng) for k in ("gate", "up", "down")}
    d16 = np.ascontiguousarray(sh["up"][..., 0:2]).view(np.float16)
    sh["up"][..., 2:4] = (d16.astype(bfloat16).astype(np.float32) * -8).astype(np.float16).view(np.uint8)
    wr = bf16_vals(rng.normal(0, 0.02, (Hx, 8)).astype(np.float32)).astype(bfloat16).view(np.uint16)
    sgw = bf16_vals(rng.normal(0, 0.02, Hx).astype(np.float32)).astype(bfloat16).view(np.uint16)
    pln = bf16_vals(1 + rng.normal(0, 0.01, Hx).astype(np.float32)).astype(bfloat16).view(np.uint16)
    L = "model.layer.0."
    tens = {L + "post_attention_layernorm.weight": ("BF16", pln), L + "moe_router.weight": ("BF16", wr),
            L + "shared_expert_gate.weight": ("BF16", sgw)}
    for k in ("gate", "up", "down"):
        tens[L + f"mlp.{k}_exps_proj.weight"] = ("I8", np.concatenate([OQX.q4nx_matrix(b) for b in ex[k]]))
        tens[L + f"mlp.share_{k}_exps_proj.weight"] = ("I8", OQX.signed_q4_matrix(sh[k]) if k == "up"
                                                       else OQX.q4nx_matrix(sh[k]))
    shas = {}
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "l0.q4nx"
        OQX.write_q4nx(path, tens)
        container_sha = hashlib.sha256(path.read_bytes()).hexdigest()
        m = RQ.Q4NX(path)
        for k in ("gate", "up", "down"):
            for e in range(Ex):
                shas[f"expert_{k}_{e}"] = sha(m.expert_w(0, k, e))
            shas[f"shared_{k}"] = sha(m.shared_w(0, k))
        shas["router"] = sha(m.bf16(L + "moe_router.weight"))
        m.mm.close()
        m.f.close()
    np.savez_compressed(HERE / "q4nx.npz", seed=11, E=Ex, F=Fx, H=Hx, container_sha=container_sha,
                        **{k: v for k, v in shas.items()})
    for f in ("gemm_q4.npz", "q4_1.npz", "router.npz", "moe.npz", "expert_pool.npz", "q4nx.npz"):
        print(f"wrote {HERE / f} ({(HERE / f).stat().st_size} B)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
