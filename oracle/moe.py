"""CPU oracle, Qwen3.6-MoE expert block -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module, and only as the checker or the timed CPU baseline. The product path (``flowmoe``) never
imports it and has no CPU fallback.

Parity pins (see ``tests/golden/make_golden.py``): ``router_block`` is checked against the
reference's ``open_kernels/model/replica_block.py:160-169`` on its own ``random_case`` fixture and
its tie known-answer test (``specs/open-engine/tests/test_prefill_batch.py:363-369``);
``moe_block_f64`` against ``open_kernels/model/replica.py:131-143`` (restated over T tokens) on
seeded inputs generated with the reference's own block generator.

Numerics contract of the block (reference citations inline):
  * router: logits = xm . Wr (fp32), softmax with max subtraction, top-k by probability with the
    lowest index on a tie, renormalised (``src/open_qwen36/block_host.cpp:766-803``);
  * experts: x -> bf16 at the gather (``src/open_qwen36/core.cpp:5204``), u = W_up x, g = W_gate x,
    h = bf16(silu(g) * u) (``open_kernels/designs/moe_batch/make_test.py:87-97``), y = W_down h;
  * combine: out = res + sum_e w_e y_e in ascending expert order (``core.cpp:5150-5165``,
    ``:5236-5255``), shared expert added as sigmoid(bf16(xm) . sgw) * down_s(silu(g_s) u_s)
    (``core.cpp:4342-4380``).
"""
from __future__ import annotations

import numpy as np

from .q4_1 import dequant_q4_1


def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 (round to nearest even) -> f32; ``open_kernels/model/replica_block.py:20-24``."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return r.view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> f32 (exact)."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def silu(x):
    return x / (1 + np.exp(-x))


def sigmoid(x):
    return 1 / (1 + np.exp(-x))


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """Post-attention RMSNorm -> xm (f32): ``Core::rmsnorm_host`` (``src/open_qwen36/core.cpp:3014-3044``,
    groups = 1): the sum of squares, the rms and the product with the weight in fp64,
    out = f32((x / sqrt(mean(x^2) + eps)) * w); the weight arrives as bf16 values."""
    xd = np.asarray(x, np.float64)
    rms = np.sqrt((xd * xd).sum(-1, keepdims=True) / xd.shape[-1] + eps)
    return ((xd / rms) * np.asarray(w, np.float64)).astype(np.float32)


def moe_stack_f64(x, layers, eps: float = 1e-6, engine_rounding: bool = True, y_bf16: bool = False):
    """x_{l+1} = x_l + MoE_l(RMSNorm_l(x_l)) over a list of layers, each a dict with ``norm_w``, ``Wr``,
    ``gate``, ``up``, ``down``, ``shared``, ``k`` (the staged_tail -> ffn_block sequence of
    ``core.cpp:4934-4957`` repeated per layer; ``replica.py:121-143``). ``y_bf16``: see ``moe_block_f64``."""
    x = np.asarray(x, np.float32)
    for L in layers:
        xm = rmsnorm(x, L["norm_w"], eps)
        _, idx, w = router_block(bf16_round(xm), L["Wr"], L["k"])
        x = moe_block_f64(xm, x, idx, w, L["gate"], L["up"], L["down"], shared=L["shared"],
                          engine_rounding=engine_rounding, y_bf16=y_bf16).astype(np.float32)
    return x


def router_block(xm: np.ndarray, Wr: np.ndarray, topk: int, bias: np.ndarray | None = None):
    """(probs [T, E], idx int32 [T, topk], w [T, topk]) in fp64.

    ``open_kernels/model/replica_block.py:160-169``: softmax over the experts, top-k by probability
    with a stable sort (so the lowest index wins a tie, as ``router_fin`` and
    ``block_host.cpp:786-795`` pick), weights renormalised over the chosen k.
    """
    if topk > Wr.shape[1]:
        raise ValueError("router_block: topk past the expert count")   # block_host.cpp:768
    lg = np.asarray(xm, np.float64) @ np.asarray(Wr, np.float64)
    if bias is not None:   # the synthetic Zipf skew of the prefill configs (not in the reference)
        lg = lg + np.asarray(bias, np.float64)
    p = np.exp(lg - lg.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    idx = np.argsort(-p, axis=-1, kind="stable")[:, :topk]
    w = np.take_along_axis(p, idx, -1)
    w /= w.sum(-1, keepdims=True)
    return p, idx.astype(np.int32), w


def router_margins(xm: np.ndarray, Wr: np.ndarray, topk: int, bias: np.ndarray | None = None) -> np.ndarray:
    """Per token, p[k-th] - p[(k+1)-th] (fp64): where this exceeds 1e-3 the ids must be bit-exact."""
    lg = np.asarray(xm, np.float64) @ np.asarray(Wr, np.float64)
    if bias is not None:
        lg = lg + np.asarray(bias, np.float64)
    p = np.exp(lg - lg.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ps = -np.sort(-p, axis=-1)
    if topk >= p.shape[1]:
        return np.full(p.shape[0], np.inf)
    return ps[:, topk - 1] - ps[:, topk]


def dispatch(idx: np.ndarray, n_experts: int, t_real: int | None = None):
    """Per-expert counts, exclusive offsets and the stable permutation of (token, slot) pairs.

    ``src/open_qwen36/core.cpp:5155-5165``: each expert's owed list holds its (token, slot) pairs
    in token-then-slot order; experts are visited in ascending order. Returns
    ``counts int32[E]``, ``offsets int32[E+1]``, ``pos int32[T, k]`` (row of each pair in the
    expert-sorted order) and ``pair int32[P]`` (the inverse: sorted row -> t*k + s).
    Raises on an expert id out of range (``core.cpp:5159-5160``).
    """
    T, k = idx.shape
    t_real = T if t_real is None else t_real
    flat = idx[:t_real].reshape(-1).astype(np.int64)
    if flat.size and (flat.min() < 0 or flat.max() >= n_experts):
        raise ValueError(f"router produced expert index out of range [0, {n_experts})")
    counts = np.bincount(flat, minlength=n_experts).astype(np.int32)
    offsets = np.zeros(n_experts + 1, np.int32)
    offsets[1:] = np.cumsum(counts)
    order = np.argsort(flat, kind="stable")            # stable: token-then-slot order within an expert
    pos = np.full(T * k, -1, np.int32)
    pos[order] = np.arange(order.size, dtype=np.int32)
    return counts, offsets, pos.reshape(T, k), order.astype(np.int32)


def expert_ffn_f64(x: np.ndarray, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray, round_h: bool = True) -> np.ndarray:
    """One expert over rows x: fp64 products, h rounded to bf16 when ``round_h`` (the engine's
    rounding point before the down product); ``round_h=False`` is ``replica.py:139-140`` exactly."""
    xt = np.asarray(x, np.float64)
    g = xt @ wg.astype(np.float64).T
    u = xt @ wu.astype(np.float64).T
    h = silu(g) * u
    if round_h:
        h = bf16_round(h.astype(np.float32)).astype(np.float64)
    return h @ wd.astype(np.float64).T


def shared_gate(xm: np.ndarray, sgw: np.ndarray, round_x: bool = True) -> np.ndarray:
    """sigmoid(bf16(xm) . sgw) per token; the dot in double as ``core.cpp:4370-4373``
    (``round_x=False``: ``replica.py:142``, the unrounded xm)."""
    x = bf16_round(np.asarray(xm, np.float32)) if round_x else np.asarray(xm, np.float32)
    d = x.astype(np.float64) @ np.asarray(sgw, np.float64)
    if round_x:
        d = d.astype(np.float32).astype(np.float64)
    return 1.0 / (1.0 + np.exp(-d))


def q4_gemm_f64(x: np.ndarray, blocks: np.ndarray) -> np.ndarray:
    """y [T, n] = x [T, k] . dequant(W)^T in fp64 over GGUF Q4_1 blocks W uint8[n, k/32, 20], x rounded to bf16
    first (the activation precision of the device path). The reference's dense prefill GEMM checks
    against the same product computed per token from its pool bytes, ``q4_1_pack.pool_reference``
    (``open_kernels/q4_1_pack.py:183-191``, used by ``designs/gemm_q4_prefill/make_test.py:89-94``)."""
    xb = bf16_round(np.asarray(x, np.float32)).astype(np.float64)
    return (xb @ dequant_q4_1(blocks).astype(np.float64).T).astype(np.float32)


def moe_block_f64(xm, res, idx, w, gate_blocks, up_blocks, down_blocks, t_real=None, shared=None,
                  engine_rounding: bool = True, y_bf16: bool = False):
    """out [T, H] = res + (shared) + sum over each token's experts, ascending expert order, fp64.

    ``gate_blocks[e]`` etc. are GGUF Q4_1 blocks (uint8[rows, K/32, 20]). ``shared`` is None or
    ``(gate_blocks, up_blocks, down_blocks, sgw)``. Rows past ``t_real`` are carried as res
    (``core.cpp:5155``, ``:3697``). This is ``open_kernels/model/replica.py:131-143`` over T tokens
    with the engine's dispatch order and rounding points; ``engine_rounding=False`` drops the two
    bf16 rounding points (x at the gather, h before down) and is then replica.py's fp64 math.
    ``y_bf16=True`` adds the rounding point of this build's expert-parallel paths, whose routed y rows
    travel between ranks as bf16 (the reference keeps them in f32, ``moe_acc.cc``): each (token, expert)
    y row is rounded to bf16 before the weighted combine; the shared expert's row is not.
    """
    xm = np.asarray(xm, np.float32)
    T, H = xm.shape
    t_real = T if t_real is None else t_real
    E = len(gate_blocks)
    out = np.asarray(res, np.float64).copy()
    xb = bf16_round(xm) if engine_rounding else xm
    if shared is not None:
        sg_b, su_b, sd_b, sgw = shared
        sh = expert_ffn_f64(xb[:t_real], dequant_q4_1(sg_b), dequant_q4_1(su_b), dequant_q4_1(sd_b), engine_rounding)
        out[:t_real] += shared_gate(xm[:t_real], sgw, engine_rounding)[:, None] * sh
    counts, offsets, pos, pair = dispatch(idx, E, t_real)
    k = idx.shape[1]
    y_pairs = np.zeros((pair.size, H), np.float64)
    for e in range(E):
        lo, hi = offsets[e], offsets[e + 1]
        if lo == hi:
            continue
        toks = pair[lo:hi] // k
        y_pairs[lo:hi] = expert_ffn_f64(xb[toks], dequant_q4_1(gate_blocks[e]), dequant_q4_1(up_blocks[e]),
                                        dequant_q4_1(down_blocks[e]), engine_rounding)
    if y_bf16:
        y_pairs = bf16_round(y_pairs.astype(np.float32)).astype(np.float64)
    wf = np.asarray(w, np.float64)
    for t in range(t_real):
        order = np.argsort(idx[t], kind="stable")          # ascending expert, as the visit order
        for s in order:
            out[t] += wf[t, s] * y_pairs[pos[t, s]]
    return out


def moe_rows_f64(rows, xm, res, idx, w, gate_blocks, up_blocks, down_blocks, shared=None, e_begin: int = 0):
    """``moe_block_f64`` for the token rows ``rows`` only (out f64 [len(rows), H]).

    The block is per token once the routing is fixed (``core.cpp:5236-5255`` adds each token's own expert
    terms into its own row; the shared expert and its gate are per token, ``core.cpp:4342-4380``), so a
    sample of rows of a full-size call is checked exactly as the whole call would be, at the cost of the
    experts those rows touch. ``gate_blocks[e]`` etc. may be any indexable of per-expert GGUF Q4_1 blocks
    (numpy arrays or device tensors, fetched and dequantised once per touched expert); expert e of the
    routing is entry ``e - e_begin``.
    """
    rows = np.asarray(rows, np.int64)
    xm = np.asarray(xm, np.float32)[rows]
    out = np.asarray(res, np.float64)[rows].copy()
    idx = np.asarray(idx)[rows]
    wf = np.asarray(w, np.float64)[rows]
    xb = bf16_round(xm)

    def host(b):
        if hasattr(b, "cpu"):   # a torch tensor: bf16 values widen to f32 exactly, bytes stay bytes
            return (b.float() if str(b.dtype) == "torch.bfloat16" else b).cpu().numpy()
        return np.asarray(b)

    if shared is not None:
        sg_b, su_b, sd_b, sgw = shared
        sh = expert_ffn_f64(xb, dequant_q4_1(host(sg_b)), dequant_q4_1(host(su_b)), dequant_q4_1(host(sd_b)))
        out += shared_gate(xm, host(sgw).astype(np.float32))[:, None] * sh
    # y of every sampled (row, slot) pair, one expert at a time (each touched expert dequantised once)
    y = np.zeros(idx.shape + (xm.shape[1],), np.float64)
    for e in sorted(set(int(v) for v in idx.reshape(-1))):
        ri, si = np.nonzero(idx == e)
        g, u, d = (dequant_q4_1(host(b[e - e_begin])) for b in (gate_blocks, up_blocks, down_blocks))
        y[ri, si] = expert_ffn_f64(xb[ri], g, u, d)
    for i in range(len(rows)):
        for s in np.argsort(idx[i], kind="stable"):       # ascending expert, the visit order
            out[i] += wf[i, s] * y[i, s]
    return out


class MoeLayerF32:
    """The timed CPU baseline: NumPy fp32 + BLAS restatement of the block.

    router_block -> per touched expert, dequantise Q4_1 once -> BLAS matmuls -> weighted scatter,
    the order of ``core.cpp:5150-5255`` (dispatch ascending expert) and ``core.cpp:4342-4380``
    (shared expert). Dequantised weights are cached per expert on first touch only within one call.
    """

    def __init__(self, Wr, gate_blocks, up_blocks, down_blocks, shared=None, topk=8):
        self.Wr = np.asarray(Wr, np.float32)
        self.gate, self.up, self.down = gate_blocks, up_blocks, down_blocks
        self.shared = shared
        self.topk = topk

    def route(self, xm):
        lg = np.asarray(xm, np.float32) @ self.Wr
        p = np.exp(lg - lg.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True, dtype=np.float64).astype(np.float32)
        idx = np.argsort(-p, axis=-1, kind="stable")[:, :self.topk].astype(np.int32)
        w = np.take_along_axis(p, idx, -1)
        w = (w / w.sum(-1, keepdims=True, dtype=np.float64)).astype(np.float32)
        return p, idx, w

    def forward(self, xm, res):
        xm = np.asarray(xm, np.float32)
        out = np.asarray(res, np.float32).copy()
        xb = bf16_round(xm)
        _, idx, w = self.route(xb)
        if self.shared is not None:
            sg_b, su_b, sd_b, sgw = self.shared
            g = xb @ dequant_q4_1(sg_b).T
            u = xb @ dequant_q4_1(su_b).T
            h = bf16_round(g / (1 + np.exp(-g)) * u)
            gate = 1.0 / (1.0 + np.exp(-(xb @ np.asarray(sgw, np.float32))))
            out += gate[:, None] * (h @ dequant_q4_1(sd_b).T)
        E = len(self.gate)
        counts, offsets, pos, pair = dispatch(idx, E)
        k = idx.shape[1]
        for e in range(E):
            lo, hi = offsets[e], offsets[e + 1]
            if lo == hi:
                continue
            pr = pair[lo:hi]
            toks, slots = pr // k, pr % k
            x = xb[toks]
            g = x @ dequant_q4_1(self.gate[e]).T
            u = x @ dequant_q4_1(self.up[e]).T
            h = bf16_round(g / (1 + np.exp(-g)) * u)
            y = h @ dequant_q4_1(self.down[e]).T
            np.add.at(out, toks, w[toks, slots][:, None] * y)
        return out, idx, w
