"""The drop-in host API of the MoE expert block.

Mirrors the reference's engine boundary for this path:
  * ``router_block(xm, Wr, topk) -> (probs, idx, w)``  -- ``host::router_block``
    (src/open_qwen36/block_host.hpp:155-159) / ``replica_block.router_block``
    (open_kernels/model/replica_block.py:160-169);
  * ``MoELayer.moe_block(xm, res, idx, w, t_real)``   -- ``Core::moe_block`` (core.hpp:844-848), with
    the gated shared expert of ``Core::ffn_block`` (core.cpp:4342-4380) folded in;
  * ``MoELayer.forward(xm, res, t_real)``             -- router + shared + experts (core.cpp:4934-4957,
    :3685-3700).
Weights are accepted in the reference's GGUF Q4_1 block layout (``q4_1_pack.random_q4_1_blocks`` /
``gguf_pool.unpack_q4`` shape ``uint8[rows, K/32, 20]``). Torch tensors appear only here, at the
boundary: device memory and the current stream are handed to libflowmoe as raw pointers.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import FM_BF16, FM_F32, FmLayer, call

Q4_1_BYTES = 20


@dataclass(frozen=True)
class MoEConfig:
    """The layer geometry: hidden size, router width, top-k, routed and shared expert intermediate sizes, and
    the expert range this rank holds (e.g. 2048/128/8/768/0 for a Qwen3-30B-A3B-shaped layer,
    2048/256/8/512/512 for a Qwen3.6-MoE-shaped one)."""
    hidden: int = 2048
    n_experts: int = 128
    top_k: int = 8
    ffn: int = 768
    shared_ffn: int = 0
    e_begin: int = 0
    e_local: int | None = None      # None: all experts (one GPU)

    @property
    def local(self) -> int:
        return self.n_experts if self.e_local is None else self.e_local

    def q4_bytes(self, rows: int, k: int) -> int:
        return rows * k // 32 * Q4_1_BYTES

    @property
    def gate_up_bytes(self) -> int:
        return 2 * self.q4_bytes(self.ffn, self.hidden)

    @property
    def down_bytes(self) -> int:
        return self.q4_bytes(self.hidden, self.ffn)


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _as_dev_u8(blocks, device) -> torch.Tensor:
    if isinstance(blocks, np.ndarray):
        b = np.ascontiguousarray(blocks, np.uint8)
        if not b.flags.writeable:   # e.g. a read-only memory map of a model file: copy once
            b = b.copy()
        blocks = torch.from_numpy(b)
    return blocks.to(device=device, dtype=torch.uint8).contiguous()


def _check_dev_u8(t, name: str, numel: int | None = None) -> None:
    """A byte buffer whose pointer goes to a kernel: a contiguous uint8 tensor on a GPU (of `numel` bytes)."""
    if not isinstance(t, torch.Tensor) or t.dtype != torch.uint8 or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous uint8 tensor on a GPU")
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{name} holds {t.numel()} bytes, not {numel}")


def q4_1_to_tiles(blocks, rows: int, k: int, device="cuda", out: torch.Tensor | None = None) -> torch.Tensor:
    """GGUF Q4_1 blocks (numpy or torch, any leading expert dims) -> the device tile layout, per matrix."""
    src = _as_dev_u8(blocks, device).reshape(-1)
    per = rows * k // 32 * Q4_1_BYTES
    if src.numel() % per:
        raise ValueError(f"{src.numel()} block bytes is not a whole number of [{rows}, {k}] matrices")
    if out is not None:
        _check_dev_u8(out, "out", src.numel())
        if out.device != src.device:
            raise ValueError(f"out is on {out.device}, the blocks on {src.device}")
    dst = torch.empty_like(src) if out is None else out.reshape(-1)
    st = _stream(src.device)
    for i in range(src.numel() // per):
        call("fm_q4_1_to_tiles", src[i * per:].data_ptr(), rows, k, dst[i * per:].data_ptr(), st)
    return dst


def gate_up_to_tiles(gate_blocks, up_blocks, F: int, k: int, device="cuda") -> torch.Tensor:
    """Per expert GGUF gate and up blocks [E, F, k/32, 20] -> the interleaved gate_up tiles [E, 2*F*k*5/8]."""
    g = _as_dev_u8(gate_blocks, device).reshape(-1)
    u = _as_dev_u8(up_blocks, device).reshape(-1)
    per = F * k // 32 * Q4_1_BYTES
    if g.numel() != u.numel() or g.numel() % per:
        raise ValueError(f"gate/up blocks are not whole [{F}, {k}] matrices of equal count")
    E = g.numel() // per
    out = torch.empty(E, 2 * per, dtype=torch.uint8, device=device)
    st = _stream(out.device)
    for e in range(E):
        call("fm_gate_up_to_tiles", g[e * per:].data_ptr(), u[e * per:].data_ptr(), F, k, out[e].data_ptr(), st)
    return out


def tiles_to_q4_1(tiles: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """The inverse permutation (tile layout -> GGUF blocks), per matrix."""
    _check_dev_u8(tiles, "tiles")
    src = tiles.reshape(-1)
    per = rows * k // 32 * Q4_1_BYTES
    if per <= 0 or src.numel() % per:
        raise ValueError(f"{src.numel()} tile bytes is not a whole number of [{rows}, {k}] matrices")
    dst = torch.empty_like(src)
    st = _stream(src.device)
    for i in range(src.numel() // per):
        call("fm_tiles_to_q4_1", src[i * per:].data_ptr(), rows, k, dst[i * per:].data_ptr(), st)
    return dst


def pool_to_q4_1(pool, n: int, k: int, rs: int = 2, chunk_bytes: int | None = None, device="cuda") -> torch.Tensor:
    """The reference's pool chunk bytes of one [n, k] matrix -> GGUF Q4_1 blocks [n, k/32, 20] (device).

    ``pool`` is what open_kernels/q4_1_pack.py ``pack_q4_1_pool`` (5120-byte chunks, bf16 scales) or
    gguf_pool/gguf_pool.py ``pack_q4_pool`` (6144-byte chunks, f32 scales) wrote for the matrix with band
    row split ``rs``; ``chunk_bytes`` is inferred from the size when not given. Raises if a scale does
    not fit fp16 exactly (a pool those packers did not write)."""
    src = _as_dev_u8(pool, device).reshape(-1)
    nch = n * k // (32 * 256)
    if chunk_bytes is None:
        chunk_bytes = src.numel() // nch if nch and src.numel() % nch == 0 else 0
    if src.numel() != nch * chunk_bytes:
        raise ValueError(f"{src.numel()} pool bytes are not {nch} chunks of {chunk_bytes} B for [{n}, {k}]")
    out = torch.empty(n, k // 32, Q4_1_BYTES, dtype=torch.uint8, device=src.device)
    bad = torch.empty(1, dtype=torch.int32, device=src.device)
    call("fm_pool_to_q4_1", src.data_ptr(), n, k, rs, chunk_bytes, out.data_ptr(), bad.data_ptr(), _stream(src.device))
    if int(bad.item()):
        raise _lib.FlowMoeError(_lib.FM_EINVAL_SHAPE, f"pool_to_q4_1: {int(bad.item())} scales do not fit fp16")
    return out


def experts_from_pool(gate_up_pool, down_pool, E: int, F: int, H: int, chunk_bytes: int | None = None,
                      device="cuda"):
    """The reference engine's MoE expert pool regions -> per-expert GGUF Q4_1 blocks on the device:
    (gate [E, F, H/32, 20], up [E, F, H/32, 20], down [E, H, F/32, 20]).

    ``gate_up_pool`` is what the engine's ``expert_stripes`` op writes (src/open_qwen36/pools.cpp:927-950):
    per expert, per 128-row stripe k, the up stripe then the gate stripe (``[up_k | gate_k]``), each stripe's
    32-row x 256-column chunks in ``stripe_transpose`` order (open_kernels/recipes/pack.py:525-530), i.e.
    the chunk law of q4_1_pack.chunk_geometry with band row split 4. ``down_pool`` is what ``expert_down``
    writes (pools.cpp:951-962): one slice per expert in ``down_perm`` order (recipes/pack.py:515-522), the
    same law for the F = 512 the reference packs. Chunks are 5120 bytes (bf16 d and m, the q4nx pool) or
    6144 (f32 d and m); ``chunk_bytes`` is inferred from the sizes when not given."""
    if F % 128 or H % 256 or F % 256 or H % 128:
        raise ValueError(f"expert pool geometry needs F % 256 == 0 and H % 256 == 0 (F={F}, H={H})")
    gu = _as_dev_u8(gate_up_pool, device).reshape(-1)
    dn = _as_dev_u8(down_pool, device).reshape(-1)
    nch = E * 2 * F * H // (32 * 256)
    if chunk_bytes is None:
        chunk_bytes = gu.numel() // nch if nch and gu.numel() % nch == 0 else 0
    if gu.numel() != nch * chunk_bytes or dn.numel() * 2 != gu.numel():
        raise ValueError(f"pool regions of {gu.numel()} and {dn.numel()} bytes are not {E} experts of "
                         f"[{F}, {H}] up/gate and [{H}, {F}] down in {chunk_bytes}-byte chunks")
    st = gu.reshape(E, F // 128, 2, -1)
    dnv = dn.reshape(E, -1)
    gate, up, down = [], [], []
    for e in range(E):
        up.append(pool_to_q4_1(st[e, :, 0].contiguous(), F, H, rs=4, chunk_bytes=chunk_bytes, device=gu.device))
        gate.append(pool_to_q4_1(st[e, :, 1].contiguous(), F, H, rs=4, chunk_bytes=chunk_bytes, device=gu.device))
        down.append(pool_to_q4_1(dnv[e], H, F, rs=4, chunk_bytes=chunk_bytes, device=gu.device))
    return torch.stack(gate), torch.stack(up), torch.stack(down)


def narrow_scales(tiles: torch.Tensor) -> torch.Tensor:
    """In place: every d and m of a tile array rounded to bf16 precision (fm_tiles_narrow_scales)."""
    _check_dev_u8(tiles, "tiles")
    n = tiles.numel()
    if n % 5120:
        raise ValueError("not a whole number of 5120-byte tiles")
    call("fm_tiles_narrow_scales", tiles.data_ptr(), n // 5120, _stream(tiles.device))
    return tiles


def _bf16(t, device) -> torch.Tensor:
    if isinstance(t, np.ndarray):
        if t.dtype == np.uint16:
            return torch.from_numpy(t.astype(np.int16, copy=False).view(np.int16)).view(torch.bfloat16).to(device)
        a = np.ascontiguousarray(t, np.float32)
        if not a.flags.writeable:   # e.g. a read-only GGUF memory map: torch wants a writable buffer
            a = a.copy()
        t = torch.from_numpy(a)
    return t.to(device=device, dtype=torch.bfloat16).contiguous()


def _size(x) -> int:
    return int(x.numel()) if isinstance(x, torch.Tensor) else int(np.asarray(x).size)


def _check_inputs(cfg: MoEConfig, gate_blocks, up_blocks, down_blocks, router_w, shared, router_bias) -> None:
    """Every host-side size check of MoELayer.from_q4_1, before any device work."""
    H, F, E = cfg.hidden, cfg.ffn, cfg.local
    if _size(gate_blocks) != E * cfg.q4_bytes(F, H) or _size(up_blocks) != E * cfg.q4_bytes(F, H):
        raise ValueError("gate/up blocks do not match [E_local, F, H/32, 20]")
    if _size(down_blocks) != E * cfg.down_bytes:
        raise ValueError("down blocks do not match [E_local, H, F/32, 20]")
    wr_shape = tuple(router_w.shape)
    if wr_shape != (H, cfg.n_experts):
        raise ValueError(f"router weight shape {wr_shape} != (H, E) = {(H, cfg.n_experts)}")
    if shared is not None:
        if cfg.shared_ffn <= 0:
            raise ValueError("shared expert weights given but cfg.shared_ffn == 0")
        sg, su, sd, sgw = shared
        FS = cfg.shared_ffn
        if _size(sg) != cfg.q4_bytes(FS, H) or _size(su) != cfg.q4_bytes(FS, H) or _size(sd) != cfg.q4_bytes(H, FS):
            raise ValueError("shared expert blocks do not match [F_s, H/32, 20] / [H, F_s/32, 20]")
        if sgw is not None and _size(sgw) != H:
            raise ValueError(f"shared gate vector has {_size(sgw)} values, not H = {H}")
    if router_bias is not None and _size(router_bias) != cfg.n_experts:
        raise ValueError(f"router bias has {_size(router_bias)} values, not E = {cfg.n_experts}")


class MoELayer:
    """One Qwen3.6-MoE expert block resident on a B200: router, routed experts, shared expert."""

    def __init__(self, cfg: MoEConfig, gate_up: torch.Tensor, down: torch.Tensor, router: torch.Tensor,
                 shared_gate_up: torch.Tensor | None = None, shared_down: torch.Tensor | None = None,
                 router_bias: torch.Tensor | None = None):
        self.cfg = cfg
        self.device = router.device
        self.gate_up, self.down, self.router = gate_up, down, router
        self.shared_gate_up, self.shared_down = shared_gate_up, shared_down
        self.router_bias = None if router_bias is None else router_bias.to(self.device, torch.float32).contiguous()
        self._L = FmLayer(cfg.hidden, cfg.n_experts, cfg.top_k, cfg.ffn, cfg.shared_ffn, cfg.e_begin, cfg.local, 0,
                          gate_up.data_ptr(), down.data_ptr(), _ptr(shared_gate_up), _ptr(shared_down),
                          router.data_ptr(), _ptr(self.router_bias))
        self._ws: torch.Tensor | None = None

    PATHS = {"auto": 0, "tc": 2, "gemv": 3}
    FIXED_ORDER = 0x100   # FM_FIXED_ORDER (include/flowmoe.h)

    @property
    def path(self) -> str:
        """Kernel choice: "auto" (the GEMV up to 128 tokens while tokens x top_k <= 1024, else the tcgen05
        grouped GEMM), or forced "tc" (tcgen05) or "gemv" (the GEMV, within the same limits; tcgen05 past
        them)."""
        return {v: k for k, v in self.PATHS.items()}[self._L.flags & 0xFF]

    @path.setter
    def path(self, name: str) -> None:
        self._L.flags = (self._L.flags & ~0xFF) | self.PATHS[name]

    @property
    def fixed_order(self) -> bool:
        """Every token's expert terms added in ascending expert order (the reference's scatter order,
        core.cpp:5163-5165): outputs bit-reproducible and independent of the other tokens of a call, so a
        prompt run layer-major (each layer over all its tokens) matches block-major bit for bit. Costs the
        tcgen05 path f32 y-row scratch and a combine kernel, the GEMV path its K splits."""
        return bool(self._L.flags & self.FIXED_ORDER)

    @fixed_order.setter
    def fixed_order(self, on: bool) -> None:
        self._L.flags = (self._L.flags | self.FIXED_ORDER) if on else (self._L.flags & ~self.FIXED_ORDER)

    # ---- construction from the reference's block layout
    @classmethod
    def from_q4_1(cls, cfg: MoEConfig, gate_blocks, up_blocks, down_blocks, router_w, shared=None, device="cuda",
                  router_bias=None, scales: str = "fp16"):
        """gate/up blocks [E_local, F, H/32, 20], down [E_local, H, F/32, 20] (numpy or torch uint8),
        router_w [H, E] (bf16 values), shared = (gate, up, down blocks, sgw [H]) or None,
        router_bias [E] f32 added to the logits (or None). scales="bf16" narrows every block's d and m
        to bf16 first: the reference's q4nx pool numerics."""
        if scales not in ("fp16", "bf16"):
            raise ValueError(f"scales must be 'fp16' or 'bf16', not {scales!r}")
        H, F, E = cfg.hidden, cfg.ffn, cfg.local
        _check_inputs(cfg, gate_blocks, up_blocks, down_blocks, router_w, shared, router_bias)
        g = _as_dev_u8(gate_blocks, device).reshape(E, -1)
        u = _as_dev_u8(up_blocks, device).reshape(E, -1)
        gate_up = gate_up_to_tiles(g, u, F, H, device)
        down = q4_1_to_tiles(_as_dev_u8(down_blocks, device), H, F, device).reshape(E, -1)
        sgu = sdn = None
        sgw = None
        if shared is not None:
            sg, su, sd, sgw = shared
            FS = cfg.shared_ffn
            sgu = gate_up_to_tiles(sg, su, FS, H, device).reshape(-1)
            sdn = q4_1_to_tiles(sd, H, FS, device)
        wr = _bf16(router_w, device)
        router = torch.empty(cfg.n_experts + 1, H, dtype=torch.bfloat16, device=device)
        sgw_t = None if sgw is None else _bf16(sgw, device).reshape(H)
        call("fm_router_pack", wr.data_ptr(), _ptr(sgw_t), H, cfg.n_experts, router.data_ptr(), _stream(device))
        if router_bias is not None and not isinstance(router_bias, torch.Tensor):
            router_bias = torch.from_numpy(np.array(router_bias, np.float32))   # a writable copy
        if scales == "bf16":
            for t in (gate_up, down, sgu, sdn):
                if t is not None:
                    narrow_scales(t)
        return cls(cfg, gate_up.reshape(-1), down.reshape(-1), router, sgu, sdn, router_bias)

    @classmethod
    def from_expert_pool(cls, cfg: MoEConfig, gate_up_pool, down_pool, router_w, shared=None, device="cuda",
                         router_bias=None, chunk_bytes: int | None = None):
        """A layer from the reference engine's expert pool regions (``experts_from_pool``) for this rank's
        cfg.local experts; router, shared expert and bias as in ``from_q4_1``. 5120-byte chunks carry bf16
        scales, so the layer computes with the q4nx pool's numerics."""
        gate, up, down = experts_from_pool(gate_up_pool, down_pool, cfg.local, cfg.ffn, cfg.hidden, chunk_bytes, device)
        return cls.from_q4_1(cfg, gate, up, down, router_w, shared=shared, device=device, router_bias=router_bias)

    # ---- workspace
    def workspace_bytes(self, T: int) -> int:
        n = ctypes.c_size_t(0)
        call("fm_workspace_size", ctypes.byref(self._L), T, ctypes.byref(n))
        return n.value

    def workspace(self, T: int) -> torch.Tensor:
        need = self.workspace_bytes(T)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
        return self._ws

    @staticmethod
    def _dtype(xm: torch.Tensor) -> int:
        if xm.dtype == torch.float32:
            return FM_F32
        if xm.dtype == torch.bfloat16:
            return FM_BF16
        raise TypeError(f"xm must be float32 or bfloat16, not {xm.dtype}")

    def _check_x(self, xm: torch.Tensor):
        if xm.device != self.device or xm.dim() != 2 or xm.shape[1] != self.cfg.hidden or not xm.is_contiguous():
            raise ValueError(f"xm must be a contiguous [T, {self.cfg.hidden}] tensor on {self.device}")

    def _check_bufs(self, T: int, **bufs):
        """Device buffers handed to the library as raw pointers: a host tensor or a wrong size would be
        read or written out of bounds by the kernels, so each is checked here (None = not given)."""
        H, k = self.cfg.hidden, self.cfg.top_k
        want = {"res": (torch.float32, (T, H)), "out": (torch.float32, (T, H)), "idx": (torch.int32, (T, k)),
                "w": (torch.float32, (T, k)), "shared_gate": (torch.float32, (T,))}
        for name, t in bufs.items():
            if t is None:
                continue
            dt, shape = want[name]
            if t.dtype != dt or tuple(t.shape) != shape or not t.is_contiguous() or t.device != self.device:
                raise ValueError(f"{name} must be a contiguous {dt} tensor of shape {shape} on {self.device}")

    # ---- the reference's entry points
    def router_block(self, xm: torch.Tensor, want_probs: bool = True):
        """(probs [T, E] f32, idx [T, k] int32, w [T, k] f32): softmax top-k, lowest index on a tie."""
        self._check_x(xm)
        T, E, k = xm.shape[0], self.cfg.n_experts, self.cfg.top_k
        probs = torch.empty(T, E, dtype=torch.float32, device=self.device) if want_probs else None
        idx = torch.empty(T, k, dtype=torch.int32, device=self.device)
        w = torch.empty(T, k, dtype=torch.float32, device=self.device)
        self.shared_gate_buf = torch.empty(T, dtype=torch.float32, device=self.device)
        ws = self.workspace(T)
        call("fm_router_topk", ctypes.byref(self._L), xm.data_ptr(), self._dtype(xm), T, _ptr(probs), idx.data_ptr(),
             w.data_ptr(), self.shared_gate_buf.data_ptr(), ws.data_ptr(), ws.numel(), _stream(self.device))
        return probs, idx, w

    def shared_gate(self, xm: torch.Tensor) -> torch.Tensor:
        """sigmoid(bf16(xm) . sgw) per token (core.cpp:4370-4373)."""
        self.router_block(xm, want_probs=False)
        return self.shared_gate_buf

    def moe_block(self, xm: torch.Tensor, res: torch.Tensor, idx: torch.Tensor, w: torch.Tensor,
                  t_real: int | None = None, shared_gate: torch.Tensor | None = None, check: bool = True,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        """out = res + shared_gate * shared(xm) + sum_e w_e * expert_e(xm), ascending expert order.
        ``check`` synchronises and raises on expert ids outside [e_begin, e_begin + e_local)
        (the reference throws, core.cpp:5159-5160)."""
        self._check_x(xm)
        T = xm.shape[0]
        t_real = T if t_real is None else t_real
        if res is None or idx is None or w is None:
            raise ValueError("moe_block needs res, idx and w")
        self._check_bufs(T, res=res, idx=idx, w=w, out=out, shared_gate=shared_gate)
        out = torch.empty_like(res) if out is None else out
        ws = self.workspace(T)
        st = _stream(self.device)
        call("fm_moe_block", ctypes.byref(self._L), xm.data_ptr(), self._dtype(xm), res.data_ptr(), idx.data_ptr(),
             w.data_ptr(), _ptr(shared_gate), T, t_real, out.data_ptr(), ws.data_ptr(), ws.numel(), st)
        if check:
            call("fm_moe_check", ws.data_ptr(), st)
        return out

    def dispatch(self, idx: torch.Tensor, t_real: int | None = None):
        """(counts [e_local], offsets [e_local + 1], pos [t_real, k], pair [P]) of the stable
        expert-sorted order (the owed lists and ascending visits of core.cpp:5155-5165)."""
        T, k = idx.shape
        t_real = T if t_real is None else t_real
        E = self.cfg.local
        counts = torch.empty(E, dtype=torch.int32, device=self.device)
        offsets = torch.empty(E + 1, dtype=torch.int32, device=self.device)
        pos = torch.empty(t_real, k, dtype=torch.int32, device=self.device)
        pair = torch.empty(max(t_real * k, 1), dtype=torch.int32, device=self.device)
        ws = self.workspace(T)
        call("fm_moe_dispatch", ctypes.byref(self._L), idx.data_ptr(), T, t_real, counts.data_ptr(),
             offsets.data_ptr(), pos.data_ptr(), pair.data_ptr(), ws.data_ptr(), ws.numel(), _stream(self.device))
        torch.cuda.current_stream(self.device).synchronize()
        return counts, offsets, pos, pair[:int(offsets[-1].item())]

    def forward(self, xm: torch.Tensor, res: torch.Tensor, t_real: int | None = None, out: torch.Tensor | None = None,
                idx: torch.Tensor | None = None, w: torch.Tensor | None = None) -> torch.Tensor:
        """Router + shared expert + routed experts (fm_moe_layer)."""
        self._check_x(xm)
        T = xm.shape[0]
        self._check_bufs(T, res=res, out=out, idx=idx, w=w)
        t_real = T if t_real is None else t_real
        out = torch.empty(T, self.cfg.hidden, dtype=torch.float32, device=self.device) if out is None else out
        ws = self.workspace(T)
        call("fm_moe_layer", ctypes.byref(self._L), xm.data_ptr(), self._dtype(xm), res.data_ptr(), T, t_real,
             out.data_ptr(), _ptr(idx), _ptr(w), ws.data_ptr(), ws.numel(), _stream(self.device))
        return out

    __call__ = forward

    def forward_norm(self, x: torch.Tensor, norm_w: torch.Tensor, eps: float = 1e-6, t_real: int | None = None,
                     out: torch.Tensor | None = None, idx: torch.Tensor | None = None,
                     w: torch.Tensor | None = None) -> torch.Tensor:
        """One layer of the MoE stack: out = x + MoE(RMSNorm(x)) (fm_moe_layer_norm). x f32 [T, H]; norm_w
        bf16 [H] (the post-attention RMSNorm weight)."""
        if x.dtype != torch.float32 or x.device != self.device or x.dim() != 2 or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous f32 [T, {self.cfg.hidden}] tensor on {self.device}")
        T = x.shape[0]
        self._check_bufs(T, out=out, idx=idx, w=w)
        t_real = T if t_real is None else t_real
        out = torch.empty_like(x) if out is None else out
        if out.data_ptr() == x.data_ptr():
            raise ValueError("out may not alias x")
        nw = norm_w.to(self.device, torch.bfloat16).contiguous()
        ws = self.workspace(T)
        call("fm_moe_layer_norm", ctypes.byref(self._L), x.data_ptr(), nw.data_ptr(), ctypes.c_float(eps), T, t_real,
             out.data_ptr(), _ptr(idx), _ptr(w), ws.data_ptr(), ws.numel(), _stream(self.device))
        return out


def router_block(xm: torch.Tensor, Wr: torch.Tensor, topk: int):
    """Functional ``host::router_block``: (probs, idx, w) for xm [T, H] and Wr [H, E] on the device.
    H is zero-padded to a multiple of 128 (exact for the dot products)."""
    H0, E = Wr.shape
    if topk > E:
        raise _lib.FlowMoeError(_lib.FM_EINVAL_SHAPE, "router_block: topk past the expert count")
    H = (H0 + 127) // 128 * 128
    dev = xm.device
    if H != H0:
        xm = torch.nn.functional.pad(xm, (0, H - H0))
        Wr = torch.nn.functional.pad(Wr, (0, 0, 0, H - H0))
    cfg = MoEConfig(hidden=H, n_experts=E, top_k=topk, ffn=128, shared_ffn=0)
    router = torch.empty(E + 1, H, dtype=torch.bfloat16, device=dev)
    wr = Wr.to(torch.bfloat16).contiguous()
    call("fm_router_pack", wr.data_ptr(), None, H, E, router.data_ptr(), _stream(dev))
    dummy = torch.empty(256, dtype=torch.uint8, device=dev)
    layer = MoELayer(cfg, dummy, dummy, router)
    return layer.router_block(xm.contiguous())
