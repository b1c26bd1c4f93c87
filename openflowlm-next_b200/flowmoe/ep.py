"""Expert parallelism: the MoE block over G ranks, one process per GPU.

The reference runs every expert on one NPU (``Core::moe_block``, src/open_qwen36/core.cpp:5150-5259),
so this module has no counterpart there; it keeps that call's result. Rank r holds experts
[r * E / G, (r + 1) * E / G); the router and the shared expert are replicated and run on each rank's
own tokens. One layer is:

  1. ``dispatch``  (device) router, stable sort of the (token, slot) pairs over all E experts, gather
                   of the sorted bf16 rows: the rows for rank g are one contiguous range;
  2. exchange      all-to-all of the per-expert counts (int32 [G, E / G]), one device->host read of
                   the split sizes, all-to-all of the rows (NCCL over NVLink on the GPU);
  3. ``experts``   (device) regroup the received rows expert-major, this rank's experts as tcgen05
                   grouped GEMMs -> unweighted bf16 y rows in the received order; out = res + the
                   gated shared expert of this rank's own tokens;
  4. exchange      the reverse all-to-all of the y rows;
  5. ``combine``   (device) out[t] += w * y over t's pairs in ascending expert order.

``ep_forward`` is the exchange logic alone, over a ``stages`` object that provides steps 1, 3 and
5: ``DeviceStages`` (libflowmoe on the GPU) in production, a CPU stand-in in the tests, so the
exchange runs unchanged over gloo ranks on CPU.

``PeerEPMoELayer`` (over a ``PeerGroup``) is the default multi-GPU layer: one ``fm_ep_peer_layer`` call
does all five steps on the device, the two exchanges being the library's own stores into the owners'
IPC-mapped buffers over NVLink, synchronised by device flags (no host step, so it can be graph-captured).
"""
from __future__ import annotations

import ctypes
from datetime import timedelta

import torch
import torch.distributed as dist

from ._lib import FM_BF16, FM_EP_MAX_RANKS, FM_F32, FmEpGroup, call
from .layer import MoEConfig, MoELayer, _stream


class ExchangeError(RuntimeError):
    """The ranks disagree about the exchange (counts that do not add up), or a peer failed."""


def expert_range(n_experts: int, rank: int, world: int) -> tuple[int, int]:
    """(e_begin, e_local) of ``rank``: the contiguous block [r * E / G, (r + 1) * E / G)."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
    el = n_experts // world
    return rank * el, el


def ep_forward(stages, x: torch.Tensor, res: torch.Tensor, t_real: int | None = None, group=None,
               timings: dict | None = None) -> torch.Tensor:
    """One MoE layer of this rank's tokens ``x`` [T, H] over the expert-parallel group.

    Every rank takes the same collective steps in the same order, whatever its token count (T may be
    0 on some ranks). Returns out [T, H] f32 = res + shared + routed experts."""
    G = dist.get_world_size(group)
    T = x.shape[0]
    t_real = T if t_real is None else t_real
    E, k, H = stages.n_experts, stages.top_k, stages.hidden
    El = E // G
    P = t_real * k
    xsend, counts, pos, idx, w, sg, xb = stages.dispatch(x, t_real)
    # counts for rank g's experts go to rank g: equal splits of El
    recv_counts = torch.empty(G * El, dtype=torch.int32, device=counts.device)
    dist.all_to_all_single(recv_counts, counts, group=group)
    host = torch.cat([counts, recv_counts]).cpu()          # the one device -> host read per layer
    send_splits = host[:E].view(G, El).sum(1).tolist()
    recv_splits = host[E:].view(G, El).sum(1).tolist()
    if sum(send_splits) != P or min(recv_splits) < 0 or int(host[E:].min()) < 0:
        raise ExchangeError(f"inconsistent counts: sent {sum(send_splits)} of {P} pairs, received {recv_splits}")
    R = sum(recv_splits)
    if R > G * stages.max_tokens * k:
        raise ExchangeError(f"received {R} rows, more than {G} ranks x {stages.max_tokens} tokens x {k} can send")
    xrecv = stages.rows(R + 1)          # one spare row: never a zero-size buffer
    dist.all_to_all_single(xrecv[:R], xsend[:P], recv_splits, send_splits, group=group)
    out, yrecv = stages.experts(xrecv, R, recv_counts, G, xb, sg, res, T, t_real)
    ysorted = stages.rows(P + 1)
    dist.all_to_all_single(ysorted[:P], yrecv[:R], send_splits, recv_splits, group=group)
    stages.combine(out, ysorted, pos, idx, w, T, t_real)
    if timings is not None:
        timings["recv_rows"] = R
        timings["send_rows"] = P
    return out


class DeviceStages:
    """Steps 1, 3 and 5 on this rank's GPU through libflowmoe (fm_ep_dispatch / fm_ep_experts /
    fm_ep_combine). ``layer`` holds this rank's experts (cfg.e_begin, cfg.e_local = its range) and
    the full router and shared expert."""

    def __init__(self, layer: MoELayer, max_tokens: int):
        self.layer = layer
        c = layer.cfg
        self.n_experts, self.top_k, self.hidden = c.n_experts, c.top_k, c.hidden
        self.max_tokens = max_tokens
        self.device = layer.device
        self._ws = None
        self._bufs: dict[str, torch.Tensor] = {}
        self._rows: list[torch.Tensor] = []
        self._row_turn = 0

    def _buf(self, name, n, dtype):
        b = self._bufs.get(name)
        if b is None or b.numel() < n or b.dtype != dtype:
            b = torch.empty(max(n, 1), dtype=dtype, device=self.device)
            self._bufs[name] = b
        return b[:n]

    def rows(self, n: int) -> torch.Tensor:
        """A bf16 [n, H] row buffer; two alternate (the received rows and the returned rows)."""
        if len(self._rows) < 2:
            self._rows = [torch.empty(0, self.hidden, dtype=torch.bfloat16, device=self.device) for _ in range(2)]
        i = self._row_turn
        self._row_turn ^= 1
        if self._rows[i].shape[0] < n:
            self._rows[i] = torch.empty(n, self.hidden, dtype=torch.bfloat16, device=self.device)
        return self._rows[i][:n]

    def _workspace(self, T, R, G):
        n = ctypes.c_size_t(0)
        call("fm_ep_workspace_size", ctypes.byref(self.layer._L), T, R, G, ctypes.byref(n))
        if self._ws is None or self._ws.numel() < n.value:
            self._ws = torch.empty(max(n.value, 256), dtype=torch.uint8, device=self.device)
        return self._ws

    def dispatch(self, x: torch.Tensor, t_real: int):
        T, H, E, k = x.shape[0], self.hidden, self.n_experts, self.top_k
        if x.dtype == torch.bfloat16:
            dt, xb = FM_BF16, x
        elif x.dtype == torch.float32:
            dt, xb = FM_F32, self._buf("xb", T * H, torch.bfloat16).view(T, H)
        else:
            raise TypeError(f"x must be float32 or bfloat16, not {x.dtype}")
        idx = self._buf("idx", T * k, torch.int32).view(T, k)
        w = self._buf("w", T * k, torch.float32).view(T, k)
        sg = self._buf("sg", T, torch.float32)
        counts = self._buf("counts", E, torch.int32)
        pos = self._buf("pos", T * k, torch.int32).view(T, k)
        xsend = self._buf("xsend", (T * k + 1) * H, torch.bfloat16).view(T * k + 1, H)
        ws = self._workspace(T, 0, 1)
        call("fm_ep_dispatch", ctypes.byref(self.layer._L), x.data_ptr(), dt, T, t_real,
             xb.data_ptr() if dt == FM_F32 else None, idx.data_ptr(), w.data_ptr(), sg.data_ptr(), counts.data_ptr(),
             pos.data_ptr(), xsend.data_ptr(), ws.data_ptr(), ws.numel(), _stream(self.device))
        return xsend, counts, pos, idx, w, sg, xb

    def experts(self, xrecv, R, recv_counts, G, xb, sg, res, T, t_real):
        out = torch.empty(T, self.hidden, dtype=torch.float32, device=self.device)
        yrecv = self.rows(R + 1)
        ws = self._workspace(T, R, G)
        call("fm_ep_experts", ctypes.byref(self.layer._L), xrecv.data_ptr(), R, recv_counts.data_ptr(), G,
             xb.data_ptr(), sg.data_ptr(), res.data_ptr(), T, t_real, out.data_ptr(), yrecv.data_ptr(), ws.data_ptr(),
             ws.numel(), _stream(self.device))
        return out, yrecv

    def combine(self, out, ysorted, pos, idx, w, T, t_real):
        call("fm_ep_combine", ctypes.byref(self.layer._L), out.data_ptr(), ysorted.data_ptr(), pos.data_ptr(),
             idx.data_ptr(), w.data_ptr(), T, t_real, _stream(self.device))

    def check(self):
        """Synchronise and raise on a device wait that gave up or an expert id out of range."""
        if self._ws is not None:
            call("fm_moe_check", self._ws.data_ptr(), _stream(self.device))


class PeerGroup:
    """The symmetric buffers of a peer-memory expert-parallel group: each rank allocates one
    (fm_ipc_alloc), the IPC handles are all-gathered over ``group`` (host objects only), each rank maps
    the others' (fm_ipc_open). ``layer`` must hold this rank's expert range."""

    def __init__(self, layer: MoELayer, t_cap: int, group=None, timeout_ms: int = 10000):
        self.layer = layer
        self.group = group
        G, r = dist.get_world_size(group), dist.get_rank(group)
        if G > FM_EP_MAX_RANKS:
            raise ValueError(f"at most {FM_EP_MAX_RANKS} ranks")
        self.g = FmEpGroup(r, G, t_cap, timeout_ms)
        sym_b, ws_b = ctypes.c_size_t(0), ctypes.c_size_t(0)
        call("fm_ep_peer_sizes", ctypes.byref(layer._L), ctypes.byref(self.g), ctypes.byref(sym_b), ctypes.byref(ws_b))
        self.sym_bytes = sym_b.value
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        call("fm_ipc_alloc", self.sym_bytes, ctypes.byref(own), handle)
        self._own = own.value
        handles = [None] * G
        dist.all_gather_object(handles, (handle.raw, t_cap, self.sym_bytes), group=group)
        if len({h[1:] for h in handles}) != 1:
            call("fm_ipc_free", self._own)
            raise ValueError(f"ranks disagree on (t_cap, buffer bytes): {[h[1:] for h in handles]}")
        handles = [h[0] for h in handles]
        self._opened = []
        for i in range(G):
            if i == r:
                self.g.sym[i] = self._own
                continue
            p = ctypes.c_void_p()
            call("fm_ipc_open", handles[i], ctypes.byref(p))
            self.g.sym[i] = p.value
            self._opened.append(p.value)
        self.ws = torch.empty(max(ws_b.value, 256), dtype=torch.uint8, device=layer.device)
        torch.cuda.synchronize(layer.device)
        dist.barrier(group=group)

    def close(self):
        """Unmap the peers' buffers and free our own, after every rank has finished with them."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.layer.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            call("fm_ipc_close", p)
        self._opened = []
        dist.barrier(group=self.group)
        call("fm_ipc_free", self._own)
        self._own = None


class PeerEPMoELayer:
    """The MoE block of one rank over peer memory: one fm_ep_peer_layer call per layer, rows and y rows
    stored straight into their owners' buffers over NVLink, no NCCL and no host round trip."""

    def __init__(self, layer: MoELayer, t_cap: int, group=None, timeout_ms: int = 10000):
        self.cfg = layer.cfg
        self.layer = layer
        self.peers = PeerGroup(layer, t_cap, group, timeout_ms)

    def forward(self, x: torch.Tensor, res: torch.Tensor, t_real: int | None = None, out: torch.Tensor | None = None,
                idx: torch.Tensor | None = None, w: torch.Tensor | None = None) -> torch.Tensor:
        layer = self.layer
        layer._check_x(x)
        T = x.shape[0]
        layer._check_bufs(T, res=res, out=out, idx=idx, w=w)
        t_real = T if t_real is None else t_real
        out = torch.empty(T, self.cfg.hidden, dtype=torch.float32, device=layer.device) if out is None else out
        ws = self.peers.ws
        call("fm_ep_peer_layer", ctypes.byref(layer._L), ctypes.byref(self.peers.g), x.data_ptr(), layer._dtype(x),
             res.data_ptr(), T, t_real, out.data_ptr(), None if idx is None else idx.data_ptr(),
             None if w is None else w.data_ptr(), ws.data_ptr(), ws.numel(), _stream(layer.device))
        return out

    __call__ = forward

    def check(self):
        """Synchronise; raise FM_ETIMEOUT if a peer did not take its step in time, or on a bad expert id."""
        call("fm_moe_check", self.peers.ws.data_ptr(), _stream(self.layer.device))

    def close(self):
        self.peers.close()


class EPMoELayer:
    """The MoE block of one rank in an expert-parallel group (``torch.distributed`` initialised, NCCL on
    the GPU). Holds only this rank's experts; ``forward(x, res)`` takes this rank's tokens."""

    def __init__(self, layer: MoELayer, max_tokens: int, group=None):
        self.group = group
        self.stages = DeviceStages(layer, max_tokens)
        self.cfg = layer.cfg

    @classmethod
    def from_q4_1(cls, cfg: MoEConfig, gate_blocks, up_blocks, down_blocks, router_w, shared=None, device="cuda",
                  router_bias=None, max_tokens: int = 8192, group=None):
        """gate/up/down blocks of THIS rank's experts only ([E / G, ...], see ``expert_range``)."""
        G, r = dist.get_world_size(group), dist.get_rank(group)
        eb, el = expert_range(cfg.n_experts, r, G)
        lcfg = MoEConfig(cfg.hidden, cfg.n_experts, cfg.top_k, cfg.ffn, cfg.shared_ffn, eb, el)
        layer = MoELayer.from_q4_1(lcfg, gate_blocks, up_blocks, down_blocks, router_w, shared=shared, device=device,
                                   router_bias=router_bias)
        return cls(layer, max_tokens, group)

    def forward(self, x: torch.Tensor, res: torch.Tensor, t_real: int | None = None,
                timings: dict | None = None) -> torch.Tensor:
        if x.shape[0] > self.stages.max_tokens:
            raise ValueError(f"{x.shape[0]} tokens on this rank, more than max_tokens={self.stages.max_tokens}")
        self.stages.layer._check_x(x)
        self.stages.layer._check_bufs(x.shape[0], res=res)
        return ep_forward(self.stages, x, res, t_real, self.group, timings)

    __call__ = forward


def init_process_group(backend: str = "nccl", timeout_s: float = 120.0):
    """torch.distributed from the torchrun environment, with a bounded collective timeout so that ranks
    waiting on a failed peer end with an error instead of waiting for good."""
    if not dist.is_initialized():
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size()


__all__ = ["EPMoELayer", "PeerEPMoELayer", "PeerGroup", "DeviceStages", "ep_forward", "expert_range", "ExchangeError",
           "init_process_group"]
