"""Benchmark of the Qwen3.6-MoE expert block on B200 -- prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flowmoe|reference] [--no-sweep]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Headline workload (the metric's 1/2/4/8-GPU line): the Qwen3.6-MoE-shaped layer
(H 2048, 256 experts, top-8, F 512, shared expert F 512 with sigmoid gate, Q4_1 weights) over T=8192
bf16 tokens per GPU. A step is one fm_moe_layer call (router, dispatch, shared + routed experts,
combine) over the step's tokens. Weights (503 MB of Q4_1) exceed the 126 MB L2, so every step
streams them from HBM. With N > 1 GPUs (torchrun, one rank per GPU) the layer is expert parallel:
rank r holds experts [r * 256 / N, (r + 1) * 256 / N), router and shared expert replicated, its own
8192 tokens; a step is one fm_ep_peer_layer call: the routed rows go to their experts' ranks as peer
stores over NVLink, each rank runs its experts, the y rows come back the same way, then the combine
(--ep nccl: the NCCL all-to-all variant instead); weak scaling, the tokens per GPU stay fixed.
  value   tokens/s of the whole job, inputs resident on the device, CUDA events, max over ranks;
  e2e     the same through the public API with pinned host buffers (flowmoe.HostPipeline): every step
          copies x (bf16) and res (f32) in and out (f32) back inside the timed region, the copies of
          neighbouring steps overlapping the kernels on their own streams;
  roofline the dominant kernel (gate_up expert GEMM): algorithmic FLOPs / its event-timed duration
          inside the timed region vs the measured dense bf16 peak (MEASURED_PEAKS.json);
  cpu_baseline the oracle port (NumPy fp32 + BLAS on all host cores) on a bounded token sample,
          rank 0 at N=1;
  sweep   BASELINE configs 2 (decode T 1..32, HBM GB/s, 16 token batches per graph replay so the
          touched experts stream from HBM), 3 (Zipf prefill T 512..8192, TFLOP/s) and 5 on one GPU
          (48-layer RMSNorm stack, decode T=64, one CUDA graph);
  stack_c36_T64_ep (N > 1 with --ep-stack) config 5 across the group: 64 decode tokens split over the
          ranks, each rank's experts of all 48 layers, one CUDA graph per rank, max over ranks.
--impl reference times only the CPU implementation (rank 0), same metric and unit.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "openflowlm-next_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402

WORKLOAD = "qwen36moe_c36_layer_T8192_per_gpu"
METRIC = "MoE-layer tokens/s"
T_HEADLINE = 8192


def headline_config(world: int) -> dict:
    """The workload both arms name (identical dicts): the C36 layer over 8192 tokens per GPU."""
    return {"workload": WORKLOAD, "hidden": 2048, "experts": 256, "top_k": 8, "ffn": 512, "shared_ffn": 512,
            "tokens_per_gpu": T_HEADLINE, "weights": "q4_1", "parallelism": f"ep{world}" if world > 1 else "single",
            "l2": "expert weights 503 MB > 126 MB L2 streamed every step"}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def dist_init(n):
    if n <= 1 or "RANK" not in os.environ:
        return 0, 1, 0
    import datetime
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


class Clocks:
    """SM clocks and throttle reasons sampled DURING the timed region: an NVML thread polling every
    ~2 ms (the timed region is tens of milliseconds, shorter than nvidia-smi's sampling period), the
    same counters nvidia-smi's clocks.sm / clocks_event_reasons report."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, index: int):
        import threading
        self.samples, self.err = [], None
        self.stop_ev = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            try:   # the CUDA device's own GPU, whatever CUDA_VISIBLE_DEVICES maps it to
                self.h = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(torch.cuda.get_device_properties(index).uuid))
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:   # no NVML: report why instead of clocks
            self.nv, self.err = None, f"nvml unavailable: {type(e).__name__}"
            return
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        while not self.samples and self.t.is_alive():   # the sampler is live before timing starts
            time.sleep(0.001)

    def _run(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((sm, rs))
            except Exception as e:
                self.err = f"nvml sample failed: {type(e).__name__}"
                return
            time.sleep(0.002)

    def stop(self):
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err], "samples": 0}
        self.stop_ev.set()
        self.t.join()
        busy = self.samples[1:] or self.samples     # the first sample is taken before the region starts
        if not busy:
            return {"sm_mhz": None, "sm_max_mhz": self.max, "reasons": [self.err or "no samples"], "samples": 0}
        reasons = sorted({n for _, r in busy for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": float(np.median([c for c, _ in busy])), "sm_max_mhz": float(self.max), "reasons": reasons,
                "samples": len(busy), "source": "nvml"}


def time_steps(fn, steps, warmup, world, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def routed_flops(cfg, pairs, T):
    f = 2.0 * pairs * 3 * cfg.hidden * cfg.ffn
    if cfg.shared_ffn:
        f += 2.0 * T * 3 * cfg.hidden * cfg.shared_ffn
    return f


def gate_up_flops(cfg, pairs, T):
    f = 2.0 * pairs * 2 * cfg.hidden * cfg.ffn
    if cfg.shared_ffn:
        f += 2.0 * T * 2 * cfg.hidden * cfg.shared_ffn
    return f


# ------------------------------------------------------------------ sweep (configs 2 and 3)
def graph_time(fn, reps=30, calls=1):
    """Capture fn in a CUDA graph and replay it: ms per layer call (fn makes `calls` of them) of the
    plain graph, and the stage durations per call from a second capture with the stage events inside it
    (its last replay)."""
    from flowmoe import _lib
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps / calls
    gp = torch.cuda.CUDAGraph()
    _lib.profile(True)
    with torch.cuda.graph(gp):
        fn()
    for _ in range(3):
        gp.replay()
    torch.cuda.synchronize()
    stages = _lib.profile_read()
    _lib.profile(False)
    del g, gp
    return ms, {k: round(v / calls, 4) for k, v in stages.items() if v}


def sweep(hbm, tfl_burst):
    import flowmoe
    from flowmoe.synth import C30, synth_layer, synth_tokens
    cfg = flowmoe.MoEConfig(**C30)
    out = {"decode": [], "prefill_zipf": []}
    layer = synth_layer(cfg, seed=0)
    expert_bytes = 3 * cfg.hidden * cfg.ffn * 5 // 8
    gu_bytes = 2 * cfg.hidden * cfg.ffn * 5 // 8
    # Each replay runs R layer calls on R different token batches, so the experts they touch together
    # (most of the layer's 377 MB) exceed the 126 MB L2 and every call streams its experts from HBM.
    R = 16
    for T in (1, 4, 8, 16, 32):
        batches = [synth_tokens(T, cfg.hidden, seed=100 * T + r) for r in range(R)]
        outs = [torch.empty_like(res) for _, res in batches]
        idxs = [torch.empty(T, cfg.top_k, dtype=torch.int32, device="cuda") for _ in range(R)]
        ws = [torch.empty(T, cfg.top_k, device="cuda") for _ in range(R)]

        def calls():
            for (x, res), o, idx, w in zip(batches, outs, idxs, ws):
                layer.forward(x, res, out=o, idx=idx, w=w)

        ms, st = graph_time(calls, calls=R)
        U = sum(int(torch.unique(i).numel()) for i in idxs) / R
        nbytes = U * expert_bytes + (cfg.n_experts + 1) * cfg.hidden * 2 + T * cfg.hidden * (2 + 4 + 4)
        gbs = nbytes / (ms * 1e-3) / 1e9
        gu = U * gu_bytes / (st["gate_up"] * 1e-3) / 1e9 if st.get("gate_up") else None
        out["decode"].append({"T": T, "experts_touched": round(U, 2), "batches_per_replay": R, "ms": round(ms, 4), "tokens_per_s": round(T / ms * 1e3, 1),
                              "GB_s": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4), "stages_ms": st,
                              "gemv_gate_up_GB_s": round(gu, 1) if gu else None,
                              "gemv_gate_up_hbm_frac": round(gu / hbm, 4) if gu else None})
    del layer
    layer = synth_layer(cfg, seed=0, zipf=1.1)
    for T in (512, 2048, 8192):
        x, res = synth_tokens(T, cfg.hidden, seed=T)
        o = torch.empty_like(res)
        idx = torch.empty(T, cfg.top_k, dtype=torch.int32, device="cuda")
        w = torch.empty(T, cfg.top_k, device="cuda")
        ms, st = graph_time(lambda: layer.forward(x, res, out=o, idx=idx, w=w), reps=10)
        cnt = torch.bincount(idx.reshape(-1).long(), minlength=cfg.n_experts)
        fl = routed_flops(cfg, T * cfg.top_k, 0) + 2.0 * T * cfg.hidden * cfg.n_experts
        tf = fl / (ms * 1e-3) / 1e12
        gu_tf = gate_up_flops(cfg, T * cfg.top_k, 0) / (st["gate_up"] * 1e-3) / 1e12 if st.get("gate_up") else None
        out["prefill_zipf"].append({"T": T, "ms": round(ms, 4), "tokens_per_s": round(T / ms * 1e3, 1),
                                    "TFLOP_s": round(tf, 2), "tensor_frac": round(tf / tfl_burst, 4), "stages_ms": st,
                                    "gate_up_TFLOP_s": round(gu_tf, 1) if gu_tf else None,
                                    "max_expert_rows": int(cnt.max()), "empty_experts": int((cnt == 0).sum())})
    # config 5 on one GPU: 48 C36 layers of x + MoE(RMSNorm(x)), decode T=64, the stack captured in one
    # CUDA graph; HBM bytes = per layer the touched experts' Q4_1 + shared expert + router
    from flowmoe.stack import MoEStack
    from flowmoe.synth import C36, synth_stack
    cfg36 = flowmoe.MoEConfig(**C36)
    del layer
    torch.cuda.empty_cache()
    layers, norms = synth_stack(cfg36, 48, seed=5)
    T = 64
    x, _ = synth_tokens(T, cfg36.hidden, seed=5)
    x = x.float()
    e_bytes = 3 * cfg36.hidden * cfg36.ffn * 5 // 8
    fixed = 3 * cfg36.hidden * cfg36.shared_ffn * 5 // 8 + (cfg36.n_experts + 1) * cfg36.hidden * 2
    stack_runs = []
    for path in ("gemv", "auto"):
        for L in layers:
            L.path = path
        stack = MoEStack(layers, norms).capture(T)   # the 48 layers as one CUDA graph
        for _ in range(3):
            stack.forward(x)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            stack.forward(x)
        b.record()
        torch.cuda.synchronize()
        stack_runs.append((a.elapsed_time(b) / 10, path))
        del stack
    ms, path = min(stack_runs)
    # bytes of one step: each layer's touched experts (one eager pass records the routing)
    idx = torch.empty(T, cfg36.top_k, dtype=torch.int32, device="cuda")
    with torch.no_grad():
        cur = x.clone()
        nbytes = 0
        for L, nw in zip(layers, norms):
            cur = L.forward_norm(cur, nw, out=torch.empty_like(cur), idx=idx)
            nbytes += int(torch.unique(idx).numel()) * e_bytes + fixed
    gbs = nbytes / (ms * 1e-3) / 1e9
    out["stack_c36_T64"] = {"layers": 48, "T": T, "path": path, "ms": round(ms, 3),
                            "tokens_per_s": round(T / ms * 1e3, 1), "GB_per_step": round(nbytes / 1e9, 2),
                            "GB_s": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
                            "both_paths_ms": {p: round(m, 3) for m, p in stack_runs}}
    del layers
    return out


# ------------------------------------------------------------------ arms
def ref_router_lib():
    """The reference's own host router (src/open_qwen36/block_host.cpp:766-803, OpenMP), compiled from its
    sources by oracle/Makefile into oracle/_ref/, or None when it was not built."""
    import ctypes
    p = ROOT / "oracle" / "_ref" / "libref_router.so"
    if not p.exists():
        return None
    lib = ctypes.CDLL(str(p))
    lib.ref_router_block.restype = ctypes.c_int
    return lib


class CpuLayer:
    """The CPU implementation of the headline layer on the host cores: the router stage is the reference's
    own C++ host::router_block when oracle/_ref holds it (else the NumPy port's router), the experts, the
    shared expert and the combine are the NumPy fp32 + BLAS port of replica.py / Core::moe_block
    (oracle.moe.MoeLayerF32). Weights: seeded GGUF Q4_1 blocks of the C36 shapes (the reference's block
    generator; the timing does not depend on their values)."""

    def __init__(self, seed=0, threads=None):
        from oracle.moe import MoeLayerF32, bf16_round
        from oracle.q4_1 import random_q4_1_blocks
        self.cores = threads or len(os.sched_getaffinity(0))
        torch.set_num_threads(self.cores)
        os.environ["OMP_NUM_THREADS"] = str(self.cores)
        rng = np.random.default_rng(seed)
        H, E, F, FS, k = 2048, 256, 512, 512, 8
        gate = [random_q4_1_blocks(F, H, rng) for _ in range(E)]
        up = [random_q4_1_blocks(F, H, rng) for _ in range(E)]
        down = [random_q4_1_blocks(H, F, rng) for _ in range(E)]
        shared = (random_q4_1_blocks(FS, H, rng), random_q4_1_blocks(FS, H, rng), random_q4_1_blocks(H, FS, rng),
                  bf16_round(rng.normal(0, 0.02, H).astype(np.float32)))
        self.Wr = bf16_round(rng.normal(0, 0.02, (H, E)).astype(np.float32))
        self.port = MoeLayerF32(self.Wr, gate, up, down, shared=shared, topk=k)
        self.x = bf16_round(rng.standard_normal((T_HEADLINE, H), dtype=np.float32))
        self.res = rng.standard_normal((T_HEADLINE, H)).astype(np.float32)
        self.ref = ref_router_lib()
        if self.ref is not None:   # the reference router replaces the port's own
            self.port.route = self._route_ref

    def _route_ref(self, xm):
        import ctypes
        xm = np.ascontiguousarray(xm, np.float32)
        T, H = xm.shape
        E, k = self.Wr.shape[1], self.port.topk
        probs = np.empty((T, E), np.float32)
        idx = np.empty((T, k), np.int32)
        w = np.empty((T, k), np.float32)
        f = ctypes.POINTER(ctypes.c_float)
        rc = self.ref.ref_router_block(ctypes.c_size_t(T), ctypes.c_size_t(H), ctypes.c_size_t(E), ctypes.c_size_t(k),
                                       xm.ctypes.data_as(f), self.Wr.ctypes.data_as(f), probs.ctypes.data_as(f),
                                       idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), w.ctypes.data_as(f))
        if rc:
            raise RuntimeError("reference router_block raised")
        return probs, idx, w

    @property
    def kind_text(self):
        r = ("router: the reference's own host::router_block (block_host.cpp, built from its sources by "
             "oracle/Makefile, OpenMP)" if self.ref is not None else "router: NumPy port")
        return f"{r}; experts, shared expert and combine: NumPy fp32 + BLAS port ({self.cores} threads)"

    def step(self, t0, n):
        """One step over tokens [t0, t0 + n) of the 8192-token batch; returns the seconds it took."""
        a = time.perf_counter()
        self.port.forward(self.x[t0:t0 + n], self.res[t0:t0 + n])
        return time.perf_counter() - a

    def router_rate(self, n=T_HEADLINE):
        """Tokens/s of the router stage alone over n tokens (the reference's C++ when built)."""
        xm = self.x[:n]
        a = time.perf_counter()
        self.port.route(xm)
        return n / (time.perf_counter() - a)


def run_reference(args):
    """The CPU implementation of the path on the host cores, rank 0 only (the other ranks exit without
    work). Same metric, unit and config dict as the flowmoe arm; each step is a bounded sample of the
    headline batch (its first tokens onwards), timed whole, so ms_per_step is the measured step time."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return 0
    cpu = CpuLayer(seed=0)
    # size the sample so that warm-up + timed steps take about two minutes
    probe = cpu.step(0, 16)
    n = int(max(16, min(1024, 16 * 120.0 / max(1e-3, probe * (args.steps + args.warmup)))))
    times = []
    for i in range(args.warmup + args.steps):
        dt = cpu.step((i * n) % (T_HEADLINE - n + 1), n)
        if i >= args.warmup:
            times.append(dt)
    step_s = float(np.median(times))
    val = n / step_s
    router = cpu.router_rate(min(T_HEADLINE, 2048))
    line = {"impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": headline_config(args.gpus),
            "cpu_baseline": {"value": round(val, 3), "unit": "tokens/s", "cores": cpu.cores, "kind": "port",
                             "sample": f"each step {n} of the 8192 tokens of the headline layer; {cpu.kind_text}",
                             "router_only_tokens_per_s": round(router, 1)},
            "e2e": {"value": round(val, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def ep_stack_measure(rank, world, args, n_layers=48, T_total=64):
    """BASELINE config 5 across the group: 48 C36 layers of x + MoE(RMSNorm(x)), T_total decode tokens
    split over the ranks, experts sharded, the stack captured into one CUDA graph per rank and replayed;
    ms per step is the max over ranks of the CUDA-event time of the replays."""
    import flowmoe
    from flowmoe.ep import expert_range
    from flowmoe.stack import EPMoEStack
    from flowmoe.synth import C36, synth_stack, synth_tokens
    eb, el = expert_range(256, rank, world)
    cfg = flowmoe.MoEConfig(**C36, e_begin=eb, e_local=el)
    layers, norms = synth_stack(cfg, n_layers, seed=5)
    Tr = T_total // world
    x, _ = synth_tokens(T_total, cfg.hidden, seed=5)
    x = x.float()[rank * Tr:(rank + 1) * Tr].contiguous()
    stack = EPMoEStack(layers, norms, t_cap=Tr).capture(Tr)
    st = torch.cuda.current_stream()
    for _ in range(3):
        stack.forward(x)
    stack.check()
    ms = max_over_ranks(time_steps(lambda: stack.forward(x), 10, 0, world, st), world)
    stack.check()
    e_bytes = 3 * cfg.hidden * cfg.ffn * 5 // 8
    stack.close()
    del stack, layers
    torch.cuda.empty_cache()
    return {"layers": n_layers, "T_total": T_total, "tokens_per_rank": Tr, "ms": round(ms, 3),
            "tokens_per_s": round(T_total / (ms * 1e-3), 1), "experts_per_gpu": el,
            "expert_bytes": e_bytes, "graph": "whole stack per rank, replayed"}


def run_flowmoe(args):
    import flowmoe
    from flowmoe import _lib
    from flowmoe.synth import C36, synth_blocks, synth_tokens
    rank, world, local = dist_init(args.gpus)
    torch.cuda.set_device(local)
    hbm, tfl_burst, tfl_sus, peak_kind = peaks()
    cfg = flowmoe.MoEConfig(**C36)
    T = T_HEADLINE
    x, res = synth_tokens(T, cfg.hidden, seed=rank)
    st = torch.cuda.current_stream()
    ep_info = {}
    if world > 1:
        # expert parallel: this rank's 256 / N experts, the replicated router and shared expert, its
        # own T tokens; two all-to-all exchanges per step over NCCL
        from flowmoe.ep import EPMoELayer, PeerEPMoELayer, expert_range
        eb, el = expert_range(cfg.n_experts, rank, world)
        cfg = flowmoe.MoEConfig(**C36, e_begin=eb, e_local=el)
        blocks = synth_blocks(cfg, seed=0)
        gate, up, down, wr, shared = blocks
        base = flowmoe.MoELayer.from_q4_1(cfg, gate, up, down, wr, shared=shared)
        if args.ep == "peer":
            # one fm_ep_peer_layer call: rows and y rows stored into their owners' buffers over NVLink
            layer = PeerEPMoELayer(base, t_cap=T)
            out = torch.empty_like(res)
            idx = torch.empty(T, cfg.top_k, dtype=torch.int32, device="cuda")

            def step():
                layer(x, res, out=out, idx=idx)

            def forward_into(xd, rd, od):
                return layer(xd, rd, out=od, idx=idx)
        else:
            layer = EPMoELayer(base, max_tokens=T)

            def step():
                layer(x, res, timings=ep_info)

            def forward_into(xd, rd, od):
                od.copy_(layer(xd, rd))
                return od
    else:
        blocks = synth_blocks(cfg, seed=0)
        gate, up, down, wr, shared = blocks
        layer = flowmoe.MoELayer.from_q4_1(cfg, gate, up, down, wr, shared=shared)
        out = torch.empty_like(res)
        idx = torch.empty(T, cfg.top_k, dtype=torch.int32, device="cuda")
        w = torch.empty(T, cfg.top_k, device="cuda")
        step = lambda: layer.forward(x, res, out=out, idx=idx, w=w)  # noqa: E731

        def forward_into(xd, rd, od):
            return layer.forward(xd, rd, out=od, idx=idx, w=w)

    # device-resident timing, with the stage events recorded live in the timed region
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clk = Clocks(local)
    _lib.profile(True)
    n0 = _lib.launch_count()
    ms = time_steps(step, args.steps, 0, world, st)
    launches = (_lib.launch_count() - n0) // max(1, args.steps) * args.steps
    stages = _lib.profile_read()
    _lib.profile(False)
    clocks = clk.stop()
    ms_max = max_over_ranks(ms, world)
    value = T * world / (ms_max * 1e-3)
    stage_ms = {k: round(v / args.steps, 4) for k, v in stages.items()}
    if world > 1:
        # the rest of the step, outside the library's stage events (NCCL exchange: the count exchange,
        # its device->host read and the two row exchanges; peer exchange: host launch gaps only)
        stage_ms["exchange"] = round(ms - sum(stages.values()) / args.steps, 4)
    pairs = ep_info.get("recv_rows", T * cfg.top_k)
    if world > 1 and args.ep == "peer":
        # rows this rank's experts received: the counts of its expert range over all ranks' tokens
        from flowmoe.ep import expert_range
        eb, el = expert_range(cfg.n_experts, rank, world)
        mine = ((idx >= eb) & (idx < eb + el)).sum().to(torch.float64)
        import torch.distributed as dist
        dist.all_reduce(mine)
        pairs = int(mine.item())
    gu_ms = stages["gate_up"] / args.steps
    # the gate_up stage events bracket the routed items only: the shared expert runs on a side stream
    # beside the dispatch (one GPU) or the row exchange (expert parallel)
    gu_tflops = gate_up_flops(cfg, pairs, 0) / (gu_ms * 1e-3) / 1e12

    # end to end through the public API with host buffers: flowmoe.HostPipeline streams each step's inputs
    # from pinned host memory and its output back, the copies of neighbouring steps overlapping the kernels
    xh = x.cpu().pin_memory()
    rh = res.cpu().pin_memory()
    oh = torch.empty(T, cfg.hidden, dtype=torch.float32).pin_memory()
    pipe = flowmoe.HostPipeline(layer if world == 1 else base, T,
                                call=lambda xd, rd, od, t_real: forward_into(xd, rd, od))
    for _ in range(2):
        pipe.submit(xh, rh, oh)
    pipe.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(st)
    pipe.wait_on(st)
    for _ in range(args.steps):
        pipe.submit(xh, rh, oh)
    pipe.join(st)
    eb.record(st)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(ea.elapsed_time(eb) / args.steps, world)
    e2e = {"value": round(T * world / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
           "h2d_bytes_per_step": x.numel() * 2 + res.numel() * 4, "d2h_bytes_per_step": oh.numel() * 4,
           "api": "flowmoe.HostPipeline (host->device, layer, device->host on three streams, two slots)"}

    ep_stack = ep_stack_measure(rank, world, args) if world > 1 and args.ep == "peer" and args.ep_stack else None

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            cl = CpuLayer(seed=0)
            n = 64
            dts = [cl.step((i * n) % (T_HEADLINE - n), n) for i in range(max(1, int(args.cpu_seconds / max(1e-3, cl.step(0, 16) * n / 16))))]
            v = n / float(np.median(dts))
            cpu = {"value": round(v, 3), "unit": "tokens/s", "cores": cl.cores, "kind": "port",
                   "sample": f"{len(dts)} steps of {n} of the 8192 tokens of the same layer; {cl.kind_text}",
                   "router_only_tokens_per_s": round(cl.router_rate(2048), 1)}
            del cl
        sw = None if args.no_sweep or world > 1 else sweep(hbm, tfl_burst)
        prof = ROOT / "profiles"
        traffic = None
        tf = prof / "traffic_gate_up.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get("bytes_per_launch")
        # the burst peak for a timed region shorter than a second (the clocks stay at their maximum), the
        # sustained one (the power cap's clocks) for a longer one
        region_s = ms * args.steps / 1e3
        peak, peak_kind_txt = (tfl_burst, "burst") if region_s < 1.0 else (tfl_sus, "sustained")
        line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": headline_config(world),
                **({"ep": {"exchange": "peer stores over NVLink" if args.ep == "peer" else "nccl all_to_all",
                           "experts_per_gpu": cfg.local, "recv_rows_rank0": pairs}} if world > 1 else {}),
                "roofline": {"bound": "tensor", "kernel": "expert_tc<gate_up> (routed items)",
                             "achieved": round(gu_tflops, 2), "peak": peak, "unit": "TFLOP/s",
                             "frac": round(gu_tflops / peak, 4), "traffic": traffic,
                             "peak_kind": f"{peak_kind} bf16 {peak_kind_txt} (timed region {region_s:.3f} s)"},
                "stages_ms": stage_ms, "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks,
                "cpu_baseline": cpu, "sweep": sw,
                **({"stack_c36_T64_ep": ep_stack} if ep_stack else {})}
        print(json.dumps(line), flush=True)
    barrier(world)
    if world > 1:
        import torch.distributed as dist
        if hasattr(layer, "close"):
            layer.close()
        dist.destroy_process_group()
    return 0


def profile_case(name: str, calls: int = 6, path: str = "auto") -> int:
    """A few plain layer calls for an ncu capture (no timing, no JSON): "decode" = C30 T=32 (GEMV path),
    "decode1" = C30 T=1, "prefill" = the headline C36 T=8192 layer; ``path`` forces a kernel choice."""
    import flowmoe
    from flowmoe.synth import C30, C36, synth_layer, synth_tokens
    cfg = flowmoe.MoEConfig(**(C36 if name == "prefill" else C30))
    T = {"decode": 32, "decode1": 1}.get(name, T_HEADLINE)
    layer = synth_layer(cfg, seed=0)
    layer.path = path
    x, res = synth_tokens(T, cfg.hidden, seed=T)
    out = torch.empty_like(res)
    for _ in range(calls):
        layer.forward(x, res, out=out)
    torch.cuda.synchronize()
    print(f"profile case {name}: {calls} calls", flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="flowmoe", choices=["flowmoe", "reference"])
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--ep", default="peer", choices=["peer", "nccl"],
                    help="N > 1: the expert-parallel exchange (peer-memory stores, or NCCL all-to-all)")
    ap.add_argument("--ep-stack", action="store_true",
                    help="N > 1: also time BASELINE config 5 (48-layer stack, 64 decode tokens) across the group")
    ap.add_argument("--profile-case", choices=["decode", "decode1", "prefill"], default=None,
                    help="run a few plain layer calls for an ncu capture and exit")
    ap.add_argument("--profile-path", default="auto", choices=["auto", "tc", "gemv"],
                    help="--profile-case: the kernel choice (MoELayer.path)")
    args = ap.parse_args()
    if args.profile_case:
        return profile_case(args.profile_case, path=args.profile_path)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_flowmoe(args)


if __name__ == "__main__":
    sys.exit(main())
