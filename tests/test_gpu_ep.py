"""Expert-parallel device stages (fm_ep_dispatch / fm_ep_experts / fm_ep_combine) against the
one-device oracle.

On one GPU the G ranks are emulated: every rank's stages run on cuda:0 and the two all-to-all
exchanges are done by slicing and concatenating the row buffers, so the regroup of rows received
from several sources is covered without a second GPU. With two or more GPUs, two processes run the
real exchange over NCCL.
"""
from __future__ import annotations

import json
import os
import socket
import sys
import time
import traceback
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cases, moe as OM

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
TOL = 2e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda:0")


def _rank_layer(c, rank, world, dev):
    import flowmoe
    from flowmoe.ep import DeviceStages, expert_range
    eb, el = expert_range(c["E"], rank, world)
    cfg = flowmoe.MoEConfig(hidden=c["H"], n_experts=c["E"], top_k=c["k"], ffn=c["F"], shared_ffn=c["FS"],
                            e_begin=eb, e_local=el)
    layer = flowmoe.MoELayer.from_q4_1(cfg, c["gate"][eb:eb + el], c["up"][eb:eb + el], c["down"][eb:eb + el],
                                       c["Wr"], shared=c["shared"], device=dev, router_bias=c.get("bias"))
    return DeviceStages(layer, max_tokens=c["T"])


def _want(c, lo, hi):
    xm = c["x"][lo:hi]
    _, idx, w = OM.router_block(xm, c["Wr"], c["k"], c.get("bias"))
    return OM.moe_block_f64(xm, c["res"][lo:hi], idx, w, c["gate"], c["up"], c["down"], shared=c["shared"])


def _rel(got, ref, res):
    return float(np.abs(got - ref).max() / max(np.abs(ref - res).max(), 1e-30))


def _emulated(c, world, shards, dev):
    stages = [_rank_layer(c, r, world, dev) for r in range(world)]
    E, k, H = c["E"], c["k"], c["H"]
    El = E // world
    st1 = []
    for r, (lo, hi) in enumerate(shards):
        x = torch.from_numpy(c["x"][lo:hi]).reshape(hi - lo, H).to(dev).to(torch.bfloat16).contiguous()
        st1.append(stages[r].dispatch(x, hi - lo))
    counts = [s[1].cpu().numpy().astype(np.int64) for s in st1]
    # dispatch exchange: rank d receives, from each source s in order, s's rows for d's experts
    send_off = [np.concatenate([[0], np.cumsum(cn.reshape(world, El).sum(1))]) for cn in counts]
    outs = []
    yrecvs, recv_splits = [], []
    for d in range(world):
        parts = [st1[s][0][send_off[s][d]:send_off[s][d + 1]] for s in range(world)]
        xrecv = torch.cat(parts + [torch.zeros(1, H, dtype=torch.bfloat16, device=dev)]).contiguous()
        R = xrecv.shape[0] - 1
        rc = torch.from_numpy(np.concatenate([cn[d * El:(d + 1) * El] for cn in counts]).astype(np.int32)).to(dev)
        lo, hi = shards[d]
        _, _, _, _, _, sg, xb = st1[d]
        res = torch.from_numpy(c["res"][lo:hi]).reshape(hi - lo, H).to(dev).contiguous()
        out, yrecv = stages[d].experts(xrecv, R, rc, world, xb, sg, res, hi - lo, hi - lo)
        outs.append(out)
        yrecvs.append(yrecv[:R].clone())
        recv_splits.append([int(p.shape[0]) for p in parts])
    # combine exchange: source s gets back, from each expert rank d in order, its rows
    for s, (lo, hi) in enumerate(shards):
        parts = []
        for d in range(world):
            off = sum(recv_splits[d][:s])
            parts.append(yrecvs[d][off:off + recv_splits[d][s]])
        ysorted = torch.cat(parts + [torch.zeros(1, H, dtype=torch.bfloat16, device=dev)]).contiguous()
        _, _, pos, idx, w, _, _ = st1[s]
        stages[s].combine(outs[s], ysorted, pos, idx, w, hi - lo, hi - lo)
    torch.cuda.synchronize()
    for s in stages:
        s.check()
    return [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("world", [1, 2, 4])
def test_ep_stages_emulated_ranks(dev, world):
    c = cases.make_case(H=256, E=16, F=128, FS=128, k=4, T=96, seed=40 + world)
    n = c["T"] // world
    shards = [(r * n, (r + 1) * n) for r in range(world)]
    outs = _emulated(c, world, shards, dev)
    for (lo, hi), got in zip(shards, outs):
        assert _rel(got, _want(c, lo, hi), c["res"][lo:hi]) < TOL


def test_ep_stages_uneven_and_empty_rank(dev):
    c = cases.make_case(H=256, E=16, F=128, FS=128, k=4, T=70, seed=77)
    shards = [(0, 50), (50, 70), (70, 70), (70, 70)]
    outs = _emulated(c, 4, shards, dev)
    for (lo, hi), got in zip(shards, outs):
        if hi > lo:
            assert _rel(got, _want(c, lo, hi), c["res"][lo:hi]) < TOL


def test_ep_stages_skewed_c36_shape(dev):
    # the C36 geometry (H 2048, 256 experts, F 512 + shared 512) with a Zipf-skewed router, 2 ranks
    c = cases.make_case(H=2048, E=256, F=512, FS=512, k=8, T=128, seed=9, zipf=1.1)
    shards = [(0, 64), (64, 128)]
    outs = _emulated(c, 2, shards, dev)
    for (lo, hi), got in zip(shards, outs):
        assert _rel(got, _want(c, lo, hi), c["res"][lo:hi]) < TOL


# ---- two processes, NCCL

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path[:0] = [str(ROOT), str(ROOT / "openflowlm-next_b200")]
    result = {"rank": rank}
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=dev)
        from flowmoe.ep import EPMoELayer
        c = cases.make_case(H=512, E=32, F=256, FS=256, k=8, T=192, seed=123)
        st = _rank_layer(c, rank, world, dev)
        layer = EPMoELayer(st.layer, max_tokens=c["T"])
        n = c["T"] // world
        lo, hi = rank * n, (rank + 1) * n
        x = torch.from_numpy(c["x"][lo:hi]).to(dev).to(torch.bfloat16).contiguous()
        res = torch.from_numpy(c["res"][lo:hi]).to(dev).contiguous()
        errs = []
        for _ in range(2):         # twice: the second call reuses every buffer
            out = layer(x, res)
            layer.stages.check()
            errs.append(_rel(out.cpu().numpy(), _want(c, lo, hi), c["res"][lo:hi]))
        result.update(ok=True, errs=errs)
    except Exception as e:
        result.update(ok=False, error=f"{type(e).__name__}: {e}", tb=traceback.format_exc()[-3000:])
    finally:
        Path(outdir, f"rank{rank}.json").write_text(json.dumps(result))
        if dist.is_initialized():
            dist.destroy_process_group()


def test_ep_nccl_two_ranks(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_nccl_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + 240
    while not ctx.join(timeout=1):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("NCCL ranks did not finish within 240 s")
    for r in range(2):
        res = json.loads(Path(tmp_path, f"rank{r}.json").read_text())
        assert res["ok"], res.get("tb")
        assert max(res["errs"]) < TOL, res


def test_ep_counts_that_do_not_add_up_are_rejected(dev):
    # the plan kernel checks the received counts against R and computes nothing when they disagree
    from flowmoe._lib import FlowMoeError
    c = cases.make_case(H=256, E=16, F=128, FS=128, k=4, T=32, seed=5)
    st = _rank_layer(c, 0, 2, dev)
    H, R = c["H"], 40
    xrecv = torch.zeros(R + 1, H, dtype=torch.bfloat16, device=dev)
    rc = torch.full((16,), 3, dtype=torch.int32, device=dev)       # 48 rows claimed, 40 sent
    x = torch.from_numpy(c["x"]).to(dev).to(torch.bfloat16)
    res = torch.from_numpy(c["res"]).to(dev)
    sg = torch.zeros(c["T"], device=dev)
    st.experts(xrecv, R, rc, 2, x, sg, res, c["T"], c["T"])
    with pytest.raises(FlowMoeError, match="do not add up"):
        st.check()


# ---- peer-memory expert parallel (fm_ep_peer_layer), two processes

def _peer_worker(rank, world, port, outdir, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path[:0] = [str(ROOT), str(ROOT / "openflowlm-next_b200")]
    result = {"rank": rank}
    import torch.distributed as dist
    layer = None
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from flowmoe.ep import PeerEPMoELayer
        c = cases.make_case(H=512, E=32, F=256, FS=256, k=8, T=192, seed=321)
        st = _rank_layer(c, rank, world, dev)
        layer = PeerEPMoELayer(st.layer, t_cap=c["T"], timeout_ms=1000 if mode == "absent" else 5000)
        n = c["T"] // world
        shards = [(0, 120), (120, 192)] if mode == "uneven" else [(i * n, (i + 1) * n) for i in range(world)]
        lo, hi = shards[rank]
        x = torch.from_numpy(c["x"][lo:hi]).reshape(hi - lo, c["H"]).to(dev).to(torch.bfloat16).contiguous()
        res = torch.from_numpy(c["res"][lo:hi]).reshape(hi - lo, c["H"]).to(dev).contiguous()
        if mode == "absent":
            # rank 1 maps the buffers, then skips the layer call: rank 0's waits must run out
            if rank == 0:
                layer(x, res)
                try:
                    layer.check()
                    result.update(ok=False, error="no timeout reported")
                except Exception as e:
                    result.update(ok=True, error=str(e))
            else:
                result.update(ok=True)
            dist.barrier()
        else:
            errs = []
            for _ in range(3):     # the epochs advance; every buffer is reused
                out = layer(x, res)
                layer.check()
                errs.append(_rel(out.cpu().numpy(), _want(c, lo, hi), c["res"][lo:hi]))
            result.update(ok=True, errs=errs)
    except Exception as e:
        result.update(ok=False, error=f"{type(e).__name__}: {e}", tb=traceback.format_exc()[-3000:])
    finally:
        Path(outdir, f"rank{rank}.json").write_text(json.dumps(result))
        try:
            if layer is not None:
                layer.close()
        finally:
            if dist.is_initialized():
                dist.destroy_process_group()


def _run_peer(mode, tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_peer_worker, args=(2, _free_port(), str(tmp_path), mode), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + 240
    while not ctx.join(timeout=1):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("peer ranks did not finish within 240 s")
    return [json.loads(Path(tmp_path, f"rank{r}.json").read_text()) for r in range(2)]


@pytest.mark.parametrize("mode", ["even", "uneven"])
def test_ep_peer_two_ranks(tmp_path, mode):
    for r in _run_peer(mode, tmp_path):
        assert r["ok"], r.get("tb")
        assert max(r["errs"]) < TOL, r


def test_ep_peer_absent_rank_times_out(tmp_path):
    res = _run_peer("absent", tmp_path)
    assert res[0]["ok"], res[0]
    assert "FM_ETIMEOUT" in res[0]["error"], res[0]


def _stack_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path[:0] = [str(ROOT), str(ROOT / "openflowlm-next_b200")]
    result = {"rank": rank}
    import torch.distributed as dist
    stack = None
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from flowmoe.stack import EPMoEStack
        rng = np.random.default_rng(77)
        cs, layers, nws = [], [], []
        for l in range(3):
            c = cases.make_case(H=512, E=32, F=256, FS=256, k=8, T=64, seed=400 + l)
            c["norm_w"] = OM.bf16_round((1.0 + rng.normal(0, 0.01, c["H"])).astype(np.float32))
            cs.append(c)
            layers.append(_rank_layer(c, rank, world, dev).layer)
            nws.append(torch.from_numpy(c["norm_w"]))
        n = 64 // world
        lo, hi = rank * n, (rank + 1) * n
        x0 = cs[0]["res"][lo:hi]
        # the oracle with this path's rounding point: routed y rows cross between ranks as bf16. Against
        # the f32-y oracle one of rank 1's tokens sits 4e-6 from a top-k tie in the third layer and flips
        # (tests/test_oracle.py::test_ep_stack_case_flips_only_through_bf16_y).
        want = OM.moe_stack_f64(x0, cs, y_bf16=True)
        stack = EPMoEStack(layers, nws, t_cap=n, timeout_ms=5000)
        x = torch.from_numpy(x0).to(dev).contiguous()
        errs = []
        got = stack.forward(x)
        stack.check()
        errs.append(float(np.abs(got.cpu().numpy() - want).max() / np.abs(want - x0).max()))
        stack.capture(n)
        for _ in range(2):       # graph replays: the epochs keep advancing on the device
            got = stack.forward(x)
            stack.check()
            errs.append(float(np.abs(got.cpu().numpy() - want).max() / np.abs(want - x0).max()))
        result.update(ok=True, errs=errs)
    except Exception as e:
        result.update(ok=False, error=f"{type(e).__name__}: {e}", tb=traceback.format_exc()[-3000:])
    finally:
        Path(outdir, f"rank{rank}.json").write_text(json.dumps(result))
        try:
            if stack is not None:
                stack.close()
        finally:
            if dist.is_initialized():
                dist.destroy_process_group()


def test_ep_stack_two_ranks_matches_oracle(tmp_path):
    """BASELINE config 5's form, small: three layers of x + MoE(RMSNorm(x)) across two ranks over peer
    memory (one shared peer group), eager and then as a replayed CUDA graph, against the fp64 oracle stack
    (with the expert-parallel bf16 y rows) on each rank's tokens."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_stack_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + 240
    while not ctx.join(timeout=1):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("stack ranks did not finish within 240 s")
    for r in range(2):
        res = json.loads(Path(tmp_path, f"rank{r}.json").read_text())
        assert res["ok"], res.get("tb")
        assert max(res["errs"]) < TOL, res
