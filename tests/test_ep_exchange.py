"""Expert-parallel exchange logic on CPU: gloo ranks (world size 2 and 4), the device stages replaced by
oracle-backed stand-ins, results against the one-device oracle (``oracle.moe.moe_block_f64``).

Faults are made on the host only: a rank whose stage raises before the exchange, a rank that reports
counts that do not add up, a rank that never joins. The others must end with an error within the
process group's timeout instead of waiting for good.
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
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bf16_tensor(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16)


class OracleStages:
    """Steps 1, 3 and 5 of the expert-parallel layer in numpy (fp64 products, the device's bf16
    rounding points: x and h rounded, y returned as bf16 rows)."""

    def __init__(self, case, rank, world, fault=None):
        from oracle.q4_1 import dequant_q4_1
        self.c = case
        self.n_experts, self.top_k, self.hidden = case["E"], case["k"], case["H"]
        self.max_tokens = 64
        self.El = case["E"] // world
        self.eb = rank * self.El
        self.fault = fault
        self.wg = [dequant_q4_1(case["gate"][e]) for e in range(self.eb, self.eb + self.El)]
        self.wu = [dequant_q4_1(case["up"][e]) for e in range(self.eb, self.eb + self.El)]
        self.wd = [dequant_q4_1(case["down"][e]) for e in range(self.eb, self.eb + self.El)]
        sg, su, sd, self.sgw = case["shared"]
        self.shared = (dequant_q4_1(sg), dequant_q4_1(su), dequant_q4_1(sd))

    def rows(self, n):
        return torch.zeros(n, self.hidden, dtype=torch.bfloat16)

    def dispatch(self, x, t_real):
        from oracle import moe
        if self.fault == "raise_in_dispatch":
            raise RuntimeError("injected: dispatch failed on this rank")
        xm = x.float().numpy()
        T, k, E = xm.shape[0], self.top_k, self.n_experts
        idx = np.zeros((T, k), np.int32)
        w = np.zeros((T, k), np.float64)
        if T:
            _, idx, w = moe.router_block(moe.bf16_round(xm), self.c["Wr"], k)
        counts, offsets, pos, pair = moe.dispatch(idx, E, t_real)
        if self.fault == "bad_counts":
            counts = counts.copy()
            counts[0] += 1
        xsend = torch.zeros(T * k + 1, self.hidden, dtype=torch.bfloat16)
        if pair.size:
            xsend[:pair.size] = x[torch.from_numpy(pair // k).long()]
        sg = moe.shared_gate(xm, self.sgw) if T else np.zeros(0)
        return (xsend, torch.from_numpy(counts), torch.from_numpy(pos), torch.from_numpy(idx),
                torch.from_numpy(w), torch.from_numpy(sg), x)

    def experts(self, xrecv, R, recv_counts, G, xb, sg, res, T, t_real):
        from oracle import moe
        rc = recv_counts.numpy().reshape(G, self.El)
        xr = xrecv[:R].float().numpy()
        yrecv = torch.zeros(R + 1, self.hidden, dtype=torch.bfloat16)
        r = 0
        for s in range(G):
            for j in range(self.El):
                n = int(rc[s, j])
                if n:
                    y = moe.expert_ffn_f64(xr[r:r + n], self.wg[j], self.wu[j], self.wd[j])
                    yrecv[r:r + n] = _bf16_tensor(y.astype(np.float32))
                r += n
        assert r == R
        out = res.double().clone()
        if t_real:
            xs = xb[:t_real].float().numpy()
            sh = moe.expert_ffn_f64(xs, *self.shared)
            out[:t_real] += torch.from_numpy(sg.numpy()[:t_real, None] * sh)
        return out, yrecv

    def combine(self, out, ysorted, pos, idx, w, T, t_real):
        y = ysorted.double()
        for t in range(t_real):
            for s in np.argsort(idx[t].numpy(), kind="stable"):
                out[t] += float(w[t, s]) * y[int(pos[t, s])]


def _case(world, seed=3):
    from oracle.cases import make_case
    return make_case(H=128, E=4 * world, F=64, FS=64, k=2, T=24, seed=seed)


def _shards(T, world, uneven):
    if uneven:   # rank 0 gets most, the last rank none
        cuts = [0] + [min(T, (i + 1) * (T // world + 3)) for i in range(world - 1)] + [T]
        cuts[-2] = T
        return [(cuts[i], cuts[i + 1]) for i in range(world)]
    n = T // world
    return [(i * n, (i + 1) * n) for i in range(world)]


def _worker(rank, world, port, outdir, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path[:0] = [str(ROOT), str(ROOT / "openflowlm-next_b200")]
    result = {"rank": rank}
    t0 = time.monotonic()
    try:
        from flowmoe.ep import ep_forward
        from oracle import moe
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        case = _case(world)
        fault = None
        if mode == "raise" and rank == 1:
            fault = "raise_in_dispatch"
        if mode == "bad_counts" and rank == 1:
            fault = "bad_counts"
        if mode == "absent" and rank == 1:
            result["skipped"] = True      # joins the group, then never takes the exchange's steps
            time.sleep(8)
            return
        lo, hi = _shards(case["T"], world, mode == "uneven")[rank]
        x = _bf16_tensor(case["x"][lo:hi]).reshape(hi - lo, case["H"])
        res = torch.from_numpy(case["res"][lo:hi]).reshape(hi - lo, case["H"])
        stages = OracleStages(case, rank, world, fault)
        out = ep_forward(stages, x, res)
        xm = case["x"][lo:hi]
        if hi > lo:
            _, idx, w = moe.router_block(moe.bf16_round(xm), case["Wr"], case["k"])
            want = moe.moe_block_f64(xm, case["res"][lo:hi], idx, w, case["gate"], case["up"], case["down"],
                                     shared=case["shared"])
            err = float(np.abs(out.numpy() - want).max() / max(np.abs(want - case["res"][lo:hi]).max(), 1e-30))
        else:
            err = 0.0
        result.update(ok=True, err=err, rows=hi - lo)
    except Exception as e:   # reported to the parent, which checks who failed and how fast
        result.update(ok=False, error=f"{type(e).__name__}: {e}", tb=traceback.format_exc()[-2000:])
    finally:
        result["seconds"] = time.monotonic() - t0
        Path(outdir, f"rank{rank}.json").write_text(json.dumps(result))
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world, mode, tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_worker, args=(world, port, str(tmp_path), mode), nprocs=world, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + 120
    while not ctx.join(timeout=1):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail(f"ranks did not finish within 120 s (mode {mode})")
    return [json.loads(Path(tmp_path, f"rank{r}.json").read_text()) for r in range(world)]


@pytest.mark.parametrize("world,mode", [(2, "even"), (2, "uneven"), (4, "even"), (4, "uneven")])
def test_ep_exchange_matches_one_device(world, mode, tmp_path):
    res = _run(world, mode, tmp_path)
    for r in res:
        assert r["ok"], r.get("tb")
        assert r["err"] < 5e-3, r       # only the bf16 rounding of the returned y rows differs
    if mode == "uneven":
        assert res[-1]["rows"] == 0


def test_ep_rank_failure_ends_peers_with_error(tmp_path):
    res = _run(2, "raise", tmp_path)
    assert not res[1]["ok"] and "injected" in res[1]["error"]
    assert not res[0]["ok"], "the surviving rank must fail, not hang or succeed"
    assert res[0]["seconds"] < 60


def test_ep_inconsistent_counts_detected(tmp_path):
    res = _run(2, "bad_counts", tmp_path)
    assert not res[1]["ok"] and "ExchangeError" in res[1]["error"]
    assert not res[0]["ok"]
    assert res[0]["seconds"] < 60


def test_ep_absent_rank_times_out(tmp_path):
    res = _run(2, "absent", tmp_path)
    assert res[1].get("skipped")
    assert not res[0]["ok"]
    assert res[0]["seconds"] < 60


def test_expert_range():
    sys.path[:0] = [str(ROOT / "openflowlm-next_b200")]
    from flowmoe.ep import expert_range
    assert expert_range(256, 3, 8) == (96, 32)
    with pytest.raises(ValueError):
        expert_range(10, 0, 4)
