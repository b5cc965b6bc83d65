"""
Multi-rank host logic on CPU (gloo, world size 2): contiguous sharding with
one fp64 all-reduce reproduces the whole-array sum, and a rank that stops
between steps is detected through the store before the next launch.
No GPU is involved; the per-rank partial is the oracle's shard sum.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    for p in (str(REPO), str(REPO / "cd-cuda-course-project_b200"), str(REPO / "cd-cuda-course-project_b200" / "src")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _worker(rank, world, port, scenario, q):
    try:
        _setup_paths()
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        import sharding
        import workloads
        from oracle import ref

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=30))
        if scenario == "sum":
            x = workloads.make_inputs("reduction", d={"n": 1_000_003}, seed=5)["x"]
            lo, hi = sharding.shard_range(x.size, world, rank)
            partial = torch.tensor([ref.reduce_sum_ref(x[lo:hi])], dtype=torch.float64)
            total = sharding.combine_partials(partial)
            q.put((rank, "ok", float(total.item()), ref.reduce_sum_ref(x)))
        elif scenario == "rank_loss":
            store = dist.distributed_c10d._get_default_store()
            mon = sharding.RankMonitor(store, rank, world, timeout_s=2.0)
            for step in range(3):
                mon.beat(step)
                mon.wait_all(step)
            if rank == 1:
                q.put((rank, "left", None, None))
                q.close()
                q.join_thread()
                os._exit(0)  # leaves between steps, nothing in flight
            mon.beat(3)
            try:
                mon.wait_all(3)
                q.put((rank, "missed", None, None))
            except sharding.RankLostError as e:
                q.put((rank, "detected", e.missing, e.step))
            q.close()
            q.join_thread()
            os._exit(0)
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc(), None))


def _run(scenario, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


def test_sharded_sum_matches_whole_sum_gloo():
    out = _run("sum")
    for rank, status, total, want in out:
        assert status == "ok", total
        assert total == pytest.approx(want, rel=1e-12)


def test_rank_loss_is_detected_between_steps():
    out = _run("rank_loss")
    assert out[1][1] == "left"
    assert out[0][1] == "detected", out[0]
    assert out[0][2] == [1] and out[0][3] == 3


def test_xrank_sum_counts_epochs_on_one_rank():
    """XrankSum without a process group: one rank, no exchange table, and the
    epoch passed to the kernel entry point starts at 1 and grows by one per call."""
    import sharding

    class FakeLib:
        def __init__(self):
            self.calls = []

        def reduce_workspace_bytes(self, n):
            return 16 + 8 * 4

        def reduce_sum_f32_xrank(self, x, n, out64, out32, ws, ws_bytes, exchange, rank, world, epoch, stream):
            self.calls.append((x, n, out64, ws_bytes, list(exchange), rank, world, epoch))

    lib = FakeLib()
    xs = sharding.XrankSum(lib, 1000, "cpu")
    assert int(xs.ws.sum()) == 0 and xs.ws_bytes == 48
    xs(111, 1000, 222, None)
    xs(111, 1000, 222, None)
    assert [c[-1] for c in lib.calls] == [1, 2]
    assert all(c[4] == [] and c[5] == 0 and c[6] == 1 for c in lib.calls)
