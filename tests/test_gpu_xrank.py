"""
The whole-job sum with the combine inside the kernel (kt_reduce_sum_f32_xrank)
through the C ABI on GPUs.

  * one rank: same sum as kt_reduce_sum_f32 and the oracle, on repeated calls
    that reuse one workspace without any reset between them;
  * a rank that never arrives: the bounded wait (2 s) runs out, the result is
    NaN and the device error word says 3, and the context stays usable (the
    failure is made by an exchange slot that nothing writes, not by a fault);
  * two ranks on two GPUs (torchrun, NCCL only for the set-up barrier):
    every rank gets the oracle's whole sum, bit-identical across ranks, over
    several sizes and epochs. Skipped with fewer than two GPUs.
"""

from __future__ import annotations

import math
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import kt_ops  # noqa: E402
import sharding  # noqa: E402
import workloads  # noqa: E402
from oracle import ref  # noqa: E402

HERE = Path(__file__).resolve().parent


def test_xrank_single_rank_matches_local(dev, lib):
    xs_by_n = {}
    for n in ((1 << 22) + 3, 1_000_001, 5, 0):
        x = workloads.make_inputs("reduction", d={"n": n}, seed=n + 1)["x"]
        xs_by_n[n] = (x, torch.from_numpy(x).to(dev))
    xsum = sharding.XrankSum(lib, 1 << 23, dev)
    stream = torch.cuda.current_stream().cuda_stream
    for rep in range(2):
        for n, (x, xd) in xs_by_n.items():
            out = torch.full((1,), float("nan"), dtype=torch.float64, device=dev)
            xsum(xd.data_ptr() if n else 0, n, out.data_ptr(), stream)
            torch.cuda.synchronize()
            got = out.item()
            want = ref.reduce_sum_ref(x)
            assert abs(got - want) <= 1e-4 * abs(want) + 1e-12, (rep, n, got, want)
            if n:
                assert got == kt_ops.reduce_sum(xd, lib=lib).item()  # same kernel body and grid
    assert xsum.epoch == 8
    assert lib.device_error() == 0


def test_xrank_missing_rank_times_out_cleanly(dev, lib):
    import kt_lib
    n = 1 << 20
    xd = torch.ones(n, device=dev)
    ws_bytes = lib.reduce_workspace_bytes(n)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    own = torch.zeros(kt_lib.KT_XRANK_EXCHANGE_BYTES, dtype=torch.uint8, device=dev)
    other = torch.zeros(kt_lib.KT_XRANK_EXCHANGE_BYTES, dtype=torch.uint8, device=dev)
    out = torch.zeros(1, dtype=torch.float64, device=dev)
    assert lib.device_error(reset=True) == 0
    # rank 0 of 2: rank 1's slot in `own` is never written, so the wait gives up
    lib.reduce_sum_f32_xrank(xd.data_ptr(), n, out.data_ptr(), None, ws.data_ptr(), ws_bytes,
                             [own.data_ptr(), other.data_ptr()], 0, 2, 1, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert math.isnan(out.item())
    assert lib.device_error(reset=True) == 3
    # the context is still usable and the workspace ticket was left at zero
    xsum = sharding.XrankSum(lib, n, dev)
    xsum(xd.data_ptr(), n, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    lib.reduce_sum_f32(xd.data_ptr(), n, out.data_ptr(), None, ws.data_ptr(), ws_bytes)
    torch.cuda.synchronize()
    assert out.item() == float(n)
    assert lib.device_error() == 0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_xrank_two_ranks_match_oracle(tmp_path):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531", str(HERE / "xrank_ranks.py"),
           str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    lines = sorted((tmp_path).glob("rank*.txt"))
    assert len(lines) == 2
    sums = [p.read_text().split() for p in lines]
    assert sums[0] == sums[1]  # identical bits on both ranks, every case
