"""
One rank of the two-GPU check of kt_reduce_sum_f32_xrank (launched by
tests/test_gpu_xrank.py under torchrun). Every rank generates its own shard of
seeded inputs, runs several calls (epochs) per size and checks the whole sum
against the oracle computed from every shard; it writes the sums it got (as
hex bit patterns) to <outdir>/rank<r>.txt so the test can compare ranks.
"""

from __future__ import annotations

import math
import sys
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "cd-cuda-course-project_b200", REPO / "cd-cuda-course-project_b200" / "src"):
    sys.path.insert(0, str(p))


def main() -> int:
    import os
    import torch
    import torch.distributed as dist

    import kt_lib
    import sharding
    import workloads
    from oracle import ref

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    lib = kt_lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    got_bits = []
    try:
        for n in (4_000_037, 1 << 24, 1001):
            lo, hi = sharding.shard_range(n, world, rank)
            x = workloads.make_inputs("reduction", d={"n": n}, seed=n % 997, part=(lo, hi))["x"]
            xd = torch.from_numpy(x).to(dev)
            parts = [None] * world
            dist.all_gather_object(parts, ref.reduce_sum_ref(x))
            want = math.fsum(parts)
            xs = sharding.XrankSum(lib, hi - lo, dev)
            out = torch.zeros(1, dtype=torch.float64, device=dev)
            for _ in range(5):
                xs(xd.data_ptr(), hi - lo, out.data_ptr(), stream)
            torch.cuda.synchronize()
            got = out.item()
            if not abs(got - want) <= 1e-4 * abs(want):
                print(f"rank {rank}: n={n} got {got} want {want}", flush=True)
                return 1
            got_bits.append(float(got).hex())
        code = lib.device_error()
        if code != 0:
            print(f"rank {rank}: device error {code}", flush=True)
            return 1
        (Path(sys.argv[1]) / f"rank{rank}.txt").write_text(" ".join(got_bits))
        dist.barrier(device_ids=[rank])
        return 0
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
