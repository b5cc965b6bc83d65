"""
sharding.py — how each family is split across GPUs (one process per GPU).

  reduction  contiguous shards of the input; each rank reduces its shard to
             an fp64 partial on its GPU and the partials are combined by one
             all-reduce (NCCL over NVLink; gloo in the CPU tests)
  softmax / layernorm   rows
  matmul     row-blocks of A (B replicated)
  attention  (batch, head) pairs

Only the reduction has an exchange step. `RankMonitor` is the host-side
failure detector: ranks publish a heartbeat per step in the process group's
store, and a rank that stops publishing is reported before the next launch
(no GPU wait is involved).
"""

from __future__ import annotations

import time
from typing import Optional


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of rank's contiguous shard of n units; shards differ in size by at most 1."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    if n < 0:
        raise ValueError("negative size")
    return rank * n // world, (rank + 1) * n // world


def combine_partials(partial, group=None):
    """Sum an fp64 partial tensor across the ranks of `group` (in place; returned)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial


def sharded_sum(x_shard, lib=None, group=None, workspace=None, out64=None):
    """Whole-job sum: this rank's shard reduced on its GPU, then combined across ranks."""
    import kt_ops
    partial = kt_ops.reduce_sum(x_shard, out64=out64, workspace=workspace, lib=lib)
    return combine_partials(partial, group)


class RankLostError(RuntimeError):
    """A rank stopped publishing heartbeats."""

    def __init__(self, missing: list[int], step: int):
        self.missing = missing
        self.step = step
        super().__init__(f"ranks {missing} did not reach step {step}")


class RankMonitor:
    """
    Store-based liveness check between steps.

        mon = RankMonitor(store, rank, world, timeout_s=2.0)
        for step in range(n):
            mon.beat(step)          # after this rank finished `step`
            mon.wait_all(step)      # before launching step + 1
    """

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, poll_s: float = 0.01,
                 prefix: str = "kt_hb"):
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = timeout_s
        self.poll_s = poll_s
        self.prefix = prefix

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank), str(step))

    def last_step(self, r: int) -> Optional[int]:
        try:
            if hasattr(self.store, "check") and not self.store.check([self._key(r)]):
                return None
            return int(self.store.get(self._key(r)).decode())
        except Exception:  # noqa: BLE001 - a missing key reads as "no beat yet"
            return None

    def wait_all(self, step: int) -> None:
        """Return when every rank reached `step`; raise RankLostError after timeout_s."""
        deadline = time.monotonic() + self.timeout_s
        while True:
            seen = [self.last_step(r) for r in range(self.world)]
            missing = [r for r, s in enumerate(seen) if s is None or s < step]
            if not missing:
                return
            if time.monotonic() >= deadline:
                raise RankLostError(missing, step)
            time.sleep(self.poll_s)
