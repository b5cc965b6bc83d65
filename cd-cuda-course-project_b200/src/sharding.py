"""
sharding.py — how each family is split across GPUs (one process per GPU).

  reduction  contiguous shards of the input; each rank reduces its shard to
             an fp64 partial on its GPU. The partials are combined inside the
             reduction kernel itself (XrankSum: peer stores into every rank's
             exchange buffer over NVLink, kt_reduce_sum_f32_xrank), or by one
             all-reduce (combine_partials: NCCL, gloo in the CPU tests)
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


class XrankSum:
    """
    Whole-job sum of per-rank shards with the combine inside the kernel
    (kt_reduce_sum_f32_xrank): one launch per step and no collective call.

        xs = XrankSum(lib, n_shard, device)          # collective: every rank
        xs(x_shard_ptr, n_shard, out64_ptr, stream)  # every rank, every step

    Set-up allocates each rank's exchange buffer with torch's symmetric memory
    (peer mappings over NVLink; multicast objects are not requested), zeroes it
    and the workspace, and agrees on them with a barrier. `epoch` counts calls
    (identical on every rank, since all ranks call once per step).
    """

    def __init__(self, lib, n_shard: int, device, group=None):
        import os
        import torch
        import torch.distributed as dist
        import kt_lib

        self.lib = lib
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if self.world > kt_lib.KT_XRANK_MAX:
            raise ValueError(f"XrankSum supports up to {kt_lib.KT_XRANK_MAX} ranks, not {self.world}")
        self.ws_bytes = max(lib.reduce_workspace_bytes(n_shard), 16)
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=device)  # ticket starts at zero
        self.ptrs: list[int] = []
        self._buf = self._hdl = None
        if self.world > 1:
            os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
            import torch.distributed._symmetric_memory as symm_mem
            g = group if group is not None else dist.group.WORLD
            self._buf = symm_mem.empty(kt_lib.KT_XRANK_EXCHANGE_BYTES, dtype=torch.uint8, device=device)
            self._buf.zero_()
            self._hdl = symm_mem.rendezvous(self._buf, g)
            self.ptrs = [int(p) for p in self._hdl.buffer_ptrs]
            if len(self.ptrs) != self.world or self.ptrs[self.rank] != self._buf.data_ptr():
                raise RuntimeError("symmetric-memory rendezvous returned an unexpected buffer table")
            torch.cuda.synchronize(device)
            dist.barrier(group=g, device_ids=[device.index])
        self.epoch = 0

    def __call__(self, x: int, n: int, out64: int, stream, out32: Optional[int] = None) -> None:
        self.epoch += 1
        self.lib.reduce_sum_f32_xrank(x, n, out64, out32, self.ws.data_ptr(), self.ws_bytes, self.ptrs,
                                      self.rank, self.world, self.epoch, stream)


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
