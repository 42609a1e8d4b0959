"""Data-parallel rank group: communicator set-up and host-side failure detection.

One process per GPU. The ranks share a torch.distributed process group (gloo,
host only) for the NCCL unique id and a key-value store; the gradient
allreduce itself runs inside each rank's training step over NCCL
(tensorgrad_b200/csrc/runtime_exec.cu).

Failure handling follows the reference's contract: every failure of a
request settles as ``{"kind": "failed", "error": ...}`` (src/compile.ts:1198-1208,
``guarded``), and when the worker dies every pending request is rejected
rather than left waiting (src/worker-proxy.ts:39-44). Across ranks that means
a rank whose peer failed or left must fail its next step, not hang in a
collective:

* a rank whose step raises records the error in the store (``abort``) before
  re-raising; a rank that leaves cleanly records ``left/<rank>``;
* before each step a rank checks those keys and waits (up to ``timeout_s``)
  for every peer to have finished the previous step; a recorded failure, a
  departure or a peer that stays behind fails the step with ``NcclError``
  before any collective is launched;
* a peer that dies inside a step is caught on the device side: the step's
  completion wait polls the communicator against ``TG_NCCL_TIMEOUT_S`` and
  aborts it (``Context.sync``).
"""
from __future__ import annotations

import time
from typing import Callable, Optional

from . import backend as BK


class RankGroup:
    """Host-side coordination of one data-parallel rank.

    ``store`` is any torch.distributed Store (the default process group's
    store when None)."""

    def __init__(self, rank: int, world: int, store=None, timeout_s: float = 300.0, prefix: str = "tg"):
        import torch.distributed as dist
        self.rank, self.world = rank, world
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.timeout_s = timeout_s
        self.prefix = prefix
        self.steps_done = 0

    def _key(self, *parts) -> str:
        return "/".join((self.prefix,) + tuple(str(p) for p in parts))

    def _get(self, key: str) -> Optional[str]:
        if self.store.check([key]):
            return self.store.get(key).decode()
        return None

    def _peer_failure(self) -> Optional[str]:
        msg = self._get(self._key("abort"))
        if msg is not None:
            return msg
        for r in range(self.world):
            if r != self.rank and self._get(self._key("left", r)) is not None:
                return f"peer rank {r} left the group"
        return None

    def before_step(self) -> None:
        """Fails with NcclError if a peer failed or left, or has not finished
        the previous step within the timeout."""
        t0 = time.monotonic()
        while True:
            why = self._peer_failure()
            if why is not None:
                raise BK.TgError("NcclError", f"step {self.steps_done + 1} not started: {why}")
            behind = [r for r in range(self.world) if r != self.rank and
                      int(self._get(self._key("done", r)) or 0) < self.steps_done]
            if not behind:
                return
            if time.monotonic() - t0 > self.timeout_s:
                raise BK.TgError("NcclError", f"step {self.steps_done + 1} not started: peer ranks {behind} did not "
                                              f"finish step {self.steps_done} within {self.timeout_s} s")
            time.sleep(0.002)

    def after_step(self) -> None:
        self.steps_done += 1
        self.store.set(self._key("done", self.rank), str(self.steps_done))

    def fail(self, err: BaseException) -> None:
        """Records this rank's failure for its peers (first failure wins)."""
        key = self._key("abort")
        if not self.store.check([key]):
            self.store.set(key, f"peer rank {self.rank} failed: {type(err).__name__}: {err}")

    def leave(self) -> None:
        self.store.set(self._key("left", self.rank), "1")

    def step(self, run: Callable[[], dict]) -> dict:
        """Runs one training step (a callable returning the reference's result
        object) under the group's checks. A failure, local or a peer's,
        settles as {"kind": "failed", "error": ...}."""
        try:
            self.before_step()
        except BK.TgError as e:
            self.fail(e)  # this rank gives up: its peers fail their next step too
            return {"kind": "failed", "error": e}
        try:
            r = run()
        except Exception as e:  # noqa: BLE001 - every failure settles as 'failed'
            r = {"kind": "failed", "error": e}
        if r.get("kind") == "failed":
            # a peer's recorded failure is the cause of a collective that broke here
            why = self._peer_failure()
            self.fail(r.get("error") or RuntimeError("step failed"))
            if why is not None and not why.startswith(f"peer rank {self.rank} "):
                return {"kind": "failed", "error": BK.TgError("NcclError", f"step {self.steps_done + 1}: {why}"),
                        "cause": r.get("error")}
            return r
        self.after_step()
        return r


def init_data_parallel(device: Optional[int] = None, timeout_s: float = 300.0):
    """Inside a torch.distributed job (RANK/WORLD_SIZE/MASTER_* set, e.g. by
    torchrun): joins a gloo process group on the host, shares the NCCL unique
    id from rank 0 and creates this rank's device context. Returns
    (Context, RankGroup)."""
    import datetime
    import os

    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank))) if device is None else device
    if not dist.is_initialized():
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    obj = [BK.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    ctx = BK.Context(local, rank, world, obj[0])
    return ctx, RankGroup(rank, world, timeout_s=timeout_s)
