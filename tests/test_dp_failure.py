"""Failure handling of data-parallel ranks, on CPU (gloo ranks, no GPU).

The failures are made on the host: a rank whose step raises, a rank that
leaves between steps, a rank that stalls after a collective, and injected
communicator set-up failures (TG_FAULT). Each surviving rank must settle its
next step as {"kind": "failed"} with an NcclError naming the cause, instead
of waiting forever: the reference rejects every pending request when its
worker dies (src/worker-proxy.ts:39-44) and maps every failure to 'failed'
(src/compile.ts:1198-1208).
"""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tensorgrad_b200 import backend as BK
from tensorgrad_b200.dist import RankGroup

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _step_body(rank, step, scenario):
    """One 'training step': a local computation and a gloo allreduce."""
    def run():
        if scenario == "raise" and rank == 1 and step == 2:
            raise RuntimeError("injected compute failure on rank 1")
        t = torch.full((16,), float(rank + step))
        dist.all_reduce(t)
        if scenario == "stall" and rank == 1 and step == 1:
            time.sleep(3.0)   # finished the collective, then stalls before reporting the step done
        return {"kind": "completed", "loss": float(t[0])}
    return run


def _rank(rank, port, scenario, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=4))
    results = []
    try:
        g = RankGroup(rank, WORLD, timeout_s=1.0, prefix=f"tg-{scenario}")
        for step in (1, 2, 3):
            if scenario == "leave" and rank == 1 and step == 2:
                g.leave()
                break
            t0 = time.monotonic()
            r = g.step(_step_body(rank, step, scenario))
            err = r.get("error")
            results.append((step, r["kind"], getattr(err, "name", type(err).__name__ if err else ""),
                            str(err) if err else "", time.monotonic() - t0))
            if r["kind"] == "failed":
                break
    finally:
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array(results, dtype=object), allow_pickle=True)
        if scenario == "stall" and rank == 0:
            time.sleep(4.0)   # rank 0 hosts the store: keep it up until the stalled rank has settled
        dist.destroy_process_group()


def _run(tmp_path, scenario):
    mp.spawn(_rank, args=(_free_port(), scenario, str(tmp_path)), nprocs=WORLD, join=True)
    return [list(np.load(str(tmp_path / f"r{r}.npy"), allow_pickle=True)) for r in range(WORLD)]


def test_peer_failure_fails_the_survivors_step(tmp_path):
    r0, r1 = _run(tmp_path, "raise")
    assert [x[1] for x in r0] == ["completed", "failed"] and [x[1] for x in r1] == ["completed", "failed"]
    step, kind, name, msg, _ = r0[1]
    assert name == "NcclError" and "peer rank 1 failed" in msg and "injected compute failure" in msg
    assert "injected compute failure" in r1[1][3]


def test_departed_peer_fails_the_next_step_before_any_collective(tmp_path):
    r0, r1 = _run(tmp_path, "leave")
    assert [x[1] for x in r1] == ["completed"]
    step, kind, name, msg, secs = r0[1]
    assert (step, kind, name) == (2, "failed", "NcclError") and "peer rank 1 left" in msg
    assert secs < 0.9          # detected before launching, not by a collective timeout


def test_stalled_peer_times_out(tmp_path):
    r0, r1 = _run(tmp_path, "stall")
    step, kind, name, msg, secs = r0[1]
    assert (step, kind, name) == (2, "failed", "NcclError")
    assert "did not finish step 1" in msg and 0.9 < secs < 2.5
    # the stalled rank learns of it before its next step's collective
    assert r1[1][1] == "failed" and "peer rank 0 failed" in r1[1][3] and r1[1][4] < 1.0


def test_injected_communicator_failures(monkeypatch):
    """TG_FAULT fakes the failing communicator call on the host: set-up that
    reports an error, and set-up that never completes (the deadline and abort
    path). Neither touches a GPU."""
    monkeypatch.setenv("TG_FAULT", "nccl_init")
    with pytest.raises(BK.TgError) as e:
        BK.Context(0, 0, 2, bytes(128))
    assert e.value.name == "NcclError" and "injected" in str(e.value)
    monkeypatch.setenv("TG_FAULT", "nccl_init_stall")
    monkeypatch.setenv("TG_NCCL_TIMEOUT_S", "0.3")
    t0 = time.monotonic()
    with pytest.raises(BK.TgError) as e:
        BK.Context(0, 0, 2, bytes(128))
    assert e.value.name == "NcclError" and "did not complete" in str(e.value) and "aborted" in str(e.value)
    assert 0.25 < time.monotonic() - t0 < 3.0
