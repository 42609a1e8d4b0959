"""Data-parallel training step on two GPUs (NCCL allreduce inside the step).

Each rank runs the C4 model on its batch shard. After one step, the flat
gradient arena holds the NCCL sum of the rank gradients; divided by the world
size it must equal the oracle's gradients for the whole batch, and the
reported loss must be the whole-batch loss. Skipped when fewer than two GPUs
are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch

from .test_gpu_ops import close

pytestmark = pytest.mark.gpu

WORLD = 2
TINY = {"vocab": 65, "T": 16, "D": 32, "layers": 2, "heads": 2, "batch": 2, "dropout": 0.2}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, out_path):
    import torch.distributed as dist
    from tensorgrad_b200 import backend as BK
    from tensorgrad_b200 import configs as CF
    from tensorgrad_b200.compile import build_training_ir, initial_params
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        obj = [BK.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx = BK.Context(rank, rank, WORLD, obj[0])
        B = TINY["batch"]
        w = CF.workload("c4", **TINY)
        ir = build_training_ir(w.make_model(), w.loss, w.inputs(B), w.optimizer)
        init = initial_params(ir.graph, ir.materialized.initFns, CF.PARAM_SEED)
        dg = BK.DeviceGraph(ctx, ir.program)
        dg.upload_params(init)
        data = CF.shard(w.data(B * WORLD), rank, WORLD)
        loss, _ = dg.step(data)
        if rank == 0:
            shapes = {n: tuple(t.shape) for n, t in ir.paramGrads.items()}
            grads = {n: dg.read_grad(n, s) for n, s in shapes.items()}
            np.savez(out_path, loss=np.array([loss]), **{f"g_{n}": g for n, g in grads.items()})
        dg.destroy()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bucket_mb", [None, "0.02"])
def test_two_gpu_step_matches_whole_batch(tmp_path, bucket_mb, monkeypatch):
    """bucket_mb "0.02" splits the gradient allreduce into many buckets that
    run on the communication stream during the backward pass."""
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    if bucket_mb:
        monkeypatch.setenv("TG_DP_BUCKET_MB", bucket_mb)
    import torch.multiprocessing as mp
    from oracle.driver import OracleTrainer
    from tensorgrad_b200 import configs as CF
    from tensorgrad_b200.compile import build_training_ir, initial_params

    out = str(tmp_path / "dp.npz")
    mp.spawn(_rank, args=(_free_port(), out), nprocs=WORLD, join=True)
    r = np.load(out)
    B = TINY["batch"] * WORLD
    w = CF.workload("c4", **{**TINY, "batch": B})
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(B), w.optimizer)
    init = initial_params(ir.graph, ir.materialized.initFns, CF.PARAM_SEED)
    orc = OracleTrainer(ir.program, init)
    ref_loss = orc.step(w.data(B))
    close(r["loss"], np.array([ref_loss]))
    for n, g in orc.grads().items():
        # the arena holds the sum over ranks of each rank's mean gradient
        close(r[f"g_{n}"] / WORLD, np.asarray(g).reshape(r[f"g_{n}"].shape), tensor_frac=1.0)


_FAULT_RANK = r"""
import os, sys, time
sys.path.insert(0, sys.argv[1])
rank, port, fault, log = int(sys.argv[2]), sys.argv[3], sys.argv[4], sys.argv[5]
os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=port, TG_FAULT=fault, TG_NCCL_TIMEOUT_S="2",
                  NCCL_NVLS_ENABLE="0")
def say(m):
    with open(log, "a") as f:
        f.write(f"{rank} {time.monotonic():.3f} {m}\n")
import torch.distributed as dist
from tensorgrad_b200 import backend as BK
from tensorgrad_b200 import configs as CF
from tensorgrad_b200.compile import build_training_ir, initial_params
dist.init_process_group("gloo", rank=rank, world_size=2)
obj = [BK.nccl_unique_id() if rank == 0 else None]
dist.broadcast_object_list(obj, src=0)
ctx = BK.Context(rank, rank, 2, obj[0])
say("context")
w = CF.workload("c4", vocab=65, T=16, D=32, layers=2, heads=2, batch=2, dropout=0.2)
ir = build_training_ir(w.make_model(), w.loss, w.inputs(2), w.optimizer)
dg = BK.DeviceGraph(ctx, ir.program)
dg.upload_params(initial_params(ir.graph, ir.materialized.initFns, CF.PARAM_SEED))
data = CF.shard(w.data(4), rank, 2)
for step in (1, 2, 3):
    try:
        dg.step(data)
        say(f"step{step} ok")
    except BK.TgError as e:
        say(f"step{step} {e.name}: {e.message}")
dg.destroy()
say("destroyed graph")
ctx.close()
say("closed context")
dist.destroy_process_group()
say("done")
"""


@pytest.mark.parametrize("fault", ["step_error:2", "step_stall:2"])
def test_two_gpu_collective_failure_aborts_the_communicator(tmp_path, fault):
    """The completion wait of a data-parallel step fails with NcclError when
    the communicator reports an error or the step does not complete within
    TG_NCCL_TIMEOUT_S; the communicator is aborted and every later step fails
    at once. The failures are injected on the host (TG_FAULT fakes the result
    of the completion check); the collectives themselves complete on both
    GPUs, so no device is left waiting. NVLS is off, and the two rank
    processes run under a time limit, so a fault in the host-side handling
    ends the test instead of holding the GPUs."""
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "rank.py"
    script.write_text(_FAULT_RANK)
    log = tmp_path / "log.txt"
    port = str(_free_port())
    procs = [subprocess.Popen(["timeout", "-s", "KILL", "120", sys.executable, str(script), root, str(r), port, fault,
                               str(log)]) for r in range(WORLD)]
    codes = [p.wait() for p in procs]
    text = log.read_text() if log.exists() else ""
    assert codes == [0, 0], f"rank exit codes {codes}; log:\n{text}"
    for r in range(WORLD):
        lines = [ln.split(" ", 2)[2] for ln in text.splitlines() if ln.startswith(f"{r} ")]
        assert lines[1] == "step1 ok", text
        assert lines[2].startswith("step2 NcclError") and "aborted" in lines[2], text
        assert lines[3].startswith("step3 NcclError") and "earlier collective failure" in lines[3], text
        assert lines[-1] == "done", text
