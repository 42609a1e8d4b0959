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
