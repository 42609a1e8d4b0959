"""Data-parallel decomposition on CPU ranks (gloo, world size 2).

Data parallelism here works as follows:
- each rank evaluates the training graph on its contiguous batch shard (configs.shard), with
  the dropout hash index offset by rank * numel;
- the flat gradients are allreduced (sum) and scaled by 1 / world before the optimizer;
- the reported loss is the mean of the rank losses.

These ranks run that decomposition with the oracle evaluator as the per-rank compute and
torch.distributed (gloo) as the collective. The averaged gradients and loss must equal those of
one process evaluating the whole batch: same dropout masks, same reduction. This is the host
logic the NCCL path on the GPU relies on (the GPU step itself is checked against the oracle in
test_gpu_train).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.driver import OracleTrainer
from tensorgrad_b200 import configs as CF
from tensorgrad_b200.compile import build_training_ir, initial_params

WORLD = 2
TINY = {"vocab": 17, "T": 8, "D": 16, "layers": 1, "heads": 2, "batch": 2, "dropout": 0.25}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _grads_and_loss(per_rank_batch, data, dp_rank):
    w = CF.workload("c4", **{**TINY, "batch": per_rank_batch})
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(per_rank_batch), w.optimizer)
    init = initial_params(ir.graph, ir.materialized.initFns, CF.PARAM_SEED)
    orc = OracleTrainer(ir.program, init, dp_rank=dp_rank)
    loss = orc.step(data)
    return {k: np.asarray(v, np.float64) for k, v in orc.grads().items()}, loss


def _rank(rank, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        B = TINY["batch"]
        full = CF.workload("c4", **TINY).data(B * WORLD)
        grads, loss = _grads_and_loss(B, CF.shard(full, rank, WORLD), rank)
        names = sorted(grads)
        flat = torch.from_numpy(np.concatenate([grads[n].reshape(-1) for n in names]))
        dist.all_reduce(flat, op=dist.ReduceOp.SUM)
        flat /= WORLD
        lt = torch.tensor([loss], dtype=torch.float64)
        dist.all_reduce(lt, op=dist.ReduceOp.SUM)
        lt /= WORLD
        if rank == 0:
            np.savez(out_path, flat=flat.numpy(), loss=lt.numpy(), names=np.array(names))
    finally:
        dist.destroy_process_group()


def test_dp_allreduce_matches_full_batch(tmp_path):
    out = str(tmp_path / "dp.npz")
    mp.spawn(_rank, args=(_free_port(), out), nprocs=WORLD, join=True)
    r = np.load(out)
    B = TINY["batch"]
    full = CF.workload("c4", **TINY).data(B * WORLD)
    grads, loss = _grads_and_loss(B * WORLD, full, 0)
    names = [str(n) for n in r["names"]]
    ref = np.concatenate([grads[n].reshape(-1) for n in names])
    # f32-stored intermediates on both sides: the DP and full-batch reductions
    # group the same terms differently, so agreement is to f32 rounding.
    assert np.max(np.abs(r["flat"] - ref)) <= 1e-5 * np.max(np.abs(ref))
    assert abs(float(r["loss"][0]) - loss) <= 1e-6 * abs(loss)


def test_dropout_offsets_partition_the_full_batch_masks():
    """Rank r's dropout mask over its shard is the slice [r*n, (r+1)*n) of the
    single-graph mask over the whole batch."""
    from oracle.evaluator import dropout_mask
    n = 64
    whole = dropout_mask(7, 3, 0.3, n * WORLD, 0)
    for r in range(WORLD):
        np.testing.assert_array_equal(dropout_mask(7, 3, 0.3, n, r * n), whole[r * n:(r + 1) * n])
