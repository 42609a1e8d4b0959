"""Training parity through the C ABI: every benchmark workload (shrunk so the
oracle finishes in seconds) trains on the GPU from the same seeded params and
data as the CPU oracle.

* loss and every gradient after step 1: per element
  |gpu - ref| <= 1e-4 * max(|ref|, 1e-2 * max|ref|) (see test_gpu_ops);
* loss after 10 steps: 1e-4 relative;
* params after 10 steps: |gpu - ref| <= 1e-4 * max|ref| per tensor. Adam
  divides each coordinate by its own running RMS, so a coordinate whose
  gradient is near zero turns the f32-vs-f64 rounding noise of that gradient
  into an O(lr) difference in its update; the error is bounded relative to
  the tensor's scale, not the coordinate's own value.
"""
import numpy as np
import pytest

from oracle.driver import OracleTrainer
from tensorgrad_b200 import backend as BK
from tensorgrad_b200 import configs as CF
from tensorgrad_b200.compile import build_training_ir, initial_params

from .test_gpu_ops import close

pytestmark = pytest.mark.gpu

TINY = {
    "c1": {},
    "c2": {"batch": 4, "hw": 12, "c1": 4, "c2": 8, "hidden": 16},
    "c3": {"batch": 256},
    "c4": {"vocab": 65, "T": 16, "D": 32, "layers": 2, "heads": 2, "batch": 4, "dropout": 0.2},
    "c5": {"vocab": 512, "T": 32, "D": 64, "layers": 2, "heads": 2, "batch": 2, "sched_steps": 10},
}


def setup(ctx, name, steps_check=10):
    w = CF.workload(name, **TINY[name])
    B = w.global_batch
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(B), w.optimizer)
    init = initial_params(ir.graph, ir.materialized.initFns, CF.PARAM_SEED)
    dg = BK.DeviceGraph(ctx, ir.program)
    dg.upload_params(init)
    orc = OracleTrainer(ir.program, init)
    return w, ir, dg, orc, w.data(B)


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_train_parity(ctx, name):
    w, ir, dg, orc, data = setup(ctx, name)
    shapes = {n: ir.graph.tensors[t.id].shape for n, t in ir.paramGrads.items()}
    try:
        lg, _ = dg.step(data)
        lo = orc.step(data)
        close([lg], [lo])
        og = orc.grads()
        for n, shp in shapes.items():
            close(dg.read_grad(n, shp), og[n].reshape(shp))
        for _ in range(9):
            lg, _ = dg.step(data)
            lo = orc.step(data)
        close([lg], [lo], rtol=1e-4)
        pg = dg.download_params({n: s for n, s in shapes.items()})
        for n in shapes:
            close(pg[n], orc.params[n].reshape(shapes[n]), tensor_frac=1.0)
    finally:
        dg.destroy()


def test_c1_thousand_steps_loss_curve(ctx):
    """Full config 1: 1000 Adam steps; the loss curve tracks the oracle's."""
    w, ir, dg, orc, data = setup(ctx, "c1")
    try:
        gl = np.array([dg.step(data)[0] for _ in range(1000)])
        ol = np.array([orc.step(data) for _ in range(1000)])  # cheap: 4k params
        # both runs converge by orders of magnitude; the curves agree to 1e-3
        # of the initial loss at every step (at the f32 noise floor of a
        # converged fit the two trajectories decorrelate, so the comparison is
        # against the curve's scale, not the tiny late values)
        assert gl[-1] < 1e-3 * gl[0] and ol[-1] < 1e-3 * ol[0]
        assert np.max(np.abs(gl - ol)) < 1e-3 * ol[0]
        assert np.max(np.abs(gl[:100] - ol[:100]) / np.abs(ol[:100])) < 1e-3
    finally:
        dg.destroy()


def test_fused_optimizer_and_launch_list(ctx):
    w, ir, dg, orc, data = setup(ctx, "c4")
    try:
        info = dg.info()
        assert info["fusedOptimizer"] == "adam"
        kinds = dg.launch_list()
        assert "gather_rows" in kinds and "embedding_grad" in kinds and "adam_flat" in kinds
        assert "one_hot" not in kinds
    finally:
        dg.destroy()
