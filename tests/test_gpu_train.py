"""Training parity through the C ABI: every benchmark workload (shrunk so the
oracle finishes in seconds) trains on the GPU from the same seeded params and
data as the CPU oracle; loss and gradients after step 1 and params after 10
steps must agree per element within 1e-4 relative
(|gpu - ref| <= 1e-4 * max(|ref|, 1e-3 * max|ref|))."""
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
            close(pg[n], orc.params[n].reshape(shapes[n]))
    finally:
        dg.destroy()


def test_c1_thousand_steps_loss_curve(ctx):
    """Full config 1: 1000 Adam steps; the loss curve tracks the oracle's."""
    w, ir, dg, orc, data = setup(ctx, "c1")
    try:
        gl, ol = [], []
        for i in range(1000):
            gl.append(dg.step(data)[0])
            if i % 50 == 0 or i == 999:
                ol.append((i, None))
        # oracle over the same 1000 steps (cheap: 4k params)
        ol = [orc.step(data) for _ in range(1000)]
        gl, ol = np.array(gl), np.array(ol)
        assert gl[-1] < 0.1 * gl[0]
        assert np.max(np.abs(gl - ol) / np.maximum(np.abs(ol), 1e-3 * np.abs(ol).max())) < 1e-2
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
