"""The public training API on the GPU (src/compile.ts:585-891 surface):
checkpoint export/import resumes a run exactly, attached forward graphs share
the trainer's params and resolve parametric batch dims per call through an
LRU of sibling graphs, and reset / setLR / uploadParams behave as the
reference's handle does."""
import numpy as np
import pytest

import tensorgrad_b200 as tg
from oracle.evaluator import eval_graph
from tensorgrad_b200 import backend as BK
from tensorgrad_b200 import configs as CF
from tensorgrad_b200 import ops as O
from tensorgrad_b200.compile import build_forward_ir

from .test_gpu_ops import close

pytestmark = pytest.mark.gpu

SHAPE = {"vocab": 65, "T": 16, "D": 32, "layers": 2, "heads": 2, "batch": 4}


def _train(ctx, seed, dropout=0.2, **over):
    w = CF.workload("c4", **{**SHAPE, "dropout": dropout, **over})
    t = tg.compile(w.make_model(), w.loss, w.inputs(w.global_batch), w.optimizer, seed=seed, ctx=ctx)
    return w, t


def _batch(w, i):
    return CF.gpt_data(w.global_batch, w.extra["T"], w.extra["V"], seed=1000 + i)


def _step(t, data):
    r = t.step(data)
    assert r["kind"] == "completed", r
    return r["loss"]


def test_checkpoint_resume_continues_the_run(ctx):
    w, a = _train(ctx, seed=1)
    for i in range(3):
        _step(a, _batch(w, i))
    blob = a.exportCheckpoint()
    ref = [_step(a, _batch(w, i)) for i in (3, 4)]
    ref_params = a.downloadParams()

    _, b = _train(ctx, seed=2)          # different init: everything comes from the blob
    b.importCheckpoint(blob)
    assert b.steps_done == 3
    got = [_step(b, _batch(w, i)) for i in (3, 4)]
    # same params, moments, step and dropout counters: the same kernels see the same bytes
    np.testing.assert_array_equal(np.array(got, np.float32), np.array(ref, np.float32))
    for n, v in b.downloadParams().items():
        np.testing.assert_array_equal(v, ref_params[n])
    a.destroy()
    b.destroy()


def test_checkpoint_resumes_the_oracle_run(ctx):
    """A checkpoint loaded into the CPU oracle (params, moments, the step and
    dropout counters from its metadata) continues the run as the GPU does:
    the next two losses and the params after them agree at the op
    tolerance."""
    from oracle.driver import OracleTrainer
    w, a = _train(ctx, seed=1)
    for i in range(3):
        _step(a, _batch(w, i))
    d = tg.loadSafetensors(a.exportCheckpoint())
    meta = d["metadata"]
    orc = OracleTrainer(a.program, {n[6:]: v for n, v in d["tensors"].items() if n.startswith("param/")})
    orc.states = {n[6:]: v.reshape(orc.states[n[6:]].shape) for n, v in d["tensors"].items()
                  if n.startswith("state/")}
    orc.t, orc.prng = int(meta["step"]), int(meta["prng"])
    for i in (3, 4):
        close([_step(a, _batch(w, i))], [orc.step(_batch(w, i))])
    got = a.downloadParams()
    for n, v in orc.params.items():
        close(got[n], v.reshape(got[n].shape))
    a.destroy()


def test_checkpoint_import_is_strict(ctx):
    w, a = _train(ctx, seed=1)
    blob = a.exportCheckpoint()
    _, other = _train(ctx, seed=1, layers=1)
    with pytest.raises(BK.TgError):
        other.importCheckpoint(blob)
    with pytest.raises(BK.TgError, match="not a tensorgrad_b200 checkpoint"):
        a.importCheckpoint(tg.saveSafetensors({"x": np.zeros(2, np.float32)}))
    a.destroy()
    other.destroy()


def _fwd_ref(model, forward, tokens, params):
    g, _, prog = build_forward_ir(model, forward, {"tokens": {"shape": list(tokens.shape), "dtype": "i32"}})
    vals = eval_graph(prog["graph"], {**params, "tokens": tokens})
    return vals[prog["loss"]]


@pytest.mark.parametrize("fuse", ["0", "1"])
def test_attach_shares_params_and_resolves_parametric_batch(ctx, fuse, monkeypatch):
    # "1": the forward graphs' attention runs as the fused forward kernel
    monkeypatch.setenv("TG_ATTN_FUSE", fuse)
    w, t = _train(ctx, seed=3, dropout=0.0)
    T = w.extra["T"]
    logits = t.attach(lambda m, x: CF.gpt_logits(m, x["tokens"]),
                      {"tokens": {"shape": [None, T], "dtype": "i32"}}, maxCachedShapes=1)
    pick = t.attach(lambda m, x: O.argmax(CF.gpt_logits(m, x["tokens"]), -1),
                    {"tokens": {"shape": [None, T], "dtype": "i32"}}, output="i32")

    def check(b, seed):
        toks = _batch(w, seed)["tokens"][:b] if b <= w.global_batch else \
            CF.gpt_data(b, T, w.extra["V"], seed=seed)["tokens"]
        params = t.downloadParams()
        ref = _fwd_ref(t.model, lambda m, x: CF.gpt_logits(m, x["tokens"]), toks, params)
        r = logits.run({"tokens": toks})
        assert r["kind"] == "completed", r
        assert r["output"].shape == (b, T, w.extra["V"])
        close(r["output"], ref)
        r2 = pick.run({"tokens": toks})
        assert r2["kind"] == "completed", r2
        am = r2["output"]
        assert am.dtype == np.int32 and am.shape == (b, T)
        # index results are exact wherever the oracle's top two logits are not a near tie
        srt = np.sort(ref, -1)
        clear = (srt[..., -1] - srt[..., -2]) > 1e-4 * np.abs(ref).max()
        np.testing.assert_array_equal(am[clear], np.argmax(ref, -1)[clear])

    check(2, 0)
    assert ("attn_fwd" in [x.split("|")[0] for x in logits.graph_for(
        {"tokens": np.zeros((2, T), np.int32)}).launch_list()]) == (fuse == "1")
    check(7, 11)                 # a second resolved shape evicts the first (LRU of 1)
    assert len(logits._cache) == 1
    _step(t, _batch(w, 0))       # the attached graphs read the trainer's updated params
    check(2, 0)
    with pytest.raises(Exception):
        logits.graph_for({"tokens": np.zeros(T + 1, np.int32)})  # does not fit [None, T]
    logits.destroy()
    pick.destroy()
    t.destroy()


def test_reset_set_lr_and_upload_params(ctx):
    w, t = _train(ctx, seed=5, dropout=0.0)   # reset keeps the dropout counter running
    init = t.downloadParams()
    first = _step(t, _batch(w, 0))
    _step(t, _batch(w, 1))
    t.reset()
    for n, v in t.downloadParams().items():
        np.testing.assert_array_equal(v, init[n])
    assert _step(t, _batch(w, 0)) == first   # seed, moments and step counter all back at zero
    t.reset({"params": False})                  # optimizer only: params untouched
    kept = t.downloadParams()
    assert any(not np.array_equal(kept[n], init[n]) for n in init)

    before = t.downloadParams()
    # zero step size. With a constant lr the AdamW shrink 1 - lr*wd was baked in
    # at compile time from the original lr (src/adam.ts:10-11), so setLR leaves it;
    # each param is either untouched or exactly shrink * p
    t.setLR(0.0)
    _step(t, _batch(w, 2))
    shrink = np.float32(1 - 3e-4 * 0.1)
    decayed = 0
    for n, v in t.downloadParams().items():
        if not np.array_equal(v, before[n]):
            np.testing.assert_array_equal(v, shrink * before[n])
            decayed += 1
    assert decayed > 0

    with pytest.raises(BK.TgError, match="missing"):
        t.uploadParams({n: v for n, v in list(before.items())[1:]})
    with pytest.raises(BK.TgError, match="unknown"):
        t.uploadParams({**before, "nope": np.zeros(1, np.float32)})
    t.uploadParams(init)
    for n, v in t.downloadParams().items():
        np.testing.assert_array_equal(v, init[n])

    r = t.step({"tokens": _batch(w, 0)["tokens"]})   # a missing input fails, it does not throw
    assert r["kind"] == "failed"
    t.destroy()
