"""Planner decisions without a GPU (tg_plan_dry): views, elementwise fusion,
embedding and optimizer patterns, and that every generated fused kernel is
valid CUDA for sm_100a (compiled here with NVRTC, as the runtime does)."""
import numpy as np
import pytest

import tensorgrad_b200 as tg
from tensorgrad_b200 import backend as BK
from tensorgrad_b200 import configs as CF
from tensorgrad_b200.build import build
from tensorgrad_b200.compile import _program, build_training_ir
from tensorgrad_b200.trace import tensor_input as T, trace_fn

TINY = {
    "c1": {},
    "c2": {"batch": 4, "hw": 12, "c1": 4, "c2": 8, "hidden": 16},
    "c3": {"batch": 256},
    "c4": {"vocab": 65, "T": 16, "D": 32, "layers": 2, "heads": 2, "batch": 4, "dropout": 0.2},
    "c5": {"vocab": 512, "T": 32, "D": 64, "layers": 2, "heads": 2, "batch": 2, "sched_steps": 10},
}


@pytest.fixture(scope="module", autouse=True)
def lib():
    build()
    return BK.load()


def plan(name):
    w = CF.workload(name, **TINY[name])
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(w.global_batch), w.optimizer)
    return BK.plan_dry(ir.program)


def kinds(r):
    return [x.split("|")[0] for x in r["launches"]]


def test_gpt_plan_has_no_layout_copies():
    r = plan("c4")
    k = kinds(r)
    # head split/merge and their gradients are strided GEMM operands or
    # written in place by the producing GEMM
    assert "permute" not in k
    assert "gather_rows" in k and "embedding_grad" in k and "adam_flat" in k
    assert "one_hot" not in k
    assert r["info"]["fusedOptimizer"] == "adam"
    assert any(x.startswith("fused_ew|") for x in r["launches"])


def test_fusion_collapses_a_chain_into_one_launch():
    g = trace_fn(lambda: tg.tanh(tg.addScalar(tg.mulScalar(T("x", [64, 48]), 2.0), 1.0)))
    prog = _program(g, {}, [], g.outputs[0], None, len(g.ops))
    r = BK.plan_dry(prog)
    assert r["launches"] == ["fused_ew|mul_scalar+add_scalar+tanh"]
    assert len(r["kernelSources"]) == 1


def test_observable_intermediate_is_not_fused_away():
    def chain(with_inner_output):
        x = T("x", [32, 8])
        y = tg.mul(x, x)
        out = tg.exp(y)
        return [out, y] if with_inner_output else out

    g = trace_fn(lambda: chain(False))
    r = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))
    assert r["launches"] == ["fused_ew|mul+exp"]
    # the intermediate is also a graph output: it keeps its own launch and storage
    g2 = trace_fn(lambda: chain(True))
    r2 = BK.plan_dry(_program(g2, {}, [], g2.outputs[0], None, len(g2.ops)))
    assert sorted(r2["launches"]) == ["exp", "mul"]


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_generated_kernels_compile_for_sm100a(name):
    nvrtc = pytest.importorskip("cuda.bindings.nvrtc")
    r = plan(name)
    src = r["kernelPreamble"] + "".join(r["kernelSources"])
    err, prog = nvrtc.nvrtcCreateProgram(src.encode(), b"fused.cu", 0, [], [])
    assert err == nvrtc.nvrtcResult.NVRTC_SUCCESS
    opts = [b"--gpu-architecture=sm_100a", b"--std=c++17", b"-default-device"]
    (err,) = nvrtc.nvrtcCompileProgram(prog, len(opts), opts)
    if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
        _, n = nvrtc.nvrtcGetProgramLogSize(prog)
        log = b" " * n
        nvrtc.nvrtcGetProgramLog(prog, log)
        pytest.fail(log.decode(errors="replace")[:2000])
    _, size = nvrtc.nvrtcGetCUBINSize(prog)
    assert size > 0


def test_data_parallel_plan_adds_one_allreduce():
    w = CF.workload("c4", **TINY["c4"])
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(w.global_batch), w.optimizer)
    one = BK.plan_dry(ir.program, world=1)
    two = BK.plan_dry(ir.program, world=2)
    assert "nccl_allreduce" not in kinds(one)
    k2 = kinds(two)
    assert k2.count("nccl_allreduce") == 1
    # the gradient allreduce precedes the fused optimizer pass
    assert k2.index("nccl_allreduce") < k2.index("adam_flat")


def test_reduction_consumes_its_elementwise_producer():
    g = trace_fn(lambda: tg.sum(tg.mul(T("x", [64, 48]), T("y", [48])), -1))
    r = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))
    assert r["launches"] == ["fused_red|sum_last:mul"]


def test_cheap_shared_producer_is_recomputed_by_each_consumer():
    def f():
        x = T("x", [64, 48])
        c = tg.sub(x, T("m", [64, 1]))          # read by two consumers
        return tg.add(tg.mul(c, c), tg.mulScalar(c, 0.5))
    g = trace_fn(f)
    r = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))
    assert len(r["launches"]) == 1 and r["launches"][0].startswith("fused_ew|")


def test_scale_after_gemm_becomes_its_alpha():
    g = trace_fn(lambda: tg.mulScalar(tg.matmul(T("a", [64, 32]), T("b", [32, 48])), 0.125))
    r = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))
    assert [x.split("|")[0] for x in r["launches"]] == ["matmul"]
    # the unscaled product is an output too: the scale stays its own launch
    g2 = trace_fn(lambda: (lambda m: [tg.mulScalar(m, 0.125), m])(tg.matmul(T("a", [64, 32]), T("b", [32, 48]))))
    r2 = BK.plan_dry(_program(g2, {}, [], g2.outputs[0], None, len(g2.ops)))
    assert sorted(x.split("|")[0] for x in r2["launches"]) == ["matmul", "mul_scalar"]


@pytest.fixture
def fuse_attention(monkeypatch):
    monkeypatch.setenv("TG_ATTN_FUSE", "1")


def test_attention_fusion_default_follows_scores_size():
    # 4 x 2 x 16 x 16 probabilities: far below the 1 GiB default threshold
    assert "attn_fwd" not in kinds(plan("c4"))


def test_attention_blocks_are_fused(fuse_attention):
    k = kinds(plan("c4"))
    layers = TINY["c4"]["layers"]
    assert k.count("attn_fwd") == layers and k.count("attn_bwd") == layers
    assert "matmul_batched" not in k and "softmax_causal_last" not in k


def _attention(observe_scores):
    def f():
        q, kk, v = T("q", [2, 2, 64, 64]), T("k", [2, 2, 64, 64]), T("v", [2, 2, 64, 64])
        s = tg.mulScalar(tg.matmul(q, tg.swapAxes(kk, -1, -2)), 0.125)
        o = tg.matmul(tg.softmaxCausal(s), v)
        return [o, s] if observe_scores else o
    g = trace_fn(f)
    return BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))


def test_observed_scores_keep_attention_unfused(fuse_attention):
    assert kinds(_attention(False)) == ["attn_fwd"]
    # the scores are an output: the chain runs op by op, the scale folded
    # into the scores GEMM
    assert kinds(_attention(True)) == ["matmul_batched", "softmax_causal_last", "matmul_batched"]


def _layernorm(x):
    d = tg.sub(x, tg.mean(x, -1, keepDims=True))
    sd = tg.sqrt(tg.addScalar(tg.mean(tg.mul(d, d), -1, keepDims=True), 1e-5))
    return tg.div(d, sd)


def test_row_values_after_a_row_reduction_run_in_its_kernel():
    """LayerNorm: the eps add and sqrt on the variance run as post ops of the
    variance's row reduction instead of a launch of their own."""
    g = trace_fn(lambda: _layernorm(T("x", [64, 48])))
    k = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"]
    assert any(x.startswith("fused_red|mean_last") and "post:add_scalar+sqrt" in x for x in k)
    assert not any(x.startswith("fused_ew|add_scalar+sqrt") for x in k)


def test_attention_dropout_is_written_by_the_softmax():
    k = kinds(plan("c4"))
    assert k.count("softmax_causal_last+dropout") == TINY["c4"]["layers"]
    assert "softmax_causal_last" not in k

    g = trace_fn(lambda: tg.dropout(tg.softmaxCausal(T("s", [2, 3, 40, 40])), 0.25))
    assert kinds(BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))) == ["softmax_causal_last+dropout"]


def test_long_row_reduction_consumes_its_producer():
    g = trace_fn(lambda: tg.sum(tg.mul(T("x", [4, 50304]), T("y", [50304])), -1))
    assert BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"] == ["fused_red|sum_last:mul"]


def test_cross_entropy_gathers_the_target_log_probability():
    """sum(logSoftmax(z) * oneHot(t)) reads one element per row (pick)."""
    k = kinds(plan("c4"))
    assert "pick" in k
    assert not any(x.startswith("fused_red|sum_last:mul") for x in plan("c4")["launches"])


def test_cross_entropy_backward_writes_no_dense_one_hot_gradient():
    """The backward of the gathered term, sum(broadcast(g) * oneHot(t)), becomes
    one value per row (row_hit) that the dlogits group reads; no [rows, V]
    one-hot gradient is written."""
    launches = plan("c4")["launches"]
    assert "row_hit" in kinds(plan("c4"))
    assert "fused_ew|broadcast_to+mul" not in launches


def test_row_sum_read_through_keepdims_reshape_is_an_epilogue():
    """sum(..., keepDims) is a row sum plus a reshape; the group that reads it
    through the reshape still runs as the reduction's epilogue (the softmax
    gradient: one launch, not two)."""
    sh = [4, 2, 64, 64]

    def f():
        dP, P = T("dp", sh), T("p", sh)
        d = tg.dropout(dP, 0.2)
        return tg.mul(tg.sub(d, tg.sum(tg.mul(d, P), -1, keepDims=True)), P)
    g = trace_fn(f)
    assert BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"] == [
        "fused_red|sum_last:dropout+mul+epi:dropout+sub+mul"]


def test_layernorm_mean_is_a_first_pass_of_the_variance_kernel():
    """LayerNorm's mean (a plain row mean of a stored tensor) runs inside the
    variance reduction's kernel as a first pass over each row: one launch for
    mean, variance and normalisation."""
    def f():
        X = T("x", [300, 384])
        d = tg.sub(X, tg.mean(X, -1, keepDims=True))
        sd = tg.sqrt(tg.addScalar(tg.mean(tg.mul(d, d), -1, keepDims=True), 1e-5))
        return tg.add(tg.div(d, sd), tg.mul(sd, sd))
    g = trace_fn(f)
    assert BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"] == [
        "fused_red|mean_last>mean_last:sub+mul+post:add_scalar+sqrt+mul+epi:sub+div+add"]
    assert "mean_last" not in plan("c4")["launches"]


def test_mean_read_before_the_variance_keeps_its_own_launch():
    """A mean that another launch reads before the variance kernel runs is not
    moved into it."""
    def f():
        X = T("x", [300, 384])
        mu = tg.mean(X, -1, keepDims=True)
        early = tg.sum(tg.mul(mu, mu))                       # reads the mean first
        d = tg.sub(X, mu)
        return tg.add(tg.mean(tg.mul(d, d), -1), early)
    g = trace_fn(f)
    launches = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"]
    assert "mean_last" in launches


@pytest.mark.parametrize("n", [96, 37])
def test_column_sum_is_stored_by_its_producer_group(n):
    """A stored elementwise result that is also column-summed: one launch
    writes both (the group becomes a column reduction that stores its value)."""
    def f():
        e = tg.mulScalar(tg.add(T("x", [300, n]), T("y", [300, n])), 3.0)
        return tg.add(e, tg.sumToShape(e, [1, n]))
    g = trace_fn(f)
    launches = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"]
    assert launches[0] == "fused_red|sum_to_shape+store:add+mul_scalar" and "colsum" not in launches


@pytest.mark.parametrize("rows,merged", [(300, True), (4096, False)])
def test_write_through_skips_large_arithmetic_heavy_groups(rows, merged):
    """A small exp group stores its value and its column sum in one launch; a
    large one (>= 4M elements) keeps the elementwise grid and a separate
    column sum."""
    def f():
        e = tg.exp(T("x", [rows, 1024]))
        return tg.add(e, tg.sumToShape(e, [1, 1024]))
    g = trace_fn(f)
    launches = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"]
    assert (launches[0] == "fused_red|sum_to_shape+store:exp") == merged
    assert ("colsum" in launches) != merged


def _transposed_row_sum(view):
    """mulScalar(mul(sub(X, view(sum(X*P, -1, keepDims))), P), 0.5) over a
    square X: the row sums of shape [64, 1] seen as [1, 64] or [64], which
    broadcast along columns, not rows."""
    def f():
        X, P = T("x", [64, 64]), T("p", [64, 64])
        s = tg.sum(tg.mul(X, P), -1, keepDims=True)
        s = tg.reshape(s, [1, 64]) if view == "row" else tg.reshape(s, [64])
        return tg.mulScalar(tg.mul(tg.sub(X, s), P), 0.5)
    return f


@pytest.mark.parametrize("view", ["row", "flat"])
def test_transposed_row_value_is_not_an_epilogue(view):
    """A row result read through a reshape that broadcasts it along the other
    axis cannot be handed out per row: the reader keeps its own launch."""
    g = trace_fn(_transposed_row_sum(view))
    launches = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"]
    assert not any("+epi:" in x for x in launches), launches
    assert len(launches) == 2


@pytest.mark.parametrize("view", ["row", "flat"])
def test_transposed_mean_is_not_a_first_pass(view):
    """A mean read through a reshape that broadcasts along columns is not
    absorbed as the first pass of a later row reduction over the same rows."""
    def f():
        X = T("x", [64, 64])
        m = tg.mean(X, -1, keepDims=True)
        m = tg.reshape(m, [1, 64]) if view == "row" else tg.reshape(m, [64])
        d = tg.sub(X, m)
        return tg.mean(tg.mul(d, d), -1)
    g = trace_fn(f)
    launches = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"]
    assert "mean_last" in launches, launches
    assert not any(">mean_last" in x for x in launches), launches


def test_launch_bytes_count_each_tensor_once():
    """The planner's algorithmic bytes per launch: distinct inputs at their own
    size (a broadcast row once) plus every output."""
    def f():
        x, b = T("x", [64, 48]), T("b", [48])
        return tg.tanh(tg.add(tg.mul(x, x), b))
    g = trace_fn(f)
    r = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))
    assert r["launches"] == ["fused_ew|mul+add+tanh"]
    assert r["launchBytes"] == [4.0 * (64 * 48 + 48 + 64 * 48)]
    c4 = plan("c4")
    by = dict(zip(kinds(c4), c4["launchBytes"]))
    assert by["adam_flat"] > 0 and by["colsum"] > 0 and by["gather_rows"] > 0
    assert all(b == 0 for k, b in zip(kinds(c4), c4["launchBytes"]) if k.startswith("matmul"))


def test_data_parallel_gradients_allreduce_in_buckets_during_backward():
    """Full C4 at world 2: the gradient allreduce is split into buckets that
    start while backward GEMMs are still to come, cover every gradient's
    padded range exactly once, and join before the fused optimizer."""
    w = CF.workload("c4", batch=8)
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(8), w.optimizer)
    r = BK.plan_dry(ir.program, world=2)
    labels = r["launches"]
    k = kinds(r)
    buckets = [i for i, x in enumerate(k) if x == "nccl_allreduce"]
    assert len(buckets) >= 2
    floats = sum(int(labels[i].split("floats=")[1].split()[0]) for i in buckets)
    padded = sum((int(np.prod(t.shape)) + 63) // 64 * 64 for t in ir.paramGrads.values())
    assert floats == padded
    last_gemm = max(i for i, x in enumerate(k) if x.startswith("matmul"))
    assert buckets[0] < last_gemm
    assert k.index("nccl_join") > buckets[-1] and k.index("nccl_join") < k.index("adam_flat")


def test_attention_gemms_with_a_causal_operand_skip_its_zero_half():
    """C4 unfused: of the six batched GEMMs per layer, the four whose operand
    is the causal probabilities (or the softmax gradient, a product with
    them) are marked causal and skip the K stages of exact-zero products."""
    w = CF.workload("c4", batch=2)
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(2), w.optimizer)
    labels = [x for x in BK.plan_dry(ir.program)["launches"] if x.startswith("matmul_batched")]
    assert len(labels) == 36
    assert sum(x.endswith(" causal") for x in labels) == 24
