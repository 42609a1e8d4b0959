"""Pins the CPU oracle (and the graph layer) to the reference's own known
answers: the finite-difference exemplars of test/grad.ts:35-235, the leakyRelu
values of test/ops.ts:49-58, the dropout seed/salt structure of
test/ops.ts:26-45, the schedule values of test/smoke.ts:411-470 and the DCE
bit-identity of test/dce.ts:79-89."""
import math

import numpy as np
import pytest

import tensorgrad_b200 as tg
from oracle.evaluator import eval_graph, dropout_mask
from tensorgrad_b200.dce import eliminateDeadCode
from tensorgrad_b200.grad import appendGrad, appendGradNormalize
from tensorgrad_b200.ir import graph_to_wire
from tensorgrad_b200.lr import lr, resolveLR
from tensorgrad_b200.trace import param_input, tensor_input, trace_fn

from ._helpers import fd_check, make_range


# ---- FD exemplars (test/grad.ts:35-146) ------------------------------------
def test_fd_mul():
    fd_check([4, 8], lambda p: tg.mean(tg.mul(p, p)))


def test_fd_mean_keepdims():
    fd_check([4, 8], lambda p: tg.mean(tg.mean(p, -1, keepDims=True)))


def test_fd_matmul():
    fd_check([4, 8], lambda p: tg.mean(tg.matmul(p, tensor_input("x", [8, 16]))),
             extra={"x": make_range([8, 16])})


def test_fd_embedding():
    fd_check([10, 4], lambda p: tg.mean(tg.embedding(p, tensor_input("idx", [3], "i32"))),
             extra={"idx": np.array([2, 5, 7], np.int32)})


def test_fd_softmax_causal():
    fd_check([4, 4], lambda p: tg.mean(tg.softmaxCausal(p)))


def test_fd_dropout_seed42():
    fd_check([4, 8], lambda p: tg.mean(tg.dropout(p, 0.1)), extra={"__prngSeed": np.array(42, np.int32)})


def test_fd_concat():
    fd_check([3, 4], lambda p: tg.mean(tg.concat([p, tensor_input("q", [3, 5])], 1)),
             extra={"q": make_range([3, 5])})


def test_fd_erf_and_gelu():
    fd_check([5], lambda p: tg.mean(tg.erf(p)))
    fd_check([5], lambda p: tg.mean(tg.gelu(p)))
    fd_check([4], lambda p: tg.mean(tg.gelu(p, approximate="tanh")))


def test_fd_conv_input_grad():
    fd_check([1, 2, 4, 4], lambda p: tg.mean(tg.conv2d(p, tensor_input("k", [3, 2, 2, 2]))),
             extra={"k": make_range([3, 2, 2, 2])})


def test_fd_conv_weight_grad_stride_pad():
    fd_check([3, 2, 2, 2], lambda p: tg.mean(tg.conv2d(tensor_input("x", [1, 2, 4, 4]), p, stride=2, padding=1)),
             extra={"x": make_range([1, 2, 4, 4])})


def test_fd_conv_groups():
    fd_check([1, 4, 4, 4], lambda p: tg.mean(tg.conv2d(p, tensor_input("k", [6, 2, 2, 2]), groups=2)),
             extra={"k": make_range([6, 2, 2, 2])})
    fd_check([6, 2, 2, 2], lambda p: tg.mean(tg.conv2d(tensor_input("x", [1, 4, 4, 4]), p, stride=2, padding=1,
                                                       groups=2)),
             extra={"x": make_range([1, 4, 4, 4])})
    fd_check([1, 3, 4, 4], lambda p: tg.mean(tg.conv2d(p, tensor_input("k", [3, 1, 3, 3]), padding=1, groups=3)),
             extra={"k": make_range([3, 1, 3, 3])})


def test_fd_narrow_split_where_causal():
    fd_check([4, 6], lambda p: tg.mean(tg.narrow(p, 1, 1, 3)))

    def split_loss(p):
        a, b = tg.split(p, [2, 4], 1)
        return tg.add(tg.mean(tg.mul(a, a)), tg.mean(tg.mul(b, b)))
    fd_check([4, 6], split_loss)
    fd_check([4, 4], lambda p: tg.mean(tg.whereCausal(p, 0)))


def test_fd_maxpool():
    fd_check([1, 2, 4, 4], lambda p: tg.mean(tg.maxPool2d(p, 2)), init=make_range([1, 2, 4, 4]))


# ---- structural known answers -----------------------------------------------
def test_stop_gradient_one_over_n():
    N = 6
    init = (np.arange(N) * 0.1 - 0.3).astype(np.float32)
    g = trace_fn(lambda: (lambda p: tg.mean(tg.add(tg.stopGradient(p), p)))(param_input("w", [N])))
    gr = appendGrad(g)
    v = eval_graph(graph_to_wire(g), {"w": init})[gr.paramGrads["w"].id]
    assert np.allclose(v, 1 / N, atol=1e-5)


def test_grouped_conv_equals_block_diagonal_dense():
    B, cin, cout, G, K, H, W = 2, 4, 6, 2, 3, 5, 5
    cpg, opg = cin // G, cout // G
    x = make_range([B, cin, H, W])
    wg = make_range([cout, cpg, K, K])
    wd = np.zeros((cout, cin, K, K), np.float32)
    for co in range(cout):
        g = co // opg
        wd[co, g * cpg:(g + 1) * cpg] = wg[co]
    g1 = trace_fn(lambda: tg.conv2d(tensor_input("x", [B, cin, H, W]), tensor_input("w", [cout, cpg, K, K]),
                                    padding=1, groups=G))
    g2 = trace_fn(lambda: tg.conv2d(tensor_input("x", [B, cin, H, W]), tensor_input("w", [cout, cin, K, K]),
                                    padding=1))
    o1 = eval_graph(graph_to_wire(g1), {"x": x, "w": wg})[g1.outputs[0]]
    o2 = eval_graph(graph_to_wire(g2), {"x": x, "w": wd})[g2.outputs[0]]
    assert np.max(np.abs(o1 - o2)) <= 1e-5


def test_normalize_grads_unit_norm_and_filter():
    N = 6
    init = make_range([N])
    holder = {}

    def body():
        p = param_input("w", [N])
        q = param_input("v", [N])
        return tg.add(tg.mean(tg.mul(p, p)), tg.mean(tg.mul(q, q)))
    g = trace_fn(body)
    gr = appendGrad(g)
    normed = appendGradNormalize(g, gr.paramGrads, lambda n: n == "w")
    assert normed["v"] is gr.paramGrads["v"]
    vals = eval_graph(graph_to_wire(g), {"w": init, "v": init})
    raw = vals[gr.paramGrads["w"].id].astype(np.float64)
    gn = vals[normed["w"].id].astype(np.float64)
    assert abs(np.linalg.norm(gn) - 1) < 1e-4
    assert np.allclose(gn, raw / (np.linalg.norm(raw) + 1e-8), atol=1e-5)
    with pytest.raises(RuntimeError):
        appendGradNormalize(g, gr.paramGrads, lambda n: n == "typo.W")


def test_leaky_relu_alpha2_values():
    g = trace_fn(lambda: tg.leakyRelu(tensor_input("x", [4]), 2))
    out = eval_graph(graph_to_wire(g), {"x": np.array([-1, -0.5, 0.5, 1], np.float32)})[g.outputs[0]]
    assert np.allclose(out, [-2, -1, 0.5, 1], atol=1e-6)


def test_dropout_zero_is_identity_and_salts_unique():
    g = trace_fn(lambda: tg.dropout(tensor_input("x", [4]), 0))
    assert not any(op["kind"] == "dropout" for op in g.ops)
    g = trace_fn(lambda: tg.dropout(tg.dropout(tensor_input("x", [4]), 0.1), 0.2))
    seeds = [op for op in g.ops if op["kind"] == "tensor_input" and op["name"] == "__prngSeed"]
    salts = [op["salt"] for op in g.ops if op["kind"] == "dropout"]
    assert len(seeds) == 1 and len(set(salts)) == len(salts)


def test_dropout_mask_keep_rate_and_scale():
    m = dropout_mask(7, 3, 0.2, 200000)
    assert set(np.unique(m)).issubset({0.0, np.float32(1.25)})
    assert abs((m > 0).mean() - 0.8) < 0.005


def test_lr_schedule_values():
    s = lr.staircase(peak=1.0, every=1, gamma=0.7)
    for step, want in [(1, 1.0), (2, 0.7), (3, 0.49), (10, 0.7 ** 9)]:
        assert abs(resolveLR(s, step) - want) < 1e-7
    s = lr.staircase(peak=0.1, every=3, gamma=0.5)
    for step, want in [(1, 0.1), (3, 0.1), (4, 0.05), (6, 0.05), (7, 0.025)]:
        assert abs(resolveLR(s, step) - want) < 1e-9
    s = lr.multiStep(peak=1.0, milestones=[3, 7], gamma=0.1)
    for step, want in [(1, 1.0), (2, 1.0), (3, 0.1), (4, 0.1), (6, 0.1), (7, 0.01), (10, 0.01)]:
        assert abs(resolveLR(s, step) - want) < 1e-9
    c = lr.cosineAnnealing(peak=1.0, final=0.0, steps=10)
    assert abs(resolveLR(c, 5) - 0.5 * (1 + math.cos(math.pi * 0.5))) < 1e-12


def test_dce_is_bit_identical():
    """Loss and grads identical before/after DCE (test/dce.ts:79-89)."""
    def build():
        x = tensor_input("x", [1, 2, 6, 6])
        w = param_input("w", [3, 2, 3, 3])
        frozen = tensor_input("k", [3, 3, 3, 3])
        h = tg.relu(tg.conv2d(x, w, padding=1))
        return tg.mean(tg.conv2d(h, frozen, padding=1))
    inputs = {"x": make_range([1, 2, 6, 6]), "w": make_range([3, 2, 3, 3]) * 0.3, "k": make_range([3, 3, 3, 3])}
    g1 = trace_fn(build)
    gr1 = appendGrad(g1)
    v1 = eval_graph(graph_to_wire(g1), inputs)
    g2 = trace_fn(build)
    gr2 = appendGrad(g2)
    n_before = len(g2.ops)
    idm = eliminateDeadCode(g2, [t.id for t in gr2.paramGrads.values()])
    assert len(g2.ops) < n_before
    v2 = eval_graph(graph_to_wire(g2), inputs)
    assert np.array_equal(v1[g1.outputs[0]], v2[g2.outputs[0]])
    assert np.array_equal(v1[gr1.paramGrads["w"].id], v2[idm[gr2.paramGrads["w"].id].id])
