"""Per-op parity: each IR op kind runs through the C ABI on the GPU and is
compared with the oracle on the same seeded inputs. Tolerance for f32:
|gpu - ref| <= 1e-4 * max(|ref|, 1e-2 * max|ref|) per element (plus a 1e-7
absolute floor for exact zeros). The oracle accumulates in f64 and the GPU in
f32, so an element that is the small difference of large terms carries an
absolute error proportional to the tensor's magnitude, not its own; the
1e-2 * max|ref| floor bounds it there. i32 outputs and dropout masks must
match bit for bit."""
import numpy as np
import pytest

import tensorgrad_b200 as tg
from oracle.evaluator import eval_graph
from tensorgrad_b200 import backend as BK
from tensorgrad_b200.compile import _program
from tensorgrad_b200.ir import graph_to_wire
from tensorgrad_b200.module import Mulberry32
from tensorgrad_b200.trace import tensor_input, trace_fn

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def close(gpu, ref, rtol=RTOL, floor=1e-7, tensor_frac=1e-2):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.maximum(np.abs(ref), tensor_frac * max(np.abs(ref).max(), 1e-30))
    err = np.abs(gpu - ref)
    ok = err <= rtol * scale + floor
    i = int(np.argmax(err / (scale + 1e-30)))
    assert ok.all(), f"max rel err {np.max(err / (scale + 1e-30)):.3e} at {i}: gpu={gpu.reshape(-1)[i]} ref={ref.reshape(-1)[i]}"


def rnd(shape, seed=1, lo=-1.0, hi=1.0):
    n = int(np.prod(shape)) if len(shape) else 1
    return (lo + (hi - lo) * Mulberry32(seed).take(n)).astype(np.float32).reshape(shape)


def run(ctx, build, inputs, exact=False, rtol=RTOL):
    g = trace_fn(build)
    prog = _program(g, {}, [], g.outputs[0], None, len(g.ops))
    prog["usesPrng"] = False  # the test passes __prngSeed itself
    dg = BK.DeviceGraph(ctx, prog)
    try:
        out, _ = dg.run(inputs)
    finally:
        dg.destroy()
    ref = eval_graph(graph_to_wire(g), inputs)[g.outputs[0]]
    if exact:
        assert np.array_equal(out, ref.reshape(out.shape))
    else:
        close(out, ref.reshape(out.shape), rtol)
    return out


T = tensor_input


def test_binops_broadcast(ctx):
    ins = {"a": rnd([4, 5, 8], 1), "b": rnd([8], 2), "c": rnd([4, 5, 1], 3), "d": rnd([5, 1], 4)}

    def build():
        A, B, C, D = T("a", [4, 5, 8]), T("b", [8]), T("c", [4, 5, 1]), T("d", [5, 1])
        x = tg.sub(tg.mul(tg.add(A, B), C), D)
        x = tg.div(x, tg.add(tg.abs(C), 0.5))
        return tg.max(tg.min(x, 0.7), -0.6)
    run(ctx, build, ins)


@pytest.mark.parametrize("name", ["exp", "tanh", "sigmoid", "erf", "sin", "cos", "relu", "neg", "abs", "gelu"])
def test_unary(ctx, name):
    fn = getattr(tg, name)
    run(ctx, lambda: fn(T("a", [3, 1000])), {"a": rnd([3, 1000], 5, -3, 3)})


@pytest.mark.parametrize("name", ["sqrt", "rsqrt", "log"])
def test_unary_positive(ctx, name):
    fn = getattr(tg, name)
    run(ctx, lambda: fn(T("a", [3, 1000])), {"a": rnd([3, 1000], 6, 0.1, 4)})


def test_compare_where(ctx):
    ins = {"a": rnd([6, 7], 7)}
    run(ctx, lambda: tg.leakyRelu(T("a", [6, 7]), 0.3), ins)
    run(ctx, lambda: tg.leakyRelu(T("a", [6, 7]), 2.0), ins)


def test_where_with_broadcast_branches(ctx):
    ins = {"a": rnd([6, 7], 7), "b": rnd([7], 8)}

    def build():
        a, b = T("a", [6, 7]), T("b", [7])
        return tg.where(tg.less(a, b), tg.mul(a, 3.0), tg.neg(b))
    run(ctx, build, ins)


def test_reductions(ctx):
    a = rnd([33, 257], 9)
    run(ctx, lambda: tg.sum(T("a", [33, 257]), -1), {"a": a})
    run(ctx, lambda: tg.mean(T("a", [33, 257]), -1, keepDims=True), {"a": a})
    run(ctx, lambda: tg.mean(T("a", [33, 257])), {"a": a})
    run(ctx, lambda: tg.sum(T("a", [33, 257]), 0), {"a": a})


def test_long_row_sum(ctx):
    a = rnd([1, 1 << 20], 10)
    run(ctx, lambda: tg.mean(T("a", [1, 1 << 20])), {"a": a})


def test_argmax_exact_with_ties(ctx):
    a = np.floor(rnd([64, 300], 11, 0, 4)).astype(np.float32)  # many ties: first max must win
    run(ctx, lambda: tg.argmax(T("a", [64, 300]), -1), {"a": a}, exact=True)
    run(ctx, lambda: tg.argmin(T("a", [64, 300]), -1), {"a": a}, exact=True)
    big = np.floor(rnd([3, 5000], 12, 0, 3)).astype(np.float32)
    run(ctx, lambda: tg.argmax(T("a", [3, 5000]), -1), {"a": big}, exact=True)


def test_softmaxes(ctx):
    a = rnd([2, 3, 40, 40], 13, -4, 4)
    run(ctx, lambda: tg.softmaxCausal(T("a", [2, 3, 40, 40])), {"a": a})
    run(ctx, lambda: tg.logSoftmax(T("a", [2, 3, 40, 40])), {"a": a})
    run(ctx, lambda: tg.softmax(T("a", [2, 3, 40, 40]), 2), {"a": a})
    w = rnd([4, 3000], 14, -4, 4)
    run(ctx, lambda: tg.logSoftmax(T("a", [4, 3000])), {"a": w})
    # the C5 vocabulary (float4 rows) and an odd width (scalar rows)
    v = rnd([3, 50304], 67, -8, 8)
    run(ctx, lambda: tg.logSoftmax(T("a", [3, 50304])), {"a": v})
    u = rnd([2, 4099], 68, -8, 8)
    run(ctx, lambda: tg.logSoftmax(T("a", [2, 4099])), {"a": u})
    s = rnd([2, 2100, 2100], 15, -2, 2)
    run(ctx, lambda: tg.softmaxCausal(T("a", [2, 2100, 2100])), {"a": s})


def test_where_causal_and_dropout_exact(ctx):
    a = rnd([2, 16, 16], 16)
    run(ctx, lambda: tg.whereCausal(T("a", [2, 16, 16]), -1e9), {"a": a}, exact=True)
    x = rnd([8, 1024], 17)
    seed = np.array(42, np.int32)
    run(ctx, lambda: tg.dropout(tg.dropout(T("x", [8, 1024]), 0.2), 0.5), {"x": x, "__prngSeed": seed}, exact=True)


def test_layout_ops(ctx):
    a = rnd([3, 4, 5, 6], 18)
    run(ctx, lambda: tg.permute(T("a", [3, 4, 5, 6]), [2, 0, 3, 1]), {"a": a}, exact=True)
    run(ctx, lambda: tg.narrow(T("a", [3, 4, 5, 6]), 2, 1, 3), {"a": a}, exact=True)
    run(ctx, lambda: tg.narrow(T("a", [3, 4, 5, 6]), 0, 1, 2), {"a": a}, exact=True)
    b = rnd([3, 4, 2, 6], 19)
    run(ctx, lambda: tg.concat([T("a", [3, 4, 5, 6]), T("b", [3, 4, 2, 6])], 2), {"a": a, "b": b}, exact=True)
    run(ctx, lambda: tg.scatterAxis(T("b", [3, 4, 2, 6]), [3, 4, 5, 6], 2, 1, 3), {"b": b}, exact=True)
    run(ctx, lambda: tg.broadcastTo(T("c", [1, 6]), [3, 4, 5, 6]), {"c": rnd([1, 6], 20)}, exact=True)
    run(ctx, lambda: tg.sumToShape(T("a", [3, 4, 5, 6]), [4, 1, 6]), {"a": a})


def test_sum_to_shape_trailing(ctx):
    """Kept leading dims, reduced trailing dims: the row-sum path (LayerNorm
    backward shape), including a long row that splits across blocks."""
    a = rnd([64, 33, 384], 61)
    run(ctx, lambda: tg.sumToShape(T("a", [64, 33, 384]), [64, 33, 1]), {"a": a})
    b = rnd([3, 40000], 62)
    run(ctx, lambda: tg.sumToShape(T("b", [3, 40000]), [3, 1]), {"b": b})


def test_softmax_causal_with_its_dropout(ctx):
    """The causal softmax kernel writing dropout(P) as a second output: the
    same masks as the elementwise dropout (bit for bit) and the same values."""
    s = rnd([2, 3, 200, 200], 66, -4, 4)
    seed = np.array(11, np.int32)

    run(ctx, lambda: tg.dropout(tg.softmaxCausal(T("s", [2, 3, 200, 200])), 0.25), {"s": s, "__prngSeed": seed})


def test_layernorm_row_post_ops(ctx):
    """Row-reduction kernels that also evaluate the per-row values after the
    sum (eps, sqrt) and write them: LayerNorm forward and a row-term use of
    the standard deviation."""
    x = rnd([300, 384], 65, -2, 2)

    def build():
        X = T("x", [300, 384])
        d = tg.sub(X, tg.mean(X, -1, keepDims=True))
        sd = tg.sqrt(tg.addScalar(tg.mean(tg.mul(d, d), -1, keepDims=True), 1e-5))
        return tg.add(tg.div(d, sd), tg.mul(sd, sd))
    run(ctx, build, {"x": x})


def test_softmax_gradient_row_epilogue(ctx):
    """The softmax gradient with dropout, P * (dropout(dP) - sum(dropout(dP) * P,
    keepDims)): one row-reduction launch whose epilogue reads the row sum
    through its keepDims reshape and recomputes the same dropout mask."""
    sh = [2, 3, 200, 200]
    dp, p = rnd(sh, 67), rnd(sh, 68, 0, 1)
    seed = np.array(5, np.int32)

    def build():
        dP, P = T("dp", sh), T("p", sh)
        d = tg.dropout(dP, 0.2)
        return tg.mulScalar(tg.mul(tg.sub(d, tg.sum(tg.mul(d, P), -1, keepDims=True)), P), 0.125)
    run(ctx, build, {"dp": dp, "p": p, "__prngSeed": seed})


@pytest.mark.parametrize("n", [96, 37])
def test_column_sum_stored_by_its_producer(ctx, n):
    """A column sum of a tensor that an elementwise group stores for other
    readers is computed by that group's launch (float4 columns and scalar)."""
    x, y = rnd([300, n], 69), rnd([300, n], 70)

    def build():
        e = tg.mulScalar(tg.add(T("x", [300, n]), T("y", [300, n])), 3.0)
        return tg.add(e, tg.sumToShape(e, [1, n]))
    run(ctx, build, {"x": x, "y": y})


def test_sum_to_shape_middle(ctx):
    """Reduced dims on both sides of the kept ones (the conv bias gradient
    [B, C, H, W] -> [C, 1, 1]), small and at the CNN benchmark's size."""
    a = rnd([3, 5, 4, 7], 63)
    run(ctx, lambda: tg.sumToShape(T("a", [3, 5, 4, 7]), [5, 1, 1]), {"a": a})
    b = rnd([128, 64, 24, 24], 64)
    run(ctx, lambda: tg.sumToShape(T("b", [128, 64, 24, 24]), [64, 1, 1]), {"b": b})


def test_scaled_gemm(ctx):
    """mul_scalar folded into the producing GEMM's alpha (tensor-core and
    SIMT paths, batched scores shape)."""
    q, kt = rnd([4, 128, 64], 70), rnd([4, 64, 128], 71)
    run(ctx, lambda: tg.mulScalar(tg.matmul(T("q", [4, 128, 64]), T("k", [4, 64, 128])), 0.125), {"q": q, "k": kt})
    a, b = rnd([7, 5], 72), rnd([5, 9], 73)
    run(ctx, lambda: tg.mulScalar(tg.matmul(T("a", [7, 5]), T("b", [5, 9])), -3.0), {"a": a, "b": b})


@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (37, 29, 53), (256, 384, 200), (130, 1, 70)])
def test_matmul_2d(ctx, M, K, N):
    run(ctx, lambda: tg.matmul(T("a", [M, K]), T("b", [K, N])), {"a": rnd([M, K], 21), "b": rnd([K, N], 22)})


def test_matmul_transposed_views_and_batched(ctx):
    a, b = rnd([2, 3, 17, 24], 23), rnd([2, 3, 19, 24], 24)
    run(ctx, lambda: tg.matmul(T("a", [2, 3, 17, 24]), tg.swapAxes(T("b", [2, 3, 19, 24]), -1, -2)),
        {"a": a, "b": b})
    x = rnd([2, 17, 3, 8], 25)

    def heads():
        h = tg.swapAxes(T("x", [2, 17, 3, 8]), 1, 2)          # [2,3,17,8] strided view
        s = tg.matmul(h, tg.swapAxes(h, -1, -2))              # [2,3,17,17]
        return tg.matmul(s, h)
    run(ctx, heads, {"x": x})
    w = rnd([24, 10], 26)
    run(ctx, lambda: tg.matmul(tg.swapAxes(T("w", [24, 10]), 0, 1), T("v", [24, 7])), {"w": w, "v": rnd([24, 7], 27)})


def test_embedding_gather_and_onehot(ctx):
    idx = np.floor(rnd([5, 7], 28, 0, 11)).astype(np.int32)
    tab = rnd([11, 12], 29)
    run(ctx, lambda: tg.embedding(T("t", [11, 12]), T("i", [5, 7], "i32")), {"t": tab, "i": idx}, exact=True)
    run(ctx, lambda: tg.oneHot(T("i", [5, 7], "i32"), 11), {"i": idx}, exact=True)


def test_conv_and_pool(ctx):
    x = rnd([2, 4, 9, 9], 30)
    w = rnd([6, 2, 3, 3], 31)
    run(ctx, lambda: tg.conv2d(T("x", [2, 4, 9, 9]), T("w", [6, 2, 3, 3]), stride=2, padding=1, groups=2),
        {"x": x, "w": w})
    q = np.floor(rnd([2, 3, 8, 8], 32, 0, 3)).astype(np.float32)
    run(ctx, lambda: tg.maxPool2d(T("x", [2, 3, 8, 8]), 2), {"x": q}, exact=True)
    run(ctx, lambda: tg.maxPool2d(T("x", [2, 3, 8, 8]), 3, stride=2, padding=1), {"x": q}, exact=True)


@pytest.mark.parametrize("shape,k,stride,pad", [([3, 4, 8, 6], 2, 2, 0), ([2, 3, 9, 7], 2, 2, 0),
                                                 ([2, 3, 9, 9], 3, 3, 1), ([2, 2, 8, 8], 3, 2, 1)])
def test_maxpool_grad(ctx, shape, k, stride, pad):
    """Max-pool gradient on exact 2x2 tilings, ragged edges, padded disjoint
    windows and overlapping windows; ties (integer-valued inputs) must route
    to the first maximum in scan order, bit for bit."""
    q = np.floor(rnd(shape, 34, 0, 3)).astype(np.float32)
    Ho = (shape[2] + 2 * pad - k) // stride + 1
    Wo = (shape[3] + 2 * pad - k) // stride + 1
    dy = rnd([shape[0], shape[1], Ho, Wo], 35)
    run(ctx, lambda: tg.maxPool2dGrad(T("x", shape), T("dy", list(dy.shape)), k, k, stride, stride, pad, pad),
        {"x": q, "dy": dy}, exact=True)


@pytest.mark.parametrize("B,Cin,H,W,Cout,k,stride,pad,groups", [
    (8, 16, 20, 20, 32, 3, 1, 1, 1),   # every contraction on the tensor-core path
    (4, 1, 28, 28, 8, 3, 1, 0, 1),     # Cin=1: K=9 forward on the SIMT path
    (3, 6, 11, 9, 9, 3, 2, 1, 3),      # groups, stride 2, ragged spatial sizes
    (2, 4, 7, 7, 4, 5, 1, 2, 2),       # 5x5 taps wider than the stride
])
def test_conv_forward_and_grads(ctx, B, Cin, H, W, Cout, k, stride, pad, groups):
    """conv2d, conv2d_input_grad and conv2d_weight_grad through the column
    gather + GEMM lowering against the oracle's direct sums."""
    Ho = (H + 2 * pad - k) // stride + 1
    Wo = (W + 2 * pad - k) // stride + 1
    x = rnd([B, Cin, H, W], 40)
    w = rnd([Cout, Cin // groups, k, k], 41)
    dy = rnd([B, Cout, Ho, Wo], 42)
    run(ctx, lambda: tg.conv2d(T("x", list(x.shape)), T("w", list(w.shape)), stride=stride, padding=pad,
                               groups=groups), {"x": x, "w": w})
    run(ctx, lambda: tg.conv2dInputGrad(T("w", list(w.shape)), T("dy", list(dy.shape)), H, W, stride, stride,
                                        pad, pad, groups), {"w": w, "dy": dy})
    run(ctx, lambda: tg.conv2dWeightGrad(T("x", list(x.shape)), T("dy", list(dy.shape)), k, k, stride, stride,
                                         pad, pad, groups), {"x": x, "dy": dy})


def test_randn_and_categorical(ctx):
    seed = np.array(5, np.int32)
    run(ctx, lambda: tg.add(tg.randn([4, 1000]), T("z", [1000])), {"z": np.zeros(1000, np.float32),
                                                                   "__prngSeed": seed}, rtol=1e-3)
    logits = rnd([16, 50], 33, -2, 2)
    run(ctx, lambda: tg.categorical(T("l", [16, 50])), {"l": logits, "__prngSeed": seed}, exact=True)


def test_fused_long_row_reduction(ctx):
    """A row reduction fused with its elementwise producer over rows longer
    than a warp handles (one block per row), as the C5 loss's
    sum(logSoftmax * oneHot)."""
    x = rnd([5, 50304], 69, -3, 3)
    y = rnd([5, 50304], 70)
    run(ctx, lambda: tg.sum(tg.mul(T("x", [5, 50304]), T("y", [5, 50304])), -1), {"x": x, "y": y})
    run(ctx, lambda: tg.mean(tg.exp(T("x", [5, 50304])), -1), {"x": x})


def test_fused_reductions_and_shared_producers(ctx):
    """Elementwise groups consumed by row and column reductions, and a cheap
    producer recomputed by each of its consumers (the LayerNorm shapes)."""
    x, y, m = rnd([256, 96], 71), rnd([96], 72), rnd([256, 1], 73)
    run(ctx, lambda: tg.mean(tg.mul(T("x", [256, 96]), T("y", [96])), -1, keepDims=True), {"x": x, "y": y})
    def square_sum():
        xx = T("x", [256, 96])
        return tg.sum(tg.mul(xx, xx), -1)
    run(ctx, square_sum, {"x": x})
    run(ctx, lambda: tg.sumToShape(tg.mulScalar(T("x", [256, 96]), 0.5), [96]), {"x": x})
    big = rnd([4096, 96], 74)
    run(ctx, lambda: tg.sumToShape(tg.mul(T("b", [4096, 96]), T("y", [96])), [1, 96]), {"b": big, "y": y})

    def shared():
        mm = T("m", [256, 1])
        c = tg.sub(T("x", [256, 96]), mm)
        return tg.add(tg.mul(c, c), tg.div(c, tg.sqrt(tg.addScalar(mm, 3.0))))
    run(ctx, shared, {"x": x, "m": np.abs(m)})


@pytest.mark.parametrize("view", ["row", "flat"])
def test_row_result_broadcast_along_columns(ctx, view):
    """A [64, 1] row sum (and a row mean) reshaped to [1, 64] or [64]
    broadcasts along columns: element (r, j) uses the value of row j."""
    x, p = rnd([64, 64], 71), rnd([64, 64], 72)
    shp = [1, 64] if view == "row" else [64]

    def build_sum():
        X, P = T("x", [64, 64]), T("p", [64, 64])
        s = tg.reshape(tg.sum(tg.mul(X, P), -1, keepDims=True), shp)
        return tg.mulScalar(tg.mul(tg.sub(X, s), P), 0.5)

    def build_mean():
        X = T("x", [64, 64])
        d = tg.sub(X, tg.reshape(tg.mean(X, -1, keepDims=True), shp))
        return tg.mean(tg.mul(d, d), -1)
    run(ctx, build_sum, {"x": x, "p": p})
    run(ctx, build_mean, {"x": x})
