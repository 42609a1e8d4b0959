"""User-facing op surface: builds IR, no numeric work (src/ops.ts:1-1197).

Function names, argument order and composite lowerings follow the reference
one-to-one, because the composites decide which IR ops the backend sees:
``gelu`` through ``erf`` (src/ops.ts:319-327), ``softmax = exp(logSoftmax)``
(:709-711), ``mean()`` as ``mulScalar(sum_last(reshape))`` (:405-412),
non-last axes through ``permute`` (:428-457, :715-749), ``embedding`` as
``oneHot @ table`` (:626-635), ``concat`` chained at 7 inputs (:788-816),
dropout/randn/categorical salts (:191-287).
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple, Union

from .ir import Tensor, add_op, capture_site, shape_size
from . import shape as S
from .shape import ShapeError, show
from .trace import current_graph, tensor_input

Num = Union[int, float]
PRNG_SEED_INPUT = "__prngSeed"


def _binop(name: str, kind: str, a: Tensor, b: Tensor, out_dtype: Optional[str] = None) -> Tensor:
    site = capture_site(name)
    if a.dtype != b.dtype:
        raise ShapeError(f"{name}: dtype mismatch ({a.dtype} vs {b.dtype})", site)
    out = S.infer_binop(name, a.shape, b.shape, site)
    return add_op(current_graph(), kind, out, out_dtype or a.dtype, site, {"a": a.id, "b": b.id})


def _num(x) -> bool:
    return isinstance(x, (int, float)) and not isinstance(x, bool)


def add(a, b) -> Tensor:
    if _num(a):
        return addScalar(b, a)
    if _num(b):
        return addScalar(a, b)
    return _binop("add", "add", a, b)


def sub(a, b) -> Tensor:
    if _num(b):
        return addScalar(a, -b)
    if _num(a):
        return _binop("sub", "sub", constScalar(a, b.dtype), b)
    return _binop("sub", "sub", a, b)


def mul(a, b) -> Tensor:
    if _num(a):
        return mulScalar(b, a)
    if _num(b):
        return mulScalar(a, b)
    return _binop("mul", "mul", a, b)


def div(a, b) -> Tensor:
    if _num(b):
        if b == 0:
            raise ShapeError("div: scalar divisor cannot be zero", capture_site("div"))
        return mulScalar(a, 1 / b)
    if _num(a):
        return _binop("div", "div", constScalar(a, b.dtype), b)
    return _binop("div", "div", a, b)


def min(a, b) -> Tensor:  # noqa: A001 - mirrors the reference's name
    if _num(a):
        return min(b, a)
    rhs = constScalar(b, a.dtype) if _num(b) else b
    return _binop("min", "min", a, rhs)


def max(a, b) -> Tensor:  # noqa: A001
    if _num(a):
        return max(b, a)
    rhs = constScalar(b, a.dtype) if _num(b) else b
    return _binop("max", "max", a, rhs)


def clamp(a: Tensor, lo: Num, hi: Num) -> Tensor:
    return min(max(a, lo), hi)


def mulScalar(a: Tensor, scalar: Num) -> Tensor:
    return add_op(current_graph(), "mul_scalar", a.shape, a.dtype, capture_site("mulScalar"),
                  {"a": a.id, "scalar": float(scalar)})


def addScalar(a: Tensor, scalar: Num) -> Tensor:
    return add_op(current_graph(), "add_scalar", a.shape, a.dtype, capture_site("addScalar"),
                  {"a": a.id, "scalar": float(scalar)})


def _unary(name: str, a: Tensor) -> Tensor:
    site = capture_site(name)
    if a.dtype != "f32":
        raise ShapeError(f"{name}: requires f32, got {a.dtype}", site)
    return add_op(current_graph(), name, a.shape, "f32", site, {"a": a.id})


def sqrt(a): return _unary("sqrt", a)
def rsqrt(a): return _unary("rsqrt", a)
def log(a): return _unary("log", a)
def exp(a): return _unary("exp", a)
def relu(a): return _unary("relu", a)
def neg(a): return _unary("neg", a)
def abs(a): return _unary("abs", a)  # noqa: A001
def tanh(a): return _unary("tanh", a)
def sigmoid(a): return _unary("sigmoid", a)
def erf(a): return _unary("erf", a)
def sin(a): return _unary("sin", a)
def cos(a): return _unary("cos", a)


def square(a: Tensor) -> Tensor:
    return mul(a, a)


def stopGradient(a: Tensor) -> Tensor:
    return add_op(current_graph(), "stop_gradient", a.shape, a.dtype, capture_site("stopGradient"),
                  {"a": a.id})


def silu(a: Tensor) -> Tensor:
    return mul(a, sigmoid(a))


def _find_or_create_seed(g) -> Tensor:
    for op in g.ops:
        if op["kind"] == "tensor_input" and op["name"] == PRNG_SEED_INPUT:
            return g.tensors[op["out"]]
    return tensor_input(PRNG_SEED_INPUT, [], "i32")


def _count_stochastic(g) -> int:
    n = 0
    for op in g.ops:
        if op["kind"] in ("dropout", "randn", "categorical_last"):
            n += 1
    return n


def dropout(x: Tensor, p: float) -> Tensor:
    """Inverted dropout with a per-call salt and the shared per-step seed."""
    if p == 0:
        return x
    site = capture_site("dropout")
    if p < 0 or p >= 1:
        raise ShapeError(f"dropout: p must be in [0, 1), got {p}", site)
    if x.dtype != "f32":
        raise ShapeError(f"dropout: requires f32, got {x.dtype}", site)
    g = current_graph()
    seed = _find_or_create_seed(g)
    salt = _count_stochastic(g)
    return add_op(g, "dropout", x.shape, "f32", site, {"a": x.id, "seed": seed.id, "p": float(p), "salt": salt})


def randn(shape: Sequence[int]) -> Tensor:
    site = capture_site("randn")
    for d in shape:
        if not isinstance(d, int) or d <= 0:
            raise ShapeError(f"randn: shape must be positive integers, got {show(shape)}", site)
    g = current_graph()
    seed = _find_or_create_seed(g)
    salt = _count_stochastic(g)
    return add_op(g, "randn", shape, "f32", site, {"seed": seed.id, "salt": salt, "shape": list(shape)})


def dropoutWithSalt(dy: Tensor, p: float, salt: int, seed_id: int) -> Tensor:
    return add_op(current_graph(), "dropout", dy.shape, "f32", capture_site("dropout"),
                  {"a": dy.id, "seed": seed_id, "p": float(p), "salt": salt})


def _categorical_last(a: Tensor) -> Tensor:
    site = capture_site("categorical")
    if a.dtype != "f32":
        raise ShapeError(f"categorical: requires f32 logits, got {a.dtype}", site)
    out = S.infer_sum_last("categorical", a.shape, site)
    g = current_graph()
    seed = _find_or_create_seed(g)
    salt = _count_stochastic(g)
    return add_op(g, "categorical_last", out, "i32", site, {"a": a.id, "seed": seed.id, "salt": salt})


def categorical(logits: Tensor, axis: int = -1) -> Tensor:
    return _axis_reducing(logits, axis, "categorical", _categorical_last)


def gelu(a: Tensor, approximate: str = "none") -> Tensor:
    if approximate == "tanh":
        c = 0.7978845608028654
        x3 = mul(mul(a, a), a)
        inner = mul(add(a, mul(x3, 0.044715)), c)
        return mul(mul(a, 0.5), add(tanh(inner), 1))
    return mul(mul(a, 0.5), add(erf(mul(a, 1 / math.sqrt(2))), 1))


def leakyRelu(a: Tensor, alpha: float = 0.01) -> Tensor:
    return where(greater(a, 0), a, mul(a, alpha))


def softplus(a: Tensor) -> Tensor:
    return add(max(a, 0), log(add(exp(neg(abs(a))), 1)))


# ---- reductions ---------------------------------------------------------

def _mean_last(a: Tensor) -> Tensor:
    site = capture_site("mean")
    if a.dtype != "f32":
        raise ShapeError(f"mean: requires f32, got {a.dtype}", site)
    return add_op(current_graph(), "mean_last", S.infer_mean_last("mean", a.shape, site), a.dtype, site, {"a": a.id})


def _sum_last(a: Tensor) -> Tensor:
    site = capture_site("sum")
    if a.dtype != "f32":
        raise ShapeError(f"sum: requires f32, got {a.dtype}", site)
    return add_op(current_graph(), "sum_last", S.infer_sum_last("sum", a.shape, site), a.dtype, site, {"a": a.id})


def _argmax_last(a: Tensor) -> Tensor:
    site = capture_site("argmax")
    if a.dtype != "f32":
        raise ShapeError(f"argmax: requires f32, got {a.dtype}", site)
    return add_op(current_graph(), "argmax_last", S.infer_sum_last("argmax", a.shape, site), "i32", site, {"a": a.id})


def argmax(a: Tensor, axis: Optional[int] = None) -> Tensor:
    if axis is None:
        return _argmax_last(reshape(a, [-1]))
    return _axis_reducing(a, axis, "argmax", _argmax_last)


def argmin(a: Tensor, axis: Optional[int] = None) -> Tensor:
    return argmax(neg(a), axis)


def mean(a: Tensor, axis: Optional[int] = None, keepDims: bool = False) -> Tensor:
    if axis is None:
        n = shape_size(a.shape)
        if n == 0:
            raise ShapeError("mean: cannot mean over zero elements", capture_site("mean"))
        return mulScalar(_sum_last(reshape(a, [-1])), 1 / n)
    return _reduce_axis(a, axis, keepDims, "mean")


def sum(a: Tensor, axis: Optional[int] = None, keepDims: bool = False) -> Tensor:  # noqa: A001
    if axis is None:
        return _sum_last(reshape(a, [-1]))
    return _reduce_axis(a, axis, keepDims, "sum")


def _back_perm(k: int, r: int) -> List[int]:
    return list(range(k)) + [r - 1] + list(range(k, r - 1))


def _reduce_axis(a: Tensor, axis_arg: int, keep: bool, kind: str) -> Tensor:
    r = len(a.shape)
    k = r + axis_arg if axis_arg < 0 else axis_arg
    if k < 0 or k >= r:
        raise ShapeError(f"{kind}: axis {axis_arg} out of range for shape {show(a.shape)}", capture_site(kind))
    is_last = k == r - 1
    inp = a if is_last else permute(a, [i for i in range(r) if i != k] + [k])
    if kind == "mean":
        red = _mean_last(inp)
        if is_last:
            return red if keep else reshape(red, red.shape[:-1])
        if not keep:
            return reshape(red, red.shape[:-1])
        return permute(red, _back_perm(k, r))
    dropped = _sum_last(inp)
    if is_last:
        return reshape(dropped, list(dropped.shape) + [1]) if keep else dropped
    if not keep:
        return dropped
    return permute(reshape(dropped, list(dropped.shape) + [1]), _back_perm(k, r))


# ---- shape ops ----------------------------------------------------------

def reshape(a: Tensor, new_shape: Sequence[int]) -> Tensor:
    site = capture_site("reshape")
    out = S.infer_reshape("reshape", a.shape, list(new_shape), site)
    return add_op(current_graph(), "reshape", out, a.dtype, site, {"a": a.id, "newShape": list(out)})


def permute(a: Tensor, perm: Sequence[int]) -> Tensor:
    site = capture_site("permute")
    out = S.infer_permute("permute", a.shape, list(perm), site)
    return add_op(current_graph(), "permute", out, a.dtype, site, {"a": a.id, "perm": list(perm)})


def swapAxes(a: Tensor, axis1: int, axis2: int) -> Tensor:
    r = len(a.shape)
    i1 = r + axis1 if axis1 < 0 else axis1
    i2 = r + axis2 if axis2 < 0 else axis2
    site = capture_site("swapAxes")
    if not (0 <= i1 < r and 0 <= i2 < r):
        raise ShapeError(f"swapAxes: axis out of range — got ({axis1}, {axis2}) for rank-{r} tensor", site)
    if i1 == i2:
        return a
    perm = list(range(r))
    perm[i1], perm[i2] = i2, i1
    return permute(a, perm)


def matmul(a: Tensor, b: Tensor) -> Tensor:
    site = capture_site("matmul")
    if a.dtype != "f32" or b.dtype != "f32":
        raise ShapeError(f"matmul: requires f32, got {a.dtype} and {b.dtype}", site)
    if len(a.shape) < 2:
        raise ShapeError(f"matmul: lhs must have rank >= 2, got {show(a.shape)}", site)
    if len(b.shape) < 2:
        raise ShapeError(f"matmul: rhs must have rank >= 2, got {show(b.shape)}", site)
    if len(b.shape) == 2:
        return add_op(current_graph(), "matmul", S.infer_matmul("matmul", a.shape, b.shape, site), "f32",
                      site, {"a": a.id, "b": b.id})
    if len(a.shape) != len(b.shape):
        raise ShapeError(f"matmul: rank mismatch — lhs {show(a.shape)} vs rhs {show(b.shape)}. When rhs "
                         f"is batched (rank > 2), lhs must have the same rank. Reshape explicitly if needed.", site)
    return add_op(current_graph(), "matmul_batched", S.infer_matmul_batched("matmul", a.shape, b.shape, site),
                  "f32", site, {"a": a.id, "b": b.id})


def oneHot(indices: Tensor, depth: int, dtype: str = "f32") -> Tensor:
    site = capture_site("oneHot")
    if indices.dtype != "i32":
        raise ShapeError(f"oneHot: indices must be i32, got {indices.dtype}", site)
    if depth <= 0:
        raise ShapeError(f"oneHot: depth must be positive, got {depth}", site)
    return add_op(current_graph(), "one_hot", tuple(indices.shape) + (depth,), dtype, site,
                  {"indices": indices.id, "depth": depth, "dtype": dtype})


def takeAlongAxis(inp: Tensor, indices: Tensor, axis: int) -> Tensor:
    site = capture_site("takeAlongAxis")
    if inp.dtype != "f32":
        raise ShapeError(f"takeAlongAxis: input must be f32, got {inp.dtype}", site)
    if indices.dtype != "i32":
        raise ShapeError(f"takeAlongAxis: indices must be i32, got {indices.dtype}", site)
    n = len(inp.shape)
    if len(indices.shape) != n:
        raise ShapeError("takeAlongAxis: input and indices must have the same rank", site)
    k = n + axis if axis < 0 else axis
    if k < 0 or k >= n:
        raise ShapeError(f"takeAlongAxis: axis {axis} out of range for rank-{n} input", site)
    for i in range(n):
        if i != k and inp.shape[i] != indices.shape[i]:
            raise ShapeError("takeAlongAxis: input and indices must match on every axis except the gather axis", site)
    perm = [i for i in range(n) if i != k] + [k]
    permuted = permute(inp, perm)
    sa = inp.shape[k]
    expanded = reshape(permuted, [1 if i == k else inp.shape[i] for i in range(n)] + [sa])
    oh = oneHot(indices, sa, "f32")
    return sum(mul(expanded, oh), -1)


def embedding(table: Tensor, indices: Tensor) -> Tensor:
    site = capture_site("embedding")
    if len(table.shape) != 2:
        raise ShapeError(f"embedding: table must be 2-d [vocab, dim], got {show(table.shape)}", site)
    if indices.dtype != "i32":
        raise ShapeError(f"embedding: indices must be i32, got {indices.dtype}", site)
    return matmul(oneHot(indices, table.shape[0], "f32"), table)


def arange(n: int, dtype: str = "i32") -> Tensor:
    site = capture_site("arange")
    if not isinstance(n, int) or n <= 0:
        raise ShapeError(f"arange: n must be a positive integer, got {n}", site)
    return add_op(current_graph(), "arange", (n,), dtype, site, {"n": n, "dtype": dtype})


def _const_fill(name: str, shape, dtype: str, value: float) -> Tensor:
    site = capture_site(name)
    for d in shape:
        if not isinstance(d, int) or d <= 0:
            raise ShapeError(f"{name}: shape must be positive integers, got {show(shape)}", site)
    return add_op(current_graph(), "const_fill", shape, dtype, site, {"value": value, "dtype": dtype})


def zeros(shape, dtype: str = "f32") -> Tensor:
    return _const_fill("zeros", shape, dtype, 0)


def ones(shape, dtype: str = "f32") -> Tensor:
    return _const_fill("ones", shape, dtype, 1)


# ---- ML primitives ------------------------------------------------------

def _softmax_causal_last(a: Tensor) -> Tensor:
    site = capture_site("softmaxCausal")
    if a.dtype != "f32":
        raise ShapeError(f"softmaxCausal: requires f32, got {a.dtype}", site)
    S.infer_where_causal("softmaxCausal", a.shape, site)
    return add_op(current_graph(), "softmax_causal_last", a.shape, "f32", site, {"a": a.id})


def softmaxCausal(a: Tensor, axis: int = -1) -> Tensor:
    return _axis_preserving(a, axis, "softmaxCausal", _softmax_causal_last)


def _log_softmax_last(a: Tensor) -> Tensor:
    site = capture_site("logSoftmax")
    if a.dtype != "f32":
        raise ShapeError(f"logSoftmax: requires f32, got {a.dtype}", site)
    return add_op(current_graph(), "log_softmax_last", a.shape, "f32", site, {"a": a.id})


def logSoftmax(a: Tensor, axis: int = -1) -> Tensor:
    return _axis_preserving(a, axis, "logSoftmax", _log_softmax_last)


def softmax(a: Tensor, axis: int = -1) -> Tensor:
    return exp(logSoftmax(a, axis))


def _axis_preserving(a: Tensor, axis_arg: int, name: str, fn) -> Tensor:
    r = len(a.shape)
    if r == 0:
        raise ShapeError(f"{name}: cannot apply to 0-d tensor", capture_site(name))
    k = r + axis_arg if axis_arg < 0 else axis_arg
    if k < 0 or k >= r:
        raise ShapeError(f"{name}: axis {axis_arg} out of range for shape {show(a.shape)}", capture_site(name))
    if k == r - 1:
        return fn(a)
    perm = [i for i in range(r) if i != k] + [k]
    return permute(fn(permute(a, perm)), _back_perm(k, r))


def _axis_reducing(a: Tensor, axis_arg: int, name: str, fn) -> Tensor:
    r = len(a.shape)
    if r == 0:
        raise ShapeError(f"{name}: cannot reduce a 0-d tensor", capture_site(name))
    k = r + axis_arg if axis_arg < 0 else axis_arg
    if k < 0 or k >= r:
        raise ShapeError(f"{name}: axis {axis_arg} out of range for shape {show(a.shape)}", capture_site(name))
    if k == r - 1:
        return fn(a)
    return fn(permute(a, [i for i in range(r) if i != k] + [k]))


def whereCausal(a: Tensor, fillValue: float) -> Tensor:
    site = capture_site("whereCausal")
    if a.dtype != "f32":
        raise ShapeError(f"whereCausal: requires f32, got {a.dtype}", site)
    S.infer_where_causal("whereCausal", a.shape, site)
    return add_op(current_graph(), "where_causal", a.shape, "f32", site, {"a": a.id, "fillValue": float(fillValue)})


def narrow(a: Tensor, axis: int, start: int, length: int) -> Tensor:
    site = capture_site("narrow")
    ax = len(a.shape) + axis if axis < 0 else axis
    end = start + length
    out = S.infer_slice_range("narrow", a.shape, ax, start, end, site)
    return add_op(current_graph(), "slice_range", out, a.dtype, site, {"a": a.id, "axis": ax, "start": start, "end": end})


def scatterAxis(a: Tensor, out_shape, axis: int, start: int, end: int) -> Tensor:
    site = capture_site("scatterAxis")
    out = S.infer_scatter_axis("scatterAxis", a.shape, tuple(out_shape), axis, start, end, site)
    return add_op(current_graph(), "scatter_axis", out, a.dtype, site,
                  {"a": a.id, "outShape": list(out_shape), "axis": axis, "start": start, "end": end})


CONCAT_INPUT_CAP = 7


def concat(tensors: Sequence[Tensor], axis: int) -> Tensor:
    site = capture_site("concat")
    if len(tensors) == 0:
        raise ShapeError("concat: needs at least one input", site)
    if len(tensors) == 1:
        return tensors[0]
    dt = tensors[0].dtype
    for t in tensors:
        if t.dtype != dt:
            raise ShapeError(f"concat: dtype mismatch ({dt} vs {t.dtype})", site)
    ax = len(tensors[0].shape) + axis if axis < 0 else axis
    layer = list(tensors)
    while len(layer) > CONCAT_INPUT_CAP:
        nxt = []
        for i in range(0, len(layer), CONCAT_INPUT_CAP):
            chunk = layer[i:i + CONCAT_INPUT_CAP]
            nxt.append(chunk[0] if len(chunk) == 1 else _concat_one(chunk, ax, site))
        layer = nxt
    return _concat_one(layer, ax, site)


def _concat_one(ts, ax, site) -> Tensor:
    out = S.infer_concat("concat", [t.shape for t in ts], ax, site)
    return add_op(current_graph(), "concat", out, ts[0].dtype, site, {"inputs": [t.id for t in ts], "axis": ax})


def stack(tensors: Sequence[Tensor], axis: int) -> Tensor:
    if not tensors:
        raise ShapeError("stack: needs at least one input", capture_site("stack"))
    t0 = tensors[0]
    ax = len(t0.shape) + 1 + axis if axis < 0 else axis
    ns = list(t0.shape[:ax]) + [1] + list(t0.shape[ax:])
    return concat([reshape(t, ns) for t in tensors], ax)


def splitHeads(x: Tensor, nHeads: int) -> Tensor:
    site = capture_site("splitHeads")
    r = len(x.shape)
    if r < 2:
        raise ShapeError(f"splitHeads: requires rank >= 2, got {r}", site)
    T, D = x.shape[-2], x.shape[-1]
    if D % nHeads:
        raise ShapeError(f"splitHeads: last dim {D} not divisible by nHeads {nHeads}", site)
    lead = list(x.shape[:-2])
    rs = reshape(x, lead + [T, nHeads, D // nHeads])
    return swapAxes(rs, len(lead), len(lead) + 1)


def mergeHeads(x: Tensor) -> Tensor:
    site = capture_site("mergeHeads")
    r = len(x.shape)
    if r < 3:
        raise ShapeError(f"mergeHeads: requires rank >= 3, got {r}", site)
    H, T, d = x.shape[-3], x.shape[-2], x.shape[-1]
    lead = list(x.shape[:-3])
    return reshape(swapAxes(x, r - 3, r - 2), lead + [T, H * d])


def split(t: Tensor, sizes: Sequence[int], axis: int) -> List[Tensor]:
    site = capture_site("split")
    ax = len(t.shape) + axis if axis < 0 else axis
    if ax < 0 or ax >= len(t.shape):
        raise ShapeError(f"split: axis {axis} out of range", site)
    total = 0
    for s in sizes:
        total += s
    if total != t.shape[ax]:
        raise ShapeError(f"split: sizes sum to {total}, but axis {ax} has size {t.shape[ax]}", site)
    out, cur = [], 0
    for s in sizes:
        out.append(narrow(t, ax, cur, s))
        cur += s
    return out


def rope(q: Tensor, k: Tensor, base: float = 10000) -> Tuple[Tensor, Tensor]:
    site = capture_site("rope")
    if q.dtype != "f32" or k.dtype != "f32":
        raise ShapeError("rope: q and k must be f32", site)
    if len(q.shape) < 2 or len(k.shape) < 2:
        raise ShapeError("rope: q and k require rank >= 2", site)
    T, D = q.shape[-2], q.shape[-1]
    if k.shape[-2] != T or k.shape[-1] != D:
        raise ShapeError("rope: q and k must share sequence and feature dims", site)
    if D % 2:
        raise ShapeError(f"rope: rotation dim must be even (rotates pairs), got {D}", site)
    half = D // 2
    idx = arange(half, "f32")
    freqs = exp(mul(idx, -math.log(base) / half))
    positions = arange(T, "f32")
    angles = mul(reshape(positions, [T, 1]), reshape(freqs, [1, half]))
    cos_h, sin_h = cos(angles), sin(angles)
    cos_f = concat([cos_h, cos_h], -1)
    sin_f = concat([sin_h, sin_h], -1)

    def rot(x):
        x1, x2 = split(x, [half, half], -1)
        rotated = concat([neg(x2), x1], -1)
        return add(mul(x, cos_f), mul(rotated, sin_f))
    return rot(q), rot(k)


def broadcastTo(a: Tensor, target) -> Tensor:
    site = capture_site("broadcastTo")
    S.infer_broadcast_to("broadcastTo", a.shape, tuple(target), site)
    return add_op(current_graph(), "broadcast_to", tuple(target), a.dtype, site, {"a": a.id, "targetShape": list(target)})


def sumToShape(a: Tensor, target) -> Tensor:
    site = capture_site("sumToShape")
    S.infer_sum_to_shape("sumToShape", a.shape, tuple(target), site)
    return add_op(current_graph(), "sum_to_shape", tuple(target), a.dtype, site, {"a": a.id, "targetShape": list(target)})


def constScalar(value: Num, dtype: str = "f32") -> Tensor:
    return add_op(current_graph(), "const_scalar", (), dtype, capture_site("constScalar"), {"value": float(value), "dtype": dtype})


def less(a, b) -> Tensor:
    if _num(a):
        return greater(b, a)
    rhs = constScalar(b, a.dtype) if _num(b) else b
    return _binop("less", "less", a, rhs, "bool")


def greater(a, b) -> Tensor:
    if _num(a):
        return less(b, a)
    rhs = constScalar(b, a.dtype) if _num(b) else b
    return _binop("greater", "greater", a, rhs, "bool")


def where(cond: Tensor, a: Tensor, b: Tensor) -> Tensor:
    site = capture_site("where")
    if cond.dtype != "bool":
        raise ShapeError(f"where: cond must be bool, got {cond.dtype}", site)
    if a.dtype != b.dtype:
        raise ShapeError(f"where: a/b dtype mismatch ({a.dtype} vs {b.dtype})", site)
    out = S.infer_where("where", cond.shape, a.shape, b.shape, site)
    return add_op(current_graph(), "where", out, a.dtype, site, {"cond": cond.id, "a": a.id, "b": b.id})


def reluGrad(x: Tensor, dy: Tensor) -> Tensor:
    site = capture_site("reluGrad")
    if x.shape != dy.shape:
        raise ShapeError(f"reluGrad: x and dy must have matching shapes, got {show(x.shape)} and {show(dy.shape)}", site)
    return add_op(current_graph(), "relu_grad", x.shape, "f32", site, {"x": x.id, "dy": dy.id})


def adamUpdateM(m: Tensor, g: Tensor, beta1: float) -> Tensor:
    site = capture_site("adamUpdateM")
    if m.shape != g.shape:
        raise ShapeError("adamUpdateM: shape mismatch", site)
    return add_op(current_graph(), "adam_update_m", m.shape, "f32", site, {"m": m.id, "g": g.id, "beta1": float(beta1)})


def adamUpdateV(v: Tensor, g: Tensor, beta2: float) -> Tensor:
    site = capture_site("adamUpdateV")
    if v.shape != g.shape:
        raise ShapeError("adamUpdateV: shape mismatch", site)
    return add_op(current_graph(), "adam_update_v", v.shape, "f32", site, {"v": v.id, "g": g.id, "beta2": float(beta2)})


def adamUpdateP(p: Tensor, mNew: Tensor, vNew: Tensor, lrt: Tensor, eps: float, decayShrink=1) -> Tensor:
    site = capture_site("adamUpdateP")
    if lrt.dtype != "f32" or len(lrt.shape) != 0:
        raise ShapeError("adamUpdateP: lrt must be a 0-d f32 scalar", site)
    if p.shape != mNew.shape:
        raise ShapeError("adamUpdateP: p/mNew shape mismatch", site)
    is_t = isinstance(decayShrink, Tensor)
    return add_op(current_graph(), "adam_update_p", p.shape, "f32", site, {
        "p": p.id, "mNew": mNew.id, "vNew": vNew.id, "lrt": lrt.id, "eps": float(eps),
        "decayShrink": 1.0 if is_t else float(decayShrink),
        "decayShrinkTensor": decayShrink.id if is_t else None})


def _pair(v, default) -> Tuple[int, int]:
    if v is None:
        return (default, default)
    if isinstance(v, int):
        return (v, v)
    return (int(v[0]), int(v[1]))


def conv2d(inp: Tensor, weight: Tensor, stride=None, padding=None, groups: int = 1) -> Tensor:
    site = capture_site("conv2d")
    if inp.dtype != "f32" or weight.dtype != "f32":
        raise ShapeError("conv2d: input and weight must be f32", site)
    sh, sw = _pair(stride, 1)
    ph, pw = _pair(padding, 0)
    out = S.infer_conv2d("conv2d", inp.shape, weight.shape, sh, sw, ph, pw, groups, site)
    return add_op(current_graph(), "conv2d", out, "f32", site, {
        "input": inp.id, "weight": weight.id, "strideH": sh, "strideW": sw, "padH": ph, "padW": pw, "groups": groups})


def conv2dInputGrad(weight, dy, inH, inW, strideH, strideW, padH, padW, groups) -> Tensor:
    site = capture_site("conv2dInputGrad")
    cout, wic = weight.shape[0], weight.shape[1]
    if dy.shape[1] != cout:
        raise ShapeError(f"conv2dInputGrad: dy's C={dy.shape[1]} doesn't match weight C_out={cout}", site)
    return add_op(current_graph(), "conv2d_input_grad", (dy.shape[0], wic * groups, inH, inW), "f32", site, {
        "weight": weight.id, "dy": dy.id, "inH": inH, "inW": inW, "strideH": strideH, "strideW": strideW,
        "padH": padH, "padW": padW, "groups": groups})


def conv2dWeightGrad(inp, dy, kH, kW, strideH, strideW, padH, padW, groups) -> Tensor:
    site = capture_site("conv2dWeightGrad")
    return add_op(current_graph(), "conv2d_weight_grad", (dy.shape[1], inp.shape[1] // groups, kH, kW), "f32", site, {
        "input": inp.id, "dy": dy.id, "kH": kH, "kW": kW, "strideH": strideH, "strideW": strideW,
        "padH": padH, "padW": padW, "groups": groups})


def maxPool2d(inp: Tensor, kernelSize, stride=None, padding=None) -> Tensor:
    site = capture_site("maxPool2d")
    if inp.dtype != "f32":
        raise ShapeError(f"maxPool2d: input must be f32, got {inp.dtype}", site)
    kh, kw = _pair(kernelSize, 1)
    sh, sw = (kh, kw) if stride is None else _pair(stride, 1)
    ph, pw = _pair(padding, 0)
    out = S.infer_max_pool2d("maxPool2d", inp.shape, kh, kw, sh, sw, ph, pw, site)
    return add_op(current_graph(), "max_pool_2d", out, "f32", site, {
        "input": inp.id, "kH": kh, "kW": kw, "strideH": sh, "strideW": sw, "padH": ph, "padW": pw})


def maxPool2dGrad(inp, dy, kH, kW, strideH, strideW, padH, padW) -> Tensor:
    return add_op(current_graph(), "max_pool_2d_grad", inp.shape, "f32", capture_site("maxPool2dGrad"), {
        "input": inp.id, "dy": dy.id, "kH": kH, "kW": kW, "strideH": strideH, "strideW": strideW,
        "padH": padH, "padW": padW})


def nearestUpsample2d(x: Tensor, factor: int) -> Tensor:
    site = capture_site("nearestUpsample2d")
    if len(x.shape) != 4:
        raise ShapeError(f"nearestUpsample2d: input must be rank-4 [B, C, H, W], got {show(x.shape)}", site)
    if not isinstance(factor, int) or factor < 1:
        raise ShapeError(f"nearestUpsample2d: factor must be a positive integer, got {factor}", site)
    if factor == 1:
        return x
    B, C, H, W = x.shape
    e = broadcastTo(reshape(x, [B, C, H, 1, W, 1]), [B, C, H, factor, W, factor])
    return reshape(e, [B, C, H * factor, W * factor])
