"""Reverse-mode autograd appended into the traced graph (src/grad.ts:1-563).

One adjoint rule per op kind, each expressed as forward-op calls so the
backward graph is ordinary IR. Cotangents accumulate with ``add`` in arrival
order (src/grad.ts:175-182), so the traced graph matches the reference's op
for op.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Optional

from . import ops as O
from .ir import Graph, Tensor
from .shape import shapes_equal
from .trace import trace_into


class GradResult:
    def __init__(self, graph: Graph, param_grads: Dict[str, Tensor], loss: Tensor):
        self.graph = graph
        self.paramGrads = param_grads
        self.loss = loss


def appendGrad(graph: Graph) -> GradResult:
    if len(graph.outputs) != 1:
        raise RuntimeError(f"autograd: expected graph with exactly 1 output (the loss); got {len(graph.outputs)}")
    loss_id = graph.outputs[0]
    loss_t = graph.tensors[loss_id]
    if len(loss_t.shape) != 0:
        raise RuntimeError(f"autograd: loss must be a rank-0 scalar; got shape {list(loss_t.shape)}.")
    n_fwd = len(graph.ops)
    fwd_ops = graph.ops[:n_fwd]
    cot: Dict[int, Tensor] = {}

    def body():
        cot[loss_id] = O.constScalar(1.0, "f32")
        for i in range(n_fwd - 1, -1, -1):
            op = fwd_ops[i]
            oc = cot.get(op["out"])
            if oc is None:
                continue
            _adjoint(op, oc, graph, cot)
        grads: Dict[str, Tensor] = {}
        for op in fwd_ops:
            if op["kind"] != "param_input":
                continue
            c = cot.get(op["out"])
            if c is None:
                t = graph.tensors[op["out"]]
                grads[op["name"]] = O.broadcastTo(O.constScalar(0.0, t.dtype), t.shape)
            else:
                grads[op["name"]] = c
        return GradResult(graph, grads, loss_t)
    return trace_into(graph, body)


def appendGradClip(graph: Graph, param_grads: Dict[str, Tensor], max_norm: float) -> Dict[str, Tensor]:
    """Global L2-norm clip: scale = min(1, maxNorm/(norm+1e-6)) (src/grad.ts:110-130)."""
    def body():
        entries = list(param_grads.items())
        if not entries:
            return param_grads
        s = O.sum(O.mul(entries[0][1], entries[0][1]))
        for _, g in entries[1:]:
            s = O.add(s, O.sum(O.mul(g, g)))
        scale = O.min(O.div(O.constScalar(max_norm, "f32"), O.add(O.sqrt(s), 1e-6)), 1)
        return {n: O.mul(g, O.broadcastTo(scale, g.shape)) for n, g in entries}
    return trace_into(graph, body)


def appendGradNormalize(graph: Graph, param_grads: Dict[str, Tensor],
                        filt: Optional[Callable[[str], bool]] = None) -> Dict[str, Tensor]:
    """Per-param g / (||g|| + 1e-8) (src/grad.ts:148-172)."""
    def body():
        out, matched = {}, 0
        for n, g in param_grads.items():
            if filt is not None and not filt(n):
                out[n] = g
                continue
            matched += 1
            norm = O.add(O.sqrt(O.sum(O.mul(g, g))), 1e-8)
            out[n] = O.div(g, O.broadcastTo(norm, g.shape))
        if filt is not None and matched == 0 and param_grads:
            raise RuntimeError("normalizeGrads: the filter matched no parameters. Param names are property "
                               "paths like 'w1.W' — available: " + ", ".join(param_grads))
        return out
    return trace_into(graph, body)


def _acc(cot: Dict[int, Tensor], tid: int, c: Tensor) -> None:
    e = cot.get(tid)
    cot[tid] = O.add(e, c) if e is not None else c


def _unb(c: Tensor, shape) -> Tensor:
    return c if shapes_equal(c.shape, shape) else O.sumToShape(c, shape)


def _inv_perm(perm):
    inv = [0] * len(perm)
    for i, p in enumerate(perm):
        inv[p] = i
    return inv


def _adjoint(op: dict, oc: Tensor, graph: Graph, cot: Dict[int, Tensor]) -> None:
    T = graph.tensors
    k = op["kind"]
    if k in ("param_input", "tensor_input", "state_input", "arange", "const_scalar", "const_fill",
             "randn", "stop_gradient", "one_hot", "less", "greater", "argmax_last", "categorical_last"):
        return
    if k == "add":
        a, b = T[op["a"]], T[op["b"]]
        _acc(cot, op["a"], _unb(oc, a.shape))
        _acc(cot, op["b"], _unb(oc, b.shape))
    elif k == "sub":
        a, b = T[op["a"]], T[op["b"]]
        _acc(cot, op["a"], _unb(oc, a.shape))
        _acc(cot, op["b"], _unb(O.mulScalar(oc, -1), b.shape))
    elif k == "mul":
        a, b = T[op["a"]], T[op["b"]]
        _acc(cot, op["a"], _unb(O.mul(oc, b), a.shape))
        _acc(cot, op["b"], _unb(O.mul(oc, a), b.shape))
    elif k == "div":
        a, b = T[op["a"]], T[op["b"]]
        _acc(cot, op["a"], _unb(O.div(oc, b), a.shape))
        numer = O.mul(oc, a)
        bsq = O.mul(b, b)
        _acc(cot, op["b"], _unb(O.mulScalar(O.div(numer, bsq), -1), b.shape))
    elif k == "mul_scalar":
        _acc(cot, op["a"], O.mulScalar(oc, op["scalar"]))
    elif k == "add_scalar":
        _acc(cot, op["a"], oc)
    elif k == "sqrt":
        c = T[op["out"]]
        _acc(cot, op["a"], O.mulScalar(O.div(oc, c), 0.5))
    elif k == "rsqrt":
        c = T[op["out"]]
        c3 = O.mul(O.mul(c, c), c)
        _acc(cot, op["a"], O.mulScalar(O.mul(oc, c3), -0.5))
    elif k == "log":
        _acc(cot, op["a"], O.div(oc, T[op["a"]]))
    elif k == "exp":
        _acc(cot, op["a"], O.mul(oc, T[op["out"]]))
    elif k == "relu":
        _acc(cot, op["a"], O.reluGrad(T[op["a"]], oc))
    elif k == "neg":
        _acc(cot, op["a"], O.mulScalar(oc, -1))
    elif k == "abs":
        a = T[op["a"]]
        _acc(cot, op["a"], O.where(O.less(a, O.constScalar(0, "f32")), O.mulScalar(oc, -1), oc))
    elif k == "tanh":
        c = T[op["out"]]
        _acc(cot, op["a"], O.mul(oc, O.sub(O.constScalar(1, "f32"), O.mul(c, c))))
    elif k == "sigmoid":
        c = T[op["out"]]
        _acc(cot, op["a"], O.mul(oc, O.sub(c, O.mul(c, c))))
    elif k == "erf":
        a = T[op["a"]]
        d = O.mulScalar(O.exp(O.mulScalar(O.mul(a, a), -1)), 2 / math.sqrt(math.pi))
        _acc(cot, op["a"], O.mul(oc, d))
    elif k == "sin":
        _acc(cot, op["a"], O.mul(oc, O.cos(T[op["a"]])))
    elif k == "cos":
        _acc(cot, op["a"], O.mul(oc, O.mulScalar(O.sin(T[op["a"]]), -1)))
    elif k == "dropout":
        _acc(cot, op["a"], O.dropoutWithSalt(oc, op["p"], op["salt"], op["seed"]))
    elif k == "concat":
        cur = 0
        for iid in op["inputs"]:
            sz = T[iid].shape[op["axis"]]
            _acc(cot, iid, O.narrow(oc, op["axis"], cur, sz))
            cur += sz
    elif k == "slice_range":
        a = T[op["a"]]
        _acc(cot, op["a"], O.scatterAxis(oc, a.shape, op["axis"], op["start"], op["end"]))
    elif k in ("min", "max"):
        a, b = T[op["a"]], T[op["b"]]
        zero = O.constScalar(0, "f32")
        a_wins = O.less(a, b) if k == "min" else O.greater(a, b)
        _acc(cot, op["a"], _unb(O.where(a_wins, oc, O.broadcastTo(zero, oc.shape)), a.shape))
        _acc(cot, op["b"], _unb(O.where(a_wins, O.broadcastTo(zero, oc.shape), oc), b.shape))
    elif k == "mean_last":
        a = T[op["a"]]
        D = a.shape[-1]
        _acc(cot, op["a"], O.mulScalar(O.broadcastTo(oc, a.shape), 1 / D))
    elif k == "sum_last":
        a = T[op["a"]]
        _acc(cot, op["a"], O.broadcastTo(O.reshape(oc, list(oc.shape) + [1]), a.shape))
    elif k == "reshape":
        _acc(cot, op["a"], O.reshape(oc, T[op["a"]].shape))
    elif k == "permute":
        _acc(cot, op["a"], O.permute(oc, _inv_perm(op["perm"])))
    elif k == "matmul":
        a, b = T[op["a"]], T[op["b"]]
        _acc(cot, op["a"], O.matmul(oc, O.swapAxes(b, -1, -2)))
        K, N = a.shape[-1], b.shape[-1]
        rows = 1
        for d in a.shape[:-1]:
            rows *= d
        a2 = O.reshape(a, [rows, K])
        oc2 = O.reshape(oc, [rows, N])
        _acc(cot, op["b"], O.sumToShape(O.matmul(O.swapAxes(a2, -1, -2), oc2), b.shape))
    elif k == "matmul_batched":
        a, b = T[op["a"]], T[op["b"]]
        _acc(cot, op["a"], O.matmul(oc, O.swapAxes(b, -1, -2)))
        _acc(cot, op["b"], O.matmul(O.swapAxes(a, -1, -2), oc))
    elif k == "broadcast_to":
        _acc(cot, op["a"], O.sumToShape(oc, T[op["a"]].shape))
    elif k == "sum_to_shape":
        _acc(cot, op["a"], O.broadcastTo(oc, T[op["a"]].shape))
    elif k == "log_softmax_last":
        c = T[op["out"]]
        sm = O.exp(c)
        s_keep = O.sum(oc, -1, keepDims=True)
        term = O.mul(sm, O.broadcastTo(s_keep, c.shape))
        _acc(cot, op["a"], O.sub(oc, term))
    elif k == "softmax_causal_last":
        c = T[op["out"]]
        dcxc = O.mul(oc, c)
        s_keep = O.sum(dcxc, -1, keepDims=True)
        inner = O.sub(oc, O.broadcastTo(s_keep, c.shape))
        _acc(cot, op["a"], O.mul(inner, c))
    elif k == "where":
        a, b = T[op["a"]], T[op["b"]]
        cond = T[op["cond"]]
        za = O.broadcastTo(O.constScalar(0, a.dtype), oc.shape)
        zb = O.broadcastTo(O.constScalar(0, b.dtype), oc.shape)
        _acc(cot, op["a"], _unb(O.where(cond, oc, za), a.shape))
        _acc(cot, op["b"], _unb(O.where(cond, zb, oc), b.shape))
    elif k == "where_causal":
        _acc(cot, op["a"], O.whereCausal(oc, 0))
    elif k == "conv2d":
        x, w = T[op["input"]], T[op["weight"]]
        _acc(cot, op["input"], O.conv2dInputGrad(w, oc, x.shape[2], x.shape[3], op["strideH"], op["strideW"],
                                                 op["padH"], op["padW"], op["groups"]))
        _acc(cot, op["weight"], O.conv2dWeightGrad(x, oc, w.shape[2], w.shape[3], op["strideH"], op["strideW"],
                                                   op["padH"], op["padW"], op["groups"]))
    elif k == "max_pool_2d":
        x = T[op["input"]]
        _acc(cot, op["input"], O.maxPool2dGrad(x, oc, op["kH"], op["kW"], op["strideH"], op["strideW"],
                                               op["padH"], op["padW"]))
    elif k in ("adam_update_m", "adam_update_v", "adam_update_p"):
        raise RuntimeError(f"autograd: cannot differentiate through {k}")
    elif k in ("conv2d_input_grad", "conv2d_weight_grad", "max_pool_2d_grad", "scatter_axis"):
        raise RuntimeError(f"autograd: cannot differentiate through {k} (it's a backward op)")
    elif k == "relu_grad":
        raise RuntimeError("autograd: cannot take second-order gradient through relu_grad — "
                           "tensorgrad does not support higher-order autodiff.")
    else:
        raise RuntimeError(f"autograd: unhandled op kind {k}")
