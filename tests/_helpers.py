"""Shared test helpers: FD harness (restating test/_fdgrad.ts) and fixtures."""
from __future__ import annotations

import numpy as np

from oracle.evaluator import eval_graph
from tensorgrad_b200.grad import appendGrad
from tensorgrad_b200.ir import graph_to_wire
from tensorgrad_b200.module import Mulberry32
from tensorgrad_b200.trace import param_input, trace_fn


def make_range(shape) -> np.ndarray:
    """sin(i*0.1)*0.5 fixture (test/grad.ts:254-259)."""
    n = int(np.prod(shape))
    return (np.sin(np.arange(n) * 0.1) * 0.5).astype(np.float32).reshape(shape)


def random_buf(size: int, seed: int = 12345) -> np.ndarray:
    """mulberry32 draws in [-0.5, 0.5) (test/_fdgrad.ts:116-127)."""
    return (Mulberry32(seed).take(size) - 0.5).astype(np.float32)


def fd_check(shape, build, extra=None, eps=1e-3, atol=5e-3, rtol=5e-3, init=None):
    """Central-difference FD vs autograd on the oracle; fails only when both
    the absolute and relative worst errors exceed tolerance (test/_fdgrad.ts:44-110)."""
    extra = extra or {}
    g = trace_fn(lambda: build(param_input("w", list(shape))))
    gr = appendGrad(g)
    w = (init.astype(np.float32).reshape(-1).copy() if init is not None
         else random_buf(int(np.prod(shape))))
    wire = graph_to_wire(g)
    vals = eval_graph(wire, {"w": w.reshape(shape), **extra})
    auto = vals[gr.paramGrads["w"].id].reshape(-1).astype(np.float64)
    loss_id = g.outputs[0]
    fd = np.zeros(w.size)
    for i in range(w.size):
        o = w[i]
        w[i] = o + np.float32(eps)
        lp = float(eval_graph(wire, {"w": w.reshape(shape), **extra})[loss_id].reshape(-1)[0])
        w[i] = o - np.float32(eps)
        lm = float(eval_graph(wire, {"w": w.reshape(shape), **extra})[loss_id].reshape(-1)[0])
        w[i] = o
        fd[i] = (lp - lm) / (2 * eps)
    absd = np.abs(auto - fd)
    rel = absd / np.maximum(np.abs(fd), 1e-6)
    assert not (absd.max() > atol and rel.max() > rtol), (absd.max(), rel.max())
    return absd.max()
