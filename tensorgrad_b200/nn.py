"""Built-in layers and losses (src/nn.ts:1-262).

Each layer's forward is composed from ops exactly as in the reference, so the
traced graph (and therefore every kernel the backend runs) is the same:
``Linear`` is ``x @ W (+ b)`` with W stored ``[in, out]``; ``LayerNorm`` is the
mean/sub/mul/mean/add/sqrt/div chain plus affine; ``crossEntropy`` is
``nllLoss(logSoftmax(logits))`` with ``nllLoss = -sum(lp * oneHot(t))``.
"""
from __future__ import annotations

from typing import Optional

from . import ops as O
from .module import Module, init
from .shape import ShapeError
from .ir import capture_site


class Linear(Module):
    def __init__(self, inDim: int, outDim: int, bias: bool = True, init=None, decay: Optional[bool] = None):
        self.inDim, self.outDim = inDim, outDim
        self.W = self.param([inDim, outDim], init=init, decay=decay)
        self.b = self.param([outDim], init=_zeros()) if bias else None

    def fwd(self, x):
        out = O.matmul(x, self.W)
        return O.add(out, self.b) if self.b is not None else out


def _zeros():
    return init.zeros()


class LayerNorm(Module):
    def __init__(self, d: int, eps: float = 1e-5, bias: bool = True, decay: bool = False):
        self.d = d
        self.eps = eps
        self.g = self.param([d], init=init.ones(), decay=decay)
        self.b = self.param([d], init=init.zeros(), decay=decay) if bias else None

    def fwd(self, x):
        m = O.mean(x, -1, keepDims=True)
        c = O.sub(x, m)
        v = O.mean(O.mul(c, c), -1, keepDims=True)
        stdev = O.sqrt(O.add(v, self.eps))
        scaled = O.mul(O.div(c, stdev), self.g)
        return O.add(scaled, self.b) if self.b is not None else scaled


class RMSNorm(Module):
    def __init__(self, d: int, eps: float = 1e-6, decay: bool = False):
        self.d = d
        self.eps = eps
        self.g = self.param([d], init=init.ones(), decay=decay)

    def fwd(self, x):
        ms = O.mean(O.mul(x, x), -1, keepDims=True)
        rstd = O.sqrt(O.add(ms, self.eps))
        return O.mul(O.div(x, rstd), self.g)


class Embedding(Module):
    def __init__(self, vocab: int, dim: int, init=None, decay: Optional[bool] = None):
        self.vocab, self.dim = vocab, dim
        self.W = self.param([vocab, dim], init=init, decay=decay)

    def fwd(self, idx):
        return O.embedding(self.W, idx)


class Conv2d(Module):
    def __init__(self, inC: int, outC: int, kernelSize, stride=None, padding=None, groups: int = 1,
                 bias: bool = True, init=None, decay: Optional[bool] = None):
        kh, kw = O._pair(kernelSize, 1)
        self.strideH, self.strideW = O._pair(stride, 1)
        self.padH, self.padW = O._pair(padding, 0)
        if not isinstance(groups, int) or groups < 1:
            raise ShapeError(f"Conv2d: groups must be a positive integer, got {groups}", capture_site("Conv2d"))
        if inC % groups or outC % groups:
            raise ShapeError(f"Conv2d: inC={inC} and outC={outC} must both be divisible by groups={groups}",
                             capture_site("Conv2d"))
        self.inC, self.outC, self.groups = inC, outC, groups
        self.W = self.param([outC, inC // groups, kh, kw], init=init, decay=decay)
        self.b = self.param([outC], init=_zeros()) if bias else None

    def fwd(self, x):
        y = O.conv2d(x, self.W, stride=(self.strideH, self.strideW), padding=(self.padH, self.padW),
                     groups=self.groups)
        if self.b is None:
            return y
        return O.add(y, O.reshape(self.b, [1, self.outC, 1, 1]))


def _reduce_loss(t, reduction: str):
    if reduction == "none":
        return t
    return O.mean(t) if reduction == "mean" else O.sum(t)


def nllLoss(logProbs, targets, reduction: str = "mean"):
    site = capture_site("nllLoss")
    if targets.dtype != "i32":
        raise ShapeError(f"nllLoss: targets must be i32, got {targets.dtype}", site)
    vocab = logProbs.shape[-1]
    target_lp = O.sum(O.mul(logProbs, O.oneHot(targets, vocab, "f32")), -1)
    per_pos = O.mul(target_lp, -1)
    return _reduce_loss(per_pos, reduction)


def crossEntropy(logits, targets, reduction: str = "mean"):
    site = capture_site("crossEntropy")
    if targets.dtype != "i32":
        raise ShapeError(f"crossEntropy: targets must be i32, got {targets.dtype}", site)
    return nllLoss(O.logSoftmax(logits), targets, reduction)
