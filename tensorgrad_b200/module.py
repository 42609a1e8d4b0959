"""Module trees, parameter placeholders and seeded init (src/module.ts:1-304).

``Mulberry32`` reproduces the reference's generator bit for bit
(src/module.ts:72-81); because its state advances by a constant each draw,
``take(n)`` evaluates n consecutive draws at once with numpy. Box-Muller
(src/module.ts:88-90) consumes two draws per value in f64 and each value is
rounded to f32 when stored, as ``Float32Array`` does. One generator stream
is shared by all params in discovery order (src/compile.ts:1173-1187).
Parameters are discovered in attribute-insertion order, recursing into child
modules and lists, with dotted path names (``layers.0.attn.W_q``).
"""
from __future__ import annotations

import copy
import math
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np

from .trace import param_input

_STEP = 0x6D2B79F5


class Mulberry32:
    """Uniform [0,1) stream identical to the reference's ``mulberry32(seed)``."""

    def __init__(self, seed: int):
        self.state = seed & 0xFFFFFFFF

    def take(self, n: int) -> np.ndarray:
        k = np.arange(1, n + 1, dtype=np.uint64)
        s = ((np.uint64(self.state) + k * np.uint64(_STEP)) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        self.state = (self.state + n * _STEP) & 0xFFFFFFFF
        t = (s ^ (s >> np.uint32(15))) * (s | np.uint32(1))
        t = t ^ (t + (t ^ (t >> np.uint32(7))) * (t | np.uint32(61)))
        return (t ^ (t >> np.uint32(14))).astype(np.float64) / 4294967296.0

    def __call__(self) -> float:
        return float(self.take(1)[0])


def mulberry32(seed: int) -> Mulberry32:
    return Mulberry32(seed)


def _gauss(size: int, std: float, rng: Mulberry32) -> np.ndarray:
    u = rng.take(2 * size)
    u1, u2 = u[0::2], u[1::2]
    z = np.sqrt(-2.0 * np.log(np.maximum(1e-10, u1))) * np.cos(2.0 * math.pi * u2)
    return (z * std).astype(np.float32)


class init:  # noqa: N801 - mirrors the reference's `init` helpers
    @staticmethod
    def randn(scale: float = 0.02) -> dict:
        return {"kind": "randn", "scale": scale}

    @staticmethod
    def zeros() -> dict:
        return {"kind": "zeros"}

    @staticmethod
    def ones() -> dict:
        return {"kind": "ones"}

    @staticmethod
    def kaiming(gain: Optional[float] = None) -> dict:
        return {"kind": "kaiming"} if gain is None else {"kind": "kaiming", "gain": gain}

    @staticmethod
    def literal(data) -> dict:
        return {"kind": "literal", "data": np.asarray(data, dtype=np.float32)}


def resolve_init(spec: Optional[dict]):
    """Init spec -> fn(size, shape, rng) -> float32 array (src/module.ts:103-129)."""
    if spec is None:
        return lambda size, shape, rng: _gauss(size, 0.02, rng)
    k = spec["kind"]
    if k == "randn":
        sc = spec["scale"]
        return lambda size, shape, rng: _gauss(size, sc, rng)
    if k == "zeros":
        return lambda size, shape, rng: np.zeros(size, np.float32)
    if k == "ones":
        return lambda size, shape, rng: np.ones(size, np.float32)
    if k == "kaiming":
        gain = spec.get("gain", math.sqrt(2))

        def f(size, shape, rng):
            fan_in = shape[0] if len(shape) else size
            return _gauss(size, gain / math.sqrt(fan_in), rng)
        return f
    if k == "literal":
        data = spec["data"]

        def g(size, shape, rng):
            if data.size != size:
                raise ValueError(f"init.literal: data length {data.size} doesn't match param size {size}")
            return data.astype(np.float32).copy()
        return g
    raise ValueError(f"unknown init kind {k!r}")


def resolve_decay(init_spec: Optional[dict], decay: Optional[bool]) -> bool:
    if decay is not None:
        return decay
    return not (init_spec is not None and init_spec["kind"] in ("zeros", "ones"))


class Param:
    """Placeholder replaced by a Tensor at materialisation."""
    __slots__ = ("shape", "dtype", "init_fn", "decay")

    def __init__(self, shape, dtype, init_fn, decay):
        self.shape = tuple(shape)
        self.dtype = dtype
        self.init_fn = init_fn
        self.decay = decay


class Module:
    """Base class for parameter trees; forward functions are free functions."""

    def param(self, shape: Sequence[int], init: Optional[dict] = None, decay: Optional[bool] = None,
              dtype: str = "f32"):
        return Param(shape, dtype, resolve_init(init), resolve_decay(init, decay))


class MaterializedParams:
    def __init__(self):
        self.tensors: Dict[str, object] = {}
        self.initFns: Dict[str, Callable] = {}
        self.decayFlags: Dict[str, bool] = {}


def _visit(node, path: str, visitor) -> None:
    if isinstance(node, Module):
        for key in list(vars(node).keys()):
            child = getattr(node, key)
            cp = f"{path}.{key}" if path else key
            _visit_child(child, cp, node, key, visitor)
    elif isinstance(node, list):
        for i, item in enumerate(node):
            cp = f"{path}.{i}" if path else str(i)
            _visit_child(item, cp, node, i, visitor)


def _visit_child(child, path, owner, key, visitor):
    if isinstance(child, (Module, list)):
        _visit(child, path, visitor)
    else:
        visitor(path, child, owner, key)


def materializeParams(root: Module) -> MaterializedParams:
    mp = MaterializedParams()

    def visit(path, val, owner, key):
        if isinstance(val, Param):
            t = param_input(path, val.shape, val.dtype)
            if isinstance(owner, list):
                owner[key] = t
            else:
                setattr(owner, key, t)
            mp.tensors[path] = t
            mp.initFns[path] = val.init_fn
            mp.decayFlags[path] = val.decay
    _visit(root, "", visit)
    return mp


def cloneModule(m):
    """Deep-clone Modules and lists, sharing Params and plain values."""
    if isinstance(m, Module):
        out = copy.copy(m)
        for key, val in list(vars(m).items()):
            setattr(out, key, cloneModule(val))
        return out
    if isinstance(m, list):
        return [cloneModule(x) for x in m]
    return m
