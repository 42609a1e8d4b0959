"""Intermediate representation: a flat SSA graph of ops over shaped tensors.

Mirrors the reference's IR data model (src/ir.ts:1-296): a ``Graph`` holds
``ops`` in construction (= topological = dispatch) order, ``tensors`` indexed by
id, ``outputs`` and named ``captures``. Each op is a plain dict with a ``kind``
discriminator, an ``out`` tensor id and kind-specific fields, using the same
field names as the reference's ``OpNode`` union so the graph serialises to the
reference's WireIR shape unchanged.

``remap_op_inputs`` is the single switch over op kinds that knows which fields
are tensor inputs (src/ir.ts:356-395); ``get_op_inputs`` is derived from it.
"""
from __future__ import annotations

import traceback
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

Shape = Tuple[int, ...]

DTYPES = ("f32", "i32", "bool")


@dataclass(frozen=True)
class CallSite:
    """Where an op was invoked; shape errors blame this frame (src/ir.ts:50-56)."""
    op_name: str
    stack: str


@dataclass(frozen=True)
class Tensor:
    """Metadata-only handle: id, static shape, dtype and producing op index."""
    id: int
    shape: Shape
    dtype: str
    source: Optional[int]
    site: Optional[CallSite] = None

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        return f"Tensor(#{self.id}, {list(self.shape)}, {self.dtype})"


@dataclass
class Graph:
    ops: List[dict] = field(default_factory=list)
    tensors: List[Tensor] = field(default_factory=list)
    outputs: List[int] = field(default_factory=list)
    captures: Dict[str, int] = field(default_factory=dict)


def make_graph() -> Graph:
    return Graph()


def capture_site(op_name: str) -> CallSite:
    """Capture the caller's stack, formatted lazily (src/ir.ts:397-401)."""
    return CallSite(op_name, "".join(traceback.format_stack(limit=8)[:-1]))


def format_site(site: CallSite) -> str:
    """First user frames outside this package (src/ir.ts:403-415)."""
    frames = []
    for line in site.stack.splitlines():
        s = line.strip()
        if s.startswith("File ") and "tensorgrad_b200" not in s:
            frames.append(s)
    if not frames:
        return f"[{site.op_name}] (no user frame found)"
    return f"[{site.op_name}]\n  " + "\n  ".join(frames[-3:])


def shape_size(shape: Sequence[int]) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def add_tensor(g: Graph, shape: Sequence[int], dtype: str, source: Optional[int],
               site: Optional[CallSite]) -> Tensor:
    t = Tensor(len(g.tensors), tuple(int(d) for d in shape), dtype, source, site)
    g.tensors.append(t)
    return t


def add_op(g: Graph, kind: str, shape: Sequence[int], dtype: str,
           site: Optional[CallSite], fields: dict) -> Tensor:
    """Append ``kind`` producing a fresh output tensor (src/ir.ts:311-323)."""
    op_index = len(g.ops)
    out = add_tensor(g, shape, dtype, op_index, site)
    node = {"kind": kind, "out": out.id}
    node.update(fields)
    g.ops.append(node)
    return out


_LEAF = {"param_input", "tensor_input", "state_input", "arange", "const_scalar", "const_fill"}
_AB = {"add", "sub", "mul", "div", "min", "max", "less", "greater", "matmul", "matmul_batched"}
_A = {"mul_scalar", "add_scalar", "sqrt", "rsqrt", "log", "exp", "relu", "neg", "abs", "tanh",
      "sigmoid", "erf", "sin", "cos", "mean_last", "sum_last", "argmax_last", "reshape", "permute",
      "softmax_causal_last", "log_softmax_last", "where_causal", "stop_gradient", "slice_range",
      "scatter_axis", "broadcast_to", "sum_to_shape"}

ALL_KINDS = frozenset(_LEAF | _AB | _A | {
    "randn", "dropout", "categorical_last", "one_hot", "where", "concat", "relu_grad",
    "adam_update_m", "adam_update_v", "adam_update_p", "conv2d", "conv2d_input_grad",
    "conv2d_weight_grad", "max_pool_2d", "max_pool_2d_grad"})


def remap_op_inputs(op: dict, f: Callable[[int], int]) -> dict:
    """Copy of ``op`` with every input tensor id passed through ``f``.

    Field order defines ``get_op_inputs`` order (src/ir.ts:356-395).
    """
    k = op["kind"]
    o = dict(op)
    if k in _LEAF:
        return o
    if k == "randn":
        o["seed"] = f(op["seed"])
    elif k in _AB:
        o["a"] = f(op["a"])
        o["b"] = f(op["b"])
    elif k in _A:
        o["a"] = f(op["a"])
    elif k in ("dropout", "categorical_last"):
        o["a"] = f(op["a"])
        o["seed"] = f(op["seed"])
    elif k == "one_hot":
        o["indices"] = f(op["indices"])
    elif k == "where":
        o["cond"] = f(op["cond"])
        o["a"] = f(op["a"])
        o["b"] = f(op["b"])
    elif k == "concat":
        o["inputs"] = [f(i) for i in op["inputs"]]
    elif k == "relu_grad":
        o["x"] = f(op["x"])
        o["dy"] = f(op["dy"])
    elif k == "adam_update_m":
        o["m"] = f(op["m"])
        o["g"] = f(op["g"])
    elif k == "adam_update_v":
        o["v"] = f(op["v"])
        o["g"] = f(op["g"])
    elif k == "adam_update_p":
        o["p"] = f(op["p"])
        o["mNew"] = f(op["mNew"])
        o["vNew"] = f(op["vNew"])
        o["lrt"] = f(op["lrt"])
        o["decayShrinkTensor"] = (f(op["decayShrinkTensor"])
                                  if op["decayShrinkTensor"] is not None else None)
    elif k == "conv2d":
        o["input"] = f(op["input"])
        o["weight"] = f(op["weight"])
    elif k == "conv2d_input_grad":
        o["weight"] = f(op["weight"])
        o["dy"] = f(op["dy"])
    elif k == "conv2d_weight_grad":
        o["input"] = f(op["input"])
        o["dy"] = f(op["dy"])
    elif k == "max_pool_2d":
        o["input"] = f(op["input"])
    elif k == "max_pool_2d_grad":
        o["input"] = f(op["input"])
        o["dy"] = f(op["dy"])
    else:
        raise ValueError(f"unknown op kind {k!r}")
    return o


def get_op_inputs(op: dict) -> List[int]:
    ids: List[int] = []

    def rec(i: int) -> int:
        ids.append(i)
        return i
    remap_op_inputs(op, rec)
    return ids


def graph_to_wire(g: Graph) -> dict:
    """JSON-ready form of a graph (the reference's WireIR.graph shape)."""
    return {
        "tensors": [{"shape": list(t.shape), "dtype": t.dtype} for t in g.tensors],
        "ops": [dict(op) for op in g.ops],
        "outputs": list(g.outputs),
        "captures": dict(g.captures),
    }
