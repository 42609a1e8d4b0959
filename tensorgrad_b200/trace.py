"""Module-global current graph and the named leaves (src/trace.ts:1-114)."""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, TypeVar, Union

from .ir import Graph, Tensor, add_op, capture_site, make_graph

_current: Optional[Graph] = None
_capture_enabled = False

T = TypeVar("T")


def current_graph() -> Graph:
    if _current is None:
        raise RuntimeError("tensorgrad: ops can only be called inside trace_fn(). "
                           "Did you forget to wrap your forward pass?")
    return _current


def is_capture_enabled() -> bool:
    return _capture_enabled


def trace_fn(fn: Callable[[], Union[Tensor, Sequence[Tensor]]]) -> Graph:
    """Run ``fn`` against a fresh graph; its return values become outputs."""
    global _current, _capture_enabled
    if _current is not None:
        raise RuntimeError("tensorgrad: nested trace_fn() is not supported")
    g = make_graph()
    _current, _capture_enabled = g, True
    try:
        res = fn()
        outs = list(res) if isinstance(res, (list, tuple)) else [res]
        for t in outs:
            g.outputs.append(t.id)
    finally:
        _current, _capture_enabled = None, False
    return g


def trace_into(g: Graph, fn: Callable[[], T]) -> T:
    """Re-enter ``g`` to append ops (autograd / optimizer passes); no captures."""
    global _current
    if _current is not None:
        raise RuntimeError("tensorgrad: trace_into() called while another trace_fn is active")
    _current = g
    try:
        return fn()
    finally:
        _current = None


def _assert_unused(g: Graph, name: str, kinds: List[str], label: str) -> None:
    for op in g.ops:
        if op["kind"] in kinds and op.get("name") == name:
            raise RuntimeError(f"tensorgrad: {label} name '{name}' already used in this trace")


def param_input(name: str, shape: Sequence[int], dtype: str = "f32") -> Tensor:
    g = current_graph()
    _assert_unused(g, name, ["param_input", "tensor_input"], "input")
    return add_op(g, "param_input", shape, dtype, capture_site("paramInput"), {"name": name})


def tensor_input(name: str, shape: Sequence[int], dtype: str = "f32") -> Tensor:
    g = current_graph()
    _assert_unused(g, name, ["param_input", "tensor_input"], "input")
    return add_op(g, "tensor_input", shape, dtype, capture_site("tensorInput"), {"name": name})


def state_input(name: str, shape: Sequence[int], dtype: str = "f32", init_value: float = 0) -> Tensor:
    g = current_graph()
    _assert_unused(g, name, ["state_input"], "state")
    return add_op(g, "state_input", shape, dtype, capture_site("stateInput"),
                  {"name": name, "initValue": init_value})
