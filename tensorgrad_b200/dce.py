"""Dead-code elimination over a traced graph (src/dce.ts:33-76).

Marks everything reachable from the outputs, the captures and ``extra_roots``;
named leaves (param/tensor/state inputs) always survive. The surviving graph is
renumbered densely in construction order; the returned map sends old tensor
ids to the new ``Tensor`` handles.
"""
from __future__ import annotations

from typing import Dict, Iterable

from .ir import Graph, Tensor, get_op_inputs, remap_op_inputs


def eliminateDeadCode(graph: Graph, extra_roots: Iterable[int] = ()) -> Dict[int, Tensor]:
    live = set()
    stack = list(graph.outputs) + list(graph.captures.values()) + list(extra_roots)
    while stack:
        tid = stack.pop()
        if tid in live:
            continue
        live.add(tid)
        src = graph.tensors[tid].source
        if src is None:
            continue
        stack.extend(get_op_inputs(graph.ops[src]))

    id_map: Dict[int, Tensor] = {}

    def map_id(old: int) -> int:
        t = id_map.get(old)
        if t is None:
            raise RuntimeError(f"dce: op input references tensor #{old} that was eliminated (internal ordering bug)")
        return t.id

    new_ops, new_tensors = [], []
    for op in graph.ops:
        named = op["kind"] in ("param_input", "tensor_input", "state_input")
        if not named and op["out"] not in live:
            continue
        old = graph.tensors[op["out"]]
        rem = remap_op_inputs(op, map_id)
        t = Tensor(len(new_tensors), old.shape, old.dtype, len(new_ops), old.site)
        rem["out"] = t.id
        new_ops.append(rem)
        new_tensors.append(t)
        id_map[op["out"]] = t
    new_outputs = [map_id(i) for i in graph.outputs]
    graph.ops[:] = new_ops
    graph.tensors[:] = new_tensors
    graph.outputs[:] = new_outputs
    for name in list(graph.captures):
        graph.captures[name] = map_id(graph.captures[name])
    return id_map
