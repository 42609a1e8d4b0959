"""Compile orchestration: the reference's public training API on the B200 backend.

Mirrors src/compile.ts: ``compile({model, loss, inputs, optimizer, seed})``
traces the model (src/compile.ts:1058-1080), appends gradients
(src/grad.ts:46), eliminates dead code (src/dce.ts:33) and appends the
optimizer (src/adam.ts:157 / src/sgd.ts:102) exactly as ``buildTrainingIR``
does (src/compile.ts:473-505), then hands the graph to the CUDA backend in
place of ``planBuffers``/``emitKernels``/``createRuntime``. Initial params
come from one ``mulberry32(seed)`` stream in param order
(src/compile.ts:1173-1187).

Results follow the reference's discriminated unions: ``step`` returns
``{'kind': 'completed', 'loss', 'captures'}``, ``{'kind': 'aborted'}`` or
``{'kind': 'failed', 'error'}`` (the ``guarded`` contract, src/compile.ts:1198-1208).
"""
from __future__ import annotations

import copy
import json
import random
from collections import OrderedDict
from typing import Callable, Dict, Optional

import numpy as np

from . import backend as BK
from .dce import eliminateDeadCode
from .grad import appendGrad
from .ir import Graph, graph_to_wire
from .lr import rebaseLR
from .module import Module, cloneModule, materializeParams, mulberry32
from .optim import appendAdam, appendSGD
from .safetensors import loadSafetensors, saveSafetensors
from .trace import tensor_input, trace_fn

CHECKPOINT_FORMAT = "tensorgrad_b200.checkpoint.v1"


def _normalize_decl(d):
    if isinstance(d, dict):
        return list(d["shape"]), d.get("dtype", "f32")
    return list(d), "f32"


def _trace_module(model: Module, forward: Callable, decls: dict):
    cloned = cloneModule(model)
    holder = {}

    def body():
        holder["mp"] = materializeParams(cloned)
        tensors = {}
        for name, d in decls.items():
            shape, dtype = _normalize_decl(d)
            if any(x is None for x in shape):
                raise ValueError(f"compile: input '{name}' has an unresolved parametric dim; "
                                 "use train.attach for polymorphic shapes")
            tensors[name] = tensor_input(name, shape, dtype)
        return forward(cloned, tensors)
    g = trace_fn(body)
    return g, holder["mp"]


def _opt_wire(kind: str, res: dict) -> dict:
    c = res["config"]
    if kind == "adam":
        return {"kind": "adam", "config": {
            "lr": c["lr"], "beta1": c["beta1"], "beta2": c["beta2"], "eps": c["eps"],
            "weightDecay": c["weightDecay"], "lrIsScheduled": c["lrIsScheduled"],
            "lrtInputName": res["lrtInputName"], "decayShrinkInputName": res["decayShrinkInputName"]}}
    return {"kind": "sgd", "config": {
        "lr": c["lr"], "momentum": c["momentum"], "nesterov": c["nesterov"], "weightDecay": c["weightDecay"],
        "lrIsScheduled": c["lrIsScheduled"], "lrInputName": res["lrInputName"]}}


def _uses_prng(g: Graph) -> bool:
    return any(op["kind"] == "tensor_input" and op["name"] == "__prngSeed" for op in g.ops)


def _program(g: Graph, grads: Dict[str, int], writebacks, loss: int, optimizer, opt_start: int) -> dict:
    states = {op["name"]: {"tensor": op["out"], "initValue": op["initValue"]}
              for op in g.ops if op["kind"] == "state_input"}
    inputs = {op["name"]: op["out"] for op in g.ops if op["kind"] == "tensor_input"}
    params = [op["name"] for op in g.ops if op["kind"] == "param_input"]
    return {"graph": graph_to_wire(g), "params": params, "inputs": inputs, "states": states,
            "paramGrads": grads, "writebacks": writebacks, "loss": loss, "optimizer": optimizer,
            "usesPrng": _uses_prng(g), "optStart": opt_start}


class TrainingIR:
    """What ``buildTrainingIR`` yields: graph, grads, loss, optimizer result."""

    def __init__(self, graph, param_grads, loss, materialized, opt_kind, opt_result, program):
        self.graph = graph
        self.paramGrads = param_grads
        self.loss = loss
        self.materialized = materialized
        self.opt_kind = opt_kind
        self.opt_result = opt_result
        self.program = program


def build_training_ir(model: Module, loss: Callable, inputs: dict, optimizer: dict) -> TrainingIR:
    """trace -> appendGrad -> DCE -> optimizer (src/compile.ts:473-505)."""
    g, mp = _trace_module(model, loss, inputs)
    gr = appendGrad(g)
    id_map = eliminateDeadCode(g, [t.id for t in gr.paramGrads.values()])
    grads = {n: id_map[t.id] for n, t in gr.paramGrads.items()}
    ptensors = {n: id_map[t.id] for n, t in mp.tensors.items()}
    loss_t = id_map[gr.loss.id]
    opt_start = len(g.ops)
    kind = optimizer["kind"]
    if kind in ("adam", "adamw"):
        res = appendAdam(g, grads, ptensors, optimizer, mp.decayFlags)
        okind = "adam"
    elif kind == "sgd":
        res = appendSGD(g, grads, ptensors, optimizer, mp.decayFlags)
        okind = "sgd"
    else:
        raise ValueError(f"compile: unknown optimizer kind {kind!r}")
    program = _program(g, {n: t.id for n, t in grads.items()}, [w.to_wire() for w in res["writebacks"]],
                       loss_t.id, _opt_wire(okind, res), opt_start)
    return TrainingIR(g, grads, loss_t, mp, okind, res, program)


def build_forward_ir(model: Module, forward: Callable, inputs: dict):
    g, mp = _trace_module(model, forward, inputs)
    eliminateDeadCode(g)
    out = g.outputs[0]
    return g, mp, _program(g, {}, [], out, None, len(g.ops))


def initial_params(graph: Graph, init_fns: Dict[str, Callable], seed: int) -> Dict[str, np.ndarray]:
    """One mulberry32 stream across params in graph order (src/compile.ts:1173-1187)."""
    rng = mulberry32(seed)
    out = {}
    for op in graph.ops:
        if op["kind"] != "param_input":
            continue
        t = graph.tensors[op["out"]]
        size = t.numel
        out[op["name"]] = init_fns[op["name"]](size, t.shape, rng).reshape(t.shape)
    return out


class Captures:
    """Named activations read back with a step (src/runtime.ts:26-75)."""

    def __init__(self, data: Dict[str, np.ndarray]):
        self._d = data

    def get(self, name: str) -> np.ndarray:
        if name not in self._d:
            raise KeyError(f"capture '{name}' was not registered")
        return self._d[name]

    def has(self, name: str) -> bool:
        return name in self._d

    def names(self):
        return list(self._d)


def _guarded(body):
    try:
        return body()
    except BK.AbortError:
        return {"kind": "aborted"}
    except Exception as e:  # noqa: BLE001 - the reference maps every failure to 'failed'
        return {"kind": "failed", "error": e}


class CompiledForward:
    """Forward executor sharing the parent's params (src/compile.ts:734-811).

    ``null`` (None) dims in the input declarations resolve per call from the
    input sizes; one sibling graph is cached per resolved shape in an LRU of
    ``maxCachedShapes`` (src/compile.ts:755-891).
    """

    def __init__(self, parent, forward, inputs, output="f32", maxCachedShapes=8, model=None, ctx=None):
        self.parent = parent
        self.forward = forward
        self.decls = inputs
        self.output = output
        self.max_cached = maxCachedShapes
        self._cache: "OrderedDict[str, BK.DeviceGraph]" = OrderedDict()
        self._model = model if model is not None else parent.model
        self._ctx = ctx or parent.ctx

    def _resolve(self, inputs):
        resolved, wild = {}, None
        for name, d in self.decls.items():
            shape, dtype = _normalize_decl(d)
            if any(x is None for x in shape):
                known = 1
                for x in shape:
                    if x is not None:
                        known *= x
                n = np.asarray(inputs[name]).size
                if n % known:
                    raise ValueError(f"input '{name}': {n} elements do not fit shape {shape}")
                w = n // known
                if wild is not None and w != wild:
                    raise ValueError("all parametric dims in one call must resolve to the same value")
                wild = w
                shape = [w if x is None else x for x in shape]
            resolved[name] = {"shape": shape, "dtype": dtype}
        return resolved

    def graph_for(self, inputs):
        decls = self._resolve(inputs)
        key = "|".join(f"{n}:{'x'.join(map(str, d['shape']))}:{d['dtype']}" for n, d in sorted(decls.items()))
        if key in self._cache:
            self._cache.move_to_end(key)
            return self._cache[key]
        g, mp, prog = build_forward_ir(self._model, self.forward, decls)
        dg = BK.DeviceGraph(self._ctx, prog, parent=self.parent.device_graph)
        self._cache[key] = dg
        if len(self._cache) > self.max_cached:
            _, old = self._cache.popitem(last=False)
            old.destroy()
        return dg

    def run(self, inputs):
        def body():
            dg = self.graph_for(inputs)
            out, caps = dg.run(inputs)
            return {"kind": "completed", "output": out, "captures": Captures(caps)}
        return _guarded(body)

    def destroy(self):
        for dg in self._cache.values():
            dg.destroy()
        self._cache.clear()


class CompiledTraining:
    """Training handle (src/compile.ts:585-722). Methods are synchronous and
    return the reference's result objects."""

    def __init__(self, model, loss, inputs, optimizer, seed=None, ctx: Optional[BK.Context] = None,
                 initial: Optional[Dict[str, np.ndarray]] = None):
        self.model = model
        self.loss_fn = loss
        self.input_decls = inputs
        self.optimizer = dict(optimizer)
        self.seed = seed if seed is not None else random.getrandbits(31)
        self.ctx = ctx or BK.default_context()
        self._build(initial)

    def _build(self, initial=None):
        self.ir = build_training_ir(self.model, self.loss_fn, self.input_decls, self.optimizer)
        self.graph = self.ir.graph
        self.program = self.ir.program
        self.paramNames = [op["name"] for op in self.graph.ops if op["kind"] == "param_input"]
        self.param_shapes = {op["name"]: self.graph.tensors[op["out"]].shape
                             for op in self.graph.ops if op["kind"] == "param_input"}
        self.device_graph = BK.DeviceGraph(self.ctx, self.program)
        self.initial = initial if initial is not None else initial_params(
            self.graph, self.ir.materialized.initFns, self.seed)
        self.device_graph.upload_params(self.initial)
        self.steps_done = 0

    def step(self, inputs: Dict[str, np.ndarray]):
        def body():
            loss, caps = self.device_graph.step(inputs)
            self.steps_done += 1
            return {"kind": "completed", "loss": loss, "captures": Captures(caps)}
        return _guarded(body)

    def attach(self, forward, inputs, output="f32", maxCachedShapes=8) -> CompiledForward:
        return CompiledForward(self, forward, inputs, output, maxCachedShapes)

    def uploadParams(self, params: Dict[str, np.ndarray]) -> None:
        for n in params:
            if n not in self.param_shapes:
                raise BK.TgError("Error", f"uploadParams: unknown param '{n}'")
        missing = [n for n in self.param_shapes if n not in params]
        if missing:
            raise BK.TgError("Error", f"uploadParams: missing params {missing}")
        self.device_graph.upload_params(params)

    def downloadParams(self) -> Dict[str, np.ndarray]:
        return self.device_graph.download_params(self.param_shapes)

    def reset(self, opts: Optional[dict] = None) -> None:
        """Re-init params from the seed and/or zero the optimizer state and its
        step counter; both by default (src/compile.ts:641-657,
        src/worker.ts:294-302). The dropout counter keeps running, as in the
        reference, so a reset run draws fresh masks."""
        opts = opts or {}
        if opts.get("params", True):
            self.device_graph.upload_params(initial_params(self.graph, self.ir.materialized.initFns, self.seed))
        if opts.get("optimizer", True):
            self.device_graph.reset_optimizer()
            self.steps_done = 0

    def setLR(self, lr) -> None:
        """New schedule whose step 1 is the next step (src/worker.ts:304-319)."""
        self.device_graph.set_lr(rebaseLR(lr, self.steps_done + 1))

    def exportCheckpoint(self) -> bytes:
        """Params, optimizer state (m, v or velocity per param) and the step and
        PRNG counters as one safetensors blob: resuming from it continues the
        run exactly. New: the reference exports only params."""
        params = self.downloadParams()
        shapes = {n: self.graph.tensors[st["tensor"]].shape for n, st in self.program["states"].items()}
        states = self.device_graph.download_states(shapes)
        step, prng = self.device_graph.counters()
        tensors = {f"param/{n}": v for n, v in params.items()}
        tensors.update({f"state/{n}": v for n, v in states.items()})
        meta = {"format": CHECKPOINT_FORMAT, "step": step, "prng": prng, "steps_done": self.steps_done,
                "optimizer": json.dumps(self.optimizer, default=str)}
        return saveSafetensors(tensors, meta)

    def importCheckpoint(self, buf: bytes) -> None:
        """Restore a blob from exportCheckpoint (strict: every param and
        state of this model, nothing else)."""
        d = loadSafetensors(buf)
        meta = d["metadata"]
        if meta.get("format") != CHECKPOINT_FORMAT:
            raise BK.TgError("Error", "importCheckpoint: not a tensorgrad_b200 checkpoint")
        params = {n[len("param/"):]: v for n, v in d["tensors"].items() if n.startswith("param/")}
        states = {n[len("state/"):]: v for n, v in d["tensors"].items() if n.startswith("state/")}
        want = set(self.program["states"])
        if set(states) != want:
            raise BK.TgError("Error", f"importCheckpoint: states {sorted(set(states) ^ want)} do not match the model")
        self.uploadParams(params)
        if states:
            self.device_graph.upload_states(states)
        self.device_graph.set_counters(int(meta["step"]), int(meta["prng"]))
        self.steps_done = int(meta.get("steps_done", meta["step"]))

    def replaceModel(self, model) -> None:
        self.device_graph.destroy()
        self.model = model
        self._build()

    def destroy(self) -> None:
        self.device_graph.destroy()


def compile(model, loss, inputs, optimizer, seed=None, ctx=None, initial=None) -> CompiledTraining:  # noqa: A001
    return CompiledTraining(model, loss, inputs, optimizer, seed, ctx, initial)


class _StandaloneParent:
    def __init__(self, ctx, dg):
        self.ctx = ctx
        self.device_graph = dg


def compileForward(model, forward, inputs, output="f32", seed=None, ctx=None):
    """Standalone forward executor that owns its params (src/compile.ts compileForward)."""
    ctx = ctx or BK.default_context()
    g, mp, prog = build_forward_ir(model, forward, inputs)
    dg = BK.DeviceGraph(ctx, prog)
    seed = seed if seed is not None else random.getrandbits(31)
    dg.upload_params(initial_params(g, mp.initFns, seed))
    fwd = CompiledForward(_StandaloneParent(ctx, dg), forward, inputs, output, model=model, ctx=ctx)
    fwd.uploadParams = lambda p: dg.upload_params(p)
    fwd.downloadParams = lambda: dg.download_params({op["name"]: g.tensors[op["out"]].shape
                                                     for op in g.ops if op["kind"] == "param_input"})
    return fwd


def trace(model, loss, inputs, optimizer) -> TrainingIR:
    """Training IR for inspection, no device (src/compile.ts:376-381)."""
    return build_training_ir(model, loss, inputs, optimizer)
