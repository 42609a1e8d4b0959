"""Multi-step training driver over the oracle evaluator — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may use it. It restates what the reference's worker does around each
evaluation, because the reference's own test evaluator has no multi-step loop:

* per-step optimizer scalars (src/worker.ts:187-206): Adam ``t += 1`` then
  ``lrt = lr_t * sqrt(1 - b2^t) / (1 - b1^t)`` and ``decayShrink = 1 - lr_t*wd``
  (src/adam.ts:134-143), both f64 stored to f32; SGD ``lr = resolveLR(lr, t)``;
* the PRNG seed counter, starting at 1 on the first step (src/worker.ts:208-214);
* writebacks applied after the step (src/buffers.ts:245-265, src/runtime.ts:354-356).

``resolve_lr`` restates src/lr.ts:69-101.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np

from .evaluator import eval_graph


def resolve_lr(s, step: int) -> float:
    """Schedule value at a 1-based step (src/lr.ts:69-101)."""
    if isinstance(s, (int, float)):
        return float(s)
    k = s["kind"]
    st = max(1, step - (s.get("startStep") or 0))
    if k == "linear":
        f = min(st / s["steps"], 1)
        return s["peak"] + (s["final"] - s["peak"]) * f
    if k == "cosineAnnealing":
        f = min(st / s["steps"], 1)
        return s["final"] + 0.5 * (s["peak"] - s["final"]) * (1 + math.cos(math.pi * f))
    if k == "warmup":
        if st <= s["steps"]:
            return s["peak"] * (st / s["steps"])
        return resolve_lr(s["after"], st - s["steps"])
    if k == "staircase":
        return s["peak"] * math.pow(s["gamma"], (st - 1) // s["every"])
    if k == "multiStep":
        return s["peak"] * math.pow(s["gamma"], sum(1 for m in s["milestones"] if st >= m))
    raise ValueError(k)


class OracleTrainer:
    """Holds params/state on the host and steps a training program on the CPU."""

    def __init__(self, program: dict, initial_params: Dict[str, np.ndarray], dp_rank: int = 0):
        self.p = program
        self.g = program["graph"]
        self.params = {k: np.asarray(v, np.float32).copy() for k, v in initial_params.items()}
        self.states: Dict[str, np.ndarray] = {}
        for name, st in program["states"].items():
            shape = self.g["tensors"][st["tensor"]]["shape"]
            self.states[name] = np.full(shape, st["initValue"], np.float32)
        self.t = 0
        self.prng = 0
        self.dp_rank = dp_rank
        self.last_vals: Optional[Dict[int, np.ndarray]] = None

    def scalars(self) -> Dict[str, np.ndarray]:
        """Advance counters and return the per-step injected inputs."""
        out: Dict[str, np.ndarray] = {}
        opt = self.p.get("optimizer")
        if opt is not None:
            c = opt["config"]
            self.t += 1
            lr_now = resolve_lr(c["lr"], self.t)
            if opt["kind"] == "adam":
                lrt = lr_now * math.sqrt(1 - math.pow(c["beta2"], self.t)) / (1 - math.pow(c["beta1"], self.t))
                out[c["lrtInputName"]] = np.array(lrt, np.float32)
                if c.get("decayShrinkInputName"):
                    out[c["decayShrinkInputName"]] = np.array(1 - lr_now * c["weightDecay"], np.float32)
            else:
                out[c["lrInputName"]] = np.array(lr_now, np.float32)
        if self.p.get("usesPrng"):
            self.prng += 1
            out["__prngSeed"] = np.array(self.prng, np.int32)
        return out

    def evaluate(self, inputs: Dict[str, np.ndarray], injected: Dict[str, np.ndarray]) -> Dict[int, np.ndarray]:
        merged = dict(self.params)
        merged.update(self.states)
        merged.update(inputs)
        merged.update(injected)
        return eval_graph(self.g, merged, self.dp_rank)

    def f32_grads(self, inputs: Dict[str, np.ndarray], params: Dict[str, np.ndarray],
                  states: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
        """The gradients of the step just taken from ``params`` and
        ``states``, re-evaluated with f32 arithmetic throughout (same injected
        scalars; nothing is updated): the f32 error floor of the graph."""
        t, prng = self.t, self.prng
        self.t, self.prng = t - 1, (prng - 1 if self.p.get("usesPrng") else prng)
        injected = self.scalars()
        self.t, self.prng = t, prng
        merged = dict(params)
        merged.update(states)
        merged.update(inputs)
        merged.update(injected)
        vals = eval_graph(self.g, merged, self.dp_rank, np.float32)
        return {n: vals[tid] for n, tid in self.p["paramGrads"].items()}

    def apply_writebacks(self, vals: Dict[int, np.ndarray]) -> None:
        for wb in self.p["writebacks"]:
            dst = self.params if wb["destKind"] == "param" else self.states
            dst[wb["destName"]] = vals[wb["source"]].astype(np.float32).copy()

    def step(self, inputs: Dict[str, np.ndarray]) -> float:
        vals = self.evaluate(inputs, self.scalars())
        self.last_vals = vals
        loss = float(vals[self.p["loss"]].reshape(-1)[0])
        self.apply_writebacks(vals)
        return loss

    def grads(self) -> Dict[str, np.ndarray]:
        assert self.last_vals is not None
        return {n: self.last_vals[t] for n, t in self.p["paramGrads"].items()}
