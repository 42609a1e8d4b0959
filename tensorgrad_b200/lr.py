"""Learning-rate schedules as serialisable data (src/lr.ts:1-119).

A schedule is a number or a dict with ``kind`` in linear / cosineAnnealing /
warmup / staircase / multiStep and an optional ``startStep``; ``resolveLR``
evaluates it at a 1-based step exactly as the reference does (f64 math).
"""
from __future__ import annotations

import math
from typing import Union

LR = Union[float, int, dict]


class lr:  # noqa: N801 - mirrors the reference's `lr` helper namespace
    @staticmethod
    def linear(peak, final, steps, startStep=None) -> dict:
        return _mk("linear", peak=peak, final=final, steps=steps, startStep=startStep)

    @staticmethod
    def cosineAnnealing(peak, final, steps, startStep=None) -> dict:
        return _mk("cosineAnnealing", peak=peak, final=final, steps=steps, startStep=startStep)

    @staticmethod
    def warmup(peak, steps, after, startStep=None) -> dict:
        return _mk("warmup", peak=peak, steps=steps, after=after, startStep=startStep)

    @staticmethod
    def staircase(peak, every, gamma, startStep=None) -> dict:
        return _mk("staircase", peak=peak, every=every, gamma=gamma, startStep=startStep)

    @staticmethod
    def multiStep(peak, milestones, gamma, startStep=None) -> dict:
        return _mk("multiStep", peak=peak, milestones=list(milestones), gamma=gamma, startStep=startStep)


def _mk(kind, **kw) -> dict:
    d = {"kind": kind}
    d.update({k: v for k, v in kw.items() if v is not None})
    return d


def _intrinsic(start, step) -> int:
    return max(1, step - (start or 0))


def resolveLR(s: LR, step: int) -> float:
    if isinstance(s, (int, float)):
        return float(s)
    k = s["kind"]
    st = _intrinsic(s.get("startStep"), step)
    if k == "linear":
        f = min(st / s["steps"], 1)
        return s["peak"] + (s["final"] - s["peak"]) * f
    if k == "cosineAnnealing":
        f = min(st / s["steps"], 1)
        return s["final"] + 0.5 * (s["peak"] - s["final"]) * (1 + math.cos(math.pi * f))
    if k == "warmup":
        if st <= s["steps"]:
            return s["peak"] * (st / s["steps"])
        return resolveLR(s["after"], st - s["steps"])
    if k == "staircase":
        return s["peak"] * math.pow(s["gamma"], (st - 1) // s["every"])
    if k == "multiStep":
        n = 0
        for m in s["milestones"]:
            if st >= m:
                n += 1
        return s["peak"] * math.pow(s["gamma"], n)
    raise ValueError(f"unknown lr schedule kind {k!r}")


def rebaseLR(s: LR, base_step: int) -> LR:
    if isinstance(s, (int, float)) or "startStep" in s:
        return s
    d = dict(s)
    d["startStep"] = base_step - 1
    return d


def isLRDynamic(s: LR) -> bool:
    return not isinstance(s, (int, float))
