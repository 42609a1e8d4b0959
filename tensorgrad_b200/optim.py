"""In-graph optimizers: Adam/AdamW (src/adam.ts:157-240) and SGD (src/sgd.ts:102-175).

Both append per-parameter update ops plus writeback declarations (new value
-> persistent param/state home), and name the per-step scalar inputs the
runtime fills (``_adam_lrt``, ``_adam_decay_shrink``, ``_sgd_lr``).
"""
from __future__ import annotations

import math
from typing import Callable, Dict, List, Optional

from . import ops as O
from .grad import appendGradClip, appendGradNormalize
from .ir import Graph, Tensor
from .lr import isLRDynamic, resolveLR
from .trace import state_input, tensor_input, trace_into


class Writeback:
    def __init__(self, source: Tensor, destName: str, destKind: str):
        self.source, self.destName, self.destKind = source, destName, destKind

    def to_wire(self) -> dict:
        return {"source": self.source.id, "destName": self.destName, "destKind": self.destKind}


def adamStepScalars(c: dict, t: int) -> dict:
    """lrt = lr_t*sqrt(1-b2^t)/(1-b1^t); decayShrink = 1 - lr_t*wd (src/adam.ts:134-143)."""
    lr_now = resolveLR(c["lr"], t)
    return {"lrt": lr_now * math.sqrt(1 - math.pow(c["beta2"], t)) / (1 - math.pow(c["beta1"], t)),
            "decayShrink": 1 - lr_now * c["weightDecay"]}


def _grad_transforms(graph, grads, cfg):
    ng = cfg.get("normalizeGrads")
    if ng:
        grads = appendGradNormalize(graph, grads, ng if callable(ng) else None)
    clip = cfg.get("clipGradNorm")
    if clip is not None and clip > 0:
        grads = appendGradClip(graph, grads, clip)
    return grads


def appendAdam(graph: Graph, param_grads: Dict[str, Tensor], param_tensors: Dict[str, Tensor],
               config: dict, decay_flags: Optional[Dict[str, bool]] = None) -> dict:
    param_grads = _grad_transforms(graph, param_grads, config)
    scheduled = isLRDynamic(config["lr"])
    initial_lr = resolveLR(config["lr"], 1)
    wd = config.get("weightDecay", 0) or 0
    wd = wd if wd > 0 else 0
    full = {"lr": config["lr"], "beta1": config.get("beta1", 0.9), "beta2": config.get("beta2", 0.999),
            "eps": config.get("eps", 1e-8), "weightDecay": wd, "lrIsScheduled": scheduled}
    filt: Callable[[str], bool] = config.get("decayFilter") or (lambda n: True)
    writebacks: List[Writeback] = []
    res = {"writebacks": writebacks, "lrtInputName": "_adam_lrt", "decayShrinkInputName": None, "config": full}

    def body():
        lrt = tensor_input("_adam_lrt", [], "f32")
        decayed = set()
        if wd > 0:
            for n in param_grads:
                if decay_flags is not None and n in decay_flags:
                    if decay_flags[n]:
                        decayed.add(n)
                elif filt(n):
                    decayed.add(n)
        shrink_t = None
        if scheduled and decayed:
            res["decayShrinkInputName"] = "_adam_decay_shrink"
            shrink_t = tensor_input("_adam_decay_shrink", [], "f32")
        for name in param_grads:
            p, g = param_tensors.get(name), param_grads.get(name)
            if p is None:
                raise RuntimeError(f"appendAdam: missing param tensor for '{name}'")
            m = state_input(f"adam_m_{name}", p.shape, "f32", 0)
            v = state_input(f"adam_v_{name}", p.shape, "f32", 0)
            ds = 1 if name not in decayed else (shrink_t if shrink_t is not None else 1 - initial_lr * wd)
            nm = O.adamUpdateM(m, g, full["beta1"])
            nv = O.adamUpdateV(v, g, full["beta2"])
            np_ = O.adamUpdateP(p, nm, nv, lrt, full["eps"], ds)
            writebacks.append(Writeback(nm, f"adam_m_{name}", "state"))
            writebacks.append(Writeback(nv, f"adam_v_{name}", "state"))
            writebacks.append(Writeback(np_, name, "param"))
        return res
    return trace_into(graph, body)


def appendSGD(graph: Graph, param_grads: Dict[str, Tensor], param_tensors: Dict[str, Tensor],
              config: dict, decay_flags: Optional[Dict[str, bool]] = None) -> dict:
    param_grads = _grad_transforms(graph, param_grads, config)
    mom = config.get("momentum", 0)
    nesterov = config.get("nesterov", False)
    if nesterov and mom <= 0:
        raise RuntimeError(f"appendSGD: nesterov requires momentum > 0 (got momentum={mom})")
    wd = config.get("weightDecay", 0)
    filt = config.get("decayFilter") or (lambda n: True)
    full = {"lr": config["lr"], "momentum": mom, "nesterov": nesterov, "weightDecay": wd,
            "lrIsScheduled": isLRDynamic(config["lr"])}
    writebacks: List[Writeback] = []

    def body():
        lr_t = tensor_input("_sgd_lr", [], "f32")
        decayed = set()
        if wd > 0:
            for n in param_grads:
                if (decay_flags[n] if (decay_flags is not None and n in decay_flags) else filt(n)):
                    decayed.add(n)
        for name in param_grads:
            p, g = param_tensors.get(name), param_grads.get(name)
            if p is None:
                raise RuntimeError(f"appendSGD: missing param tensor for '{name}'")
            g_eff = O.add(g, O.mulScalar(p, wd)) if name in decayed else g
            if mom > 0:
                v = state_input(f"sgd_v_{name}", p.shape, "f32", 0)
                v_new = O.add(O.mulScalar(v, mom), g_eff)
                upd = O.add(g_eff, O.mulScalar(v_new, mom)) if nesterov else v_new
                writebacks.append(Writeback(v_new, f"sgd_v_{name}", "state"))
            else:
                upd = g_eff
            p_new = O.sub(p, O.mul(O.broadcastTo(lr_t, p.shape), upd))
            writebacks.append(Writeback(p_new, name, "param"))
        return {"writebacks": writebacks, "lrInputName": "_sgd_lr", "config": full}
    return trace_into(graph, body)
