"""The five benchmark workloads (models, losses, optimizers, seeded data).

Model code uses only the public op surface, exactly as a user of the
reference would write it (the reference's own samples follow the same
patterns: samples/mlp-sin/spec.ts, samples/mnist-cnn/spec.ts,
samples/makemore/spec.ts, samples/transformer/spec.ts). Data is synthetic:
one ``mulberry32(1234)`` stream per config with the shapes and value
distributions the benchmark specifies, standing in for the datasets.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, Optional

import numpy as np

from . import ops as O
from .lr import lr as LRS
from .module import Module, Mulberry32
from .nn import Conv2d, LayerNorm, Linear, crossEntropy

DATA_SEED = 1234
PARAM_SEED = 42


# --------------------------------------------------------------------- C1 --
class MLP(Module):
    def __init__(self, hidden=64):
        self.l1 = Linear(1, hidden)
        self.l2 = Linear(hidden, hidden)
        self.l3 = Linear(hidden, 1)


def mlp_loss(p: MLP, x):
    h = O.relu(p.l1.fwd(x["x"]))
    h = O.relu(p.l2.fwd(h))
    diff = O.sub(p.l3.fwd(h), x["y"])
    return O.mean(O.mul(diff, diff))


def mlp_data(B: int, seed: int = DATA_SEED):
    u = Mulberry32(seed).take(B)
    x = (-math.pi + 2 * math.pi * u).astype(np.float32).reshape(B, 1)
    return {"x": x, "y": np.sin(x.astype(np.float64)).astype(np.float32)}


# --------------------------------------------------------------------- C2 --
class CNN(Module):
    def __init__(self, c1=32, c2=64, hw=28, hidden=128, classes=10):
        self.conv1 = Conv2d(1, c1, 3)
        self.conv2 = Conv2d(c1, c2, 3)
        side = (hw - 4) // 2
        self.fc1 = Linear(c2 * side * side, hidden)
        self.fc2 = Linear(hidden, classes)


def cnn_loss(m: CNN, x):
    h = O.relu(m.conv1.fwd(x["x"]))
    h = O.relu(m.conv2.fwd(h))
    h = O.maxPool2d(h, 2)
    h = O.reshape(h, [h.shape[0], -1])
    h = O.relu(m.fc1.fwd(h))
    return crossEntropy(m.fc2.fwd(h), x["y"])


def cnn_data(B: int, hw: int = 28, classes: int = 10, seed: int = DATA_SEED):
    r = Mulberry32(seed)
    x = r.take(B * hw * hw).astype(np.float32).reshape(B, 1, hw, hw)
    y = np.floor(classes * r.take(B)).astype(np.int32)
    return {"x": x, "y": y}


# --------------------------------------------------------------------- C3 --
class CharMLP(Module):
    def __init__(self, vocab=27, ctx=3, emb=10, hidden=200):
        self.C = self.param([vocab, emb])
        self.l1 = Linear(ctx * emb, hidden)
        self.l2 = Linear(hidden, vocab)
        self.ctx, self.emb = ctx, emb


def charmlp_loss(m: CharMLP, x):
    e = O.embedding(m.C, x["ids"])                       # [B, ctx, emb]
    h = O.reshape(e, [e.shape[0], m.ctx * m.emb])        # concat of the context embeddings
    h = O.tanh(m.l1.fwd(h))
    return crossEntropy(m.l2.fwd(h), x["targets"])


def charmlp_data(B: int, vocab=27, ctx=3, seed: int = DATA_SEED):
    r = Mulberry32(seed)
    ids = np.floor(vocab * r.take(B * ctx)).astype(np.int32).reshape(B, ctx)
    tg = np.floor(vocab * r.take(B)).astype(np.int32)
    return {"ids": ids, "targets": tg}


# ------------------------------------------------------------------ C4/C5 --
class Attention(Module):
    def __init__(self, D):
        self.q = Linear(D, D, bias=False)
        self.k = Linear(D, D, bias=False)
        self.v = Linear(D, D, bias=False)
        self.o = Linear(D, D, bias=False)


class FFN(Module):
    def __init__(self, D):
        self.up = Linear(D, 4 * D)
        self.down = Linear(4 * D, D)


class Block(Module):
    def __init__(self, D):
        self.ln1 = LayerNorm(D)
        self.attn = Attention(D)
        self.ln2 = LayerNorm(D)
        self.mlp = FFN(D)


class GPT(Module):
    def __init__(self, vocab, T, D, layers, heads, dropout=0.0):
        self.tok_emb = self.param([vocab, D])
        self.pos_emb = self.param([T, D])
        self.layers = [Block(D) for _ in range(layers)]
        self.lnf = LayerNorm(D)
        self.head = Linear(D, vocab, bias=False)
        self.T, self.D, self.H, self.p = T, D, heads, dropout


def gpt_logits(m: GPT, tokens):
    T, H = m.T, m.H
    x = O.add(O.embedding(m.tok_emb, tokens), O.embedding(m.pos_emb, O.arange(T)))
    x = O.dropout(x, m.p)
    scale = 1 / math.sqrt(m.D // H)
    for blk in m.layers:
        h = blk.ln1.fwd(x)
        q = O.splitHeads(blk.attn.q.fwd(h), H)
        k = O.splitHeads(blk.attn.k.fwd(h), H)
        v = O.splitHeads(blk.attn.v.fwd(h), H)
        att = O.softmaxCausal(O.mul(O.matmul(q, O.swapAxes(k, -1, -2)), scale))
        att = O.dropout(att, m.p)
        a = blk.attn.o.fwd(O.mergeHeads(O.matmul(att, v)))
        x = O.add(x, O.dropout(a, m.p))
        f = blk.mlp.down.fwd(O.gelu(blk.mlp.up.fwd(blk.ln2.fwd(x))))
        x = O.add(x, O.dropout(f, m.p))
    return m.head.fwd(m.lnf.fwd(x))


def gpt_loss(m: GPT, x):
    return crossEntropy(gpt_logits(m, x["tokens"]), x["targets"])


def gpt_data(B: int, T: int, vocab: int, seed: int = DATA_SEED):
    r = Mulberry32(seed)
    seq = np.floor(vocab * r.take(B * (T + 1))).astype(np.int32).reshape(B, T + 1)
    return {"tokens": np.ascontiguousarray(seq[:, :T]), "targets": np.ascontiguousarray(seq[:, 1:])}


# ------------------------------------------------------------------ table --
@dataclass
class Workload:
    name: str
    make_model: Callable[[], Module]
    loss: Callable
    inputs: Callable[[int], dict]          # per-rank batch -> input decls
    data: Callable[[int], Dict[str, np.ndarray]]  # global batch -> arrays
    optimizer: dict
    global_batch: int
    flops_per_sample: float                 # algorithmic training FLOPs per sample
    extra: dict = field(default_factory=dict)


def _gpt_flops(V, T, D, L, causal=True):
    # 6 * (linear params) * tokens + attention QK^T and PV, fwd + 2x bwd
    lin = L * (4 * D * D + 2 * 4 * D * D) + D * V
    attn_pairs = T * (T + 1) / 2 if causal else T * T
    attn = L * 2 * 2 * attn_pairs * D       # QK^T and PV, 2 flops per MAC, fwd
    return 6 * lin * T + 3 * attn


def workload(name: str, **over) -> Workload:
    if name == "c1":
        B = over.get("batch", 256)
        return Workload("mlp_1-64-64-1", lambda: MLP(over.get("hidden", 64)), mlp_loss,
                        lambda b: {"x": [b, 1], "y": [b, 1]}, lambda b: mlp_data(b),
                        {"kind": "adam", "lr": 0.005}, B, 6.0 * 4353)
    if name == "c2":
        B = over.get("batch", 128)
        hw = over.get("hw", 28)
        c1, c2 = over.get("c1", 32), over.get("c2", 64)
        return Workload("cnn_mnist_shape", lambda: CNN(c1, c2, hw, over.get("hidden", 128)), cnn_loss,
                        lambda b: {"x": [b, 1, hw, hw], "y": {"shape": [b], "dtype": "i32"}},
                        lambda b: cnn_data(b, hw), {"kind": "adam", "lr": 1e-3}, B, 9.21e9 / 128)
    if name == "c3":
        B = over.get("batch", 4096)
        return Workload("char_mlp_27x3", lambda: CharMLP(), charmlp_loss,
                        lambda b: {"ids": {"shape": [b, 3], "dtype": "i32"},
                                   "targets": {"shape": [b], "dtype": "i32"}},
                        lambda b: charmlp_data(b), {"kind": "sgd", "lr": 0.1, "momentum": 0.9},
                        B, 0.30e9 / 4096)
    if name in ("c4", "c5"):
        if name == "c4":
            V, T, D, L, H, B, p = 65, 256, 384, 6, 6, 64, 0.2
            opt = {"kind": "adamw", "lr": 3e-4, "weightDecay": 0.1}
        else:
            V, T, D, L, H, B, p = 50304, 1024, 768, 12, 12, 256, 0.0
            opt = {"kind": "adamw", "lr": LRS.cosineAnnealing(peak=6e-4, final=6e-5,
                                                               steps=over.get("sched_steps", 1000)),
                   "weightDecay": 0.1}
        V, T, D = over.get("vocab", V), over.get("T", T), over.get("D", D)
        L, H, B, p = over.get("layers", L), over.get("heads", H), over.get("batch", B), over.get("dropout", p)
        return Workload(f"gpt_d{D}_L{L}_T{T}_V{V}", lambda: GPT(V, T, D, L, H, p), gpt_loss,
                        lambda b: {"tokens": {"shape": [b, T], "dtype": "i32"},
                                   "targets": {"shape": [b, T], "dtype": "i32"}},
                        lambda b: gpt_data(b, T, V), opt, B, _gpt_flops(V, T, D, L),
                        {"V": V, "T": T, "D": D, "L": L, "H": H})
    raise ValueError(name)


def shard(data: Dict[str, np.ndarray], rank: int, world: int) -> Dict[str, np.ndarray]:
    """Contiguous batch slice [r*B/W, (r+1)*B/W) for each input."""
    out = {}
    for k, v in data.items():
        b = v.shape[0] // world
        out[k] = np.ascontiguousarray(v[rank * b:(rank + 1) * b])
    return out
