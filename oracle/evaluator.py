"""CPU oracle for the tensorgrad IR — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker (or the timed CPU
baseline); the product path never routes through it.

A numpy restatement of the reference's CPU evaluator ``test/_eval.ts``
(``evalGraph``/``evalOp``, test/_eval.ts:21-787): every op is evaluated in
float64 from its float32/int32 inputs and its result is rounded to float32
(int32 for i32/bool) when stored, as the reference's JS doubles are when
written into a ``Float32Array``. Sums and dot products therefore accumulate
in f64 (test/_eval.ts:214-218, :283-287).

Three op families are defined by the reference's WGSL kernels rather than by
``_eval.ts``, and follow ``src/codegen.ts``:
  * ``adam_update_m/v/p`` — ``_eval.ts`` throws for them (test/_eval.ts:611-614);
    formulas from src/codegen.ts:841-905, constants rounded to f32.
  * ``dropout``/``randn``/``categorical_last`` — the PCG hash in exact u32
    arithmetic as in the WGSL (src/codegen.ts:212-268, :409-445). The JS
    restatement multiplies ``h * 747796405`` in f64 (test/_eval.ts:569),
    which drops low bits once the product passes 2^53, so it disagrees with
    the GPU kernel it mirrors; the WGSL is the reference's product, so this
    oracle follows it. The dropout keep test is ``f32(h) / 2^32 >= f32(p)``
    with ``f32(p)`` from ``p.toFixed(8)`` (src/codegen.ts:263-265).

Graphs are the JSON wire form (``tensors``/``ops``/``outputs``/``captures``).
"""
from __future__ import annotations

from typing import Dict

import numpy as np

F32 = np.float32
F64 = np.float64
# Accumulation type of vf() operands. f64 is the oracle; the tests switch it
# to f32 (eval_graph(..., accum=np.float32)) only to measure how far any f32
# evaluation of the same graph lands from the f64 one.
_ACC = [F64]


def _np_dtype(dt: str):
    return np.float32 if dt == "f32" else np.int32


def shape_size(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def _store(x, shape, dtype: str) -> np.ndarray:
    return np.ascontiguousarray(np.broadcast_to(np.asarray(x), shape)).astype(_np_dtype(dtype)).reshape(shape)


def pcg_hash(x: np.ndarray) -> np.ndarray:
    """One PCG output permutation on uint32 (src/codegen.ts:224-227)."""
    h = (x.astype(np.uint64) * np.uint64(747796405) + np.uint64(2891336453)) & np.uint64(0xFFFFFFFF)
    h = h.astype(np.uint32)
    sh = (h >> np.uint32(28)) + np.uint32(4)
    h = ((h >> sh) ^ h).astype(np.uint64) * np.uint64(277803737) & np.uint64(0xFFFFFFFF)
    h = h.astype(np.uint32)
    return (h >> np.uint32(22)) ^ h


def _salt_const(salt: int) -> np.uint32:
    return np.uint32((salt * 0x9E3779B1) & 0xFFFFFFFF)


def f32_literal(x: float) -> np.float32:
    """The f32 value of a WGSL literal printed with ``toFixed(8)``."""
    return np.float32(float(f"{x:.8f}"))


def dropout_mask(seed: int, salt: int, p: float, n: int, offset: int = 0) -> np.ndarray:
    """Per-element multiplier (0 or f32(1/(1-p))) for elements offset..offset+n-1."""
    idx = (np.arange(offset, offset + n, dtype=np.uint64) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    h = pcg_hash(np.uint32(seed & 0xFFFFFFFF) ^ _salt_const(salt) ^ idx)
    u = h.astype(np.float32) / np.float32(4294967296.0)
    keep = u >= f32_literal(p)
    return np.where(keep, f32_literal(1.0 / (1.0 - p)), np.float32(0.0)).astype(np.float32)


def _erf_as(x: np.ndarray) -> np.ndarray:
    """Abramowitz & Stegun 7.1.26, as the reference evaluates erf (test/_eval.ts:193-198)."""
    s = np.sign(x)
    ax = np.abs(x)
    t = 1.0 / (1.0 + 0.3275911 * ax)
    p = t * (0.254829592 + t * (-0.284496736 + t * (1.421413741 + t * (-1.453152027 + t * 1.061405429))))
    return s * (1.0 - p * np.exp(-ax * ax))


_UNARY = {
    "sqrt": np.sqrt,
    "rsqrt": lambda x: 1.0 / np.sqrt(x),
    "log": np.log,
    "exp": np.exp,
    "relu": lambda x: np.maximum(x, 0.0),
    "neg": lambda x: -x,
    "abs": np.abs,
    "tanh": np.tanh,
    "sin": np.sin,
    "cos": np.cos,
    "erf": _erf_as,
    "sigmoid": lambda x: 0.5 + 0.5 * np.tanh(0.5 * x),
}

_BIN = {
    "add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide,
    "min": np.minimum, "max": np.maximum,
}


def _conv_patches(x: np.ndarray, kh, kw, sh, sw, ph, pw, hout, wout, pad_value=0.0):
    """[B,C,H,W] -> [B,C,kh,kw,hout,wout] window view (padded)."""
    B, C, H, W = x.shape
    xp = np.full((B, C, H + 2 * ph + kh * sh + kh, W + 2 * pw + kw * sw + kw), pad_value, dtype=x.dtype)
    xp[:, :, ph:ph + H, pw:pw + W] = x
    out = np.empty((B, C, kh, kw, hout, wout), dtype=x.dtype)
    for i in range(kh):
        for j in range(kw):
            out[:, :, i, j] = xp[:, :, i:i + sh * hout:sh, j:j + sw * wout:sw]
    return out


def eval_op(op: dict, vals: Dict[int, np.ndarray], inputs: Dict[str, np.ndarray], g: dict,
            dp_rank: int = 0) -> np.ndarray:
    """Evaluate one op (test/_eval.ts:94-787). ``dp_rank`` shifts the element
    index fed to the dropout hash by ``dp_rank * numel`` so a batch shard sees
    the same mask as the matching slice of the full-batch graph."""
    T = g["tensors"]
    out_t = T[op["out"]]
    shape = tuple(out_t["shape"])
    dt = out_t["dtype"]
    k = op["kind"]

    def v(i):
        return vals[i]

    def vf(i):
        return vals[i].astype(_ACC[0])

    if k in ("param_input", "tensor_input"):
        if op["name"] not in inputs:
            raise KeyError(f"eval: missing input '{op['name']}'")
        return np.asarray(inputs[op["name"]]).astype(_np_dtype(dt)).reshape(shape)
    if k == "state_input":
        if op["name"] in inputs:
            return np.asarray(inputs[op["name"]]).astype(_np_dtype(dt)).reshape(shape)
        return np.full(shape, op["initValue"] if dt == "f32" else 0, dtype=_np_dtype(dt))
    if k in ("const_scalar", "const_fill"):
        return _store(op["value"], shape, dt)
    if k == "arange":
        return np.arange(op["n"]).astype(_np_dtype(dt))
    if k in _BIN:
        return _store(_BIN[k](vf(op["a"]), vf(op["b"])), shape, dt)
    if k == "mul_scalar":
        return _store(vf(op["a"]) * op["scalar"], shape, dt)
    if k == "add_scalar":
        return _store(vf(op["a"]) + op["scalar"], shape, dt)
    if k in _UNARY:
        with np.errstate(all="ignore"):
            return _store(_UNARY[k](vf(op["a"])), shape, dt)
    if k in ("mean_last", "sum_last"):
        a = vf(op["a"])
        s = a.sum(axis=-1)
        if k == "mean_last":
            s = s / a.shape[-1]
        return _store(s.reshape(shape), shape, dt)
    if k == "argmax_last":
        return np.argmax(v(op["a"]), axis=-1).astype(np.int32).reshape(shape)
    if k in ("reshape", "stop_gradient"):
        return v(op["a"]).reshape(shape).copy()
    if k == "permute":
        return np.ascontiguousarray(np.transpose(v(op["a"]), op["perm"]))
    if k in ("matmul", "matmul_batched"):
        return _store(np.matmul(vf(op["a"]), vf(op["b"])), shape, dt)
    if k == "one_hot":
        idx = v(op["indices"]).astype(np.int64)
        D = op["depth"]
        out = np.zeros(idx.shape + (D,), dtype=_np_dtype(dt))
        ok = (idx >= 0) & (idx < D)
        flat = out.reshape(-1, D)
        rows = np.nonzero(ok.reshape(-1))[0]
        flat[rows, idx.reshape(-1)[rows]] = 1
        return out
    if k in ("less", "greater"):
        a, b = vf(op["a"]), vf(op["b"])
        r = (a < b) if k == "less" else (a > b)
        return _store(r.astype(np.int32), shape, dt)
    if k == "where":
        c = v(op["cond"]) != 0
        return _store(np.where(c, vf(op["a"]), vf(op["b"])), shape, dt)
    if k == "log_softmax_last":
        a = vf(op["a"])
        m = a.max(axis=-1, keepdims=True)
        ls = np.log(np.exp(a - m).sum(axis=-1, keepdims=True)) + m
        return _store(a - ls, shape, dt)
    if k == "softmax_causal_last":
        a = vf(op["a"])
        D = a.shape[-1]
        mask = np.tril(np.ones((D, D), dtype=bool))
        am = np.where(mask, a, -np.inf)
        m = am.max(axis=-1, keepdims=True)
        e = np.where(mask, np.exp(am - m), 0.0)
        return _store(e / e.sum(axis=-1, keepdims=True), shape, dt)
    if k == "where_causal":
        a = vf(op["a"])
        D = a.shape[-1]
        mask = np.tril(np.ones((D, D), dtype=bool))
        return _store(np.where(mask, a, op["fillValue"]), shape, dt)
    if k == "slice_range":
        sl = [slice(None)] * len(shape)
        sl[op["axis"]] = slice(op["start"], op["end"])
        return np.ascontiguousarray(v(op["a"])[tuple(sl)])
    if k == "scatter_axis":
        out = np.zeros(shape, dtype=_np_dtype(dt))
        sl = [slice(None)] * len(shape)
        sl[op["axis"]] = slice(op["start"], op["end"])
        out[tuple(sl)] = v(op["a"])
        return out
    if k == "concat":
        return np.concatenate([v(i) for i in op["inputs"]], axis=op["axis"]).astype(_np_dtype(dt))
    if k == "broadcast_to":
        return _store(v(op["a"]), shape, dt)
    if k == "sum_to_shape":
        a = vf(op["a"])
        lead = a.ndim - len(shape)
        s = a.sum(axis=tuple(range(lead))) if lead > 0 else a
        axes = tuple(i for i, d in enumerate(shape) if d == 1 and s.shape[i] != 1)
        if axes:
            s = s.sum(axis=axes, keepdims=True)
        return _store(s, shape, dt)
    if k == "relu_grad":
        return _store(np.where(vf(op["x"]) > 0, vf(op["dy"]), 0.0), shape, dt)
    if k == "dropout":
        a = v(op["a"]).astype(F32)
        seed = int(v(op["seed"]).reshape(-1)[0]) & 0xFFFFFFFF
        mask = dropout_mask(seed, op["salt"], op["p"], a.size, dp_rank * a.size).reshape(a.shape)
        return (a * mask).astype(F32)
    if k == "randn":
        seed = int(v(op["seed"]).reshape(-1)[0]) & 0xFFFFFFFF
        n = shape_size(shape)
        idx = np.arange(n, dtype=np.uint64).astype(np.uint32)
        h1 = pcg_hash(np.uint32(seed) ^ _salt_const(op["salt"]) ^ idx)
        h2 = pcg_hash(h1)
        u1 = np.maximum(np.float32(1e-10), h1.astype(np.float32) / np.float32(4294967296.0)).astype(F64)
        u2 = (h2.astype(np.float32) / np.float32(4294967296.0)).astype(F64)
        return _store((np.sqrt(-2.0 * np.log(u1)) * np.cos(2 * np.pi * u2)).reshape(shape), shape, dt)
    if k == "categorical_last":
        a = vf(op["a"])
        seed = int(v(op["seed"]).reshape(-1)[0]) & 0xFFFFFFFF
        idx = np.arange(a.size, dtype=np.uint64).astype(np.uint32)
        h = pcg_hash(np.uint32(seed) ^ _salt_const(op["salt"]) ^ idx)
        u = np.maximum(np.float32(1e-10), h.astype(np.float32) / np.float32(4294967296.0)).astype(F64)
        gmb = -np.log(-np.log(u))
        return np.argmax(a + gmb.reshape(a.shape), axis=-1).astype(np.int32).reshape(shape)
    if k == "adam_update_m":
        b1 = op["beta1"]
        return (float(F32(b1)) * vf(op["m"]) + float(F32(1 - b1)) * vf(op["g"])).astype(F32)
    if k == "adam_update_v":
        b2 = op["beta2"]
        gg = vf(op["g"])
        return (float(F32(b2)) * vf(op["v"]) + float(F32(1 - b2)) * gg * gg).astype(F32)
    if k == "adam_update_p":
        shrink = float(v(op["decayShrinkTensor"]).reshape(-1)[0]) if op["decayShrinkTensor"] is not None \
            else float(F32(op["decayShrink"]))
        lrt = float(v(op["lrt"]).reshape(-1)[0])
        r = shrink * vf(op["p"]) - lrt * vf(op["mNew"]) / (np.sqrt(vf(op["vNew"])) + float(F32(op["eps"])))
        return r.astype(F32)
    if k == "conv2d":
        x, w = vf(op["input"]), vf(op["weight"])
        B, cin, H, W = x.shape
        cout, cpg, kh, kw = w.shape
        G = op["groups"]
        hout, wout = shape[2], shape[3]
        pt = _conv_patches(x, kh, kw, op["strideH"], op["strideW"], op["padH"], op["padW"], hout, wout)
        pt = pt.reshape(B, G, cpg, kh, kw, hout, wout)
        wg = w.reshape(G, cout // G, cpg, kh, kw)
        out = np.einsum("bgcijhw,gocij->bgohw", pt, wg, optimize=True)
        return _store(out.reshape(shape), shape, dt)
    if k == "conv2d_input_grad":
        w, dy = vf(op["weight"]), vf(op["dy"])
        cout, cpg, kh, kw = w.shape
        G = op["groups"]
        B, cin, H, W = shape
        sh, sw, ph, pw = op["strideH"], op["strideW"], op["padH"], op["padW"]
        hout, wout = dy.shape[2], dy.shape[3]
        dyg = dy.reshape(B, G, cout // G, hout, wout)
        wg = w.reshape(G, cout // G, cpg, kh, kw)
        full = np.zeros((B, G, cpg, H + 2 * ph + kh * sh + kh, W + 2 * pw + kw * sw + kw), dtype=F64)
        for i in range(kh):
            for j in range(kw):
                contrib = np.einsum("bgohw,goc->bgchw", dyg, wg[:, :, :, i, j], optimize=True)
                full[:, :, :, i:i + sh * hout:sh, j:j + sw * wout:sw] += contrib
        out = full[:, :, :, ph:ph + H, pw:pw + W].reshape(shape)
        return _store(out, shape, dt)
    if k == "conv2d_weight_grad":
        x, dy = vf(op["input"]), vf(op["dy"])
        B, cin, H, W = x.shape
        cout, cpg, kh, kw = shape
        G = op["groups"]
        hout, wout = dy.shape[2], dy.shape[3]
        pt = _conv_patches(x, kh, kw, op["strideH"], op["strideW"], op["padH"], op["padW"], hout, wout)
        pt = pt.reshape(B, G, cpg, kh, kw, hout, wout)
        dyg = dy.reshape(B, G, cout // G, hout, wout)
        out = np.einsum("bgcijhw,bgohw->gocij", pt, dyg, optimize=True)
        return _store(out.reshape(shape), shape, dt)
    if k in ("max_pool_2d", "max_pool_2d_grad"):
        x = v(op["input"]).astype(F32)
        kh, kw, sh, sw, ph, pw = op["kH"], op["kW"], op["strideH"], op["strideW"], op["padH"], op["padW"]
        B, C, H, W = x.shape
        if k == "max_pool_2d":
            hout, wout = shape[2], shape[3]
        else:
            hout, wout = T[op["dy"]]["shape"][2], T[op["dy"]]["shape"][3]
        pt = _conv_patches(x, kh, kw, sh, sw, ph, pw, hout, wout, pad_value=-np.inf)
        flat = pt.reshape(B, C, kh * kw, hout, wout)
        # Strict '>' scan from -3.4e38: the first maximum in (kh, kw) order wins
        # (test/_eval.ts:716-779); np.argmax also returns the first maximum.
        arg = np.argmax(flat, axis=2)
        mx = np.take_along_axis(flat, arg[:, :, None], axis=2)[:, :, 0]
        valid = mx > F32(-3.4e38)
        if k == "max_pool_2d":
            return np.where(valid, mx, F32(-3.4e38)).astype(F32)
        dy = v(op["dy"]).astype(F64)
        out = np.zeros((B, C, H + 2 * ph + kh * sh + kh, W + 2 * pw + kw * sw + kw), dtype=F64)
        ai, aj = arg // kw, arg % kw
        bi, ci = np.meshgrid(np.arange(B), np.arange(C), indexing="ij")
        for ho in range(hout):
            for wo in range(wout):
                sel = valid[:, :, ho, wo]
                hh = ho * sh + ai[:, :, ho, wo]
                ww = wo * sw + aj[:, :, ho, wo]
                np.add.at(out, (bi[sel], ci[sel], hh[sel], ww[sel]), dy[:, :, ho, wo][sel])
        return _store(out[:, :, ph:ph + H, pw:pw + W], shape, dt)
    raise ValueError(f"eval: unhandled op kind {k}")


def eval_graph(g: dict, inputs: Dict[str, np.ndarray], dp_rank: int = 0, accum=F64) -> Dict[int, np.ndarray]:
    """Evaluate every op in order (test/_eval.ts:21-27). ``accum`` is the
    arithmetic type of elementwise ops, reductions and contractions: f64 for
    the oracle; f32 gives a plain single-precision CPU evaluation whose
    distance from the oracle is the f32 error floor of the graph."""
    vals: Dict[int, np.ndarray] = {}
    prev, _ACC[0] = _ACC[0], accum
    try:
        for op in g["ops"]:
            vals[op["out"]] = eval_op(op, vals, inputs, g, dp_rank)
    finally:
        _ACC[0] = prev
    return vals
