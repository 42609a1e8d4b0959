"""Shape inference with trailing-suffix broadcasting (src/shape.ts:1-373).

Broadcasting is right-aligned NumPy broadcasting restricted the same way the
reference restricts it: equal dims unify, size-1 dims broadcast, anything else
is a ``ShapeError`` that names the user's call site.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

from .ir import CallSite, format_site, shape_size

Shape = Tuple[int, ...]


class ShapeError(Exception):
    """Shape/dtype constraint violation; ``name`` matches the reference's."""
    name = "ShapeError"

    def __init__(self, message: str, site: Optional[CallSite] = None):
        super().__init__(f"{message}\n  at {format_site(site)}" if site else message)


def fail(msg: str, site: Optional[CallSite]):
    raise ShapeError(msg, site)


def show(shape: Sequence[int]) -> str:
    return "[" + ", ".join(str(d) for d in shape) + "]"


def shapes_equal(a: Sequence[int], b: Sequence[int]) -> bool:
    return tuple(a) == tuple(b)


def broadcast_trailing(a: Sequence[int], b: Sequence[int]) -> Optional[Shape]:
    rank = max(len(a), len(b))
    out = []
    for i in range(rank):
        ai, bi = i - (rank - len(a)), i - (rank - len(b))
        av = 1 if ai < 0 else a[ai]
        bv = 1 if bi < 0 else b[bi]
        if av == bv:
            out.append(av)
        elif av == 1:
            out.append(bv)
        elif bv == 1:
            out.append(av)
        else:
            return None
    return tuple(out)


def infer_binop(name, a, b, site) -> Shape:
    r = broadcast_trailing(a, b)
    if r is None:
        fail(f"{name}: incompatible shapes {show(a)} and {show(b)}. Trailing-suffix broadcasting "
             f"only — the smaller shape must be a suffix of the larger, with size-1 axes "
             f"broadcasting to any size.", site)
    return r


def infer_mean_last(name, a, site) -> Shape:
    if len(a) == 0:
        fail(f"{name}: cannot reduce a 0-d tensor", site)
    return tuple(a[:-1]) + (1,)


def infer_sum_last(name, a, site) -> Shape:
    if len(a) == 0:
        fail(f"{name}: cannot reduce a 0-d tensor", site)
    return tuple(a[:-1])


def infer_reshape(name, a, new_shape, site) -> Shape:
    infer_idx, known = -1, 1
    for i, d in enumerate(new_shape):
        if d == -1:
            if infer_idx != -1:
                fail(f"{name}: at most one -1 dim allowed in newShape {show(new_shape)}", site)
            infer_idx = i
        elif d <= 0:
            fail(f"{name}: invalid dim {d} in newShape {show(new_shape)}", site)
        else:
            known *= d
    total = shape_size(a)
    out = list(new_shape)
    if infer_idx != -1:
        if total % known != 0:
            fail(f"{name}: cannot reshape {show(a)} (size {total}) to {show(new_shape)} — known "
                 f"dims multiply to {known}", site)
        out[infer_idx] = total // known
    elif known != total:
        fail(f"{name}: size mismatch — input {show(a)} has {total} elements but newShape "
             f"{show(new_shape)} has {known}", site)
    return tuple(out)


def infer_permute(name, a, perm, site) -> Shape:
    if len(perm) != len(a):
        fail(f"{name}: perm length {len(perm)} must equal input rank {len(a)}", site)
    seen = set()
    for p in perm:
        if p < 0 or p >= len(a):
            fail(f"{name}: perm index {p} out of range for rank {len(a)}", site)
        if p in seen:
            fail(f"{name}: perm has duplicate index {p}", site)
        seen.add(p)
    return tuple(a[p] for p in perm)


def infer_matmul(name, a, b, site) -> Shape:
    if len(a) < 2:
        fail(f"{name}: lhs must have rank >= 2, got {show(a)}", site)
    if a[-1] != b[0]:
        fail(f"{name}: inner dims don't match — {show(a)} · {show(b)} (last axis of lhs = {a[-1]}, "
             f"first axis of rhs = {b[0]})", site)
    return tuple(a[:-2]) + (a[-2], b[1])


def infer_matmul_batched(name, a, b, site) -> Shape:
    if len(a) != len(b):
        fail(f"{name}: ranks must match (got {len(a)} vs {len(b)}).", site)
    if tuple(a[:-2]) != tuple(b[:-2]):
        fail(f"{name}: batch dims must match — {show(a)} vs {show(b)}", site)
    if a[-1] != b[-2]:
        fail(f"{name}: inner dims don't match — last axis of lhs = {a[-1]}, second-to-last of "
             f"rhs = {b[-2]}", site)
    return tuple(a[:-2]) + (a[-2], b[-1])


def infer_where_causal(name, a, site) -> Shape:
    if len(a) < 2:
        fail(f"{name}: requires rank >= 2, got {show(a)}", site)
    if a[-1] != a[-2]:
        fail(f"{name}: last two axes must be equal (square mask), got {show(a)}", site)
    return tuple(a)


def infer_slice_range(name, a, axis, start, end, site) -> Shape:
    if len(a) == 0:
        fail(f"{name}: cannot slice 0-d tensor", site)
    if axis < 0 or axis >= len(a):
        fail(f"{name}: axis {axis} out of range for shape {show(a)}", site)
    if start < 0 or end > a[axis] or start >= end:
        fail(f"{name}: invalid range [{start}, {end}) for axis {axis} of size {a[axis]}", site)
    out = list(a)
    out[axis] = end - start
    return tuple(out)


def infer_scatter_axis(name, a, out_shape, axis, start, end, site) -> Shape:
    if len(out_shape) == 0:
        fail(f"{name}: cannot scatter into 0-d tensor", site)
    if axis < 0 or axis >= len(out_shape):
        fail(f"{name}: axis {axis} out of range for output shape {show(out_shape)}", site)
    if start < 0 or end > out_shape[axis] or start >= end:
        fail(f"{name}: invalid range [{start}, {end}) for axis {axis}", site)
    if len(a) != len(out_shape):
        fail(f"{name}: input rank {len(a)} must equal output rank {len(out_shape)}", site)
    for i, d in enumerate(out_shape):
        exp = end - start if i == axis else d
        if a[i] != exp:
            fail(f"{name}: input {show(a)} doesn't match output {show(out_shape)} at axis {i}", site)
    return tuple(out_shape)


def infer_concat(name, shapes, axis, site) -> Shape:
    first = shapes[0]
    if axis < 0 or axis >= len(first):
        fail(f"{name}: axis {axis} out of range for shape {show(first)}", site)
    total = first[axis]
    for i, s in enumerate(shapes[1:], 1):
        if len(s) != len(first):
            fail(f"{name}: input {i} has rank {len(s)}, expected {len(first)}", site)
        for d in range(len(first)):
            if d != axis and s[d] != first[d]:
                fail(f"{name}: input {i} has shape {show(s)}, must match {show(first)} except "
                     f"along axis {axis}", site)
        total += s[axis]
    out = list(first)
    out[axis] = total
    return tuple(out)


def infer_broadcast_to(name, a, target, site) -> Shape:
    if len(a) > len(target):
        fail(f"{name}: source rank {len(a)} > target rank {len(target)}", site)
    off = len(target) - len(a)
    for i, av in enumerate(a):
        if av != target[off + i] and av != 1:
            fail(f"{name}: cannot broadcast {show(a)} to {show(target)}", site)
    return tuple(target)


def infer_sum_to_shape(name, a, target, site) -> Shape:
    if len(target) > len(a):
        fail(f"{name}: target rank {len(target)} > source rank {len(a)}", site)
    off = len(a) - len(target)
    for i, tv in enumerate(target):
        if a[off + i] != tv and tv != 1:
            fail(f"{name}: cannot sum-reduce {show(a)} to {show(target)}", site)
    return tuple(target)


def infer_where(name, c, a, b, site) -> Shape:
    ab = broadcast_trailing(a, b)
    if ab is None:
        fail(f"{name}: a/b incompatible: {show(a)} vs {show(b)}", site)
    r = broadcast_trailing(c, ab)
    if r is None:
        fail(f"{name}: cond {show(c)} incompatible with broadcast(a, b) {show(ab)}", site)
    return r


def conv_out(name, n, k, s, p, axis, site) -> int:
    if k < 1:
        fail(f"{name}: {axis} kernel must be >= 1, got {k}", site)
    if s < 1:
        fail(f"{name}: {axis} stride must be >= 1, got {s}", site)
    if p < 0:
        fail(f"{name}: {axis} padding must be >= 0, got {p}", site)
    out = (n + 2 * p - k) // s + 1
    if out < 1:
        fail(f"{name}: {axis} output size would be {out}", site)
    return out


def infer_conv2d(name, x, w, sh, sw, ph, pw, groups, site) -> Shape:
    if len(x) != 4:
        fail(f"{name}: input must be rank-4 [B, C_in, H, W], got {show(x)}", site)
    if len(w) != 4:
        fail(f"{name}: weight must be rank-4 [C_out, C_in/groups, K_h, K_w], got {show(w)}", site)
    if not isinstance(groups, int) or groups < 1:
        fail(f"{name}: groups must be a positive integer, got {groups}", site)
    B, cin, H, W = x
    cout, wic, kh, kw = w
    if cin % groups or cout % groups:
        fail(f"{name}: channels must be divisible by groups={groups}", site)
    if cin // groups != wic:
        fail(f"{name}: input C_in={cin} doesn't match weight C_in={wic} (groups={groups})", site)
    return (B, cout, conv_out(name, H, kh, sh, ph, "H", site), conv_out(name, W, kw, sw, pw, "W", site))


def infer_max_pool2d(name, x, kh, kw, sh, sw, ph, pw, site) -> Shape:
    if len(x) != 4:
        fail(f"{name}: input must be rank-4 [B, C, H, W], got {show(x)}", site)
    B, C, H, W = x
    return (B, C, conv_out(name, H, kh, sh, ph, "H", site), conv_out(name, W, kw, sw, pw, "W", site))
