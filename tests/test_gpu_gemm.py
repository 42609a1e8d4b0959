"""tcgen05 3xTF32 GEMM parity: every operand layout the planner produces
(A and B each K-major or MN-major), ragged tiles, batched head views, and a
large-K reduction, against the f64 oracle at the op tolerance. Row strides
that are not a multiple of 16 bytes (a vocabulary of 65 or 70) are staged into
padded copies before the tensor-core GEMM."""
import numpy as np
import pytest

import tensorgrad_b200 as tg
from tensorgrad_b200.trace import tensor_input as T

from .test_gpu_ops import rnd, run

T_ = T

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,K,N", [(300, 200, 260), (128, 64, 128), (1000, 96, 70), (256, 200, 30), (256, 30, 200),
                                   (2048, 384, 65), (2048, 65, 384), (384, 4096, 65)])
def test_gemm_layouts(ctx, ta, tb, M, K, N):
    a = rnd([K, M] if ta else [M, K], 40)
    b = rnd([N, K] if tb else [K, N], 41)

    def build():
        A = T("a", list(a.shape))
        B = T("b", list(b.shape))
        return tg.matmul(tg.swapAxes(A, 0, 1) if ta else A, tg.swapAxes(B, 0, 1) if tb else B)
    run(ctx, build, {"a": a, "b": b})


def test_gemm_attention_views(ctx):
    B_, Tn, H, d = 2, 128, 3, 64
    x = rnd([B_, Tn, H * d], 42)
    y = rnd([B_, Tn, H * d], 43)

    def build():
        q = tg.splitHeads(T("x", [B_, Tn, H * d]), H)
        k = tg.splitHeads(T("y", [B_, Tn, H * d]), H)
        s = tg.mul(tg.matmul(q, tg.swapAxes(k, -1, -2)), 0.125)
        return tg.mergeHeads(tg.matmul(s, k))
    run(ctx, build, {"x": x, "y": y})


def test_gemm_long_k_weight_grad_shape(ctx):
    x = rnd([8192, 96], 44)
    dy = rnd([8192, 160], 45)
    run(ctx, lambda: tg.matmul(tg.swapAxes(T("x", [8192, 96]), 0, 1), T("dy", [8192, 160])), {"x": x, "dy": dy})


def test_gemm_tc_error_flag_clear(ctx):
    import ctypes
    from tensorgrad_b200 import backend as BK
    lib = BK.load()
    assert lib.tg_debug_gemm_error(1) == 0


def test_gemm_split_k_batched(ctx):
    """Few output tiles and a long K: the K range is split over CTAs and the
    partial tiles are summed in split order."""
    a = rnd([3, 64, 2048], 46)
    b = rnd([3, 2048, 96], 47)
    run(ctx, lambda: tg.matmul(T("a", [3, 64, 2048]), T("b", [3, 2048, 96])), {"a": a, "b": b})


def test_gemm_simt_split_k_unaligned(ctx):
    """65-wide rows (not 16-byte aligned, so not TMA-describable) with a long
    K: the CUDA-core kernel splits K and sums the partial tiles in order."""
    x = rnd([8192, 96], 48)
    dy = rnd([8192, 65], 49)
    run(ctx, lambda: tg.matmul(tg.swapAxes(T("x", [8192, 96]), 0, 1), T("dy", [8192, 65])), {"x": x, "dy": dy})


@pytest.mark.parametrize("T", [256, 384])
@pytest.mark.parametrize("form", ["PV", "PtV", "XP", "XPt"])
def test_gemm_skips_the_zero_half_of_a_causal_operand(ctx, T, form):
    """A causal softmax's result is exactly zero above its diagonal, so a
    batched GEMM with it as an operand skips the K stages of those products
    (A = P: k below the tile's end; A = P^T: k from the tile's start; B = P or
    P^T: the same for output columns). Results match the dense oracle."""
    B_, H, d = 2, 3, 64
    s = rnd([B_, H, T, T], 90, -3, 3)
    v = rnd([B_, H, T, d], 91)
    x = rnd([B_, H, d, T], 92)

    def build():
        P = tg.softmaxCausal(T_("s", [B_, H, T, T]))
        if form == "PV":
            return tg.matmul(P, T_("v", [B_, H, T, d]))
        if form == "PtV":
            return tg.matmul(tg.swapAxes(P, -1, -2), T_("v", [B_, H, T, d]))
        if form == "XP":
            return tg.matmul(T_("x", [B_, H, d, T]), P)
        return tg.matmul(T_("x", [B_, H, d, T]), tg.swapAxes(P, -1, -2))
    inputs = {"s": s, "v": v} if form in ("PV", "PtV") else {"s": s, "x": x}
    from tensorgrad_b200.compile import _program
    from tensorgrad_b200.trace import trace_fn
    from tensorgrad_b200 import backend as BK
    g = trace_fn(build)
    labels = BK.plan_dry(_program(g, {}, [], g.outputs[0], None, len(g.ops)))["launches"]
    assert any(l.startswith("matmul_batched") and l.endswith("causal") for l in labels), labels
    run(ctx, build, inputs)

