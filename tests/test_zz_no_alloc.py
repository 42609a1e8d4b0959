"""The allocation-free column-sum entry point (tg_colsum_noalloc).

It exists for callers that may not allocate device memory (a host whose own
pool owns the GPU's memory, or a latency-critical loop that must not call
cudaMalloc). This checks, through the C ABI, that two calls in a row give the
same column sums as the regular path (a sum_to_shape graph run with tg_run,
which allocates its scratch in the graph's arena), within the tolerance the
other GPU tests use, including shapes at both extremes of the chunking.

The file sorts last so that a run stopping at the first failure has already
run every other test.
"""
import numpy as np
import pytest

import tensorgrad_b200 as tg
from tensorgrad_b200 import backend as BK
from tensorgrad_b200.trace import tensor_input as T

from .test_gpu_ops import close, rnd, run

pytestmark = pytest.mark.gpu


def _noalloc(lib, torch, x: np.ndarray) -> np.ndarray:
    outer, inner = x.shape
    xd = torch.from_numpy(x).cuda()
    od = torch.empty(inner, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.tg_colsum_noalloc(xd.data_ptr(), od.data_ptr(), outer, inner, stream)
    assert rc == 0, lib.tg_last_error_message().decode()
    torch.cuda.synchronize()
    return od.cpu().numpy()


def test_colsum_noalloc_matches_regular_path(ctx):
    import torch
    lib = BK.load()
    for call, (outer, inner, seed) in enumerate([(16384, 384, 50), (4096, 1536, 51)]):
        x = rnd([outer, inner], seed)
        ref = run(ctx, lambda: tg.sumToShape(T("x", [outer, inner]), [inner]), {"x": x})
        got = _noalloc(lib, torch, x)
        close(got, ref)
        assert np.array_equal(got, ref), f"call {call}: same kernel, same order, should be identical"


def test_colsum_noalloc_extreme_shapes(ctx):
    """The chunking bounds the partial sums: chunks x columns <= 8 x SMs x 128,
    which stays under the fixed array for up to 256 SMs. Very wide rows, very
    long columns and a near-worst case on 148 SMs ([128, 75648]: two chunks of
    75648 columns, 151296 partial sums) match the regular path."""
    import torch
    lib = BK.load()
    for outer, inner, seed in [(64, 140000, 52), (200000, 3, 53), (128, 75648, 54)]:
        x = rnd([outer, inner], seed)
        ref = run(ctx, lambda: tg.sumToShape(T("x", [outer, inner]), [inner]), {"x": x})
        np.testing.assert_array_equal(_noalloc(lib, torch, x), ref)
