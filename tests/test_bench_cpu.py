"""bench.py helpers that run without a GPU."""
from bench import gemm_flops_of


def test_gemm_flops_come_from_gemm_launch_labels():
    labels = [
        "matmul|M=16384 N=384 K=384 b=1 Ak Bmn",
        "matmul_batched|M=256 N=64 K=256 b=384 Ak Bmn",
        "matmul|M=384 N=65 K=16384 b=1 Amn Bmn padded",
        "attn_fwd|B=32 H=12 T=1024 D=64",          # a fused kernel's matmuls are not GEMM launches
        "fused_ew|add+mul",
        "conv2d_gemm|M=10 N=10 K=10 b=1",
    ]
    assert gemm_flops_of(labels) == [2.0 * 16384 * 384 * 384, 2.0 * 256 * 64 * 256 * 384, 2.0 * 384 * 65 * 16384]
