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


def test_memory_bound_rooflines_from_launch_bytes():
    from bench import memory_bound_rooflines
    labels = ["fused_ew|add+mul", "matmul|M=1 N=1 K=1 b=1", "fused_ew|exp", "colsum"]
    prof = [1.0, 5.0, 1.0, 0.5]                     # ms
    nbytes = [4e9, 0.0, 2e9, 1e9]
    r = memory_bound_rooflines(labels, prof, nbytes, hbm=6000.0)
    assert r["fused_ew"]["launches"] == 2 and r["fused_ew"]["gbs"] == 3000.0
    assert r["fused_ew"]["frac"] == 0.5
    assert r["colsum"]["gbs"] == 2000.0
    assert "matmul" not in r
    assert r["all"]["bytes"] == 7e9 and abs(r["all"]["gbs"] - 7e9 / 2.5e-3 / 1e9) < 1e-9


def test_traffic_from_an_ncu_raw_csv(tmp_path):
    from bench import ncu_traffic
    p = tmp_path / "raw.csv"
    p.write_text('"ID","Kernel Name","dram__bytes_read.sum","dram__bytes_write.sum"\n'
                 '"","","Mbyte","Kbyte"\n'
                 '"0","void tg::gemm_tc_kernel<0>(...)","10.5","500"\n'
                 '"1","tgew_0123","99","99"\n'
                 '"2","void tg::gemm_tc_kernel<1>(...)","20.5","1,500"\n')
    assert abs(ncu_traffic(str(p), r"gemm_tc") - ((10.5e6 + 0.5e6) + (20.5e6 + 1.5e6)) / 2) < 1e-3
