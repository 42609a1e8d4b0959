"""Benchmark: train samples/sec for the GPT d384 L6 T256 config (config 4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c4]

One step = forward + backward + AdamW update of GPT(V=65, T=256, d=384,
L=6, H=6, dropout 0.2) on 64 sequences per GPU (weak scaling: global batch
64*N, data-parallel gradient allreduce over NCCL). Prints one JSON line.

* value: samples/s with inputs resident on the device, K steps timed with CUDA
  events on the backend's stream, max over ranks.
* e2e: samples/s through the public step call (host inputs -> H2D each step,
  loss D2H each step), same K.
* roofline: the dominant kernel class of one step, measured live with events
  around every launch (tg_profile_step).
* cpu_baseline: the CPU oracle (numpy restatement of the reference's CPU
  evaluator, f64 accumulate) on a bounded sample, rank 0 only.
* --impl reference: times that CPU path alone on the same config and prints
  the reference line (the reference is a browser WebGPU library; its own CPU
  evaluator is the only implementation runnable here).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from tensorgrad_b200 import configs as CF  # noqa: E402

METRIC = "train samples/sec (GPT d384 L6 T256, config 4)"
UNIT = "samples/s"
# launch classes whose roofline is HBM bandwidth (their algorithmic bytes come
# from the planner, tg_launch_bytes)
MEMORY_BOUND = ("fused_ew", "fused_red", "softmax_causal_last+dropout", "softmax_causal_last", "log_softmax_last",
                "colsum", "rowsum", "dropout", "adam_flat", "sgd_flat", "gather_rows", "embedding_grad")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def gemm_flops_of(labels):
    """Algorithmic FLOPs (2·M·N·K per batch entry) of the GEMM launches, read
    from their launch labels ("matmul|M=.. N=.. K=.. b=.. ..."). Matmuls that
    a fused kernel computes (attention) are not GEMM launches and not counted."""
    fl = []
    for lab in labels:
        kind, _, rest = lab.partition("|")
        if kind not in ("matmul", "matmul_batched"):
            continue
        f = dict(kv.split("=", 1) for kv in rest.split() if "=" in kv)
        fl.append(2.0 * int(f["M"]) * int(f["N"]) * int(f["K"]) * int(f.get("b", 1)))
    return fl


def ncu_traffic(csv_path, kernel_regex):
    """Mean dram__bytes_read.sum + dram__bytes_write.sum per launch of the
    kernels matching kernel_regex in an `ncu --csv --page raw` export."""
    import csv
    import re
    rows = list(csv.reader(open(csv_path)))
    hdr = next(i for i, r in enumerate(rows) if "Kernel Name" in r)
    h = rows[hdr]
    kn, rd, wr = h.index("Kernel Name"), h.index("dram__bytes_read.sum"), h.index("dram__bytes_write.sum")
    unit = rows[hdr + 1] if rows[hdr + 1] and rows[hdr + 1][kn] == "" else None
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    tot = []
    for r in rows[hdr + 1 + (1 if unit else 0):]:
        if len(r) > max(kn, rd, wr) and re.search(kernel_regex, r[kn]):
            f = lambda c: float(r[c].replace(",", "")) * (scale.get(unit[c], 1) if unit else 1)
            tot.append(f(rd) + f(wr))
    return sum(tot) / len(tot) if tot else None


def memory_bound_rooflines(labels, prof, nbytes, hbm):
    """Per class of HBM-bound launches: algorithmic bytes of one step, the
    class's live event time, achieved GB/s and its fraction of the measured
    copy bandwidth."""
    out, tb, tm = {}, 0.0, 0.0
    for lab, t, b in zip(labels, prof, nbytes):
        k = lab.split("|")[0]
        if k not in MEMORY_BOUND or b <= 0:
            continue
        c = out.setdefault(k, {"launches": 0, "bytes": 0.0, "ms": 0.0})
        c["launches"] += 1
        c["bytes"] += b
        c["ms"] += t
        tb += b
        tm += t
    for c in out.values():
        c["gbs"] = c["bytes"] / (c["ms"] * 1e-3) / 1e9 if c["ms"] > 0 else None
        c["frac"] = c["gbs"] / hbm if c["gbs"] else None
    out = dict(sorted(out.items(), key=lambda kv: -kv[1]["ms"]))
    out["all"] = {"bytes": tb, "ms": tm, "gbs": tb / (tm * 1e-3) / 1e9 if tm > 0 else None,
                  "frac": tb / (tm * 1e-3) / 1e9 / hbm if tm > 0 else None}
    return out


def cpu_baseline(w, sample_batch: int, threads: int):
    """Times one oracle training step on `sample_batch` sequences."""
    from oracle.driver import OracleTrainer
    from tensorgrad_b200.compile import build_training_ir, initial_params
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(sample_batch), w.optimizer)
    init = initial_params(ir.graph, ir.materialized.initFns, CF.PARAM_SEED)
    orc = OracleTrainer(ir.program, init)
    data = w.data(sample_batch)
    t0 = time.perf_counter()
    orc.step(data)
    dt = time.perf_counter() - t0
    return sample_batch / dt, dt


def run_reference(args, w):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sample = 2
    vals = []
    for _ in range(max(1, args.steps)):
        v, dt = cpu_baseline(w, sample, threads)
        vals.append(v)
    v = float(np.median(vals))
    metric = METRIC if args.config == "c4" else f"train samples/sec ({w.name}, config {args.config[1:]})"
    line = {"impl": "reference", "metric": metric, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sample / v,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (mulberry32 seed 1234 tokens)",
            "config": {"workload": w.name, "global_batch": sample, "seq_len": w.extra.get("T"),
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"one training step of {w.name} at batch {sample} (full model) per timed "
                                       "step; numpy restatement of the reference CPU evaluator"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


MODEL_DESC = {
    "c1": "MLP 1-64-64-1 ReLU, Adam",
    "c2": "CNN conv3x3 1-32, 32-64, maxpool, 9216-128-10, Adam",
    "c3": "char MLP V27 ctx3 emb10 hidden200, SGD momentum",
    "c4": "GPT V65 T256 d384 L6 H6 dropout0.2, AdamW",
    "c5": "GPT V50304 T1024 d768 L12 H12, AdamW cosine",
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours")
    ap.add_argument("--config", default="c4")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU (default: the config's; smaller only for profiling captures)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-out", default=None, help="write per-launch (label, ms) of one profiled step as JSON")
    ap.add_argument("--traffic-csv", default=None,
                    help="ncu --csv --page raw export of GEMM launches of this workload (dram__bytes_read/write): "
                         "fills roofline.traffic; without it traffic is null")
    args = ap.parse_args()
    w = CF.workload(args.config, **({"batch": args.batch} if args.batch else {}))
    if args.impl == "reference":
        return run_reference(args, w)

    import torch
    from tensorgrad_b200 import backend as BK
    from tensorgrad_b200.compile import build_training_ir, initial_params

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from tensorgrad_b200.dist import init_data_parallel
        ctx, _group = init_data_parallel(local)
    else:
        ctx = BK.Context(local, rank, world, None)
    # weak scaling: a fixed batch per rank. c5 names its global batch at 8 GPUs
    # (256 = 32 per GPU), so its per-rank batch is 32 unless --batch says otherwise
    per_rank = 32 if args.config == "c5" and not args.batch else w.global_batch
    gb = per_rank * world
    ir = build_training_ir(w.make_model(), w.loss, w.inputs(per_rank), w.optimizer)
    init = initial_params(ir.graph, ir.materialized.initFns, CF.PARAM_SEED)
    dg = BK.DeviceGraph(ctx, ir.program)
    dg.upload_params(init)
    data = CF.shard(w.data(gb), rank, world)
    in_bytes = sum(v.nbytes for v in data.values())

    stream = torch.cuda.ExternalStream(ctx.stream())

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    # warm-up (captures the CUDA graph on the first step)
    dg.set_inputs(data)
    for _ in range(args.warmup):
        dg.launch_step()
    dg.read_loss()

    # value: resident inputs, device-timed
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            dg.launch_step()
        e1.record(stream)
        loss = dg.read_loss()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    barrier()
    # e2e: public step call with host buffers
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dg.step(data)
    e2e_ms = (time.perf_counter() - t0) * 1000.0
    ms_t = torch.tensor([ms, e2e_ms], dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(ms_t[0]), float(ms_t[1])

    # per-launch profile (outside the timed region)
    labels = dg.launch_list()
    kinds = [x.split("|")[0] for x in labels]
    prof_raw = dg.profile_step()
    # An event after every launch adds a fixed delay per launch that the
    # step's own graph does not have; its size is the profiled total minus the
    # measured step time, spread evenly over the launches.
    ev_over = max(0.0, (sum(prof_raw) - ms / args.steps) / max(1, len(prof_raw)))
    prof = [max(t - ev_over, 1e-4) for t in prof_raw]
    if args.profile_out and rank == 0:
        with open(args.profile_out, "w") as f:
            json.dump([[lab, t] for lab, t in zip(labels, prof)], f)
    by_kind = {}
    for k, t in zip(kinds, prof):
        by_kind[k] = by_kind.get(k, 0.0) + t
    hbm, bf16, bf16s, src = peaks()
    gemm_ms = sum(t for k, t in zip(kinds, prof) if k in ("matmul", "matmul_batched"))
    gemm_fl = sum(gemm_flops_of(labels))
    dom = max(by_kind.items(), key=lambda kv: kv[1])[0]
    n_gemm = sum(1 for k in kinds if k in ("matmul", "matmul_batched"))
    roof = {"bound": "tensor", "kernel": "matmul+matmul_batched (all GEMM launches of one step)",
            "achieved": gemm_fl / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None, "peak": bf16,
            "unit": "TFLOP/s", "peak_source": f"{src} bf16 dense (MEASURED_PEAKS.json)",
            # DRAM bytes per GEMM launch from an ncu capture of this workload, when one is given
            "traffic": ncu_traffic(args.traffic_csv, r"gemm_tc") if args.traffic_csv else None,
            "traffic_unit": "bytes per launch (average over the captured GEMM launches)",
            "gemm_launches_per_step": n_gemm}
    roof["frac"] = roof["achieved"] / bf16 if roof["achieved"] else None
    roof["frac_of_3xtf32_effective"] = roof["achieved"] / (bf16 / 6.0) if roof["achieved"] else None
    roof["dominant_kind"] = dom
    roof["step_share"] = {k: round(v / sum(prof), 4) for k, v in sorted(by_kind.items(), key=lambda kv: -kv[1])[:8]}
    roof["memory_bound"] = memory_bound_rooflines(labels, prof, dg.launch_bytes(), hbm)
    roof["memory_bound_peak_gbs"] = hbm
    roof["profile"] = {"method": "CUDA events after every launch of one graph-replayed step",
                       "event_overhead_us_per_launch": ev_over * 1e3, "raw_total_ms": sum(prof_raw)}

    value = args.steps * gb / (ms * 1e-3)
    e2e = args.steps * gb / (e2e_ms * 1e-3)
    metric = METRIC if args.config == "c4" else f"train samples/sec ({w.name}, config {args.config[1:]})"
    line = {"metric": metric, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (mulberry32 seed 1234 tokens, random-init params seed 42)",
            "config": {"workload": w.name, "model": MODEL_DESC.get(args.config, w.name), "global_batch": gb,
                       "per_rank_batch": per_rank, "seq_len": w.extra.get("T"), "parallelism": f"dp{world}",
                       "l2": "inputs and activations exceed L2 (126 MB) every step"},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": 4},
            "gpu_launches": len(kinds) * args.steps, "roofline": roof, "clocks": clk.summary(),
            "loss": loss, "steps_per_s": args.steps / (ms * 1e-3),
            "tokens_per_s": value * w.extra["T"] if "T" in w.extra else None,
            "tflops_algorithmic": w.flops_per_sample * value / 1e12}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, dt = cpu_baseline(w, 2, os.cpu_count() or 1)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"one oracle training step at batch 2 ({dt:.1f} s); numpy f64 "
                                          "restatement of the reference CPU evaluator"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    dg.destroy()
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
