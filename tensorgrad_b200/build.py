"""Build libtgcuda.so in-tree from tensorgrad_b200/csrc (nvcc, sm_100a).

Each .cu compiles to an object under tensorgrad_b200/_build/ (rebuilt when
the source or any header is newer), then all link into
tensorgrad_b200/libtgcuda.so with the static CUDA runtime and NCCL.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtgcuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(HERE, "..", "include")]


def _nccl_link():
    for d in ("/usr/lib/x86_64-linux-gnu", "/usr/local/lib"):
        if os.path.exists(os.path.join(d, "libnccl.so")) or os.path.exists(os.path.join(d, "libnccl.so.2")):
            return ["-L" + d, "-l:libnccl.so.2"]
    return ["-lnccl"]


def build(verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".hpp", ".h"))]
    headers.append(os.path.join(HERE, "..", "include", "tensorgrad_b200.h"))
    hdr_mtime = max(os.path.getmtime(h) for h in headers if os.path.exists(h))

    def one(src):
        sp = os.path.join(CSRC, src)
        obj = os.path.join(OUT_DIR, src[:-3] + ".o")
        if os.path.exists(obj) and os.path.getmtime(obj) > max(os.path.getmtime(sp), hdr_mtime):
            return obj, False
        cmd = [NVCC, *ARCH, *FLAGS, "-c", sp, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, file=sys.stderr)
        return obj, True

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(one, srcs))
    objs = [o for o, _ in results]
    changed = any(c for _, c in results)
    if changed or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", *_nccl_link(),
               "-L/usr/local/cuda/lib64", "-lnvrtc", "-Xlinker", "-rpath=/usr/local/cuda/lib64"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
