"""ctypes binding of libtgcuda.so (the C ABI in include/tensorgrad_b200.h).

There is no CPU fallback: if the library or a GPU is missing, every entry
point raises ``BackendUnavailable``.
"""
from __future__ import annotations

import ctypes as C
import json
import os
from typing import Dict, List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtgcuda.so")

_lib = None

EXPORTED = [
    "tg_nccl_unique_id", "tg_ctx_create", "tg_ctx_destroy", "tg_graph_create", "tg_graph_info",
    "tg_upload_params", "tg_download_params", "tg_upload_states", "tg_download_states", "tg_get_counters",
    "tg_set_counters", "tg_step", "tg_run", "tg_set_inputs", "tg_launch_step",
    "tg_read_loss", "tg_stream", "tg_reset_optimizer", "tg_set_lr", "tg_destroy_graph", "tg_read_grad",
    "tg_read_tensor", "tg_launch_list", "tg_profile_step", "tg_launch_bytes", "tg_debug_gemm_error", "tg_debug_gemm_dbg", "tg_debug_gemm_trace", "tg_colsum_noalloc", "tg_plan_dry", "tg_last_error_name", "tg_last_error_message",
]


class BackendUnavailable(RuntimeError):
    name = "Error"


class TgError(RuntimeError):
    """Backend failure carrying the reference-style error name."""

    def __init__(self, name: str, message: str):
        super().__init__(f"{name}: {message}")
        self.name = name
        self.message = message


class AbortError(TgError):
    def __init__(self, message: str):
        super().__init__("AbortError", message)


def load(path: str = LIB_PATH):
    """Loads the C ABI library (TG_LIB names another build of it, for A/B
    measurements of build-time variants)."""
    global _lib
    if _lib is not None:
        return _lib
    path = os.environ.get("TG_LIB", path)
    if not os.path.exists(path):
        raise BackendUnavailable(f"{path} is missing; run `python -m tensorgrad_b200.build`")
    lib = C.CDLL(path)
    vp, ip, sz = C.c_void_p, C.c_int, C.c_size_t
    cpp = C.POINTER(C.c_char_p)
    vpp = C.POINTER(C.c_void_p)
    szp = C.POINTER(C.c_size_t)
    sig = {
        "tg_nccl_unique_id": [C.c_char_p],
        "tg_ctx_create": [ip, ip, ip, C.c_char_p, C.POINTER(vp)],
        "tg_ctx_destroy": [vp],
        "tg_graph_create": [vp, ip, ip, C.c_char_p, sz],
        "tg_graph_info": [vp, ip, C.c_char_p, sz, szp],
        "tg_launch_list": [vp, ip, C.c_char_p, sz, szp],
        "tg_upload_params": [vp, ip, ip, cpp, vpp, szp],
        "tg_download_params": [vp, ip, ip, cpp, vpp, szp],
        "tg_upload_states": [vp, ip, ip, cpp, vpp, szp],
        "tg_download_states": [vp, ip, ip, cpp, vpp, szp],
        "tg_get_counters": [vp, ip, C.POINTER(C.c_int64), C.POINTER(C.c_int64)],
        "tg_set_counters": [vp, ip, C.c_int64, C.c_int64],
        "tg_step": [vp, ip, ip, cpp, vpp, szp, C.POINTER(C.c_float), vpp],
        "tg_run": [vp, ip, ip, cpp, vpp, szp, vp, vpp],
        "tg_set_inputs": [vp, ip, ip, cpp, vpp, szp, ip],
        "tg_launch_step": [vp, ip],
        "tg_read_loss": [vp, ip, C.POINTER(C.c_float)],
        "tg_stream": [vp, C.POINTER(vp)],
        "tg_reset_optimizer": [vp, ip],
        "tg_set_lr": [vp, ip, C.c_char_p, sz],
        "tg_destroy_graph": [vp, ip],
        "tg_read_grad": [vp, ip, C.c_char_p, vp],
        "tg_read_tensor": [vp, ip, ip, vp],
        "tg_profile_step": [vp, ip, C.POINTER(C.c_float), ip, C.POINTER(C.c_int)],
        "tg_launch_bytes": [vp, ip, C.POINTER(C.c_double), ip, C.POINTER(C.c_int)],
        "tg_debug_gemm_error": [ip],
        "tg_debug_gemm_dbg": [C.POINTER(C.c_int)],
        "tg_debug_gemm_trace": [C.POINTER(C.c_longlong), ip],
        "tg_colsum_noalloc": [vp, vp, C.c_int64, C.c_int64, vp],
        "tg_plan_dry": [C.c_char_p, sz, ip, C.c_char_p, sz, szp],
    }
    for name, args in sig.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = C.c_int
    lib.tg_last_error_name.restype = C.c_char_p
    lib.tg_last_error_message.restype = C.c_char_p
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != 0:
        lib = load()
        name = lib.tg_last_error_name().decode()
        msg = lib.tg_last_error_message().decode()
        if name == "AbortError":
            raise AbortError(msg)
        raise TgError(name or "Error", msg)


def _names(names: Sequence[str]):
    arr = (C.c_char_p * len(names))(*[n.encode() for n in names])
    return arr


def plan_dry(program: dict, world: int = 1) -> dict:
    """Plans `program` without a GPU (views, fusion, storage, launches).

    Returns {"info": ..., "launches": [label per kernel launch of one step],
    "kernelSources": [CUDA source of each fused elementwise kernel]}."""
    lib = load()
    data = json.dumps(program, separators=(",", ":")).encode()
    need = C.c_size_t()
    _check(lib.tg_plan_dry(data, len(data), world, None, 0, C.byref(need)))
    buf = C.create_string_buffer(need.value + 1)
    _check(lib.tg_plan_dry(data, len(data), world, buf, len(buf), C.byref(need)))
    return json.loads(buf.value.decode())


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    _check(load().tg_nccl_unique_id(buf))
    return buf.raw


class Context:
    """One device (and, for data parallelism, one rank of an NCCL communicator)."""

    def __init__(self, device: int = 0, rank: int = 0, world: int = 1, nccl_id: Optional[bytes] = None):
        lib = load()
        self.device, self.rank, self.world = device, rank, world
        h = C.c_void_p()
        _check(lib.tg_ctx_create(device, rank, world, nccl_id, C.byref(h)))
        self.h = h
        self._next_id = 1

    def new_graph_id(self) -> int:
        i = self._next_id
        self._next_id += 1
        return i

    def stream(self) -> int:
        s = C.c_void_p()
        _check(load().tg_stream(self.h, C.byref(s)))
        return s.value or 0

    def close(self) -> None:
        if self.h:
            _check(load().tg_ctx_destroy(self.h))
            self.h = None


class DeviceGraph:
    """A compiled program living on one context."""

    def __init__(self, ctx: Context, program: dict, parent: Optional["DeviceGraph"] = None,
                 graph_id: Optional[int] = None):
        self.ctx = ctx
        self.lib = load()
        self.id = graph_id if graph_id is not None else ctx.new_graph_id()
        self.program = program
        data = json.dumps(program, separators=(",", ":")).encode()
        _check(self.lib.tg_graph_create(ctx.h, self.id, parent.id if parent else -1, data, len(data)))
        g = program["graph"]
        self.tensors = g["tensors"]
        self.capture_names = list(g["captures"].keys())
        self.input_tensors = {k: v for k, v in program["inputs"].items()}
        self._loss = (C.c_float * 1)()

    def info(self) -> dict:
        need = C.c_size_t()
        buf = C.create_string_buffer(1 << 16)
        _check(self.lib.tg_graph_info(self.ctx.h, self.id, buf, len(buf), C.byref(need)))
        return json.loads(buf.value.decode())

    def launch_list(self) -> List[str]:
        need = C.c_size_t()
        _check(self.lib.tg_launch_list(self.ctx.h, self.id, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value + 1)
        _check(self.lib.tg_launch_list(self.ctx.h, self.id, buf, len(buf), C.byref(need)))
        return [s for s in buf.value.decode().split("\n") if s]

    def profile_step(self) -> List[float]:
        n = C.c_int()
        cap = 1 << 16
        buf = (C.c_float * cap)()
        _check(self.lib.tg_profile_step(self.ctx.h, self.id, buf, cap, C.byref(n)))
        return [buf[i] for i in range(min(n.value, cap))]

    def launch_bytes(self) -> List[float]:
        """Algorithmic bytes per launch (0 where not accounted), in
        launch_list order."""
        n = C.c_int()
        cap = 1 << 16
        buf = (C.c_double * cap)()
        _check(self.lib.tg_launch_bytes(self.ctx.h, self.id, buf, cap, C.byref(n)))
        return [buf[i] for i in range(min(n.value, cap))]

    # -- params -----------------------------------------------------------
    def upload_params(self, params: Dict[str, np.ndarray]) -> None:
        names = list(params)
        arrs = [np.ascontiguousarray(params[n], dtype=np.float32).reshape(-1) for n in names]
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        sizes = (C.c_size_t * len(arrs))(*[a.size for a in arrs])
        _check(self.lib.tg_upload_params(self.ctx.h, self.id, len(names), _names(names), ptrs, sizes))

    def download_params(self, shapes: Dict[str, tuple]) -> Dict[str, np.ndarray]:
        names = list(shapes)
        outs = [np.empty(shapes[n], np.float32) for n in names]
        ptrs = (C.c_void_p * len(outs))(*[a.ctypes.data for a in outs])
        sizes = (C.c_size_t * len(outs))(*[a.size for a in outs])
        _check(self.lib.tg_download_params(self.ctx.h, self.id, len(names), _names(names), ptrs, sizes))
        return dict(zip(names, outs))

    def upload_states(self, states: Dict[str, np.ndarray]) -> None:
        names = list(states)
        arrs = [np.ascontiguousarray(states[n], dtype=np.float32).reshape(-1) for n in names]
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        sizes = (C.c_size_t * len(arrs))(*[a.size for a in arrs])
        _check(self.lib.tg_upload_states(self.ctx.h, self.id, len(names), _names(names), ptrs, sizes))

    def download_states(self, shapes: Dict[str, tuple]) -> Dict[str, np.ndarray]:
        names = list(shapes)
        outs = [np.empty(shapes[n], np.float32) for n in names]
        ptrs = (C.c_void_p * len(outs))(*[a.ctypes.data for a in outs])
        sizes = (C.c_size_t * len(outs))(*[a.size for a in outs])
        _check(self.lib.tg_download_states(self.ctx.h, self.id, len(names), _names(names), ptrs, sizes))
        return dict(zip(names, outs))

    def counters(self):
        """(optimizer steps taken, PRNG seed counter)."""
        a, b = C.c_int64(), C.c_int64()
        _check(self.lib.tg_get_counters(self.ctx.h, self.id, C.byref(a), C.byref(b)))
        return a.value, b.value

    def set_counters(self, step: int, prng: int) -> None:
        _check(self.lib.tg_set_counters(self.ctx.h, self.id, int(step), int(prng)))

    # -- steps ------------------------------------------------------------
    def _pack(self, inputs: Dict[str, np.ndarray]):
        names, arrs = [], []
        for n, v in inputs.items():
            if n not in self.input_tensors:
                raise TgError("Error", f"unknown input '{n}'")
            t = self.tensors[self.input_tensors[n]]
            dt = np.float32 if t["dtype"] == "f32" else np.int32
            a = np.ascontiguousarray(v, dtype=dt).reshape(-1)
            names.append(n)
            arrs.append(a)
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        sizes = (C.c_size_t * len(arrs))(*[a.nbytes for a in arrs])
        return names, arrs, ptrs, sizes

    def _capture_bufs(self):
        bufs = []
        for n in self.capture_names:
            t = self.tensors[self.program["graph"]["captures"][n]]
            bufs.append(np.empty(t["shape"], np.float32 if t["dtype"] == "f32" else np.int32))
        ptrs = (C.c_void_p * len(bufs))(*[b.ctypes.data for b in bufs]) if bufs else None
        return bufs, ptrs

    def step(self, inputs: Dict[str, np.ndarray]):
        names, arrs, ptrs, sizes = self._pack(inputs)
        bufs, cptrs = self._capture_bufs()
        _check(self.lib.tg_step(self.ctx.h, self.id, len(names), _names(names), ptrs, sizes, self._loss, cptrs))
        return float(self._loss[0]), dict(zip(self.capture_names, bufs))

    def run(self, inputs: Dict[str, np.ndarray]):
        names, arrs, ptrs, sizes = self._pack(inputs)
        out_t = self.tensors[self.program["graph"]["outputs"][0]]
        out = np.empty(out_t["shape"], np.float32 if out_t["dtype"] == "f32" else np.int32)
        bufs, cptrs = self._capture_bufs()
        _check(self.lib.tg_run(self.ctx.h, self.id, len(names), _names(names), ptrs, sizes,
                               C.c_void_p(out.ctypes.data), cptrs))
        return out, dict(zip(self.capture_names, bufs))

    def set_inputs(self, inputs: Dict[str, object], device_src: bool = False) -> None:
        """Copy inputs in; with device_src, values are (ptr, nbytes) device pointers."""
        if device_src:
            names = list(inputs)
            ptrs = (C.c_void_p * len(names))(*[inputs[n][0] for n in names])
            sizes = (C.c_size_t * len(names))(*[inputs[n][1] for n in names])
            _check(self.lib.tg_set_inputs(self.ctx.h, self.id, len(names), _names(names), ptrs, sizes, 1))
            return
        names, arrs, ptrs, sizes = self._pack(inputs)
        _check(self.lib.tg_set_inputs(self.ctx.h, self.id, len(names), _names(names), ptrs, sizes, 0))

    def launch_step(self) -> None:
        _check(self.lib.tg_launch_step(self.ctx.h, self.id))

    def read_loss(self) -> float:
        _check(self.lib.tg_read_loss(self.ctx.h, self.id, self._loss))
        return float(self._loss[0])

    def read_grad(self, name: str, shape) -> np.ndarray:
        out = np.empty(shape, np.float32)
        _check(self.lib.tg_read_grad(self.ctx.h, self.id, name.encode(), C.c_void_p(out.ctypes.data)))
        return out

    def read_tensor(self, tid: int) -> np.ndarray:
        t = self.tensors[tid]
        out = np.empty(t["shape"], np.float32 if t["dtype"] == "f32" else np.int32)
        _check(self.lib.tg_read_tensor(self.ctx.h, self.id, tid, C.c_void_p(out.ctypes.data)))
        return out

    def reset_optimizer(self) -> None:
        _check(self.lib.tg_reset_optimizer(self.ctx.h, self.id))

    def set_lr(self, lr) -> None:
        d = json.dumps(lr).encode()
        _check(self.lib.tg_set_lr(self.ctx.h, self.id, d, len(d)))

    def destroy(self) -> None:
        if self.ctx.h:
            _check(self.lib.tg_destroy_graph(self.ctx.h, self.id))


_contexts: Dict[tuple, Context] = {}


def default_context(device: Optional[int] = None) -> Context:
    """Single-rank context for ``device`` (env TG_DEVICE, default 0), shared per process."""
    if device is None:
        device = int(os.environ.get("TG_DEVICE", "0"))
    key = (device, 0, 1)
    if key not in _contexts:
        _contexts[key] = Context(device, 0, 1, None)
    return _contexts[key]
