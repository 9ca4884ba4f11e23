"""ctypes binding of libanvil_cuda.so (include/anvil_cuda.h) and the per-device model handle.

The library is the product path of the `cuda` target: there is no CPU fallback. If it is missing, or no sm_100
device is visible, every entry point here raises (ImportError / RuntimeError) instead of computing anything.
Status codes map to the exception types the reference raises for the same failures (anvil/runtime/api.py:104-141,
anvil/semantics.py:47-84): ValueError, MemoryError, RuntimeError, TimeoutError, OverflowError, IndexError,
NotImplementedError.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parents[1] / "_lib" / "libanvil_cuda.so"

OP_GEMM, OP_LUT, OP_LUT_MUL, OP_ADD_REQUANT, OP_NORM, OP_SOFTMAX, OP_TRANSPOSE, OP_EMBED, OP_ATTENTION, OP_COPY = \
    range(1, 11)
F_CAUSAL, F_CHECKED, F_LUT, F_BIAS, F_CENTER, F_SIMT, F_BIAS_RND, F_RESIDUAL, F_SPLIT = 1, 2, 4, 8, 16, 32, 64, 128, 256
ABI_VERSION = 2
LOC_CONST = 1 << 63
LOC_NONE = (1 << 64) - 1

KIND_NAMES = {OP_GEMM: "gemm", OP_LUT: "lut", OP_LUT_MUL: "lut_mul", OP_ADD_REQUANT: "add_requant",
              OP_NORM: "norm", OP_SOFTMAX: "softmax", OP_TRANSPOSE: "transpose", OP_EMBED: "embed",
              OP_ATTENTION: "attention", OP_COPY: "copy"}

EXPORTS = ("anvil_abi_version", "anvil_last_error", "anvil_device_count", "anvil_cuda_init", "anvil_model_create",
           "anvil_model_prepare", "anvil_model_run", "anvil_model_enqueue", "anvil_model_clear_flags",
           "anvil_model_wait", "anvil_model_record", "anvil_model_wait_ticket", "anvil_model_selftest_timeout", "anvil_model_run_device", "anvil_model_time_launches", "anvil_model_read",
           "anvil_model_write", "anvil_model_read_const", "anvil_model_arena", "anvil_model_describe",
           "anvil_model_free",
           "anvil_gemm_requant")


class AnvilOp(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("flags", ctypes.c_uint32), ("in_bytes", ctypes.c_int32),
                ("in2_bytes", ctypes.c_int32), ("out_bytes", ctypes.c_int32), ("op_index", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8), ("off", ctypes.c_uint64 * 8),
                ("mult", ctypes.c_int64), ("shift", ctypes.c_int64), ("ma", ctypes.c_int64), ("mb", ctypes.c_int64),
                ("one", ctypes.c_int64), ("ss_shift", ctypes.c_int64), ("ss_init", ctypes.c_int64),
                ("mult2", ctypes.c_int64), ("shift2", ctypes.c_int64), ("aux", ctypes.c_int64 * 8)]


class AnvilIO(ctypes.Structure):
    _fields_ = [("offset", ctypes.c_uint64), ("host", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


_lib = None
_lock = threading.Lock()


def load_library(path: str | os.PathLike | None = None):
    """Load (once) and return the ctypes library; raises ImportError if the .so is missing."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise ImportError(f"{p} is missing: build it with `python -m anvil.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(str(p))
        vp, i32, i64, u32, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64
        sig = {
            "anvil_abi_version": ([], i32),
            "anvil_last_error": ([], ctypes.c_char_p),
            "anvil_device_count": ([ctypes.POINTER(i32)], i32),
            "anvil_cuda_init": ([i32], i32),
            "anvil_model_create": ([i32, vp, u64, ctypes.POINTER(vp)], i32),
            "anvil_model_prepare": ([vp, ctypes.POINTER(AnvilOp), i32, u64], i32),
            "anvil_model_run": ([vp, ctypes.POINTER(AnvilIO), i32, ctypes.POINTER(AnvilIO), i32,
                                 ctypes.POINTER(ctypes.c_float)], i32),
            "anvil_model_run_device": ([vp, i32, i32, ctypes.POINTER(ctypes.c_float)], i32),
            "anvil_model_time_launches": ([vp, i32, ctypes.POINTER(ctypes.c_float)], i32),
            "anvil_model_enqueue": ([vp, ctypes.POINTER(AnvilIO), i32, ctypes.POINTER(AnvilIO), i32, vp], i32),
            "anvil_model_clear_flags": ([vp], i32),
            "anvil_model_wait": ([vp], i32),
            "anvil_model_record": ([vp, ctypes.POINTER(u64)], i32),
            "anvil_model_wait_ticket": ([vp, u64], i32),
            "anvil_model_selftest_timeout": ([vp, u64], i32),
            "anvil_model_read": ([vp, u64, vp, u64], i32),
            "anvil_model_write": ([vp, u64, vp, u64], i32),
            "anvil_model_read_const": ([vp, u64, vp, u64], i32),
            "anvil_model_arena": ([vp, ctypes.POINTER(u64), ctypes.POINTER(u64)], i32),
            "anvil_model_describe": ([vp, i32, ctypes.POINTER(i64)], i32),
            "anvil_model_free": ([vp], None),
            "anvil_gemm_requant": ([vp, vp, vp, i64, i64, i64, ctypes.c_int32, ctypes.c_int32, u32, vp], i32),
        }
        for name, (args, res) in sig.items():
            f = getattr(lib, name)
            f.argtypes = args
            f.restype = res
        if lib.anvil_abi_version() != ABI_VERSION:
            raise ImportError(f"{p}: ABI version {lib.anvil_abi_version()} != {ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


_ERRORS = {-1: ValueError, -2: MemoryError, -3: RuntimeError, -4: TimeoutError, -5: OverflowError,
           -6: IndexError, -7: NotImplementedError}


def check(rc: int, what: str = "libanvil_cuda"):
    if rc != 0:
        msg = load_library().anvil_last_error().decode(errors="replace")
        raise _ERRORS.get(rc, RuntimeError)(f"{what}: {msg}")


def device_count() -> int:
    n = ctypes.c_int(0)
    check(load_library().anvil_device_count(ctypes.byref(n)))
    return n.value


class DeviceModel:
    """One model replica on one device: const region, arena, launch list (C handle anvil_model*)."""

    def __init__(self, device: int, const_blob: np.ndarray):
        self.lib = load_library()
        self.device = device
        self._h = ctypes.c_void_p()
        blob = np.ascontiguousarray(const_blob, dtype=np.uint8)
        check(self.lib.anvil_model_create(device, blob.ctypes.data if blob.size else None, blob.nbytes,
                                          ctypes.byref(self._h)), "anvil_model_create")
        self.prepared_key = None
        self.n_ops = 0

    def prepare(self, ops: list[AnvilOp], arena_bytes: int, key=None):
        arr = (AnvilOp * max(1, len(ops)))(*ops)
        check(self.lib.anvil_model_prepare(self._h, arr, len(ops), int(arena_bytes)), "anvil_model_prepare")
        self.prepared_key = key
        self.n_ops = len(ops)

    def run(self, inputs: list[tuple[int, np.ndarray]], outputs: list[tuple[int, np.ndarray]], timing=False):
        """inputs/outputs: (arena offset, contiguous host array). Returns per-op microseconds or None."""
        ins = (AnvilIO * max(1, len(inputs)))(*[AnvilIO(o, a.ctypes.data, a.nbytes) for o, a in inputs])
        outs = (AnvilIO * max(1, len(outputs)))(*[AnvilIO(o, a.ctypes.data, a.nbytes) for o, a in outputs])
        us = (ctypes.c_float * max(1, self.n_ops))() if timing else None
        check(self.lib.anvil_model_run(self._h, ins, len(inputs), outs, len(outputs), us), "anvil_model_run")
        return list(us)[: self.n_ops] if timing else None

    def enqueue(self, inputs: list[tuple[int, np.ndarray]], outputs: list[tuple[int, np.ndarray]],
                after: "DeviceModel | None" = None):
        """anvil_model_enqueue: copies in, the launch chain, copies out, on this model's stream, without waiting;
        with `after`, chained behind that model's latest copies in and launch chain (a pipeline stage). The host
        arrays must stay alive (and unmodified) until wait() returns."""
        ins = (AnvilIO * max(1, len(inputs)))(*[AnvilIO(o, a.ctypes.data, a.nbytes) for o, a in inputs])
        outs = (AnvilIO * max(1, len(outputs)))(*[AnvilIO(o, a.ctypes.data, a.nbytes) for o, a in outputs])
        check(self.lib.anvil_model_enqueue(self._h, ins, len(inputs), outs, len(outputs),
                                           after._h if after is not None else None), "anvil_model_enqueue")

    def clear_flags(self):
        check(self.lib.anvil_model_clear_flags(self._h), "anvil_model_clear_flags")

    def wait(self):
        """Synchronise this model's stream and raise if a device check fired since clear_flags()."""
        check(self.lib.anvil_model_wait(self._h), "anvil_model_wait")

    def record(self) -> int:
        """anvil_model_record: a ticket for everything enqueued on this model so far (its device checks are
        snapshotted and cleared in stream order)."""
        t = ctypes.c_uint64(0)
        check(self.lib.anvil_model_record(self._h, ctypes.byref(t)), "anvil_model_record")
        return t.value

    def wait_ticket(self, ticket: int):
        """Block until the ticket's work is done; raise if a device check fired in it."""
        check(self.lib.anvil_model_wait_ticket(self._h, int(ticket)), "anvil_model_wait_ticket")

    def selftest_timeout(self, wait_ns: int):
        """Run the device wait-bound self-test: raises TimeoutError after about wait_ns (the expected outcome)."""
        check(self.lib.anvil_model_selftest_timeout(self._h, int(wait_ns)), "anvil_model_selftest_timeout")

    def time_launches(self, iters: int = 5) -> list:
        """Per-launch device microseconds inside CUDA-graph replays of the prepared chain, the shortest of `iters`
        replays per launch (anvil_model_time_launches)."""
        us = (ctypes.c_float * max(1, self.n_ops))()
        check(self.lib.anvil_model_time_launches(self._h, int(iters), us), "anvil_model_time_launches")
        return [float(us[i]) for i in range(self.n_ops)]

    def run_device(self, iters: int = 1, use_graph: bool = True) -> float:
        ms = ctypes.c_float(0)
        check(self.lib.anvil_model_run_device(self._h, int(iters), int(bool(use_graph)), ctypes.byref(ms)),
              "anvil_model_run_device")
        return ms.value

    def read(self, offset: int, out: np.ndarray):
        check(self.lib.anvil_model_read(self._h, int(offset), out.ctypes.data, out.nbytes), "anvil_model_read")
        return out

    def read_const(self, offset: int, out: np.ndarray):
        check(self.lib.anvil_model_read_const(self._h, int(offset), out.ctypes.data, out.nbytes),
              "anvil_model_read_const")
        return out

    def write(self, offset: int, data: np.ndarray):
        data = np.ascontiguousarray(data)
        check(self.lib.anvil_model_write(self._h, int(offset), data.ctypes.data, data.nbytes), "anvil_model_write")

    def describe(self, op: int) -> tuple[int, int, int, int]:
        """The launch shape of prepared op `op` (anvil_model_describe): GEMM (BN, CTAs per tile, tiles, CTAs),
        attention (hd, 0, work items, CTAs), zeros otherwise."""
        info = (ctypes.c_int64 * 4)()
        check(self.lib.anvil_model_describe(self._h, int(op), info), "anvil_model_describe")
        return tuple(int(v) for v in info)

    def pointers(self) -> tuple[int, int]:
        a, c = ctypes.c_uint64(0), ctypes.c_uint64(0)
        check(self.lib.anvil_model_arena(self._h, ctypes.byref(a), ctypes.byref(c)))
        return a.value, c.value

    def close(self):
        if self._h:
            self.lib.anvil_model_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm_requant(a_ptr: int, bt_ptr: int, out_ptr: int, m: int, n: int, k: int, mult: int, shift: int,
                 flags: int = 0, stream: int = 0):
    """Device-pointer int8 GEMM + requant (include/anvil_cuda.h anvil_gemm_requant)."""
    lib = load_library()
    check(lib.anvil_gemm_requant(a_ptr, bt_ptr, out_ptr, m, n, k, mult, shift, flags, stream or None),
          "anvil_gemm_requant")
