"""Compile driver for the `cuda` target: a PyTorch module or an anvil.graph module -> CompiledModel whose run()
executes on B200s through libanvil_cuda.so.

Mirrors the reference driver anvil/driver.py (RunOutput :56-76, _resolve_model :90-116, _checked_graph :119-132,
CompiledModel :168-327, compile :330-335) with the tiny-gpu lowering/scheduling/codegen replaced by
anvil.runtime.program (graph -> launch list) and the simulator dispatch replaced by the `cuda` backend:

    cm = anvil.compile(block, (x_example,), calib)          # torch module: capture + quantize (anvil.frontend)
    cm = anvil.compile(module, consts=consts)               # graph IR (+ consts), proved free of int32 overflow
    res = cm.run(x_float, "cuda")                           # quantize x, run on the GPU, read back, dequantize
    res = cm.run(xq, "cuda", quantized=True)                # integer inputs
    res.output, res.ints["out"], res.cycles                 # float output, int values, per-kernel device us
    print(cm.summary())

Batching: where the reference runs one sample per job, the cuda target also takes a leading batch dim on every
input (all inputs the same batch); values then carry it, exactly as the oracle's batch=True evaluation. With
CudaParams(devices=(0, 1, ...)) the batch is split into contiguous shards, one per device, each device running
its own replica of the const region and launch list; there is no collective on the compute path.
"""
from __future__ import annotations

import math
import threading
from dataclasses import dataclass, field

import numpy as np

from .ir import graph as g

BACKENDS = ("cuda",)
PIPELINE_MODELS = 4          # device models (arenas + streams) a pipelined run rotates over
PIPELINE_TOKENS = 8192       # "auto" pipeline chunk size, in tokens. c3 batch 64 on one B200, pinned buffers, calls
                             # queued by submit(), copies on the device's shared copy streams: 8 chunks over 4 models
                             # 1.23 ms per call, over 3 models 1.30 ms; 4 chunks 1.30 ms, 16 chunks 1.67 ms
NOMINAL_PEAKS = {"int8_tops": 4500.0, "hbm_gbs": 7700.0}    # B200 dense int8 tensor and HBM3e, NVIDIA's figures
GUARD_BYTES = 256            # canary bytes after every buffer of a guarded (stray-write checked) run
MAX_OUTSTANDING = 32         # submit() calls queued at once (each holds one completion ticket per device model)


@dataclass(frozen=True)
class CudaParams:
    """Execution parameters of the cuda target (the analogue of the reference's GpuParams, api.py:22-63).

    devices   CUDA device ordinals; a batch is sharded across them (contiguous, ceil(B / G) each)
    checked   check every int32 intermediate on the device (OverflowError like the oracle); None: only when
              the static overflow proof does not hold for the graph. False on a graph the proof rejects runs the
              unchecked 32-bit arithmetic anyway (with a RuntimeWarning): the outputs are then exact only on inputs
              where no intermediate leaves int32, and where the oracle would raise OverflowError they are
              unspecified
    fuse      apply launch fusions (LUT epilogues, fused attention); keep="all" runs disable them
    gemm      "auto" | "tc" (tcgen05 wherever the shape allows) | "simt" (CUDA-core kernel everywhere)
    pipeline  equal chunks a device's share of a run is split into, so one chunk's host<->device copies overlap
              another chunk's kernels (the chunks go round-robin over PIPELINE_MODELS device models, each with its
              own arena and stream); "auto": chunks of about PIPELINE_TOKENS tokens; 1 disables it. keep="all" and
              timing runs are never split.
    """
    devices: tuple = (0,)
    checked: bool | None = None
    fuse: bool = True
    gemm: str = "auto"
    pipeline: int | str = "auto"

    def __post_init__(self):
        if not self.devices or any(not isinstance(d, int) or d < 0 for d in self.devices):
            raise ValueError(f"CudaParams.devices = {self.devices!r}: need non-negative ints")
        if len(set(self.devices)) != len(self.devices):
            raise ValueError(f"CudaParams.devices = {self.devices!r}: a device may appear once")
        if self.gemm not in ("auto", "tc", "simt"):
            raise ValueError(f"CudaParams.gemm = {self.gemm!r}: auto, tc or simt")
        if self.pipeline != "auto" and (not isinstance(self.pipeline, int) or self.pipeline < 1):
            raise ValueError(f"CudaParams.pipeline = {self.pipeline!r}: 'auto' or a chunk count >= 1")


class RunOutput:
    """Result of CompiledModel.run (anvil/driver.py:56-76): `ints` holds every readable value as an integer array
    in its graph dtype (int8 / int16 / int32); `output` / `outputs` are the dequantized graph outputs, computed
    on first access."""

    def __init__(self, model, ints: dict, cycles: dict, result=None, job=None, stray=None):
        self._model = model
        self.ints = ints                # sym -> int array of every value readable after the run
        self.cycles = cycles            # launch label -> device microseconds (None unless run(..., timing=True))
        self.result = result            # CudaRunResult
        self.job = job                  # the DeviceProgram of the first device
        self._outs = None
        self._stray = stray             # guarded runs: [(device, region, byte offset)] the run must not have changed

    def stray_writes(self, *, scratch_ok: bool = True) -> list:
        """Bytes the run changed that it must not have (anvil/driver.py:66-71): outside every planned arena
        buffer (alignment gaps, the canary after each buffer, past the plan) or anywhere in the const region
        (weights, LUTs, biases), as (device, "arena" | "const", byte offset). Empty for a correct launch chain.
        Needs a run(..., guard=True), which fills the arena with a canary pattern before the run and reads the
        arena and the const region back after it. `scratch_ok` is accepted for the reference's signature: this
        target has no shared scratch words."""
        if self._stray is None:
            raise ValueError("stray_writes() needs a run(..., guard=True): only a guarded run records the memory")
        return list(self._stray)

    @property
    def outputs(self) -> list:
        if self._outs is None:
            self._outs = [self._model.dequantize(s, self.ints[s]) for s in self._model.outputs]
        return self._outs

    @property
    def output(self) -> np.ndarray:
        return self.outputs[0]

    @property
    def total_cycles(self):
        c = list(self.cycles.values())
        return None if any(v is None for v in c) else sum(c)


@dataclass
class CudaRunResult:
    batch: int
    shards: list                        # [(device, batch)]
    kernel_us: dict = field(default_factory=dict)


def _wait_tickets(tickets):
    """Wait on every (DeviceModel, ticket); then raise the first device error among them (none is left pending)."""
    errs = []
    for dm, t in tickets:
        try:
            dm.wait_ticket(t)
        except Exception as e:
            errs.append(e)
    if errs:
        raise errs[0]


class PendingRun:
    """A run queued by CompiledModel.submit: its copies and kernels are on the device streams; wait() blocks until
    they are done and returns the RunOutput that run() would have returned (or raises its error). The input and
    output arrays must stay alive and unmodified until then (the object holds references to them)."""

    def __init__(self, model, batch, batched, shards, tickets, keep):
        self._model = model
        self._batch, self._batched, self._shards = batch, batched, shards
        self._tickets = tickets           # [(DeviceModel, ticket)]
        self._keep = keep                 # (bound inputs, per-shard input copies, outputs)
        self._result = None
        self._error = None

    def done(self) -> bool:
        """True once wait() has collected the run (it never blocks)."""
        return self._tickets is None

    def _finish(self):
        if self._tickets is None:
            return
        tickets, self._tickets = self._tickets, None
        try:
            _wait_tickets(tickets)
        except Exception as e:
            self._error = e
        bound, _, ints = self._keep
        self._keep = None
        if self._error is None:
            m = self._model
            ints = dict(ints)
            for sym in m.inputs:
                ints.setdefault(sym, bound[sym])
            if not self._batched:
                ints = {k: v[0] if v.ndim and v.shape[0] == 1 and k not in m._const_syms() else v
                        for k, v in ints.items()}
            prog = m.program(self._shards[0][1], "outputs")
            cycles = {d.label: None for d in prog.devops}
            self._result = RunOutput(m, ints, cycles, CudaRunResult(self._batch, self._shards, cycles), prog)

    def wait(self) -> RunOutput:
        """Block until the run is done (holding the model's lock, so a submit() from another thread waits for it);
        return its RunOutput or raise its device error, again on every later call."""
        with self._model._lock:
            self._finish()
            if self in self._model._outstanding:
                self._model._outstanding.remove(self)
        if self._error is not None:
            raise self._error
        return self._result


def _resolve_model(model, example_inputs, calib_inputs, consts, quant_kw, prove=True):
    from .frontend import Quantized
    from .frontend.numerics import prove_no_overflow

    graph_path = isinstance(model, (Quantized, g.Module)) or (
        isinstance(model, tuple) and len(model) == 2 and isinstance(model[0], g.Module))
    if graph_path and quant_kw:
        raise TypeError(f"anvil.compile got unexpected keyword argument(s) {sorted(quant_kw)} (extra keywords go to "
                        "quantize, which only runs for a torch module)")
    if isinstance(model, Quantized):
        return model.module, dict(model.consts), model
    if isinstance(model, tuple) and len(model) == 2 and isinstance(model[0], g.Module):
        return _checked_graph(model[0], dict(model[1]), prove, prove_no_overflow)
    if isinstance(model, g.Module):
        return _checked_graph(model, dict(consts or {}), prove, prove_no_overflow)
    try:
        import torch
    except ImportError:
        torch = None
    if torch is not None and isinstance(model, torch.nn.Module):
        from .frontend import from_torch
        if example_inputs is None or calib_inputs is None:
            raise ValueError("compiling a torch module needs example_inputs and calib_inputs")
        q = from_torch(model, example_inputs, calib_inputs, **quant_kw)
        return q.module, dict(q.consts), q
    raise TypeError(f"cannot compile a {type(model).__name__}: expected a torch.nn.Module, anvil.frontend.Quantized, "
                    "an anvil.graph module or (module, consts)")


def _checked_graph(module, consts, prove, prove_fn):
    """Every non-inline const needs its values and, unless prove=False, the int32 overflow proof must hold
    (anvil/driver.py:119-132). prove=False compiles anyway and runs every kernel in checked mode."""
    need = [op.sym_str for op in g.func_of(module).ops if isinstance(op, g.ConstOp) and op.value is None]
    missing = [s for s in need if s not in consts]
    if missing:
        raise ValueError(f"no values for graph consts {missing}: pass consts= or a (module, consts) pair")
    unknown = sorted(set(consts) - set(need))
    if unknown:
        raise ValueError(f"consts {unknown} name no graph const of the module")
    if prove:
        prove_fn(module, consts)
    return module, consts, None


class CompiledModel:
    """A graph ready for the cuda target: per batch size a lowered launch list and memory plan, per device a
    replica of the const region (built lazily on the first run)."""

    def __init__(self, module, consts, params: CudaParams | None = None, *, quantized=None, proven=None):
        from .frontend.numerics import prove_no_overflow

        if isinstance(params, dict):
            params = CudaParams(**params)
        self.params = params or CudaParams()
        if not isinstance(self.params, CudaParams):
            raise TypeError(f"params must be a CudaParams (or a dict of its fields), not {type(self.params).__name__}")
        self.module, self.consts, self.quantized = module, consts, quantized
        self.func = g.func_of(module)
        if not [op for op in self.func.ops if not isinstance(op, (g.InputOp, g.ConstOp, g.OutputOp))]:
            raise ValueError("the graph has no operations to compile (its outputs are its inputs)")
        self.meta = g.graph_meta(module)
        self.in_dtypes = {op.sym_str: g.qt(op.result).dtype for op in self.func.ops if isinstance(op, g.InputOp)}
        if proven is None:
            try:
                prove_no_overflow(module, consts)
                proven = True
            except (OverflowError, ValueError):
                proven = False
        self.proven = proven
        self.checked = (not proven) if self.params.checked is None else bool(self.params.checked)
        if not self.checked and not proven:
            import warnings
            warnings.warn("checked=False on a graph whose static int32 proof fails: the outputs are exact only on "
                          "inputs where no int32 intermediate overflows (where the oracle raises OverflowError they "
                          "are unspecified)", RuntimeWarning, stacklevel=2)
        from .runtime.program import ConstPool
        self._pool = ConstPool()
        self._programs = {}          # (batch, keep) -> DeviceProgram
        self._devices = {}           # device -> DeviceModel
        self._pool_size_at_upload = {}
        self._pipes = {}             # device -> [DeviceModel] for pipelined runs
        self._tail = {}              # device -> the pipelined model that took the latest chunk (cross-call chaining)
        self._outstanding = []       # PendingRuns of submit() not waited on yet
        self._lock = threading.Lock()

    # ------------------------------------------------------------------------------------- programs
    def program(self, batch: int = 1, keep: str = "outputs", guard: bool = False):
        """The launch list for `batch` samples (cached); guard=True gives the debug layout of a stray-write check
        (no buffer reuse, GUARD_BYTES of canary after every buffer)."""
        from .runtime.program import lower_program
        key = (int(batch), keep, bool(guard))
        if key not in self._programs:
            self._programs[key] = lower_program(self.module, self.consts, self._pool, batch, keep,
                                                checked=self.checked, fuse=self.params.fuse, gemm=self.params.gemm,
                                                guard=GUARD_BYTES if guard else 0)
        return self._programs[key]

    @property
    def plan(self):
        return self.program(1).plan

    @property
    def footprint(self) -> int:
        return self.plan.footprint

    def _pipe_models(self, device: int, size: int, count: int) -> list:
        """`count` replicas on `device` prepared for chunks of `size` samples (constants uploaded once each)."""
        from .runtime.cuda import DeviceModel
        prog = self.program(size, "outputs")              # lowered first: it may add constants to the pool
        pipes = self._pipes.setdefault(device, {})
        if self._pool_size_at_upload.get(("pipe", device)) != self._pool.size:
            self._finish_outstanding()                    # no model is freed under queued work
            self._tail.pop(device, None)
            for ms in pipes.values():
                for m in ms:
                    m.close()
            pipes.clear()
            self._pool_size_at_upload[("pipe", device)] = self._pool.size
        ms = pipes.setdefault(size, [])
        while len(ms) < count:
            ms.append(DeviceModel(device, self._pool.blob()))
        for m in ms[:count]:
            if m.prepared_key != (size, "outputs"):
                self._finish_outstanding()
                m.prepare(prog.ops, prog.plan.arena, key=(size, "outputs"))
        return ms[:count]

    def _chunk_plan(self, b: int, keep: str, timing: bool) -> list:
        """Sample counts of the chunks a shard of b samples runs as ([b]: one launch chain)."""
        if keep != "outputs" or timing or b < 2:
            return [b]
        if self.params.pipeline != "auto":
            n = min(int(self.params.pipeline), b)
            while b % n:
                n -= 1
            return [b // n] * n
        per = max(1, PIPELINE_TOKENS // max(1, self._tokens_per_sample()))       # samples per chunk
        want = max(1, round(b / per))
        divs = [n for n in range(1, b + 1) if b % n == 0]
        n = min(divs, key=lambda k: (abs(k - want), k))
        return [b // n] * n

    def _chunks(self, b: int, keep: str, timing: bool) -> int:
        return len(self._chunk_plan(b, keep, timing))

    def _tokens_per_sample(self) -> int:
        """Rows of the first input per sample (sequence length for (T, d) or (T,) inputs)."""
        shape = self.meta[self.inputs[0]][1]
        return int(shape[0]) if len(shape) else 1

    def _device_model(self, device: int):
        from .runtime.cuda import DeviceModel
        dm = self._devices.get(device)
        if dm is None or self._pool_size_at_upload.get(device) != self._pool.size:
            if dm is not None:
                dm.close()
            dm = DeviceModel(device, self._pool.blob())
            self._devices[device] = dm
            self._pool_size_at_upload[device] = self._pool.size
        return dm

    # -------------------------------------------------------------------------------- (de)quantization
    @property
    def inputs(self) -> list:
        return [op.sym_str for op in self.func.ops if isinstance(op, g.InputOp)]

    @property
    def outputs(self) -> list:
        for op in self.func.ops:
            if isinstance(op, g.OutputOp):
                return [v.owner.sym_str for v in op.values]
        return []

    def scale(self, sym):
        return self.meta[sym][0]

    def quantize_input(self, x, sym=None):
        """Float array -> integers by the input's scale (round half to even, saturating at the input's dtype;
        anvil/driver.py:233-241)."""
        sym = sym or self.inputs[0]
        s = self.scale(sym)
        if s is None:
            raise ValueError(f"input {sym!r} has no scale: pass integer inputs with quantized=True")
        lo, hi = {"i8": (-128, 127), "i16": (-(1 << 15), (1 << 15) - 1), "i32": (-(1 << 31), (1 << 31) - 1)}[
            self.meta[sym][2]]
        return np.clip(np.rint(np.asarray(x, dtype=np.float64) / s), lo, hi).astype(np.int64)

    def dequantize(self, sym, ints):
        s = self.scale(sym)
        return np.asarray(ints, dtype=np.float64) * (1.0 if s is None else s)

    def _bind_inputs(self, x, quantized):
        """-> ({sym: array with a leading batch dim}, batch, batched?)."""
        xs = list(x) if isinstance(x, (list, tuple)) else [x]
        if len(xs) != len(self.inputs):
            raise ValueError(f"{len(xs)} inputs for graph inputs {self.inputs}")
        out, batch, batched = {}, None, None
        for sym, v in zip(self.inputs, xs):
            v = np.asarray(v)
            shape = tuple(self.meta[sym][1])
            if v.shape == shape:
                b, v = 1, v.reshape((1,) + shape)
                isb = False
            elif v.ndim == len(shape) + 1 and tuple(v.shape[1:]) == shape:
                b, isb = v.shape[0], True
            elif v.size == math.prod(shape) and (v.ndim <= 1 or tuple(d for d in v.shape if d != 1) == tuple(
                    d for d in shape if d != 1)):
                # a flat array or extra size-1 dims (anvil/driver.py:254-261); a transposed input is an error
                b, v, isb = 1, v.reshape((1,) + shape), False
            else:
                raise ValueError(f"input {sym!r}: shape {v.shape} != {shape} (or a leading batch dim + {shape})")
            if b < 1:
                raise ValueError(f"input {sym!r}: empty batch")
            if batch is not None and (b != batch or isb != batched):
                raise ValueError(f"inputs disagree on the batch: {batch} vs {b}")
            batch, batched = b, isb
            out[sym] = self._check_int_input(sym, v) if quantized else self._quantize_checked(sym, v)
        return out, batch, batched

    def _quantize_checked(self, sym, v):
        if self.meta[sym][0] is None:
            raise ValueError(f"input {sym!r} has no scale: pass integer inputs with quantized=True")
        if not np.all(np.isfinite(np.asarray(v, dtype=np.float64))):
            raise ValueError(f"input {sym!r} has NaN or infinite values")
        return self.quantize_input(v, sym)

    def _check_int_input(self, sym, v):
        """quantized=True: integer values inside the input's own dtype (anvil/driver.py:270-280)."""
        if v.dtype.kind not in "iub":
            raise ValueError(f"input {sym!r}: quantized=True needs integer values, got dtype {v.dtype}")
        dt = self.in_dtypes.get(sym, "i8")
        bits = {"i8": 8, "i16": 16, "i32": 32}[dt]
        lo, hi = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
        info = np.iinfo(v.dtype) if v.dtype.kind in "iu" else None
        if info is not None and info.min >= lo and info.max <= hi:
            return v                              # the array's dtype cannot hold an out-of-range value
        if v.size and (int(v.min()) < lo or int(v.max()) > hi):
            raise ValueError(f"input {sym!r}: values in [{v.min()}, {v.max()}] outside {dt} [{lo}, {hi}]")
        return v

    # --------------------------------------------------------------------------------------------- runs
    def run(self, x, backend: str = "cuda", *, quantized=False, keep="outputs", timing=False, out=None,
            guard=False) -> RunOutput:
        """Quantize `x` (unless quantized=True), run the launch chain on the GPU(s), read back. `out` may map graph
        output syms to caller-owned C-contiguous arrays of the output's dtype and (batch,) + shape (pinned memory
        makes the read-back a DMA at full bus speed); those outputs are written there and returned as those
        arrays. guard=True is a debug run for RunOutput.stray_writes(): the chain runs on the guarded layout (no
        buffer reuse, canary bytes after every buffer) in one piece per device, and the arena and const region are
        compared with what they held before."""
        if backend not in BACKENDS:
            raise ValueError(f"unknown backend {backend!r}: this build runs {', '.join(BACKENDS)} (the tiny-gpu "
                             "simulators isasim/rtl/verilator are not part of it)")
        if keep not in ("outputs", "all"):
            raise ValueError(f"keep must be 'outputs' or 'all', not {keep!r}")
        bound, batch, batched = self._bind_inputs(x, quantized)
        out = self._check_out(out, batch)
        ints, kus, shards, stray = self._run_cuda(bound, batch, keep, timing, out, bool(guard))
        if not batched:
            ints = {k: v[0] if v.ndim and v.shape[0] == 1 and k not in self._const_syms() else v
                    for k, v in ints.items()}
        prog = self.program(shards[0][1], keep, bool(guard))
        cycles = {}
        for d, us in zip(prog.devops, kus if kus is not None else [None] * len(prog.devops)):
            cycles[d.label] = (cycles.get(d.label) or 0) + us if us is not None else None
        return RunOutput(self, ints, cycles, CudaRunResult(batch, shards, cycles), prog, stray)

    def submit(self, x, backend: str = "cuda", *, quantized=False, out=None) -> PendingRun:
        """run(x, backend, quantized=..., out=...) without waiting: the inputs' copies in, the launch chain and the
        outputs' copies out are queued on the device(s) behind any earlier submit() or run(), and the returned
        PendingRun's wait() gives the RunOutput. Consecutive submits overlap one call's copies with another's
        kernels, which a synchronous run() cannot do across its own start and end. Pass pinned (page-locked) input
        and `out` arrays: a copy out to pageable memory makes the queuing call itself wait for it. keep="all",
        timing and guarded runs are synchronous only (use run()); a graph whose outputs are not whole contiguous
        buffers also runs synchronously here, and its PendingRun is already complete."""
        if backend not in BACKENDS:
            raise ValueError(f"unknown backend {backend!r}: this build runs {', '.join(BACKENDS)} (the tiny-gpu "
                             "simulators isasim/rtl/verilator are not part of it)")
        bound, batch, batched = self._bind_inputs(x, quantized)
        out = self._check_out(out, batch)
        shards = self._shards(batch)
        with self._lock:
            plans = {hi - lo: self._chunk_plan(hi - lo, "outputs", False) for _, lo, hi in shards}
            sync = not all(self._pipelinable(self.program(c, "outputs")) for p in plans.values() for c in set(p))
        if sync:
            res = self.run(x, backend, quantized=quantized, out=out)
            pr = PendingRun(self, batch, batched, [(d, hi - lo) for d, lo, hi in shards], [], (bound, None, {}))
            pr._tickets, pr._keep, pr._result = None, None, res
            return pr
        from .runtime.program import NP
        full = dict(out)
        for sym in self.outputs:            # the shards' copies out land straight in these arrays
            if sym not in full:
                full[sym] = np.empty((batch,) + tuple(self.meta[sym][1]), dtype=NP[self.meta[sym][2]])
        with self._lock:
            self._outstanding = [p for p in self._outstanding if p._tickets is not None]
            while len(self._outstanding) >= MAX_OUTSTANDING:      # bounded queue: collect the oldest run first
                self._outstanding.pop(0)._finish()
            tickets, copies = [], []
            try:
                for d, lo, hi in shards:
                    _, tk, ins = self._enqueue_pipelined(d, {k: v[lo:hi] for k, v in bound.items()}, hi - lo,
                                                         plans[hi - lo], {k: v[lo:hi] for k, v in full.items()})
                    tickets += tk
                    copies.append(ins)
            except BaseException:
                _wait_tickets(tickets)
                raise
            pr = PendingRun(self, batch, batched, [(d, hi - lo) for d, lo, hi in shards], tickets,
                            (bound, copies, full))
            self._outstanding.append(pr)
        return pr

    def _finish_outstanding(self):
        """Collect every queued submit() (their errors stay with their PendingRuns); called with the lock held
        before a device model is re-prepared or freed."""
        for p in list(self._outstanding):
            p._finish()
        self._outstanding = []

    def _check_out(self, out, batch):
        if not out:
            return {}
        from .runtime.program import NP
        for sym, arr in out.items():
            if sym not in self.outputs:
                raise ValueError(f"out: {sym!r} is not a graph output ({self.outputs})")
            want = (batch,) + tuple(self.meta[sym][1])
            if not isinstance(arr, np.ndarray) or arr.shape != want or arr.dtype != NP[self.meta[sym][2]] or \
                    not arr.flags.c_contiguous or not arr.flags.writeable:
                raise ValueError(f"out[{sym!r}] must be a writable C-contiguous {NP[self.meta[sym][2]].__name__} "
                                 f"array of shape {want}")
        return out

    def _const_syms(self):
        return {op.sym_str for op in self.func.ops if isinstance(op, g.ConstOp)}

    def _shards(self, batch):
        devs = list(self.params.devices)
        n = min(len(devs), batch)
        per = -(-batch // n)
        out, lo = [], 0
        for d in devs[:n]:
            hi = min(batch, lo + per)
            if hi > lo:
                out.append((d, lo, hi))
            lo = hi
        return out

    def _run_cuda(self, bound, batch, keep, timing, out=None, guard=False):
        shards = self._shards(batch)
        results, errors = [None] * len(shards), [None] * len(shards)

        def work(i, dev, lo, hi):
            try:
                results[i] = self._run_shard(dev, {k: v[lo:hi] for k, v in bound.items()}, hi - lo, keep, timing,
                                             {k: v[lo:hi] for k, v in (out or {}).items()}, guard)
            except BaseException as e:            # re-raised on the calling thread
                errors[i] = e

        with self._lock:
            for b in {hi - lo for _, lo, hi in shards}:        # lower (and pack consts) before any upload
                self.program(b, keep, guard)
            if len(shards) == 1:
                work(0, *shards[0])
            else:
                ts = [threading.Thread(target=work, args=(i, *s)) for i, s in enumerate(shards)]
                for t in ts:
                    t.start()
                for t in ts:
                    t.join()
        for e in errors:
            if e is not None:
                raise e
        ints = {}
        for k in results[0][0]:
            if out and k in out:
                ints[k] = out[k]                      # the shards were written in place
                continue
            parts = [r[0][k] for r in results]
            ints[k] = parts[0] if k in self._const_syms() or len(parts) == 1 else np.concatenate(parts, axis=0)
        stray = None
        if guard:
            stray = [(d, region, off) for (d, _, _), r in zip(shards, results) for region, off in r[2]]
        return ints, results[0][1], [(d, hi - lo) for d, lo, hi in shards], stray

    def _run_shard(self, device, bound, b, keep, timing, out=None, guard=False):
        plan = [b] if guard else self._chunk_plan(b, keep, timing)
        if len(plan) > 1 and all(self._pipelinable(self.program(c, keep)) for c in set(plan)):
            return self._run_pipelined(device, bound, b, plan, out) + (None,)
        prog = self.program(b, keep, guard)
        dm = self._device_model(device)
        if dm.prepared_key != (b, keep, guard):
            dm.prepare(prog.ops, prog.plan.arena, key=(b, keep, guard))
        canary = None
        if guard:
            canary = canary_bytes(prog.plan.arena)
            dm.write(0, canary)
        ins = []
        for sym, (off, shape, dtype) in prog.inputs.items():
            arr = np.ascontiguousarray(bound[sym], dtype={"i8": np.int8, "i16": np.int16, "i32": np.int32}[dtype])
            ins.append((off, arr))
        want = self._readable(prog, keep)
        roots, direct, outs = {}, {}, []
        for sym, v in want.items():
            if out and sym in out and v.contiguous and out[sym].nbytes == prog.buffers[v.root]:
                direct[sym] = out[sym]            # DMA straight into the caller's buffer
                outs.append((prog.plan.addresses[v.root], out[sym]))
            else:
                roots.setdefault(v.root, None)
        for r in roots:
            buf = np.empty(prog.buffers[r], dtype=np.uint8)
            roots[r] = buf
            outs.append((prog.plan.addresses[r], buf))
        kus = dm.run(ins, outs, timing=timing)
        stray = None
        if guard:
            after = dm.read(0, np.empty(prog.plan.arena, dtype=np.uint8))
            consts_after = dm.read_const(0, np.empty(self._pool.size, dtype=np.uint8))
            stray = stray_bytes(prog.plan.inside(), canary, after, self._pool.blob(), consts_after)
        ints = dict(direct)
        for sym, v in want.items():
            if sym in direct:
                continue
            ints[sym] = _apply_view(roots[v.root], v)
            if out and sym in out:
                out[sym][...] = ints[sym]
                ints[sym] = out[sym]
        for sym in self.inputs:
            ints.setdefault(sym, bound[sym])
        return ints, kus, stray

    def _pipelinable(self, prog) -> bool:
        """Every graph output is a whole, contiguous arena buffer (copied per chunk straight into its rows)."""
        for sym, v in self._readable(prog, "outputs").items():
            nbytes = int(np.prod(self.meta[sym][1], dtype=np.int64)) * prog.batch * {"i8": 1, "i16": 2, "i32": 4}[
                self.meta[sym][2]]
            if not v.contiguous or prog.buffers[v.root] != nbytes:
                return False
        return True

    def _run_pipelined(self, device, bound, b, plan, out=None):
        """The shard as a pipelined run (_enqueue_pipelined), waited on before returning."""
        res, tickets, _ = self._enqueue_pipelined(device, bound, b, plan, out)
        _wait_tickets(tickets)
        ints = dict(res)
        for sym in self.inputs:
            ints.setdefault(sym, bound[sym])
        return ints, None

    def _enqueue_pipelined(self, device, bound, b, plan, out=None):
        """The shard as chunks of plan[i] samples, each enqueued on a device model prepared for its size: equal-size
        chunks rotate over PIPELINE_MODELS models (own stream and arena each), so while one chunk's kernels run the
        next chunk's inputs are copied in and the previous chunk's outputs copied out, straight between the
        caller's arrays and the device. The first chunk is chained behind the latest chunk of an earlier call on
        the device, so back-to-back calls keep the bus and the SMs busy across call boundaries. Returns the output
        arrays, a completion ticket per model used and the input arrays the copies read (which must outlive the
        tickets), without waiting."""
        from .runtime.program import NP
        sizes = sorted(set(plan))
        counts = {c: min(PIPELINE_MODELS, plan.count(c)) for c in sizes}
        models = {c: self._pipe_models(device, c, counts[c]) for c in sizes}
        prog0 = self.program(plan[0], "outputs")
        ins = {sym: np.ascontiguousarray(bound[sym], dtype=NP[dtype]) for sym, (_, _, dtype) in prog0.inputs.items()}
        res = {}
        for sym in self._readable(prog0, "outputs"):
            full = (b,) + tuple(self.meta[sym][1])
            if out and sym in out:
                res[sym] = out[sym]
            else:
                res[sym] = np.empty(full, dtype=NP[self.meta[sym][2]])
        used = [m for c in sizes for m in models[c]]
        live = {id(m) for ms in self._pipes.get(device, {}).values() for m in ms}
        prev = self._tail.get(device)
        prev = prev if prev is not None and id(prev) in live else None
        for dm in used:
            dm.clear_flags()
        turn = {c: 0 for c in sizes}
        enqueued = []
        try:
            lo = 0
            for c in plan:
                prog = self.program(c, "outputs")
                dm = models[c][turn[c] % counts[c]]
                turn[c] += 1
                hi = lo + c
                dm.enqueue([(off, ins[sym][lo:hi]) for sym, (off, _, _) in prog.inputs.items()],
                           [(prog.plan.addresses[v.root], res[sym][lo:hi])
                            for sym, v in self._readable(prog, "outputs").items()],
                           after=prev if prev is not dm else None)
                if dm not in enqueued:
                    enqueued.append(dm)
                lo, prev = hi, dm
                self._tail[device] = dm
        except BaseException:
            # what was queued still runs on the caller's arrays: let it finish before the error propagates
            try:
                _wait_tickets([(dm, dm.record()) for dm in enqueued])
            except Exception:
                pass
            raise
        return res, [(dm, dm.record()) for dm in used], ins

    def _readable(self, prog, keep):
        want = {}
        for sym, v in prog.outputs:
            if not v.const and sym is not None:
                want[sym] = v
        if keep == "all":
            for sym, v in prog.views.items():
                want.setdefault(sym, v)
        return want

    def readable(self, keep="outputs") -> list:
        prog = self.program(1, keep)
        return list(self._readable(prog, keep)) + [s for s in self.inputs]

    # ------------------------------------------------------------------------------------------ summary
    def summary(self, batch: int = 1, kernel_us: dict | None = None, peaks: dict | None = None) -> str:
        """Per launch: label, kernel, shape, algorithmic ops / bytes; with `kernel_us` (RunOutput.cycles of a
        timing=True run, label -> device us) the achieved rate and its fraction of the roofline that bounds the
        kernel (ops against the dense int8 tensor peak, bytes against HBM bandwidth); then the fusions and the plan
        (the reference's summary, anvil/driver.py:324-327). `peaks` = {"int8_tops": ..., "hbm_gbs": ...} gives the
        denominators (default: B200 nominal, 4500 dense int8 TOP/s and 7700 GB/s). When the first device's model
        is prepared for this batch, each launch also shows the tile shape the library chose."""
        from .runtime.cuda import KIND_NAMES, OP_ATTENTION, OP_GEMM
        pk = dict(NOMINAL_PEAKS, **(peaks or {}))
        prog = self.program(batch)
        dm = self._devices.get(self.params.devices[0])
        shapes = dm is not None and dm.prepared_key == (batch, "outputs", False)
        rows = []
        for i, d in enumerate(prog.devops):
            f = d.fields
            kname = KIND_NAMES.get(d.kind, str(d.kind))
            if d.kind == OP_GEMM:
                kname += "[simt]" if f.get("flags", 0) & 32 else "[tcgen05]"
            dims = "x".join(str(v) for v in f.get("dims", []))
            w = d.work
            work = (f"{w['ops'] / 1e6:10.2f} Mop" if "ops" in w else f"{w.get('bytes', 0) / 1e6:10.2f} MB ")
            shape = ""
            if shapes and d.kind in (OP_GEMM, OP_ATTENTION):
                a, b, tiles, ctas = dm.describe(i)
                if d.kind == OP_GEMM:
                    shape = f" [{'pair ' if b == 2 else ''}BN {a}, {tiles} tiles, {ctas} CTAs]" if a else \
                        f" [{tiles} blocks]"
                else:
                    shape = f" [{tiles} items, {ctas} CTAs]"
            t = ""
            if kernel_us and d.label in kernel_us and kernel_us[d.label]:
                us = kernel_us[d.label]
                if "ops" in w:
                    rate = w["ops"] / (us * 1e-6) / 1e12
                    t = f" {us:9.2f} us {rate:8.1f} TOP/s {rate / pk['int8_tops']:6.1%} of int8"
                else:
                    rate = w.get("bytes", 0) / (us * 1e-6) / 1e9
                    t = f" {us:9.2f} us {rate:8.1f} GB/s  {rate / pk['hbm_gbs']:6.1%} of HBM"
            rows.append(f"{d.label:>16} {kname:<18} {dims:<24} {work}{t}{shape}")
        extra = [f"fusions: {', '.join(prog.fused) or 'none'}", f"checked: {self.checked} (proof "
                 f"{'holds' if self.proven else 'fails'})", prog.plan.report()]
        if kernel_us:
            extra.append(f"roofline denominators: {pk['int8_tops']} int8 TOP/s, {pk['hbm_gbs']} GB/s")
        return "\n".join(rows + extra)


def canary_bytes(n: int) -> np.ndarray:
    """The canary a guarded run fills the arena with: n pseudo-random bytes from a fixed seed (no constant byte
    value that a kernel might happen to write)."""
    return np.random.default_rng(0xA5C0FFEE).integers(0, 256, n, dtype=np.uint8)


def stray_bytes(inside: np.ndarray, canary: np.ndarray, after: np.ndarray, blob: np.ndarray,
                consts_after: np.ndarray) -> list:
    """[("arena" | "const", byte offset)] of the bytes a run changed that it must not have: arena bytes outside
    every planned buffer (`inside` False) that no longer hold the canary, and const bytes that differ from the
    uploaded blob (the reference's JobPlan.stray_writes, anvil/codegen/__init__.py:150-168, in bytes)."""
    n = min(len(inside), len(after), len(canary))
    arena = np.flatnonzero((after[:n] != canary[:n]) & ~inside[:n])
    m = min(len(blob), len(consts_after))
    const = np.flatnonzero(np.asarray(consts_after[:m]) != np.asarray(blob[:m]))
    return [("arena", int(o)) for o in arena] + [("const", int(o)) for o in const]


def _apply_view(buf: np.ndarray, v) -> np.ndarray:
    """The value of view `v` over its root buffer's bytes, as a fresh array of the view's dtype."""
    from .runtime.program import NP
    arr = buf.view(NP[v.dtype])
    if v.contiguous:
        return arr[: v.numel].reshape(v.shape)
    isz = arr.itemsize
    return np.lib.stride_tricks.as_strided(arr[v.offset:], v.shape, [s * isz for s in v.strides]).copy()


def compile(model, example_inputs=None, calib_inputs=None, params: CudaParams | None = None, schedules=None, *,
            consts=None, prove=True, **quant_kw) -> CompiledModel:  # noqa: A001
    """anvil.compile (anvil/driver.py:330-335). `schedules` is accepted for signature parity and ignored: the
    cuda target picks its kernels from the shapes. prove=False skips the static int32 proof for a graph-IR model
    and runs every kernel in checked mode instead."""
    module, cs, q = _resolve_model(model, example_inputs, calib_inputs, consts, quant_kw, prove)
    return CompiledModel(module, cs, params, quantized=q)
