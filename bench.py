"""Benchmark of the cuda target on a BASELINE.json configuration (default: c3, the GPT-2-small int8 block).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]

One process per GPU (torchrun for N > 1, NCCL process group for the barrier and the max-over-ranks timing only).
Scaling is weak: every rank runs the config's full batch of independent sequences on its own GPU; there is no
collective on the data path.

ours (default) prints one JSON line with
  value         whole-job tokens/s with the inputs already in HBM: K steps of the launch chain (CUDA-graph replay of
                every kernel) timed with CUDA events on the model's stream, max over ranks
  e2e           the same metric through the public API, cm.submit(x_int8, "cuda", quantized=True, out=...) per
                step with the previous step waited on (two steps in flight): per step the H2D copy of the quantized
                input from pinned memory, every kernel, the D2H read of the output into a pinned buffer the caller
                owns; run_value gives the synchronous cm.run(...) per step
  roofline      the dominant kernel family of the step: algorithmic int8 ops (or bytes) per launch / average
                launch time (CUDA events per launch on the model's stream), against 2 x the measured dense bf16
                peak (int8 dense rate = 2 x bf16 on B200) or the measured copy bandwidth; traffic from the
                committed ncu summary; roofline_int8_gemm gives the same for the tcgen05 GEMMs
  gemm_sweep_c4 config c4 (the int8 GEMM + requant sweep) as one-op graphs, sampled rows bit-exact
  cpu_baseline  the oracle port (numpy restatement of anvil.interp) on rank 0 at N = 1, one bounded sample
  clocks        nvidia-smi samples taken during the timed region
--impl reference times that CPU oracle alone (rank 0), with a process pool over all host cores.
--profile-runs R (with --batch) only runs the chain R times: the command the committed ncu summaries profile.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "anvil-compiler_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "tokens/s per B200 (int8 block, bit-exact to anvil.interp); int8 GEMM % peak"
CPU_SAMPLE_SEQS = 1


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


INT8_SPEC_TOPS = 4500.0       # B200 dense int8 tensor peak, NVIDIA's nominal figure (the 9 POPS one is 2:4 sparse)


def int8_peak_measured(device=None):
    """This GPU's dense int8 GEMM rate, measured here: torch._int_mm (cuBLASLt int8 -> int32) on 8192^3, best of 10
    launches timed with CUDA events. None when the library GEMM is unavailable."""
    import torch
    try:
        n = 8192
        g = torch.Generator(device="cuda").manual_seed(0)
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g).t().contiguous().t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    except Exception:
        return None


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region: NVML every ~5 ms on a background thread
    (the recipe's nvidia-smi clocks line, at a rate a millisecond-scale region can catch), nvidia-smi as fallback."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, device):
        self.device, self.sm, self.max, self.reasons, self._stop = device, [], None, set(), False
        self.times, self.err = [], None

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.device]) if vis else self.device
            self.h, self.nv = nv.nvmlDeviceGetHandleByIndex(idx), nv
            self.max = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
        except Exception as e:
            self.nv, self.err = None, f"{type(e).__name__}: {e}"[:120]
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t0 = time.perf_counter()
        self.t.start()
        return self

    def _run(self):
        while not self._stop:
            if self.nv is not None:
                try:
                    self.sm.append(float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)))
                    self.times.append(time.perf_counter() - self.t0)
                    r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    self.reasons |= {k for k, bit in self.REASONS.items() if r & bit}
                except Exception as e:
                    self.nv, self.err = None, f"{type(e).__name__}: {e}"[:120]
            time.sleep(0.002)

    def __exit__(self, *a):
        self.region_s = time.perf_counter() - self.t0
        self._stop = True
        self.t.join(timeout=2)
        if not self.sm:                          # NVML unavailable: one nvidia-smi reading
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.device}", "--query-gpu=clocks.sm,clocks.max.sm",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=20).stdout.split(",")
                self.sm, self.max = [float(out[0])], float(out[1])
            except Exception:
                pass

    def summary(self):
        out = {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max,
               "reasons": sorted(self.reasons), "samples": len(self.sm),
               "region_ms": round(1000 * getattr(self, "region_s", 0.0), 2),
               "sample_ms": [round(1000 * t, 2) for t in (self.times[:1] + self.times[-1:])]}
        if self.err:
            out["nvml_error"] = self.err
        return out


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _pg(ws, backend):
    if ws == 1:
        return None
    import datetime
    import torch.distributed as dist
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600))
    return dist


def _max_over_ranks(dist, v, device=None):
    if dist is None:
        return v
    import torch
    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(dist, device=None):
    if dist is not None:
        import torch
        if device is not None:
            dist.barrier(device_ids=[device])
        else:
            dist.barrier()


# --------------------------------------------------------------------------------------------- CPU oracle

_WORKER = {}


def _pool_init(payload):
    """Spawned worker: single-threaded numpy, the graph parsed once from its text form."""
    os.environ["OMP_NUM_THREADS"] = "1"
    os.environ["OPENBLAS_NUM_THREADS"] = "1"
    os.environ["MKL_NUM_THREADS"] = "1"
    from anvil.ir import parse_ir
    text, consts, in_sym, shape, scale, dtype = payload
    _WORKER["g"] = (parse_ir(text), {k: np.asarray(v) for k, v in consts.items()}, in_sym, shape, scale, dtype)


def _oracle_worker(seed):
    from oracle import interp
    module, consts, in_sym, shape, scale, dtype = _WORKER["g"]
    rng = np.random.default_rng(seed)
    if scale is not None:
        lo, hi = (-128, 127) if dtype == "i8" else (-(1 << 15), (1 << 15) - 1)
        xq = np.clip(np.rint(rng.standard_normal((1,) + tuple(shape)) / scale), lo, hi).astype(np.int64)
    else:
        xq = rng.integers(0, consts_vocab(consts), (1,) + tuple(shape))
    t = time.perf_counter()
    interp.run(module, {in_sym: xq}, consts, batch=True)
    return time.perf_counter() - t


def consts_vocab(consts):
    for k, v in consts.items():
        if k.endswith(".wte"):
            return v.shape[0]
    return 2


def cpu_baseline(cfg, cm, gen, seqs=CPU_SAMPLE_SEQS):
    """The oracle on `seqs` sequences in this process (BLAS threads as numpy starts them); tokens/s."""
    from anvil import workloads as W
    from oracle import interp
    x = gen(seqs)
    xq = cm.quantize_input(x) if cm.meta[cm.inputs[0]][0] is not None else x
    t = time.perf_counter()
    interp.run(cm.module, {cm.inputs[0]: xq}, cm.consts, batch=True)
    dt = time.perf_counter() - t
    seq = W.CONFIGS[cfg].seq
    return {"value": seqs * seq / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{seqs} sequence(s) of T={seq} through oracle.interp (numpy; exact int8 products via "
                      f"float64 BLAS), {dt:.2f} s"}


REFERENCE_BUDGET_S = 240.0


def run_reference(args):
    """The CPU oracle (the numpy restatement of anvil.interp) on the host cores: a spawn pool, one sequence of the
    config per worker per step."""
    ws, rank, local = _dist()
    if rank != 0:
        return 0
    import multiprocessing as mp
    from anvil import workloads as W
    from anvil.ir import print_ir
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    cores = max(1, min(cores, args.max_workers))
    cfg = args.config
    seq = W.CONFIGS[cfg].seq
    cm, _ = W.compile_config(cfg)
    in_sym = cm.inputs[0]
    payload = (print_ir(cm.module), cm.consts, in_sym, cm.meta[in_sym][1], cm.meta[in_sym][0], cm.meta[in_sym][2])
    ctx = mp.get_context("spawn")
    times = []
    # a step is one whole sequence per worker (several seconds of single-threaded numpy); the timed steps stop
    # early, with the count reported, once REFERENCE_BUDGET_S has passed, so any --steps ends within minutes
    t_start = None
    with ctx.Pool(cores, initializer=_pool_init, initargs=(payload,)) as pool:
        for step in range(args.warmup + args.steps):
            t = time.perf_counter()
            pool.map(_oracle_worker, [step * cores + i for i in range(cores)])
            dt = time.perf_counter() - t
            if step >= args.warmup:
                times.append(dt)
                t_start = t_start if t_start is not None else t
                if time.perf_counter() - t_start > REFERENCE_BUDGET_S:
                    break
    tok = cores * seq
    value = tok * len(times) / sum(times)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": len(times),
            "steps_requested": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8/int32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": cfg, "tokens_per_step": tok,
                       "sample": f"{cores} sequences of T={seq} per step, one per worker process"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{cores} sequences of T={seq} per step on a spawn pool of {cores} processes "
                                       "(oracle.interp, the numpy restatement of anvil.interp, one thread each)"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------- our arm

def run_ours(args):
    import torch
    from anvil import workloads as W
    from anvil.driver import CudaParams
    from anvil.runtime import cuda as C

    ws, rank, local = _dist()
    json_fd = 1
    if ws > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        # NCCL's banner and communicator set-up lines (one per rank: rank, device, bus id) are printed to the
        # process's stdout: point file descriptor 1 at stderr for everything the libraries print, and keep a copy
        # of the real stdout for the one JSON line
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        sys.stdout.flush()
        json_fd = os.dup(1)
        os.dup2(2, 1)
    torch.cuda.set_device(local)
    dist = _pg(ws, "nccl")
    cfg = args.config
    c = W.CONFIGS[cfg]
    batch = args.batch or c.batch
    cm, gen = W.compile_config(cfg, params=CudaParams(devices=(local,)))
    prog = cm.program(batch)
    dm = cm._device_model(local)
    dm.prepare(prog.ops, prog.plan.arena, key=(batch, "outputs", False))
    # inputs: quantized once on the host, in pinned memory (the e2e path copies them in every step)
    x = gen(batch)
    xq = cm.quantize_input(x) if cm.meta[cm.inputs[0]][0] is not None else x
    dt_in = {"i8": torch.int8, "i16": torch.int16, "i32": torch.int32}[cm.meta[cm.inputs[0]][2]]
    pinned = torch.empty(xq.shape, dtype=dt_in, pin_memory=True)
    pinned.numpy()[...] = xq
    xin = pinned.numpy()
    off = prog.inputs[cm.inputs[0]][0]
    dm.write(off, xin)
    if args.profile_runs:                   # profiling harness: plain launches of the chain, nothing timed
        for _ in range(args.profile_runs):
            dm.run([(off, xin)], [])
        print(json.dumps({"profile_runs": args.profile_runs, "launches_per_run": len(prog.ops), "batch": batch}))
        dm.close()
        return 0
    # correctness gate on the very program the timed loop replays: one CUDA-graph replay of the prepared batch,
    # then sampled sequences of its outputs (first, middle, last) against the oracle; the same sequences are checked
    # again after the timed replays
    sample = sorted({0, batch // 2, batch - 1})
    want = None
    if not args.skip_check:
        from oracle import interp
        want = interp.run(cm.module, {cm.inputs[0]: np.asarray(xq[sample])}, cm.consts, batch=True)
        dm.run_device(1, use_graph=True)
        _gate(cm, prog, dm, sample, want, "before the timed replays")
    tokens = batch * c.seq
    # warm-up (also captures the CUDA graph)
    dm.run_device(max(1, args.warmup), use_graph=True)
    torch.cuda.synchronize()
    _barrier(dist, local)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        _barrier(dist, local)
        ms = dm.run_device(args.steps, use_graph=True)
        torch.cuda.synchronize()
        _barrier(dist, local)
    ms = _max_over_ranks(dist, ms, f"cuda:{local}")
    ms_step = ms / args.steps
    value = ws * tokens / (ms_step / 1000.0)
    # per-launch device times for the roofline, taken while the GPU is still at its working clocks (a burst of graph
    # replays first): CUDA events recorded inside graph replays of the chain, between consecutive launches (the
    # launches follow each other as in the timed replays); also, for comparison, events around each launch of
    # separately issued chains (best of five), which add each launch's host-side issue cost
    dm.run_device(max(20, args.warmup), use_graph=True)
    timing_how = "CUDA events recorded inside graph replays of the chain between consecutive launches, best of 10"
    try:
        kus_graph = dm.time_launches(10)
    except Exception as e:                                   # a driver without event nodes in captured graphs
        kus_graph, timing_how = None, f"events around separately issued launches ({type(e).__name__})"
    kus_sep = None
    for _ in range(5):
        k = dm.run([(off, xin)], [], timing=True)
        kus_sep = k if kus_sep is None else [min(a, b) for a, b in zip(kus_sep, k)]
    kus = kus_graph if kus_graph is not None else kus_sep
    if want is not None:
        _gate(cm, prog, dm, sample, want, "after the timed replays")
    hbm, bf16, src = _peaks()
    i8peak = int8_peak_measured()
    roofs = _rooflines(prog, kus, hbm, bf16, src, C, i8peak)
    by_kind = {k: round(r["total_us"], 2) for k, r in roofs.items()}
    dominant = max(roofs, key=lambda k: roofs[k]["total_us"])
    roofline = {k: v for k, v in roofs[dominant].items() if k != "total_us"}
    roofline["traffic"] = _traffic_from_profiles(dominant)
    gemm_roof = {k: v for k, v in roofs["gemm"].items() if k != "total_us"} if "gemm" in roofs else None
    norm_roof = {k: v for k, v in roofs["norm"].items() if k != "total_us"} if "norm" in roofs else None
    if norm_roof is not None:
        norm_roof["traffic"] = _traffic_from_profiles("norm")
    # e2e through the public API, quantized input from pinned memory and the output read back into pinned memory
    # every step. Headline form: each step is cm.submit(...) and the step before it is waited on right after (two
    # steps in flight, outputs alternating between two pinned buffers), so one step's copies overlap its neighbours'
    # kernels and copies across the call boundary; every step's H2D, chain and D2H complete inside the timed
    # region. Also reported: the synchronous cm.run(...) per step.
    def pinned_outs():
        o = {}
        for s_ in cm.outputs:
            shape, dt = (batch,) + tuple(cm.meta[s_][1]), cm.meta[s_][2]
            o[s_] = torch.empty(shape, dtype={"i8": torch.int8, "i16": torch.int16, "i32": torch.int32}[dt],
                                pin_memory=True).numpy()
        return o
    out_step = sum(int(np.prod(cm.meta[s_][1])) * batch * {"i8": 1, "i16": 2, "i32": 4}[cm.meta[s_][2]]
                   for s_ in cm.outputs)
    # two steps in flight need two output buffers (a buffer is reused only after the step that filled it was waited
    # on); above 8 GB of output per step (c5's logits) one pinned buffer and one step in flight
    depth = 2 if out_step <= (8 << 30) else 1
    outs = [pinned_outs() for _ in range(depth)]

    def submitted(n):
        pend, last = [], None
        for step in range(n):
            pend.append(cm.submit(xin, "cuda", quantized=True, out=outs[step % depth]))
            if len(pend) >= depth:
                last = pend.pop(0).wait()
        for p_ in pend:
            last = p_.wait()
        return last

    submitted(max(3, args.warmup))
    torch.cuda.synchronize()
    t = time.perf_counter()
    res = submitted(args.steps)
    e2e_s = (time.perf_counter() - t) / args.steps
    e2e_s = _max_over_ranks(dist, e2e_s, f"cuda:{local}")
    run_times = []
    for step in range(args.warmup + min(args.steps, 50)):
        torch.cuda.synchronize()
        t = time.perf_counter()
        cm.run(xin, "cuda", quantized=True, out=outs[0])
        run_times.append(time.perf_counter() - t)
    run_s = _max_over_ranks(dist, statistics.mean(run_times[args.warmup:]), f"cuda:{local}")
    out_bytes = sum(np.asarray(res.ints[s]).nbytes for s in cm.outputs)
    bus_ms = _bus_bound_ms(xin.nbytes, out_bytes, local)
    strong = _strong_scaling(cm, dm, xin, batch, c.seq, ws, dist, local, args) if ws > 1 else None
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/int32", "data": "synthetic",
            "config": {"workload": cfg, "batch_per_gpu": batch, "seq_len": c.seq, "n_embd": c.cfg.n_embd,
                       "n_head": c.cfg.n_head, "n_layer": c.cfg.n_layer, "tokens_per_step_per_gpu": tokens,
                       "parallelism": f"replicas{ws}",
                       "l2": "inputs larger than L2 (activations of one step >> 126 MB)",
                       "launches": len(prog.ops), "fusions": prog.fused},
            "e2e": {"value": ws * tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(xin.nbytes),
                    "d2h_bytes_per_step": int(out_bytes), "api": "cm.submit(x, 'cuda', quantized=True, out=...) "
                    "then .wait() on the previous step", "steps_in_flight": depth,
                    "run_value": ws * tokens / run_s, "run_api": "cm.run(x, 'cuda', quantized=True, out=...) per "
                    "step (synchronous)",
                    "bus_ms_per_step": bus_ms,
                    "bound": "the larger of the step's device time and bus_ms_per_step (the step's H2D and D2H bytes "
                             "copied alone, both directions at once, pinned memory, best of 5)"},
            "roofline": roofline,
            "roofline_int8_gemm": gemm_roof,
            "roofline_norm": norm_roof,
            "kernel_us_by_kind": dict(sorted(by_kind.items(), key=lambda kv: -kv[1])),
            "launch_us": [[d.label, C.KIND_NAMES[d.kind], round(u, 2)] for d, u in zip(prog.devops, kus)],
            "launch_timing": timing_how,
            "launch_us_separate": [round(u, 2) for u in kus_sep],
            "gpu_launches": sum(1 for d in prog.devops if d.kind != C.OP_COPY) * args.steps,
            "clocks": clk.summary()}
    if strong is not None:
        line["strong_scaling"] = strong
    if rank == 0 and ws == 1 and not args.no_sweep:
        line["gemm_sweep_c4"] = gemm_sweep(i8peak or 2 * bf16)
    if rank == 0 and ws == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(cfg, cm, gen)
    if rank == 0:
        sys.stdout.flush()
        os.write(json_fd, (json.dumps(line) + "\n").encode())
    dm.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def _bus_bound_ms(h2d_bytes, d2h_bytes, local):
    """Milliseconds to move one step's input to the device and its output back with nothing else running: one H2D
    and one D2H copy of those sizes between pinned host buffers and device buffers, issued together on two streams
    (both directions of the bus busy at once), best of five. The end-to-end figure cannot beat it."""
    import torch
    dev = torch.device(f"cuda:{local}")
    hi = torch.empty(h2d_bytes, dtype=torch.uint8, pin_memory=True)
    ho = torch.empty(d2h_bytes, dtype=torch.uint8, pin_memory=True)
    di = torch.empty(h2d_bytes, dtype=torch.uint8, device=dev)
    do = torch.empty(d2h_bytes, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    best = float("inf")
    for _ in range(6):
        torch.cuda.synchronize(dev)
        t = time.perf_counter()
        with torch.cuda.stream(s1):
            di.copy_(hi, non_blocking=True)
        with torch.cuda.stream(s2):
            ho.copy_(do, non_blocking=True)
        torch.cuda.synchronize(dev)
        best = min(best, time.perf_counter() - t)
    del hi, ho, di, do
    return 1000.0 * best


def _strong_scaling(cm, dm, xin, global_batch, seq, ws, dist, local, args):
    """The config's stated batch as one fixed global batch split across the ws ranks (ceil(B / ws) sequences per
    rank, contiguous shards as CudaParams(devices=...) splits them): device-timed graph replays of each rank's
    shard, max over ranks, whole-job tokens/s."""
    import torch
    per = -(-global_batch // ws)
    prog = cm.program(per)
    dm.prepare(prog.ops, prog.plan.arena, key=(per, "outputs", False))
    rank = int(os.environ.get("RANK", "0"))
    lo = min(rank * per, global_batch - per)
    dm.write(prog.inputs[cm.inputs[0]][0], np.ascontiguousarray(xin[lo:lo + per]))
    dm.run_device(max(1, args.warmup), use_graph=True)
    torch.cuda.synchronize()
    _barrier(dist, local)
    ms = dm.run_device(args.steps, use_graph=True)
    torch.cuda.synchronize()
    _barrier(dist, local)
    ms = _max_over_ranks(dist, ms, f"cuda:{local}") / args.steps
    return {"global_batch": global_batch, "batch_per_gpu": per, "ms_per_step": ms,
            "value": global_batch * seq / (ms / 1000.0), "unit": "tokens/s", "scaling": "strong"}


def _gate(cm, prog, dm, sample, want, when):
    """The graph outputs of sequences `sample`, read from the device arena of the prepared program, must equal the
    oracle's (`want`, computed on those sequences); exits non-zero otherwise."""
    from anvil.driver import _apply_view
    for sym, v in prog.outputs:
        if sym is None or v.const:
            continue
        buf = dm.read(prog.plan.addresses[v.root], np.empty(prog.buffers[v.root], dtype=np.uint8))
        got = _apply_view(buf, v)[sample]
        if not np.array_equal(got, want.values[sym]):
            bad = np.argwhere(got != want.values[sym])
            raise SystemExit(f"bench: {sym} of sequences {sample} differs from the oracle {when} "
                             f"({len(bad)} values, first at {bad[0].tolist()})")


# What each family's ncu capture shows it waits on (the summaries under profiles/ give the figures).
LIMITERS = {
    "attention": "integer issue of the 16 softmax warps (about 23 instructions per kept score element across the "
                 "requant / row-sum / probability passes; ALU pipe the busiest), not the tensor pipe or DRAM",
    "gemm": "K = 3072: the tensor pipe (88 % active); K = 768: the epilogue warps draining each accumulator "
            "(requant, bias, LUT or residual, pack, TMA store)",
    "norm": "instruction issue and row-load latency of one warp per 768-byte row",
}


def _rooflines(prog, kus, hbm, bf16, src, C, i8peak=None):
    """Per kernel family: algorithmic ops (tensor-bound families) or bytes (HBM-bound) per launch over the average
    CUDA-event launch time. Tensor families are measured against this GPU's int8 GEMM rate measured in the same run
    (torch._int_mm, 8192^3) when it could be, with the fractions of 2 x the measured dense bf16 rate and of the 4.5
    POPS dense-int8 spec alongside; HBM families against the measured copy bandwidth."""
    fam = {}
    for d, u in zip(prog.devops, kus):
        k = C.KIND_NAMES[d.kind]
        f = fam.setdefault(k, {"n": 0, "us": 0.0, "ops": 0, "bytes": 0})
        f["n"] += 1
        f["us"] += u
        f["ops"] += d.work.get("ops", 0)
        f["bytes"] += d.work.get("bytes", 0)
    out = {}
    for k, f in fam.items():
        avg = f["us"] / f["n"]
        extra = {}
        if f["ops"]:
            ach = f["ops"] / f["n"] / (avg * 1e-6) / 1e12
            unit, bound = "TOP/s", "tensor"
            if i8peak:
                peak, ps = i8peak, "int8 GEMM rate measured in this run (torch._int_mm, 8192^3, best of 10)"
            else:
                peak, ps = 2 * bf16, f"2 x {src} bf16_tflops {bf16} (dense int8 = 2 x dense bf16 on B200)"
            extra = {"frac_of_2x_bf16": ach / (2 * bf16), "frac_of_int8_spec": ach / INT8_SPEC_TOPS}
            per = {"ops_per_launch": f["ops"] / f["n"]}
        else:
            ach = f["bytes"] / f["n"] / (avg * 1e-6) / 1e9
            peak, unit, bound = hbm, "GB/s", "hbm"
            ps = f"{src} hbm_gbs {hbm}"
            per = {"bytes_per_launch": f["bytes"] / f["n"]}
        out[k] = {"kernel": k, "bound": bound, "achieved": ach, "peak": peak, "unit": unit, "frac": ach / peak,
                  **extra, "peak_source": ps, "avg_launch_us": avg, "launches_per_step": f["n"],
                  "total_us": f["us"], **per}
        if k in LIMITERS:
            out[k]["limiter"] = LIMITERS[k]
    return out


def _library_int8_us(a, b, reps):
    """torch._int_mm (cuBLASLt int8 -> int32, no requant) on the same operands, B column-major like the tcgen05
    kernel's BT input: `reps` launches captured in one CUDA graph, replayed and timed with CUDA events, mean
    microseconds per launch, best of three replays (the same accounting as the graph replays of the sweep, with no
    host launch gaps). None when the library GEMM is unavailable."""
    import torch
    try:
        ta = torch.from_numpy(a).cuda()
        tb = torch.from_numpy(np.ascontiguousarray(b.T)).cuda().t()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                out = torch._int_mm(ta, tb)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                out = torch._int_mm(ta, tb)
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = float("inf")
        for _ in range(3):
            torch.cuda.synchronize()
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1000 / reps)
        del g, out
        return best
    except Exception:
        return None


def gemm_sweep(peak_tops, reps=20):
    """Config c4: int8 GEMM + requant at M in {1024, 8192, 65536}, K = N in {768, 3072, 4096}, each shape as a
    one-op graph (qlinear: A an input, B a constant) through anvil.compile on the cuda target: the same tcgen05 GEMM
    kernels and tile choice as anvil_gemm_requant, timed as `reps` CUDA-graph replays with CUDA events on the
    model's stream (the standalone entry point synchronises on its status words every call, so it is not what a
    kernel timing should wrap), best of three; 8 sampled rows per shape checked bit-exact against the oracle.
    Operands of the smaller shapes stay in L2 across replays. Beside each shape: the library int8 GEMM's time on the
    same operands (int32 output, no requant) and its ratio to ours (above 1: ours is faster)."""
    import warnings
    from anvil import workloads as W
    from anvil.driver import CudaParams, compile as anvil_compile
    from anvil.ir import GraphBuilder
    from oracle import semantics as osem
    res = []
    for m, k, n in W.GEMM_SWEEP:
        a, b, mult, s = W.gemm_case(m, k, n)
        g = GraphBuilder("c4")
        x = g.input("a", [m, k], "i8")
        g.output(g.qlinear("out", x, g.const("b", [k, n], "i8"), int(mult), int(s)))
        with warnings.catch_warnings():          # the data is U[-127, 127]: no intermediate can overflow
            warnings.simplefilter("ignore", RuntimeWarning)
            cm = anvil_compile(g.module(), consts={"b": b.astype(np.int64)}, prove=False,
                               params=CudaParams(checked=False, gemm="tc"))
        prog = cm.program(1)
        dm = cm._device_model(0)
        dm.prepare(prog.ops, prog.plan.arena, key=(1, "outputs", False))
        dm.write(prog.inputs["a"][0], a)
        dm.run_device(3, use_graph=True)
        us = min(dm.run_device(reps, use_graph=True) * 1000 / reps for _ in range(3))
        lib_us = _library_int8_us(a, b, reps)
        (sym, v), = [(sy, vw) for sy, vw in prog.outputs if sy is not None]
        out = dm.read(prog.plan.addresses[v.root], np.empty((m, n), dtype=np.int8))
        rows = np.random.default_rng(m + k).choice(m, 8, replace=False)
        want = osem.requant(osem.matmul_i8(a[rows].astype(np.int64), b.astype(np.int64)), mult, s)
        exact = bool(np.array_equal(out[rows].astype(np.int64), want))
        tops = 2 * m * n * k / (us * 1e-6) / 1e12
        res.append({"M": m, "K": k, "N": n, "us": round(us, 2), "tops": round(tops, 1),
                    "frac": round(tops / peak_tops, 4), "rows_exact": exact, "kernel": prog.devops[0].label,
                    "library_int8_us": None if lib_us is None else round(lib_us, 2),
                    "vs_library_same_shape": None if lib_us is None else round(lib_us / us, 3),
                    "l2": "operands larger than L2" if m * k + k * n > 126e6 else "operands fit L2 (warm)"})
        dm.close()
    return res


def _traffic_from_profiles(kind):
    """DRAM bytes (read + write) per launch of `kind` from the committed ncu summary, if there is one."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(kind)
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 200 for this arm, 3 for --impl reference)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3", choices=["c1", "c2", "c3", "c5"])
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--max-workers", type=int, default=64)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--profile-runs", type=int, default=0,
                    help="run the launch chain this many times without timing (the ncu profiling harness)")
    ap.add_argument("--skip-check", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        if args.steps is None:
            args.steps = 3
        return run_reference(args)
    if args.steps is None:
        args.steps = 200
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
