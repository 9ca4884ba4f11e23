"""Benchmark of the cuda target on a BASELINE.json configuration (default: c3, the GPT-2-small int8 block).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]

One process per GPU (torchrun for N > 1, NCCL process group for the barrier and the max-over-ranks timing only).
Scaling is weak: every rank runs the config's full batch of independent sequences on its own GPU; there is no
collective on the data path.

ours (default) prints one JSON line with
  value         whole-job tokens/s with the inputs already in HBM: K steps of the launch chain (CUDA-graph replay of
                every kernel) timed with CUDA events on the model's stream, max over ranks
  e2e           the same metric through the public API, cm.run(x_int8, "cuda", quantized=True): per step the H2D
                copy of the quantized input from pinned memory, every kernel, the D2H read of the output
  roofline      the dominant kernel family (the tcgen05 GEMMs): algorithmic int8 ops per launch / average launch
                time (CUDA events per launch on the model's stream), against 2 x the measured dense bf16 peak
                (int8 dense rate = 2 x bf16 on B200); traffic from an ncu capture when one is committed
  cpu_baseline  the oracle port (numpy restatement of anvil.interp) on rank 0 at N = 1, one bounded sample
  clocks        nvidia-smi samples taken during the timed region
--impl reference times that CPU oracle alone (rank 0), with a process pool over all host cores.
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


class ClockSampler:
    """nvidia-smi clocks / throttle reasons every 200 ms on a background thread (the recipe's clocks line)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device, self.rows, self.proc = device, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


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
    with ctx.Pool(cores, initializer=_pool_init, initargs=(payload,)) as pool:
        for step in range(args.warmup + args.steps):
            t = time.perf_counter()
            pool.map(_oracle_worker, [step * cores + i for i in range(cores)])
            dt = time.perf_counter() - t
            if step >= args.warmup:
                times.append(dt)
    tok = cores * seq
    value = tok * len(times) / sum(times)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
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
    if ws > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(local)
    dist = _pg(ws, "nccl")
    cfg = args.config
    c = W.CONFIGS[cfg]
    batch = args.batch or c.batch
    cm, gen = W.compile_config(cfg, params=CudaParams(devices=(local,)))
    prog = cm.program(batch)
    dm = cm._device_model(local)
    dm.prepare(prog.ops, prog.plan.arena, key=(batch, "outputs"))
    # inputs: quantized once on the host, in pinned memory (the e2e path copies them in every step)
    x = gen(batch)
    xq = cm.quantize_input(x) if cm.meta[cm.inputs[0]][0] is not None else x
    dt_in = {"i8": torch.int8, "i16": torch.int16, "i32": torch.int32}[cm.meta[cm.inputs[0]][2]]
    pinned = torch.empty(xq.shape, dtype=dt_in, pin_memory=True)
    pinned.numpy()[...] = xq
    xin = pinned.numpy()
    off = prog.inputs[cm.inputs[0]][0]
    dm.write(off, xin)
    # correctness gate: one sequence of the device result against the oracle (rank 0, before timing)
    if rank == 0 and not args.skip_check:
        from oracle import interp
        res = cm.run(xin[:1] if len(cm.params.devices) else xin, "cuda", quantized=True)
        want = interp.run(cm.module, {cm.inputs[0]: np.asarray(xq[:1])}, cm.consts, batch=True)
        for s in cm.outputs:
            if not np.array_equal(res.ints[s], want.values[s]):
                raise SystemExit(f"bench: {s} differs from the oracle")
        dm.prepare(prog.ops, prog.plan.arena, key=(batch, "outputs"))
        dm.write(off, xin)
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
    # per-launch device times (CUDA events on the model's stream) for the roofline
    dm.write(off, xin)
    kus = dm.run([(off, xin)], [], timing=True)
    for _ in range(2):
        kus2 = dm.run([(off, xin)], [], timing=True)
        kus = [min(a, b) for a, b in zip(kus, kus2)]
    gemm_ops = sum(d.work.get("ops", 0) for d in prog.devops if d.kind == C.OP_GEMM)
    gemm_us = sum(u for d, u in zip(prog.devops, kus) if d.kind == C.OP_GEMM)
    n_gemm = sum(1 for d in prog.devops if d.kind == C.OP_GEMM)
    by_kind = {}
    for d, u in zip(prog.devops, kus):
        k = C.KIND_NAMES[d.kind]
        by_kind[k] = by_kind.get(k, 0.0) + u
    hbm, bf16, src = _peaks()
    peak_tops = 2 * bf16
    achieved = gemm_ops / (gemm_us * 1e-6) / 1e12 if gemm_us else 0.0
    roofline = {"bound": "tensor", "kernel": "qgemm_tc (tcgen05 kind::i8)", "achieved": achieved,
                "peak": peak_tops, "unit": "TOP/s", "frac": achieved / peak_tops,
                "peak_source": f"2 x {src} bf16_tflops {bf16} (dense int8 = 2 x bf16 on B200)",
                "ops_per_launch": gemm_ops / max(1, n_gemm), "avg_launch_us": gemm_us / max(1, n_gemm),
                "traffic": _traffic_from_profiles(), "launches_per_step": n_gemm}
    # e2e through the public API
    e2e_times = []
    for step in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t = time.perf_counter()
        res = cm.run(xin, "cuda", quantized=True)
        e2e_times.append(time.perf_counter() - t)
    e2e_s = statistics.mean(e2e_times[args.warmup:])
    e2e_s = _max_over_ranks(dist, e2e_s, f"cuda:{local}")
    out_bytes = sum(np.asarray(res.ints[s]).nbytes for s in cm.outputs)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/int32", "data": "synthetic",
            "config": {"workload": cfg, "batch_per_gpu": batch, "seq_len": c.seq, "n_embd": c.cfg.n_embd,
                       "n_head": c.cfg.n_head, "n_layer": c.cfg.n_layer, "tokens_per_step_per_gpu": tokens,
                       "parallelism": f"replicas{ws}",
                       "l2": "inputs larger than L2 (activations of one step >> 126 MB)",
                       "launches": len(prog.ops), "fusions": prog.fused},
            "e2e": {"value": ws * tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(xin.nbytes),
                    "d2h_bytes_per_step": int(out_bytes)},
            "roofline": roofline,
            "kernel_us_by_kind": {k: round(v, 2) for k, v in sorted(by_kind.items(), key=lambda kv: -kv[1])},
            "gpu_launches": sum(1 for d in prog.devops if d.kind != C.OP_COPY) * args.steps,
            "clocks": clk.summary()}
    if rank == 0 and ws == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(cfg, cm, gen)
    if rank == 0:
        print(json.dumps(line), flush=True)
    dm.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def _traffic_from_profiles():
    """DRAM bytes per GEMM launch from the committed ncu summary, if there is one (else null)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("qgemm_tc_bytes_per_launch")
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3", choices=["c1", "c2", "c3", "c5"])
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--max-workers", type=int, default=64)
    ap.add_argument("--skip-check", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
