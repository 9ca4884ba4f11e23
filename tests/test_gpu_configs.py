"""BASELINE configurations and the persistent kernels' multi-tile paths on a B200 vs the CPU oracle (marked gpu).

The round-robin persistent kernels only show their steady state when every CTA walks several work items: the
CTA-pair GEMM's TMEM accumulator ping-pong and barrier phase flips after the first tile, the fused attention's
rotation of score buffers and its deferred output epilogue. The shapes here give each CTA (or CTA pair) three or
more items, and every output value is compared with the oracle. Then each BASELINE configuration runs through
the public API (anvil.compile(...).run(x, "cuda")) at its stated shape (c5 at one sequence: the oracle takes about
a minute per sequence). Tolerance: none (integer outputs must be identical).
"""
import numpy as np
import pytest

import anvil
from anvil.driver import CudaParams
from oracle import interp
from oracle import semantics as sem

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    assert torch.cuda.is_available(), "a gpu test needs a CUDA device"
    return torch


def _equal(got, want, what):
    g, w = np.asarray(got), np.asarray(want)
    assert g.shape == w.shape, (what, g.shape, w.shape)
    if not np.array_equal(g, w):
        bad = np.argwhere(g != w)
        raise AssertionError(f"{what}: {len(bad)} of {g.size} differ, first at {bad[0].tolist()}: "
                             f"{g[tuple(bad[0])]} != {w[tuple(bad[0])]}")


def _oracle_by_sequence(module, inputs, consts):
    """The oracle's values of a batched run, one sequence at a time (bounded host memory), stacked."""
    n = len(next(iter(inputs.values())))
    runs = [interp.run(module, {k: v[i:i + 1] for k, v in inputs.items()}, consts, batch=True).values
            for i in range(n)]
    return {s: np.concatenate([r[s] for r in runs]) for s in runs[0] if s not in consts}


_COMPILED = {}


def _config(name):
    """(CompiledModel, generator) of a BASELINE config, compiled once per test session (c5 takes a minute)."""
    if name not in _COMPILED:
        from anvil import workloads as W
        _COMPILED[name] = W.compile_config(name)
    return _COMPILED[name]


def _launch_shapes(cm, batch):
    """(kind, describe tuple) of every launch of the program prepared on device 0 for `batch`."""
    prog = cm.program(batch)
    dm = cm._device_model(cm.params.devices[0])
    assert dm.prepared_key == (batch, "outputs", False)
    return [(d.kind, dm.describe(i)) for i, d in enumerate(prog.devops)]


# ------------------------------------------------------------------------------- multi-tile persistent paths

@pytest.mark.parametrize("T,K,N,kind", [(8192, 768, 3072, "lut"), (20480, 3072, 768, "residual"),
                                        (20480, 768, 768, "bias")])
@pytest.mark.parametrize("checked", [False, True])
def test_pair_gemm_three_or_more_tiles_per_cluster(T, K, N, kind, checked, monkeypatch):
    """CTA-pair GEMMs where every cluster runs at least three 256-row tiles (the accumulator ping-pong and the
    phase flips of every barrier after the first tile), with LUT, fused residual (unchecked) and bias epilogues,
    checked and unchecked, every output vs the oracle."""
    from test_gpu_parity import _pair_gemm_case
    from anvil.runtime import cuda as C
    monkeypatch.setenv("ANVIL_GEMM_PAIR", "1")
    module, consts, inputs = _pair_gemm_case(T + K + N, T, K, N, kind)
    want = interp.run(module, inputs, consts)
    cm = anvil.compile(module, consts=consts, params=CudaParams(checked=checked, gemm="tc"))
    res = cm.run([inputs[s] for s in cm.inputs], "cuda", quantized=True)
    gemms = [info for k, info in _launch_shapes(cm, 1) if k == C.OP_GEMM]
    assert gemms and gemms[0][1] == 2, f"expected CTA-pair tiles, got {gemms}"
    bn, _, tiles, ctas = gemms[0]
    assert tiles >= 3 * (ctas // 2), f"{tiles} tiles on {ctas // 2} clusters"
    for s in cm.outputs:
        _equal(res.ints[s], want.values[s], s)


def test_gemm_requant_full_output_65536():
    """anvil_gemm_requant at 65536 x 768 x 768 (config c4's largest M at its smallest K = N): every output value
    vs requant(matmul_i8) of the oracle."""
    torch = _torch()
    from anvil import workloads as W
    from anvil.runtime import cuda as C
    m, k, n = 65536, 768, 768
    a, b, mult, s = W.gemm_case(m, k, n)
    want = sem.requant(sem.matmul_i8(a.astype(np.int64), b.astype(np.int64)), mult, s)
    ta = torch.from_numpy(a).cuda()
    tbt = torch.from_numpy(np.ascontiguousarray(b.T)).cuda()
    out = torch.empty((m, n), dtype=torch.int8, device="cuda")
    torch.cuda.synchronize()
    C.gemm_requant(ta.data_ptr(), tbt.data_ptr(), out.data_ptr(), m, n, k, mult, s, 0,
                   torch.cuda.current_stream().cuda_stream)
    _equal(out.cpu().numpy().astype(np.int64), want, "out")


@pytest.mark.parametrize("m,n,k", [(1024, 768, 768), (8192, 768, 768), (1024, 3072, 3072), (700, 200, 96)])
def test_gemm_requant_tile_choices_bit_exact(m, n, k):
    """The standalone entry point at shapes whose tile choice is not the widest single-CTA tile (narrow tiles to
    fill the SMs, CTA pairs): bit-exact, unchecked and checked."""
    torch = _torch()
    from anvil import workloads as W
    from anvil.runtime import cuda as C
    a, b, mult, s = W.gemm_case(m, k, n)
    want = sem.requant(sem.matmul_i8(a.astype(np.int64), b.astype(np.int64)), mult, s)
    ta = torch.from_numpy(a).cuda()
    tbt = torch.from_numpy(np.ascontiguousarray(b.T)).cuda()
    for flags in (0, C.F_CHECKED):
        out = torch.full((m, n), 77, dtype=torch.int8, device="cuda")
        torch.cuda.synchronize()
        C.gemm_requant(ta.data_ptr(), tbt.data_ptr(), out.data_ptr(), m, n, k, mult, s, flags,
                       torch.cuda.current_stream().cuda_stream)
        _equal(out.cpu().numpy().astype(np.int64), want, f"out (flags {flags})")


def test_fused_attention_many_items_per_cta():
    """The fused attention at B = 16, H = 12, T = 1024 (config c3's shape at 16 sequences): 1536 work items on
    148 CTAs, so every CTA walks about ten items through its score-buffer rotation and deferred output epilogue."""
    from graphs import attention_graph
    m, c, x = attention_graph(1024 + 768 + 12, 1024, 768, 12, True)
    batch = 16
    rng = np.random.default_rng(8)
    xb = {k: np.stack([v] + [rng.integers(-128, 128, v.shape) for _ in range(batch - 1)]) for k, v in x.items()}
    want = _oracle_by_sequence(m, xb, c)
    cm = anvil.compile(m, consts=c, params=CudaParams(pipeline=1))       # one launch chain over the 16 sequences
    res = cm.run([xb[s] for s in cm.inputs], "cuda", quantized=True)
    from anvil.runtime import cuda as C
    attn = [info for k, info in _launch_shapes(cm, batch) if k == C.OP_ATTENTION]
    assert attn and attn[0][2] >= 3 * attn[0][3], attn
    for s in cm.outputs:
        _equal(res.ints[s], want[s], s)


# ------------------------------------------------------------------------------------- BASELINE configs

def test_c1_block_full():
    """Config c1 (block d32 h2 T8, batch 1, seed 0) through anvil.compile(...).run: every output vs the oracle."""
    from anvil import workloads as W
    cm, gen = W.compile_config("c1")
    xq = cm.quantize_input(gen(1))
    want = interp.run(cm.module, {cm.inputs[0]: xq}, cm.consts, batch=True)
    res = cm.run(xq, "cuda", quantized=True)
    for s in cm.outputs:
        _equal(res.ints[s], want.values[s], s)
    res = cm.run(xq, "cuda", quantized=True, keep="all")              # every value of the unfused chain
    for s, v in want.values.items():
        if s not in cm.consts:
            _equal(res.ints[s], v, s)


def test_c2_model_256_sequences():
    """Config c2 (2-layer d64 h4 T16 V64) at its stated batch of 256 sequences through the public API."""
    from anvil import workloads as W
    cm, gen = W.compile_config("c2")
    ids = np.asarray(gen(256))
    want = interp.run(cm.module, {cm.inputs[0]: ids}, cm.consts, batch=True)
    res = cm.run(ids, "cuda", quantized=True)
    for s in cm.outputs:
        _equal(res.ints[s], want.values[s], s)


def test_c3_block_64_sequences_sampled():
    """Config c3 at its stated batch of 64 sequences (the bench's timed program): the whole batch runs on the GPU;
    sequences 0, 31 and 63 are compared in full with the oracle."""
    from anvil import workloads as W
    cm, gen = W.compile_config("c3", params=CudaParams(pipeline=1))
    xq = cm.quantize_input(gen(64))
    res = cm.run(xq, "cuda", quantized=True)
    sample = [0, 31, 63]
    want = interp.run(cm.module, {cm.inputs[0]: xq[sample]}, cm.consts, batch=True)
    for s in cm.outputs:
        _equal(np.asarray(res.ints[s])[sample], want.values[s], s)


def test_c5_model_one_sequence_every_logit():
    """Config c5 (12-layer GPT-2-small int8, vocab 50304, T 1024, seed 4): one sequence, all 1024 x 50304 logits
    vs the oracle."""
    cm, gen = _config("c5")
    ids = np.asarray(gen(1))
    want = interp.run(cm.module, {cm.inputs[0]: ids}, cm.consts, batch=True)
    res = cm.run(ids, "cuda", quantized=True)
    for s in cm.outputs:
        _equal(res.ints[s], want.values[s], s)


def test_c5_float_path_tolerance():
    """Config c5's stated float-path tolerance (tests/test_frontend.py states and explains it): one sequence, the
    integer logits from the GPU (bit-exact to the oracle, checked above) against the float model."""
    from test_frontend import float_path_error
    cm, gen = _config("c5")
    max_lsb, rms, gain = float_path_error(cm, np.asarray(gen(1)),
                                          lambda xq: cm.run(xq, "cuda", quantized=True).ints[cm.outputs[0]])
    assert max_lsb <= 90 and rms <= 0.85 and 0.6 <= gain <= 1.1, (max_lsb, rms, gain)


# --------------------------------------------------------------------------------------------- multi-GPU

def test_two_devices_in_one_process():
    """CudaParams(devices=(0, 1)): the batch splits into two contiguous shards, one host thread per device, each
    device its own replica of the constants; the reassembled outputs equal the oracle's (needs two GPUs)."""
    torch = _torch()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from anvil import workloads as W
    cm, gen = W.compile_config("c3", params=CudaParams(devices=(0, 1)))
    xq = cm.quantize_input(gen(5))
    want = interp.run(cm.module, {cm.inputs[0]: xq}, cm.consts, batch=True)
    res = cm.run(xq, "cuda", quantized=True)
    assert [d for d, _ in res.result.shards] == [0, 1] and [b for _, b in res.result.shards] == [3, 2]
    for s in cm.outputs:
        _equal(res.ints[s], want.values[s], s)


def test_two_devices_submitted():
    """submit() with CudaParams(devices=(0, 1)): each device's shard is queued on that device's models without a
    host thread per device; two runs queued back to back, waited in reverse order, equal the oracle (needs two
    GPUs)."""
    torch = _torch()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from anvil import workloads as W
    cm, gen = W.compile_config("c3", params=CudaParams(devices=(0, 1)))
    xs = [cm.quantize_input(gen(4)), cm.quantize_input(gen(4))[::-1].copy()]
    pend = [cm.submit(x, "cuda", quantized=True) for x in xs]
    for x, p in reversed(list(zip(xs, pend))):
        res = p.wait()
        assert [d for d, _ in res.result.shards] == [0, 1]
        want = interp.run(cm.module, {cm.inputs[0]: x}, cm.consts, batch=True)
        for s in cm.outputs:
            _equal(res.ints[s], want.values[s], s)
