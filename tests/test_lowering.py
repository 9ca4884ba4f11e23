"""Host-side lowering of graphs to the cuda launch list, checked on the CPU: the emulated launch list
(tests/devemu.py: every anvil_op executed in numpy on a byte arena laid out by the memory plan) must equal the
oracle bit for bit. This covers views, strided copies, B^T operands, the LUT-epilogue and attention fusions, the
head-major V^T epilogue and the liveness offsets without a GPU."""
import numpy as np
import pytest

import anvil
from anvil.driver import CudaParams
from anvil import memplan
from devemu import run_program
from graphs import attention_graph, random_case
from oracle import interp


def _check(got, want, syms):
    for s in syms:
        assert np.array_equal(np.asarray(got[s]), np.asarray(want[s])), s


@pytest.mark.parametrize("seed", range(30))
def test_random_graph_launch_list(seed):
    m, c, x, want = random_case(seed, batch=3)
    cm = anvil.compile(m, consts=c, prove=False)
    for keep in ("outputs", "all"):
        got = run_program(cm, x, keep)
        syms = cm.outputs if keep == "outputs" else [k for k in got]
        _check(got, want.values, syms)


@pytest.mark.parametrize("T,C,nh,causal,T2", [(64, 128, 2, True, None), (48, 128, 2, False, None),
                                              (40, 256, 2, True, None), (32, 128, 2, False, 48),
                                              (36, 64, 2, True, None)])
def test_attention_fusion_launch_list(T, C, nh, causal, T2):
    m, c, x = attention_graph(T + C, T, C, nh, causal, T2)
    rng = np.random.default_rng(3)
    xb = {k: np.stack([v, rng.integers(-128, 128, v.shape)]) for k, v in x.items()}
    want = interp.run(m, xb, c, batch=True)
    cm = anvil.compile(m, consts=c)
    prog = cm.program(2)
    fusable = (C // nh) in (64, 128) and (T2 or T) % 16 == 0
    assert any("attention" in f for f in prog.fused) == fusable
    if fusable and T2 is None:
        assert any("vT_epilogue" in f for f in prog.fused)
    _check(run_program(cm, xb), want.values, cm.outputs)
    # keep="all" disables fusions and still matches every value
    got = run_program(cm, xb, "all")
    _check(got, want.values, [k for k in got])


def test_nanogpt_block_lowering_fuses_and_matches():
    from anvil import workloads as W
    cfg = W.GPTConfig(vocab_size=1, block_size=64, n_layer=1, n_head=2, n_embd=128)
    mod = W.build_block(cfg, 11)
    import torch
    rng = np.random.default_rng(0)
    cal = rng.standard_normal((4, 64, 128))
    cm = anvil.compile(mod, (torch.zeros(1, 64, 128),), [cal])
    prog = cm.program(2)
    assert any("attention" in f for f in prog.fused) and any("lut_epilogue" in f for f in prog.fused)
    xq = cm.quantize_input(rng.standard_normal((2, 64, 128)))
    want = interp.run(cm.module, {"x": xq}, cm.consts, batch=True)
    _check(run_program(cm, {"x": xq}), want.values, cm.outputs)


def test_qkv_projections_lower_to_one_split_gemm():
    """The q, k, v linears of a block whose width is whole 256-column tiles become one split-output GEMM (q and k
    side by side, v transposed for the attention), and the emulated launch list still equals the oracle."""
    from anvil import workloads as W
    from anvil.runtime import cuda as C
    cfg = W.GPTConfig(vocab_size=1, block_size=64, n_layer=1, n_head=4, n_embd=256)
    mod = W.build_block(cfg, 12)
    import torch
    rng = np.random.default_rng(1)
    cm = anvil.compile(mod, (torch.zeros(1, 64, 256),), [rng.standard_normal((4, 64, 256))])
    prog = cm.program(2)
    assert any(f.endswith(":qkv_split") for f in prog.fused)
    splits = [o for o in prog.ops if o.kind == C.OP_GEMM and o.flags & C.F_SPLIT]
    assert len(splits) == 1 and splits[0].dims[2] == 3 * 256 and splits[0].dims[5] == 2 * 256
    xq = cm.quantize_input(rng.standard_normal((2, 64, 256)))
    want = interp.run(cm.module, {"x": xq}, cm.consts, batch=True)
    _check(run_program(cm, {"x": xq}), want.values, cm.outputs)


def test_plan_reuses_and_never_overlaps_live_buffers():
    m, c, x, _ = random_case(3, batch=4)
    cm = anvil.compile(m, consts=c, prove=False)
    for keep in ("outputs", "all"):
        prog = cm.program(4, keep)
        plan = prog.plan
        assert not memplan.check_disjoint(plan.bufs.values(), plan.addresses)
        assert all(a % memplan.ALIGN == 0 for a in plan.addresses.values())
    assert cm.program(4).plan.arena <= cm.program(4).plan.unshared


@pytest.mark.parametrize("seed", range(30, 50))
def test_random_graph_unchecked_fusions(seed):
    """With checked=False every fusion applies; on inputs the oracle accepted no intermediate overflowed, so the
    32-bit epilogues are exact and the launch list must still match."""
    m, c, x, want = random_case(seed, batch=2)
    cm = anvil.compile(m, consts=c, prove=False, params=CudaParams(checked=False))
    _check(run_program(cm, x), want.values, cm.outputs)
