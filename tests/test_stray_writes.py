"""Stray-write detection (the reference's RunOutput.stray_writes, anvil/driver.py:66-71): a guarded run lays the
arena out without buffer reuse and with canary bytes after every buffer, fills it with the canary, runs, and
reports every byte outside the planned buffers that changed, plus every changed const byte.

CPU tests: the guarded plan's layout; the comparison on planted before/after images; and the emulated launch list
(tests/devemu.py) of a guarded program, clean and with one op's output offset moved into a guard region (the
planted mistake). The GPU test (marked gpu) checks that guarded runs of real graphs report nothing and stay
bit-exact.
"""
import copy

import numpy as np
import pytest

import anvil
from anvil import memplan
from anvil.driver import GUARD_BYTES, canary_bytes, stray_bytes
from anvil.runtime import cuda as C
from devemu import Emu
from graphs import random_case
from oracle import interp


def _guarded(seed=3, batch=2):
    m, c, x, want = random_case(seed, batch=batch)
    cm = anvil.compile(m, consts=c, prove=False)
    return cm, x, want, cm.program(batch, "outputs", guard=True)


def test_guarded_plan_separates_every_buffer():
    cm, _, _, prog = _guarded()
    plan = prog.plan
    assert plan.guard == GUARD_BYTES
    spans = sorted((plan.addresses[s], plan.addresses[s] + b.size) for s, b in plan.bufs.items())
    for (_, end), (start, _) in zip(spans, spans[1:]):
        assert start - end >= GUARD_BYTES                       # no reuse, a guard after every buffer
    assert plan.arena - spans[-1][1] >= GUARD_BYTES
    inside = plan.inside()
    assert inside.sum() == sum(b.size for b in plan.bufs.values())
    assert cm.program(2).plan.guard == 0 and cm.program(2).plan.arena < plan.arena


def test_stray_bytes_on_planted_images():
    inside = np.zeros(4096, dtype=bool)
    inside[256:1000] = True
    canary = canary_bytes(4096)
    blob = np.arange(512, dtype=np.uint8)
    after, consts = canary.copy(), blob.copy()
    after[300:900] ^= 0x5A                                      # writes inside a buffer: allowed
    assert stray_bytes(inside, canary, after, blob, consts) == []
    after[1000] ^= 1                                            # one byte past the buffer
    after[4095] ^= 0xFF                                         # the arena's last byte
    consts[17] += 1                                             # a weight byte
    assert stray_bytes(inside, canary, after, blob, consts) == [("arena", 1000), ("arena", 4095), ("const", 17)]


def _emulate(prog, blob, x):
    emu = Emu(blob, prog.plan.arena)
    canary = canary_bytes(prog.plan.arena)
    emu.arena[:] = canary
    for sym, (off, shape, dtype) in prog.inputs.items():
        emu.put(off, np.asarray(x[sym]).ravel(), {"i8": 1, "i16": 2, "i32": 4}[dtype])
    emu.run(prog.ops)
    return stray_bytes(prog.plan.inside(), canary, emu.arena, blob, emu.blob)


@pytest.mark.parametrize("seed", [3, 7, 11])
def test_emulated_guarded_chain_writes_only_its_buffers(seed):
    cm, x, want, prog = _guarded(seed)
    assert _emulate(prog, cm._pool.blob(), x) == []


def test_planted_out_of_plan_store_is_reported():
    """One launch's output offset moved into the guard after its buffer (the planted mistake): the stores that
    land past the buffer are reported, as arena offsets inside that guard region."""
    cm, x, want, prog = _guarded(5)
    ops = [copy.copy(o) for o in prog.ops]
    i = next(k for k, o in enumerate(ops) if o.kind in (C.OP_GEMM, C.OP_ADD_REQUANT, C.OP_LUT))
    slot = {C.OP_GEMM: 2, C.OP_ADD_REQUANT: 2, C.OP_LUT: 2}[ops[i].kind]
    d = prog.devops[i]
    buf = d.writes[0]
    start, size = prog.plan.addresses[buf], prog.buffers[buf]
    ops[i].off[slot] = start + 128                              # the last 128 bytes spill into the guard
    bad = type(prog)(*[ops if f == "ops" else getattr(prog, f) for f in prog.__dataclass_fields__])
    stray = _emulate(bad, cm._pool.blob(), x)
    assert stray and all(r == "arena" and start + size <= o < start + size + GUARD_BYTES for r, o in stray)


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [3, 1001, 1004])
def test_guarded_gpu_runs_report_no_stray_writes(seed):
    """Guarded runs on the GPU (fuzz graphs; seeds above 1000 run the tcgen05 GEMMs): nothing outside the planned
    buffers or in the const region changes, and the outputs stay bit-exact."""
    m, c, x, want = random_case(seed, batch=2, big=seed > 1000)
    cm = anvil.compile(m, consts=c, prove=False)
    res = cm.run([x[s] for s in cm.inputs], "cuda", quantized=True, guard=True)
    assert res.stray_writes() == []
    for s in cm.outputs:
        assert np.array_equal(res.ints[s], want.values[s]), s
    with pytest.raises(ValueError):
        cm.run([x[s] for s in cm.inputs], "cuda", quantized=True).stray_writes()


@pytest.mark.gpu
def test_guarded_c3_block_reports_no_stray_writes():
    """The c3 block (fused attention, CTA-pair GEMMs with TMA tile stores, the V^T epilogue, LayerNorm rows) at 2
    sequences on the guarded layout: no stray byte, outputs bit-exact."""
    from anvil import workloads as W
    cm, gen = W.compile_config("c3")
    xq = cm.quantize_input(gen(2))
    want = interp.run(cm.module, {cm.inputs[0]: xq}, cm.consts, batch=True)
    res = cm.run(xq, "cuda", quantized=True, guard=True)
    assert res.stray_writes() == []
    for s in cm.outputs:
        assert np.array_equal(res.ints[s], want.values[s]), s
