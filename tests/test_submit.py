"""CompiledModel.submit / PendingRun.wait on the CPU: the device models are replaced by an emulator (tests/devemu.py
runs each enqueued chunk's launch list in numpy) that keeps the C library's ticket contract (anvil_model_record
snapshots and clears the model's check words, anvil_model_wait_ticket reports the snapshot once). Checks that
queued runs return what the oracle returns, in any wait order, that chunks chain across calls, that a device
error is reported by the run whose work raised it and by no other, and that a bounded queue collects the oldest
run. The GPU path of the same API is tested in tests/test_gpu_parity.py."""
from __future__ import annotations

import numpy as np
import pytest

import anvil
from anvil import driver as D
from anvil.runtime import cuda as C
from devemu import Emu
from graphs import attention_graph
from oracle import interp


class EmuModel:
    """Stands in for runtime.cuda.DeviceModel: enqueue runs the chunk at once; check words are a plain int."""
    instances = []
    fail_next = set()          # ids of models whose next enqueue sets a check word

    def __init__(self, device, blob):
        self.device, self.blob = device, np.asarray(blob, dtype=np.uint8)
        self.prepared_key, self.flags, self.next, self.snap = None, 0, 0, {}
        self.afters = []
        EmuModel.instances.append(self)

    def prepare(self, ops, arena_bytes, key=None):
        self.ops, self.arena_bytes, self.prepared_key = list(ops), int(arena_bytes), key

    def clear_flags(self):
        self.flags = 0

    def enqueue(self, inputs, outputs, after=None):
        self.afters.append(after)
        emu = Emu(self.blob, self.arena_bytes)
        for off, a in inputs:
            emu.arena[off:off + a.nbytes] = np.frombuffer(np.ascontiguousarray(a).tobytes(), dtype=np.uint8)
        emu.run(self.ops)
        for off, a in outputs:
            a.reshape(-1).view(np.uint8)[...] = emu.arena[off:off + a.nbytes]
        if id(self) in EmuModel.fail_next:
            EmuModel.fail_next.discard(id(self))
            self.flags = 1

    def record(self):
        t = self.next
        self.snap[t], self.flags = self.flags, 0
        self.next += 1
        return t

    def wait_ticket(self, t):
        if t not in self.snap:
            raise ValueError(f"ticket {t} is not outstanding")
        if self.snap.pop(t):
            raise OverflowError("emulated device check")

    def close(self):
        pass


@pytest.fixture
def emu_models(monkeypatch):
    EmuModel.instances.clear()
    EmuModel.fail_next.clear()
    monkeypatch.setattr(C, "DeviceModel", EmuModel)
    return EmuModel


def _compiled(pipeline=4):
    mod, consts, _ = attention_graph(0, 16, 64, 2)
    return anvil.compile(mod, consts=consts, params=D.CudaParams(devices=(0,), pipeline=pipeline))


def _inputs(batch, seed):
    return np.random.default_rng(seed).integers(-128, 128, (batch, 16, 64))


def _want(cm, x):
    res = interp.run(cm.module, {"x": x}, cm.consts, batch=True)
    return {s: res.values[s] for s in cm.outputs}


def test_queued_runs_match_the_oracle_in_any_wait_order(emu_models):
    cm = _compiled()
    assert cm._pipelinable(cm.program(2, "outputs"))
    xs = [_inputs(8, s) for s in range(3)]
    pend = [cm.submit(x, quantized=True) for x in xs]
    assert not any(p.done() for p in pend)
    for i in (2, 0, 1):
        got = pend[i].wait()
        for sym, w in _want(cm, xs[i]).items():
            assert np.array_equal(got.ints[sym], w), (i, sym)
        assert pend[i].done()
    assert cm._outstanding == []


def test_chunks_chain_across_calls(emu_models, monkeypatch):
    monkeypatch.setattr(D, "PIPELINE_MODELS", 4)
    cm = _compiled()
    p1 = cm.submit(_inputs(8, 1), quantized=True)
    models = list(EmuModel.instances)
    p2 = cm.submit(_inputs(8, 2), quantized=True)
    p1.wait(), p2.wait()
    # four chunks per call round-robin over four models: the second call's first chunk waits behind the first
    # call's last chunk (another model), and no chunk is chained behind its own model
    firsts = [m for m in models if m.afters]
    assert len(firsts) == 4
    assert models[0].afters[0] is None and models[0].afters[1] is models[3]
    for m in models:
        assert all(a is not m for a in m.afters)


def test_a_device_error_belongs_to_the_run_that_raised_it(emu_models):
    cm = _compiled()
    x1, x2, x3 = (_inputs(8, s) for s in (4, 5, 6))
    p1 = cm.submit(x1, quantized=True)
    EmuModel.fail_next.add(id(EmuModel.instances[2]))       # the second call's third chunk raises a check
    p2 = cm.submit(x2, quantized=True)
    p3 = cm.submit(x3, quantized=True)
    got = p3.wait()
    assert np.array_equal(got.ints[cm.outputs[0]], _want(cm, x3)[cm.outputs[0]])
    with pytest.raises(OverflowError):
        p2.wait()
    with pytest.raises(OverflowError):                      # the error stays with its run
        p2.wait()
    p1.wait()


def test_the_queue_is_bounded(emu_models, monkeypatch):
    monkeypatch.setattr(D, "MAX_OUTSTANDING", 2)
    cm = _compiled()
    pend = [cm.submit(_inputs(8, s), quantized=True) for s in range(4)]
    assert [p.done() for p in pend] == [True, True, False, False]
    assert len(cm._outstanding) == 2
    for p in pend:
        p.wait()


def test_submit_validates_like_run(emu_models):
    cm = _compiled()
    with pytest.raises(ValueError, match="unknown backend"):
        cm.submit(_inputs(2, 0), "isasim", quantized=True)
    with pytest.raises(ValueError):
        cm.submit(np.zeros((2, 16, 63), dtype=np.int64), quantized=True)
