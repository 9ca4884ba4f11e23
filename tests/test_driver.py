"""anvil.compile / CompiledModel host logic on the CPU: argument checking with the reference's error types
(anvil/driver.py:90-132, 248-280), quantization, and a loud failure when the GPU path cannot run."""
import numpy as np
import pytest

import anvil
from anvil.driver import CudaParams
from anvil.ir import GraphBuilder
from anvil.runtime import cuda as C


def _graph(overflow=False):
    g = GraphBuilder("g")
    x = g.input("x", [4, 8], scale=0.05)
    g.output(g.qlinear("y", x, g.const("w", [8, 8]), (1 << 22) if overflow else 3, 10, 0.1))
    return g.module(), {"w": np.full((8, 8), 100)}


def test_compile_checks_like_the_reference():
    m, c = _graph()
    with pytest.raises(ValueError):
        anvil.compile(m)                                     # missing const values
    with pytest.raises(ValueError):
        anvil.compile(m, consts={**c, "zz": np.zeros(2)})   # unknown const
    with pytest.raises(TypeError):
        anvil.compile(object())
    with pytest.raises(TypeError):
        anvil.compile((m, c), headroom=2.0)
    mo, co = _graph(overflow=True)
    with pytest.raises(OverflowError):
        anvil.compile(mo, consts=co)
    cm = anvil.compile(mo, consts=co, prove=False)
    assert cm.checked and not cm.proven
    assert anvil.compile(m, consts=c).checked is False
    with pytest.raises(ValueError):
        CudaParams(devices=())
    with pytest.raises(ValueError):
        CudaParams(gemm="wmma")


def test_inputs_are_validated_and_quantized():
    m, c = _graph()
    cm = anvil.compile(m, consts=c)
    with pytest.raises(ValueError):
        cm.run(np.zeros((4, 8)), "isasim")
    with pytest.raises(ValueError):
        cm._bind_inputs(np.zeros((8, 4)), False)
    with pytest.raises(ValueError):
        cm._bind_inputs(np.full((4, 8), np.nan), False)
    with pytest.raises(ValueError):
        cm._bind_inputs(np.full((4, 8), 200), True)
    with pytest.raises(ValueError):
        cm._bind_inputs(np.zeros((4, 8)), True)              # float with quantized=True
    xs = np.array([0.5, 1.5, 2.5, -0.5, -1.5, 1000.0, -1000.0]) * 0.05
    q = cm.quantize_input(xs)
    assert list(q) == list(np.clip(np.rint(xs / 0.05), -128, 127).astype(int))   # half to even, saturating
    assert q[-2:].tolist() == [127, -128]
    bound, batch, batched = cm._bind_inputs(np.zeros((5, 4, 8)), False)
    assert batch == 5 and batched
    bound, batch, batched = cm._bind_inputs(np.zeros(32), False)
    assert batch == 1 and not batched


def test_shards_split_the_batch_contiguously():
    m, c = _graph()
    cm = anvil.compile(m, consts=c, params=CudaParams(devices=(0, 1, 2)))
    assert cm._shards(7) == [(0, 0, 3), (1, 3, 6), (2, 6, 7)]
    assert cm._shards(2) == [(0, 0, 1), (1, 1, 2)]


def test_run_fails_loudly_without_a_gpu():
    if C.device_count() > 0:
        pytest.skip("a GPU is visible")
    m, c = _graph()
    cm = anvil.compile(m, consts=c)
    with pytest.raises((NotImplementedError, RuntimeError, ImportError)):
        cm.run(np.zeros((4, 8)), "cuda")


def test_summary_lists_every_launch():
    m, c = _graph()
    text = anvil.compile(m, consts=c).summary(batch=2)
    assert "gemm" in text and "footprint" in text and "checked: False" in text


def test_summary_gives_the_roofline_fraction_of_each_timed_launch():
    """With measured microseconds (RunOutput.cycles of a timing run) every launch shows its achieved rate and the
    fraction of the roofline bounding it: ops against the int8 tensor peak, bytes against HBM bandwidth."""
    m, c = _graph()
    cm = anvil.compile(m, consts=c)
    labels = [d.label for d in cm.program(2).devops]
    text = cm.summary(batch=2, kernel_us={lab: 10.0 for lab in labels}, peaks={"int8_tops": 1000.0, "hbm_gbs": 5000.0})
    rows = text.splitlines()[:len(labels)]
    assert all(" us " in r and "% of " in r for r in rows)
    d = cm.program(2).devops[0]
    if "ops" in d.work:
        want = d.work["ops"] / 10e-6 / 1e12 / 1000.0
        assert f"{want:6.1%}" in rows[0]
    assert "1000.0 int8 TOP/s, 5000.0 GB/s" in text
