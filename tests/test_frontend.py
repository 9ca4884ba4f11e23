"""torch -> anvil.graph for the nanoGPT family (CPU): capture patterns, quantization, and the float-path tolerance
of the integer graph against the torch module (the model.measure method of the reference, anvil/model.py:302-342).

Stated tolerances (max |dequantized int output - float output| in output LSBs, and RMS error / RMS output):
    c1 block (n_embd 32, T 8):                 max <= 2 LSB,  rms <= 3 %
    c2 2-layer model (vocab 64, n_embd 64):     max <= 8 LSB,  rms <= 8 %
The float path runs on the dequantized integer input (input-quantisation free, as the reference measures).
"""
import numpy as np
import pytest

import anvil
from anvil import workloads as W
from anvil.frontend import UnsupportedOpError, capture
from oracle import interp

TOL = {"c1": (2.0, 0.03), "c2": (8.0, 0.08)}


def test_capture_matches_the_block_structure():
    mod, ex, cal, gen = W.module_and_data("c1")
    fg = capture(mod, (ex,))
    ops = [n.op for n in fg.nodes]
    assert ops.count("layernorm") == 2 and ops.count("linear") == 6 and ops.count("add") == 2
    assert ops.count("softmax") == 1 and ops.count("gelu") == 1
    assert ops.count("split_heads") == 3 and ops.count("merge_heads") == 1
    sm = [n for n in fg.nodes if n.op == "softmax"][0]
    assert sm.attrs["causal"]
    assert "return add_1" in fg.text()


def test_model_capture_has_embedding_and_tied_head():
    mod, ex, cal, gen = W.module_and_data("c2")
    fg = capture(mod, (ex,))
    emb = [n for n in fg.nodes if n.op == "embed"]
    assert len(emb) == 1 and emb[0].attrs["wpe"].shape == (16, 64)
    head = fg.outputs[0]
    assert head.op == "linear" and head.attrs["bias"] is None
    assert np.array_equal(head.attrs["weight"], emb[0].attrs["wte"])     # tied


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_float_path_within_stated_tolerance(name):
    cm, gen = W.compile_config(name)
    x = gen(32)
    if cm.meta[cm.inputs[0]][0] is not None:
        xq = cm.quantize_input(x)
        xin = xq * cm.scale(cm.inputs[0])
    else:
        xq = xin = x
    got = interp.run(cm.module, {cm.inputs[0]: xq}, cm.consts, batch=True)
    ref = cm.quantized.reference(xin)
    o = cm.outputs[0]
    deq, r = got.values[o] * cm.scale(o), ref[o]
    max_lsb = np.abs(deq - r).max() / cm.scale(o)
    rms = np.sqrt(((deq - r) ** 2).mean() / (r ** 2).mean())
    assert max_lsb <= TOL[name][0] and rms <= TOL[name][1], (max_lsb, rms)


def test_zero_biases_leave_reference_qlinears():
    cm, _ = W.compile_config("c1")
    assert not any(getattr(op, "bias", None) is not None for op in cm.func.ops if op.name.endswith("qlinear"))
    assert cm.proven


def test_unsupported_op_is_named():
    import torch

    class Odd(torch.nn.Module):
        def forward(self, x):
            return torch.tanh(x)

    with pytest.raises(UnsupportedOpError, match="tanh"):
        capture(Odd(), (torch.zeros(1, 4, 8),))
