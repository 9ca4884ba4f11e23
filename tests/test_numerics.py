"""Host constant builders and the int32 overflow proof, pinned to the reference's own quantize.py (CPU)."""
import gzip
import json
from pathlib import Path

import numpy as np
import pytest

from anvil.frontend import numerics as Q
from anvil.ir import GraphBuilder

GOLDEN = Path(__file__).parent / "golden"


def test_primitives_equal_reference_quantize_module():
    with gzip.open(GOLDEN / "reference_quantize.json.gz", "rt") as f:
        cases = json.load(f)["cases"]
    assert len(cases) > 80
    for c in cases:
        fn = getattr(Q, c["fn"])
        if "raises" in c:
            with pytest.raises((ValueError, OverflowError)) as e:
                fn(*c["args"])
            assert type(e.value).__name__ == c["raises"]
            continue
        out = fn(*c["args"])
        want = c["out"]
        if c["fn"] in ("rmsnorm_lut", "rmsnorm_lut_wide", "silu_lut"):
            assert np.array_equal(out[0], want[0]), c["fn"]
            assert list(out[1:]) == list(want[1:]), c["fn"]
        elif c["fn"] == "fixed_point":
            assert [list(out[0]), out[1]] == want
        elif isinstance(want, list):
            assert np.array_equal(out, want), c["fn"]
        else:
            assert out == want, c["fn"]


def test_fixed_point_known_answers():
    with pytest.raises(OverflowError):
        Q.fixed_point([1.0], [1 << 31])
    with pytest.raises(ValueError):
        Q.fixed_point([1e-12, 1.0], [1 << 24, 1 << 24])
    (m,), s = Q.fixed_point([0.37], [1 << 20], max_shift=12)
    assert s == 12 and m == round(0.37 * 4096)


def test_proof_covers_extensions_and_rejects_overflow():
    g = GraphBuilder("p")
    x = g.input("x", [4, 32])
    h = g.layernorm_int("h", x, g.const("w", [32]), g.const("lut", [1024], "i32"), 1, 4)
    g.output(g.qlinear("y", h, g.const("fc", [32, 8]), 3, 12, bias=g.const("b", [8], "i32")))
    consts = {"w": np.full(32, 127), "lut": np.full(1024, 100), "fc": np.full((32, 8), 127), "b": np.full(8, 10)}
    worst = Q.prove_no_overflow(g.module(), consts)
    assert worst["y"] == (128 * 127 * 32 + 10) * 3 + (1 << 11)
    consts["lut"] = np.full(1024, 1 << 20)
    with pytest.raises(OverflowError):
        Q.prove_no_overflow(g.module(), consts)


def test_gelu_lut_is_monotone_where_gelu_is():
    lut, s = Q.gelu_lut(0.05)
    x = np.arange(-128, 128) * 0.05
    assert lut.shape == (256,) and np.abs(lut).max() == 127
    assert (np.diff(lut[x > -0.75]) >= 0).all()
    assert np.allclose(lut * s, Q.gelu(x), atol=s)
