"""anvil.graph without xDSL: builder verification and the generic MLIR text round trip (CPU)."""
import gzip
import json
from pathlib import Path

import numpy as np
import pytest

from anvil.ir import GraphBuilder, ParseError, VerifyException, parse_ir, print_ir

GOLDEN = Path(__file__).parent / "golden"


@pytest.mark.parametrize("name", ["frozen_model.json.gz", "frozen_model_i8.json.gz"])
def test_reference_printed_graphs_round_trip_byte_exact(name):
    with gzip.open(GOLDEN / name, "rt") as f:
        text = json.load(f)["ir"]
    m = parse_ir(text)
    assert print_ir(m) == text
    assert len(m.ops[0].ops) == 76


def _ext_graph():
    g = GraphBuilder("ext")
    ids = g.input("ids", [8], "i32")
    x = g.embed("x", ids, g.const("wte", [16, 32]), g.const("wpe", [8, 32]), 900, 700, 11, 0.02)
    h = g.layernorm_int("h", x, g.const("w", [32]), g.const("lut", [1024], "i32"), 1, 12, 0.03,
                        bias=g.const("b", [32]))
    y = g.qlinear("y", h, g.const("fc", [32, 64]), 77, 14, 0.04, bias=g.const("fcb", [64], "i32"),
                  lut=g.const("gelu", [256]))
    z = g.qmatmul("z", y, g.transpose("fcT", g.const("fc2", [16, 64]), [1, 0]), 5, 9)
    g.output(z, g.const("inline", [2, 2], value=np.array([[1, -2], [3, 4]])))
    return g.module()


def test_extension_ops_round_trip():
    m = _ext_graph()
    text = print_ir(m)
    assert "anvil.graph.layernorm_int" in text and "anvil.graph.embed" in text and "operandSegmentSizes" in text
    assert print_ir(parse_ir(text)) == text


@pytest.mark.parametrize("bad", [
    lambda g, x: g.qlinear("q", x, g.const("w", [3, 4]), 1, 32),                       # shift > 31
    lambda g, x: g.qlinear("q", x, g.const("w", [5, 4]), 1, 3),                        # contraction mismatch
    lambda g, x: g.lut("l", x, g.const("t", [128])),                                   # LUT not 256 entries
    lambda g, x: g.softmax_lut("p", x, g.const("e", [256], "i32"), 200),               # one > 127 for i8
    lambda g, x: g.rmsnorm_int("r", x, g.const("w", [4]), g.const("l", [64], "i32"), 1, 3),   # weight length
    lambda g, x: g.qlinear("q", x, g.input("w2", [3, 4]), 1, 3),                       # weight not a const
    lambda g, x: g.transpose("t", x, [0, 0]),
    lambda g, x: g.reshape("r", x, [5]),
])
def test_verifier_rejects(bad):
    g = GraphBuilder("bad")
    x = g.input("x", [2, 3])
    with pytest.raises(VerifyException):
        bad(g, x)


def test_parse_errors():
    with pytest.raises(ParseError):
        parse_ir('builtin.module {\n  "anvil.graph.func"() <{sym_name = "f"}> ({\n    %0 = "anvil.graph.bogus"() : () -> '
                 '!anvil.graph.qtensor<4xi8>\n  }) : () -> ()\n}\n')
    with pytest.raises(ParseError):
        parse_ir('builtin.module {\n  "anvil.graph.func"() <{sym_name = "f"}> ({\n    "anvil.graph.output"(%9) : '
                 '(!anvil.graph.qtensor<4xi8>) -> ()\n  }) : () -> ()\n}\n')
