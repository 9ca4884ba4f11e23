"""CPU oracle (test infrastructure only): whole-tensor numpy interpreter for anvil.graph.

Restates the reference interpreter anvil/interp/graph.py:43-92 (the stand-in for `anvil.interp`, which cannot be
imported here: it needs xdsl and the missing xf submodule). Ops evaluate in program order through
oracle.semantics; after every op the result's shape and dtype range are re-checked (anvil/interp/graph.py:35-40).

    run(module, {"x": x}, consts)               one sample: x has the graph input's shape
    run(module, {"x": xs}, consts, batch=True)  xs has one leading batch dim; every value keeps it, consts do not
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import semantics as sem

try:                                   # the graph IR data structure comes from the package under test
    from anvil.ir import graph as g
except ImportError:                    # pragma: no cover - tests put the package on sys.path
    raise


@dataclass
class GraphResult:
    outputs: list                                   # graph.output operands, in order
    values: dict = field(default_factory=dict)      # sym -> array for every op that carries a sym


def _check_type(op, val, lead=()):
    t = g.qt(op.result)
    if list(val.shape) != list(lead) + list(t.dims):
        raise ValueError(f"{op.name} {op.sym_str!r}: shape {list(val.shape)} != declared {list(t.dims)}")
    sem.check_dtype(val, t.dtype, f"{op.name} {op.sym_str!r}")
    return val


def run(m, inputs: dict, consts: dict | None = None, *, batch: bool = False) -> GraphResult:
    """Evaluate the graph (anvil/interp/graph.py:43-92). `inputs` binds graph.input by sym; `consts` binds
    graph.const without an inline value."""
    consts = consts or {}
    env, res = {}, GraphResult([])
    lead, nb, is_const = (), 0, set()
    if batch:
        first = next(iter(inputs.values()))
        lead, nb = (int(np.shape(first)[0]),), 1
    for op in g.func_of(m).ops:
        v = lambda x: env[id(x)]  # noqa: E731
        if isinstance(op, g.InputOp):
            val = np.asarray(inputs[op.sym_str], dtype=np.int64)
        elif isinstance(op, g.ConstOp):
            is_const.add(id(op.result))
            val = op.value if op.value is not None else np.asarray(consts[op.sym_str], dtype=np.int64)
        elif isinstance(op, (g.QMatmulOp, g.QLinearOp)):
            lut = None if op.lut is None else v(op.lut)
            bias = None if op.bias is None else v(op.bias)
            val = sem.qmatmul(v(op.a), v(op.b), op.M, op.s, lut, g.qt(op.result).dtype, bias)
        elif isinstance(op, g.LutOp):
            val = sem.lut_i8(v(op.x), v(op.table))
        elif isinstance(op, g.LutMulOp):
            val = sem.swiglu_lut(v(op.x), v(op.y), v(op.table), op.M, op.s)
        elif isinstance(op, g.RmsNormIntOp):
            val = sem.rmsnorm_wide(v(op.x), v(op.w), v(op.lut), op.M, op.s, op.ss_shift_int, op.ss_init_int,
                                   g.qt(op.x).dtype)
        elif isinstance(op, g.LayerNormIntOp):
            bias = None if op.bias is None else v(op.bias)
            val = sem.layernorm_int(v(op.x), v(op.w), v(op.lut), op.M, op.s, op.ss_shift_int, op.ss_init_int,
                                    g.qt(op.x).dtype, bias)
        elif isinstance(op, g.SoftmaxLutOp):
            val = sem.softmax_lut(v(op.x), v(op.lut), op.one, op.causal_bool)
        elif isinstance(op, g.AddRequantOp):
            val = sem.add_requant(v(op.a), v(op.b), op.Ma, op.Mb, op.s, g.qt(op.result).dtype)
        elif isinstance(op, g.EmbedOp):
            val = sem.embed(v(op.ids), v(op.wte), v(op.wpe), op.Ma, op.Mb, op.s)
        elif isinstance(op, g.TransposeOp):
            k = 0 if id(op.x) in is_const else nb
            val = np.transpose(v(op.x), list(range(k)) + [p + k for p in op.perm_list])
        elif isinstance(op, g.ReshapeOp):
            k = () if id(op.x) in is_const else lead
            val = v(op.x).reshape(list(k) + list(g.qt(op.result).dims))
        elif isinstance(op, g.OutputOp):
            res.outputs = [v(x) for x in op.values]
            continue
        else:
            raise NotImplementedError(op.name)
        if isinstance(op, (g.TransposeOp, g.ReshapeOp)) and id(op.x) in is_const:
            is_const.add(id(op.result))
        env[id(op.result)] = _check_type(op, val, () if id(op.result) in is_const else lead)
        if op.sym_str is not None:
            res.values[op.sym_str] = env[id(op.result)]
    return res
