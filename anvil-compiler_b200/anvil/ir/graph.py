"""anvil.graph without xDSL: quantized tensor ops on SSA values of type qtensor<shape x dtype[, scale]>.

The op set, operand order, property names and verify rules follow the reference dialect
(anvil/ir/graph.py:1-25 for the op table, :181-343 for the verifiers, :361-455 for GraphBuilder), so a graph built
here and one built by the reference print the same generic MLIR text (anvil.ir.text) and evaluate the same way.
Three ops are extensions for the nanoGPT family the reference frontend rejects (anvil/frontend/capture.py:476-478,
162-173); each reduces to a reference op in a degenerate case:

    qlinear (x, w[, lut][, bias]) {M, s}   bias: an i32 const [N] added to the accumulator before the requant
                                           (bias = 0 is exactly the reference qlinear)
    layernorm_int (x, w, lut[, bias]) {M, s[, ss_shift, ss_init]}
                                           rmsnorm_int of the mean-centred row, plus an optional i8 bias
                                           (a row whose sum is 0, with no bias, is exactly rmsnorm_int)
    embed (ids, wte, wpe) {Ma, Mb, s}      add_requant(wte[ids[t]], wpe[t]) -> i8 (row gather + residual add)

Values are plain Python objects (``Value``) owned by ops; ops live in one ``FuncOp`` inside a ``Module``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

DTYPES = {"i8": 8, "i16": 16, "i32": 32}
WIDE = ("i8", "i16")                       # residual-stream dtypes


class VerifyException(ValueError):
    """A graph op or type breaks a dialect rule (the reference raises xdsl's VerifyException)."""


@dataclass(frozen=True)
class QTensorType:
    """qtensor<4x8xi8, 3.7e-02>: dims, element dtype and optional per-tensor scale (anvil/ir/graph.py:67-113)."""
    dims: tuple
    dtype: str = "i8"
    qscale: float | None = None

    def __init__(self, shape: Sequence[int], dtype: str = "i8", scale: float | None = None):
        if dtype not in DTYPES:
            raise ValueError(f"dtype {dtype!r} not in {sorted(DTYPES)}")
        object.__setattr__(self, "dims", tuple(int(d) for d in shape))
        object.__setattr__(self, "dtype", dtype)
        object.__setattr__(self, "qscale", None if scale is None else float(scale))
        if any(d < 1 for d in self.dims):
            raise VerifyException(f"qtensor dims must be positive, got {list(self.dims)}")

    @property
    def shape(self) -> list[int]:
        return list(self.dims)

    @property
    def numel(self) -> int:
        return math.prod(self.dims)

    @property
    def itemsize(self) -> int:
        return DTYPES[self.dtype] // 8


class Value:
    """An SSA value: the single result of `owner`."""
    __slots__ = ("type", "owner")

    def __init__(self, type_: QTensorType, owner=None):
        self.type = type_
        self.owner = owner

    def __repr__(self):
        sym = getattr(self.owner, "sym_str", None)
        return f"Value({sym or self.owner.name if self.owner else '?'}: {list(self.type.dims)}x{self.type.dtype})"


def qt(value) -> QTensorType:
    if not isinstance(value, Value):
        raise VerifyException(f"expected a qtensor value, got {value!r}")
    return value.type


def _expect(op, cond, msg):
    if not cond:
        raise VerifyException(f"{op.name}: {msg}")


def _check_shift(op, *names):
    for n in names:
        s = op.props[n]
        _expect(op, 0 <= s <= 31, f"{n}={s} outside [0, 31]")


def _lut256_i8(op, value):
    t = qt(value)
    _expect(op, list(t.dims) == [256] and t.dtype == "i8", f"LUT must be 256 x i8, got {list(t.dims)} x {t.dtype}")


class Op:
    """Base graph op. `operands` is the flat operand list; `slots` names them (optional slots may be None)."""
    name = "anvil.graph.op"
    slots: tuple = ()                 # operand names, in order
    optional: tuple = ()              # operand names that may be absent
    int_props: tuple = ()             # required integer properties
    opt_int_props: tuple = ()         # optional integer properties (absent = not printed)

    def __init__(self, operands: dict | None = None, props: dict | None = None, result_type: QTensorType | None = None,
                 sym: str | None = None):
        operands = dict(operands or {})
        self._ops = {n: operands.get(n) for n in self.slots}
        unknown = set(operands) - set(self.slots)
        if unknown:
            raise VerifyException(f"{self.name}: unknown operands {sorted(unknown)}")
        for n in self.slots:
            if self._ops[n] is None and n not in self.optional:
                raise VerifyException(f"{self.name}: missing operand {n}")
        self.props = dict(props or {})
        self.sym = sym
        self.result = Value(result_type, self) if result_type is not None else None

    # reference-style attribute access: op.a, op.b, op.lut, op.M, op.s ...
    def __getattr__(self, item):
        d = self.__dict__
        if "_ops" in d and item in d["_ops"]:
            return d["_ops"][item]
        if "props" in d and item in d["props"]:
            return d["props"][item]
        if item in type(self).opt_int_props:
            return None
        raise AttributeError(f"{type(self).__name__} has no attribute {item!r}")

    @property
    def operands(self) -> list:
        return [v for v in self._ops.values() if v is not None]

    @property
    def operand_map(self) -> dict:
        return dict(self._ops)

    @property
    def results(self) -> list:
        return [self.result] if self.result is not None else []

    @property
    def sym_str(self) -> str | None:
        return self.sym

    def verify(self):
        pass

    def __repr__(self):
        return f"<{self.name} {self.sym!r}>"


class FuncOp:
    name = "anvil.graph.func"

    def __init__(self, sym_name: str, ops: Sequence[Op] = ()):
        self.sym_name = sym_name
        self.ops: list[Op] = list(ops)

    def add_op(self, op):
        self.ops.append(op)


class Module:
    """builtin.module holding anvil.graph funcs."""
    name = "builtin.module"

    def __init__(self, funcs: Sequence[FuncOp] = ()):
        self.ops = list(funcs)

    def verify(self):
        for f in self.ops:
            verify_func(f)
        return self


class InputOp(Op):
    name = "anvil.graph.input"


class ConstOp(Op):
    name = "anvil.graph.const"

    def __init__(self, props=None, result_type=None, sym=None, value=None):
        super().__init__({}, props, result_type, sym)
        self.value = None if value is None else np.asarray(value, dtype=np.int64).reshape(result_type.dims)

    def verify(self):
        _expect(self, self.sym is not None or self.value is not None, "needs a sym or an inline value")
        if self.value is not None:
            _expect(self, list(self.value.shape) == list(qt(self.result).dims), "value shape != result shape")


class _MatmulBase(Op):
    slots = ("a", "b", "lut", "bias")
    optional = ("lut", "bias")
    int_props = ("M", "s")

    def verify(self):
        a, b, r = qt(self.a), qt(self.b), qt(self.result)
        ad, bd, rd = list(a.dims), list(b.dims), list(r.dims)
        _expect(self, a.dtype == b.dtype == "i8" and r.dtype in WIDE, "operands must be i8, the result i8 or i16")
        _expect(self, r.dtype == "i8" or self.lut is None, "a LUT epilogue needs an i8 result")
        _expect(self, len(ad) >= 2 and (len(bd) == 2 or (len(bd) == len(ad) and bd[:-2] == ad[:-2])),
                f"shapes {ad} @ {bd}: need (..., M, K) @ (K, N) or (..., M, K) @ (..., K, N)")
        _expect(self, ad[-1] == bd[-2], f"contraction mismatch {ad} @ {bd}")
        _expect(self, rd == ad[:-1] + [bd[-1]], f"result {rd} != {ad[:-1] + [bd[-1]]}")
        _check_shift(self, "s")
        if self.lut is not None:
            _lut256_i8(self, self.lut)
        if self.bias is not None:
            bt = qt(self.bias)
            _expect(self, isinstance(self.bias.owner, ConstOp), "bias operand must be an anvil.graph.const")
            _expect(self, bt.dtype == "i32" and list(bt.dims) == [bd[-1]], f"bias must be i32 [{bd[-1]}]")


class QMatmulOp(_MatmulBase):
    name = "anvil.graph.qmatmul"

    def verify(self):
        super().verify()
        _expect(self, self.bias is None, "a bias needs a qlinear (const weight)")


class QLinearOp(_MatmulBase):
    name = "anvil.graph.qlinear"

    def verify(self):
        super().verify()
        _expect(self, isinstance(self.b.owner, ConstOp), "weight operand must be an anvil.graph.const")
        _expect(self, len(qt(self.b).dims) == 2, "weight operand must be (K, N)")


class LutOp(Op):
    name = "anvil.graph.lut"
    slots = ("x", "table")

    def verify(self):
        _expect(self, qt(self.x).dtype == qt(self.result).dtype == "i8", "x and result must be i8")
        _expect(self, qt(self.x).dims == qt(self.result).dims, "shape changes")
        _lut256_i8(self, self.table)


class LutMulOp(Op):
    name = "anvil.graph.lut_mul"
    slots = ("x", "y", "table")
    int_props = ("M", "s")

    def verify(self):
        x, y, r = qt(self.x), qt(self.y), qt(self.result)
        _expect(self, x.dtype == y.dtype == r.dtype == "i8", "operands and result must be i8")
        _expect(self, x.dims == y.dims == r.dims, f"shapes {list(x.dims)}, {list(y.dims)} -> {list(r.dims)}")
        _lut256_i8(self, self.table)
        _check_shift(self, "s")


class _NormBase(Op):
    int_props = ("M", "s")
    opt_int_props = ("ss_shift", "ss_init")

    @property
    def ss_shift_int(self) -> int:
        return int(self.props.get("ss_shift") or 0)

    @property
    def ss_init_int(self) -> int:
        return int(self.props.get("ss_init") or 0)

    def _verify_norm(self):
        x, w, lut, r = qt(self.x), qt(self.w), qt(self.lut), qt(self.result)
        _expect(self, w.dtype == r.dtype == "i8" and x.dtype in WIDE, "x must be i8 or i16, w and result i8")
        _expect(self, 0 <= self.ss_shift_int <= 30, f"ss_shift={self.ss_shift_int} outside [0, 30]")
        _expect(self, 0 <= self.ss_init_int < 1 << 31, f"ss_init={self.ss_init_int} outside int32")
        _expect(self, list(w.dims) == list(x.dims[-1:]), f"weight {list(w.dims)} != [{x.dims[-1]}]")
        _expect(self, len(lut.dims) == 1 and lut.dtype == "i32", "rsqrt LUT must be 1-D i32")
        _expect(self, r.dims == x.dims, "shape changes")
        _check_shift(self, "s")


class RmsNormIntOp(_NormBase):
    name = "anvil.graph.rmsnorm_int"
    slots = ("x", "w", "lut")

    def verify(self):
        self._verify_norm()


class LayerNormIntOp(_NormBase):
    """Extension: integer LayerNorm. Per row of d entries: mean = floor((sum + d // 2) / d), xc = x - mean, then
    rmsnorm_int's sum of (rounded-shifted) squares, rsqrt index and requant on xc, then + bias (i8 [d]) and one
    clamp to int8."""
    name = "anvil.graph.layernorm_int"
    slots = ("x", "w", "lut", "bias")
    optional = ("bias",)

    def verify(self):
        self._verify_norm()
        if self.bias is not None:
            bt = qt(self.bias)
            _expect(self, bt.dtype == "i8" and list(bt.dims) == list(qt(self.x).dims[-1:]), "bias must be i8 [d]")


class SoftmaxLutOp(Op):
    name = "anvil.graph.softmax_lut"
    slots = ("x", "lut")
    int_props = ("one",)

    @property
    def causal_bool(self) -> bool:
        return bool(self.props["causal"])

    def verify(self):
        x, lut, r = qt(self.x), qt(self.lut), qt(self.result)
        _expect(self, x.dtype == "i8" and len(x.dims) >= 2, "scores must be i8 with rank >= 2")
        _expect(self, list(lut.dims) == [256] and lut.dtype == "i32", "exp LUT must be 256 x i32")
        _expect(self, r.dims == x.dims, "shape changes")
        one = self.props["one"]
        _expect(self, one >= 1 and (r.dtype == "i32" or one <= 127), f"one={one} does not fit result {r.dtype}")


class AddRequantOp(Op):
    name = "anvil.graph.add_requant"
    slots = ("a", "b")
    int_props = ("Ma", "Mb", "s")

    def verify(self):
        a, b, r = qt(self.a), qt(self.b), qt(self.result)
        _expect(self, {a.dtype, b.dtype, r.dtype} <= set(WIDE), "operands and result must be i8 or i16")
        _expect(self, a.dims == b.dims == r.dims, f"shapes {list(a.dims)} + {list(b.dims)} -> {list(r.dims)}")
        _check_shift(self, "s")


class EmbedOp(Op):
    """Extension: token + position embedding, x[t] = add_requant(wte[ids[t]], wpe[t], Ma, Mb, s) (i8 result)."""
    name = "anvil.graph.embed"
    slots = ("ids", "wte", "wpe")
    int_props = ("Ma", "Mb", "s")

    def verify(self):
        ids, wte, wpe, r = qt(self.ids), qt(self.wte), qt(self.wpe), qt(self.result)
        _expect(self, ids.dtype == "i32" and len(ids.dims) == 1, "ids must be i32 [T]")
        _expect(self, wte.dtype == wpe.dtype == "i8" and len(wte.dims) == 2 and len(wpe.dims) == 2,
                "wte and wpe must be i8 (rows, d)")
        _expect(self, wte.dims[1] == wpe.dims[1], "wte and wpe widths differ")
        _expect(self, ids.dims[0] <= wpe.dims[0], f"{ids.dims[0]} positions > {wpe.dims[0]} wpe rows")
        _expect(self, r.dtype == "i8" and list(r.dims) == [ids.dims[0], wte.dims[1]], "result must be i8 [T, d]")
        _check_shift(self, "s")


class TransposeOp(Op):
    name = "anvil.graph.transpose"
    slots = ("x",)

    @property
    def perm_list(self) -> list[int]:
        return [int(p) for p in self.props["perm"]]

    def verify(self):
        x, r, p = qt(self.x), qt(self.result), self.perm_list
        _expect(self, sorted(p) == list(range(len(x.dims))), f"perm {p} is not a permutation of rank {len(x.dims)}")
        _expect(self, list(r.dims) == [x.dims[i] for i in p] and r.dtype == x.dtype, "result type mismatch")


class ReshapeOp(Op):
    name = "anvil.graph.reshape"
    slots = ("x",)

    def verify(self):
        x, r = qt(self.x), qt(self.result)
        _expect(self, x.numel == r.numel and x.dtype == r.dtype, "reshape changes size or dtype")


class OutputOp(Op):
    name = "anvil.graph.output"

    def __init__(self, values):
        super().__init__({}, {}, None, None)
        self.values = list(values)

    @property
    def operands(self) -> list:
        return list(self.values)


OPS = {c.name: c for c in (InputOp, ConstOp, QMatmulOp, QLinearOp, LutOp, LutMulOp, RmsNormIntOp, LayerNormIntOp,
                           SoftmaxLutOp, AddRequantOp, EmbedOp, TransposeOp, ReshapeOp, OutputOp)}
EXTENSIONS = ("anvil.graph.layernorm_int", "anvil.graph.embed")


def verify_func(func: FuncOp):
    seen = set()
    for op in func.ops:
        for v in op.operands:
            if id(v) not in seen:
                raise VerifyException(f"{op.name} {op.sym!r}: operand defined after its use (or in another func)")
        op.verify()
        for r in op.results:
            seen.add(id(r))


# ----------------------------------------------------------------------------------------------------- builder

class GraphBuilder:
    """Appends verified graph ops to a func; every method returns the result value (anvil/ir/graph.py:361-455).

        g = GraphBuilder("mlp"); x = g.input("x", [4, 8], scale=0.03); ...; g.output(out); module = g.module()
    """

    def __init__(self, sym_name: str):
        self.func = FuncOp(sym_name)
        self._module = None

    def _add(self, op):
        self.func.add_op(op)
        op.verify()
        return op.result if op.result is not None else op

    def input(self, sym, shape, dtype="i8", scale=None):
        return self._add(InputOp({}, {}, QTensorType(shape, dtype, scale), sym))

    def const(self, sym, shape, dtype="i8", scale=None, value=None):
        return self._add(ConstOp({}, QTensorType(shape, dtype, scale), sym, value))

    def _mm(self, cls, sym, a, b, m, s, scale, lut, dtype="i8", bias=None):
        out = list(qt(a).dims[:-1]) + [qt(b).dims[-1]]
        return self._add(cls({"a": a, "b": b, "lut": lut, "bias": bias}, {"M": int(m), "s": int(s)},
                             QTensorType(out, dtype, scale), sym))

    def qmatmul(self, sym, a, b, m, s, scale=None, lut=None, dtype="i8"):
        return self._mm(QMatmulOp, sym, a, b, m, s, scale, lut, dtype)

    def qlinear(self, sym, x, w, m, s, scale=None, lut=None, dtype="i8", bias=None):
        return self._mm(QLinearOp, sym, x, w, m, s, scale, lut, dtype, bias)

    def lut(self, sym, x, table, scale=None):
        return self._add(LutOp({"x": x, "table": table}, {}, QTensorType(qt(x).dims, "i8", scale), sym))

    def lut_mul(self, sym, x, y, table, m, s, scale=None):
        return self._add(LutMulOp({"x": x, "y": y, "table": table}, {"M": int(m), "s": int(s)},
                                  QTensorType(qt(x).dims, "i8", scale), sym))

    @staticmethod
    def _norm_props(m, s, ss_shift, ss_init):
        p = {"M": int(m), "s": int(s)}
        if ss_shift:
            p["ss_shift"] = int(ss_shift)
        if ss_init:
            p["ss_init"] = int(ss_init)
        return p

    def rmsnorm_int(self, sym, x, w, lut, m, s, scale=None, ss_shift=0, ss_init=0):
        return self._add(RmsNormIntOp({"x": x, "w": w, "lut": lut}, self._norm_props(m, s, ss_shift, ss_init),
                                      QTensorType(qt(x).dims, "i8", scale), sym))

    def layernorm_int(self, sym, x, w, lut, m, s, scale=None, ss_shift=0, ss_init=0, bias=None):
        return self._add(LayerNormIntOp({"x": x, "w": w, "lut": lut, "bias": bias},
                                        self._norm_props(m, s, ss_shift, ss_init),
                                        QTensorType(qt(x).dims, "i8", scale), sym))

    def softmax_lut(self, sym, x, lut, one, causal=True, scale=None, dtype="i8"):
        return self._add(SoftmaxLutOp({"x": x, "lut": lut}, {"one": int(one), "causal": bool(causal)},
                                      QTensorType(qt(x).dims, dtype, scale), sym))

    def add_requant(self, sym, a, b, ma, mb, s, scale=None, dtype="i8"):
        return self._add(AddRequantOp({"a": a, "b": b}, {"Ma": int(ma), "Mb": int(mb), "s": int(s)},
                                      QTensorType(qt(a).dims, dtype, scale), sym))

    def embed(self, sym, ids, wte, wpe, ma, mb, s, scale=None):
        return self._add(EmbedOp({"ids": ids, "wte": wte, "wpe": wpe}, {"Ma": int(ma), "Mb": int(mb), "s": int(s)},
                                 QTensorType([qt(ids).dims[0], qt(wte).dims[1]], "i8", scale), sym))

    def transpose(self, sym, x, perm=None, scale=None):
        t = qt(x)
        perm = list(perm) if perm is not None else list(range(len(t.dims)))[::-1]
        sc = t.qscale if scale is None else scale
        return self._add(TransposeOp({"x": x}, {"perm": [int(p) for p in perm]},
                                     QTensorType([t.dims[i] for i in perm], t.dtype, sc), sym))

    def reshape(self, sym, x, shape, scale=None):
        t = qt(x)
        return self._add(ReshapeOp({"x": x}, {}, QTensorType(shape, t.dtype, t.qscale if scale is None else scale),
                                   sym))

    def output(self, *values):
        self._add(OutputOp(values))

    def module(self) -> Module:
        """The builtin.module holding the func (built once; later calls return the same module)."""
        if self._module is None:
            self._module = Module([self.func]).verify()
        return self._module


def funcs(module) -> list[FuncOp]:
    return [op for op in module.ops if isinstance(op, FuncOp)]


def func_of(m) -> FuncOp:
    if isinstance(m, FuncOp):
        return m
    fs = funcs(m)
    if len(fs) != 1:
        raise ValueError(f"expected one anvil.graph.func, found {len(fs)}")
    return fs[0]


def graph_meta(module) -> dict:
    """sym -> (scale, shape, dtype) for every graph value that carries a sym (anvil/driver.py:79-87)."""
    out = {}
    for op in func_of(module).ops:
        if isinstance(op, OutputOp) or not op.results:
            continue
        ty = qt(op.result)
        out[op.sym_str] = (ty.qscale, tuple(ty.dims), ty.dtype)
    return out
