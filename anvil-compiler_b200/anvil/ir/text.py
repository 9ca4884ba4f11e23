"""Generic MLIR text form of anvil.graph modules, without xDSL.

print_ir(module) writes what the reference's xDSL printer writes for a graph module (anvil/ir/__init__.py:22-25,
the frozen graphs in data/*/model_graph.json.gz are examples): one op per line,

    %5 = "anvil.graph.qlinear"(%3, %4) <{M = 6102 : i64, s = 21 : i64, sym = "L0.q"}> : (!anvil.graph.qtensor<...>,
         !anvil.graph.qtensor<...>) -> !anvil.graph.qtensor<16x32xi8, 3.29447435909011044e-02>

with properties in builder order (op props first, then sym), scales printed with 17 significant decimals, perms as
`array<i64: ...>`, inline const values as `dense<...> : tensor<...xi32>`. parse_ir reads that subset back and
verifies it, so print_ir(parse_ir(t)) == t for every reference-printed graph. An op with both optional matmul
operands (the lut epilogue and the bias extension) records which are present in `operandSegmentSizes`, as xDSL
does for ops with several optional operands.
"""
from __future__ import annotations

import re

import numpy as np

from . import graph as g

# ------------------------------------------------------------------------------------------------- printing


def _type_str(t: g.QTensorType) -> str:
    dims = "".join(f"{d}x" for d in t.dims)
    sc = "" if t.qscale is None else f", {t.qscale:.17e}"
    return f"!anvil.graph.qtensor<{dims}{t.dtype}{sc}>"


def _dense(value: np.ndarray) -> str:
    def rec(a):
        if a.ndim == 0:
            return str(int(a))
        return "[" + ", ".join(rec(x) for x in a) + "]"
    v = np.asarray(value)
    body = rec(v) if v.ndim else str(int(v))
    return f"dense<{body}> : tensor<{''.join(f'{d}x' for d in v.shape)}i32>"


def _props_str(op) -> str:
    parts = []
    if isinstance(op, g._MatmulBase) and op.bias is not None:
        segs = [1, 1, int(op.lut is not None), 1]
        parts.append(f"operandSegmentSizes = array<i32: {', '.join(map(str, segs))}>")
    if isinstance(op, g.ConstOp) and op.value is not None:
        parts.append(f"value = {_dense(op.value)}")
    for k, v in op.props.items():
        if k == "perm":
            parts.append(f"perm = array<i64: {', '.join(str(int(p)) for p in v)}>")
        elif isinstance(v, bool):
            parts.append(f"{k} = {'true' if v else 'false'}")
        else:
            parts.append(f"{k} = {int(v)} : i64")
    if op.sym is not None:
        parts.append(f'sym = "{op.sym}"')
    return "" if not parts else " <{" + ", ".join(parts) + "}>"


def print_ir(module) -> str:
    funcs = g.funcs(module) if isinstance(module, g.Module) else [module]
    lines = ["builtin.module {"]
    for f in funcs:
        lines.append(f'  "anvil.graph.func"() <{{sym_name = "{f.sym_name}"}}> ({{')
        names = {}
        for op in f.ops:
            ins = ", ".join(names[id(v)] for v in op.operands)
            in_types = ", ".join(_type_str(v.type) for v in op.operands)
            if op.result is not None:
                nm = f"%{len(names)}"
                names[id(op.result)] = nm
                lines.append(f'    {nm} = "{op.name}"({ins}){_props_str(op)} : ({in_types}) -> {_type_str(op.result.type)}')
            else:
                lines.append(f'    "{op.name}"({ins}){_props_str(op)} : ({in_types}) -> ()')
        lines.append("  }) : () -> ()")
    lines.append("}")
    return "\n".join(lines) + "\n"


# -------------------------------------------------------------------------------------------------- parsing

_TYPE = re.compile(r"!anvil\.graph\.qtensor<((?:\d+x)+)(i8|i16|i32)(?:,\s*([-+0-9.eEinfa]+))?>")
_OP = re.compile(r'^\s*(?:(%[\w.$-]+)\s*=\s*)?"([\w.]+)"\((.*?)\)\s*(?:<\{(.*)\}>)?\s*:\s*\((.*)\)\s*->\s*(.*?)\s*$')
_FUNC = re.compile(r'^\s*"anvil\.graph\.func"\(\)\s*<\{sym_name\s*=\s*"([^"]*)"\}>\s*\(\{\s*$')


class ParseError(ValueError):
    pass


def _parse_type(s: str) -> g.QTensorType:
    m = _TYPE.fullmatch(s.strip())
    if not m:
        raise ParseError(f"not a qtensor type: {s!r}")
    dims = [int(d) for d in m.group(1).rstrip("x").split("x")]
    return g.QTensorType(dims, m.group(2), None if m.group(3) is None else float(m.group(3)))


def _split_top(s: str, sep=",") -> list[str]:
    """Split on `sep` outside <>, [] and quotes."""
    out, depth, cur, q = [], 0, [], False
    for ch in s:
        if ch == '"':
            q = not q
        elif not q and ch in "<[(":
            depth += 1
        elif not q and ch in ">])":
            depth -= 1
        if ch == sep and depth == 0 and not q:
            out.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        out.append("".join(cur))
    return [p.strip() for p in out]


def _parse_dense(s: str):
    m = re.fullmatch(r"dense<(.*)>\s*:\s*tensor<((?:\d+x)*)i\d+>", s.strip(), re.S)
    if not m:
        raise ParseError(f"unsupported const value {s[:60]!r}")
    shape = [int(d) for d in m.group(2).rstrip("x").split("x") if d]
    nums = [int(v) for v in re.findall(r"-?\d+", m.group(1))]
    if len(nums) == 1 and np.prod(shape, dtype=np.int64) > 1:         # splat
        nums = nums * int(np.prod(shape))
    return np.asarray(nums, dtype=np.int64).reshape(shape)


def _parse_props(s: str | None) -> dict:
    props = {}
    if not s:
        return props
    for part in _split_top(s):
        k, v = part.split("=", 1)
        k, v = k.strip(), v.strip()
        if v.startswith("array<"):
            props[k] = [int(x) for x in re.findall(r"-?\d+", v.split(":", 1)[1])]
        elif v.startswith('"'):
            props[k] = v.strip('"')
        elif v in ("true", "false"):
            props[k] = v == "true"
        elif v.startswith("dense<"):
            props[k] = _parse_dense(v)
        else:
            props[k] = int(v.split(":")[0].strip())
    return props


def parse_ir(text: str) -> g.Module:
    """Parse (and verify) the generic form print_ir writes."""
    funcs, func, env = [], None, {}
    for ln, line in enumerate(text.splitlines(), 1):
        st = line.strip()
        if not st or st in ("builtin.module {", "}", "}) : () -> ()") or st.startswith("//"):
            if st == "}) : () -> ()" and func is not None:
                funcs.append(func)
                func = None
            continue
        m = _FUNC.match(line)
        if m:
            func, env = g.FuncOp(m.group(1)), {}
            continue
        m = _OP.match(line)
        if not m or func is None:
            raise ParseError(f"line {ln}: cannot parse {st[:80]!r}")
        res, name, ins, props_s, _in_types, out_type = m.groups()
        if name not in g.OPS:
            raise ParseError(f"line {ln}: unknown op {name!r}")
        cls = g.OPS[name]
        try:
            operands = [env[v.strip()] for v in ins.split(",") if v.strip()]
        except KeyError as e:
            raise ParseError(f"line {ln}: undefined value {e}") from None
        props = _parse_props(props_s)
        sym = props.pop("sym", None)
        segs = props.pop("operandSegmentSizes", None)
        if cls is g.OutputOp:
            op = g.OutputOp(operands)
        elif cls is g.ConstOp:
            value = props.pop("value", None)
            op = g.ConstOp(props, _parse_type(out_type), sym, value)
        else:
            slots = list(cls.slots)
            if segs is not None:
                named, i = {}, 0
                for slot, n in zip(slots, segs):
                    if n:
                        named[slot] = operands[i]
                        i += n
            else:
                if len(operands) > len(slots):
                    raise ParseError(f"line {ln}: {name} takes at most {len(slots)} operands")
                named = dict(zip(slots, operands))
            op = cls(named, props, _parse_type(out_type), sym)
        func.add_op(op)
        try:
            op.verify()
        except g.VerifyException as e:
            raise ParseError(f"line {ln}: {e}") from None
        if res is not None:
            env[res] = op.result
    if func is not None:
        raise ParseError("unterminated anvil.graph.func")
    return g.Module(funcs).verify()
