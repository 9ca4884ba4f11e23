"""torch.export -> a small float op graph (FGraph) that anvil.frontend.quantize lowers to anvil.graph.

    fg = capture(module, (x,))           # x: (B, T, C) float or (B, T) token ids; the leading dim is the batch
    print(fg.text())
    acts = fg.evaluate([xs])             # float64 activations of every node on a batch (torch)

Follows the reference frontend's pipeline (anvil/frontend/capture.py:1-27, 672-697): export the module in eval
mode, treat every node that depends only on parameters, buffers and literals as a constant, and pattern-match the
rest into the frontend op set. The ATen ops are matched at the level torch.export emits them (linear, layer_norm,
rms_norm, gelu, silu, embedding, split, view/reshape, transpose/permute, scaled_dot_product_attention, softmax,
matmul, add, mul); anything else raises UnsupportedOpError naming the op.

Frontend ops (per-sample shapes, the batch dim dropped):
    input                         graph input (float activations, or int64 token ids)
    embed (ids) {wte, wpe}        wte[ids] + wpe[0:T]  (nn.Embedding pair of nanoGPT; extension)
    layernorm (x) {weight, bias, eps}                                   (extension)
    rmsnorm (x) {weight, eps}
    linear (x) {weight, bias, rows}  x @ W[rows].T + b; `rows` from a split of the output (one linear per chunk)
    matmul (a, b) {factor}        (a @ b) * factor (None or ("inv_sqrt", n) or ("mul", c))
    softmax (x) {causal}
    gelu (x) {approximate}, silu (x), mul (a, b), add (a, b)
    transpose (x) {perm}, reshape (x)
    split_heads (x) {nh}, merge_heads (x) {nh}   (T, C) <-> (nh, T, hd)
"""
from __future__ import annotations

import math
import operator
from dataclasses import dataclass, field


class UnsupportedOpError(NotImplementedError):
    """An op (or a use of an op) outside the frontend's patterns; the message names the ATen op."""


class FNode:
    """One frontend op: `op` (the op set in the module docstring), a unique `name`, its operand nodes `inputs`,
    op attributes `attrs` (weights as float64 numpy arrays) and the per-sample result `shape` (no batch dim).
    Nodes compare by identity: two nodes with the same fields are still two values."""

    __slots__ = ("op", "name", "inputs", "attrs", "shape")

    def __init__(self, op: str, name: str, inputs, attrs: dict, shape):
        self.op, self.name, self.inputs = op, name, list(inputs)
        self.attrs, self.shape = dict(attrs), tuple(shape)

    def __repr__(self):
        return f"FNode({self.op} {self.name} {list(self.shape)})"


class FGraph:
    """A captured float graph: `nodes` in evaluation order, the `inputs` and `outputs` among them, and the
    example batch size. Lookups by name and the users of a node come from indexes built on first use (the graph
    is not changed after capture)."""

    def __init__(self, nodes, inputs, outputs, batch: int = 1):
        self.nodes, self.inputs, self.outputs, self.batch = list(nodes), list(inputs), list(outputs), batch
        self._by_name = None
        self._users = None

    def node(self, name) -> FNode:
        if self._by_name is None:
            self._by_name = {n.name: n for n in self.nodes}
        return self._by_name[name]

    def users(self, node) -> list:
        """The nodes that read `node`, in evaluation order (once each)."""
        if self._users is None:
            idx = {}
            for n in self.nodes:
                for i in {id(x): x for x in n.inputs}.values():
                    idx.setdefault(id(i), []).append(n)
            self._users = idx
        return list(self._users.get(id(node), ()))

    def text(self) -> str:
        def attr_text(at):
            return ", ".join(f"{k}={_fmt(at[k])}" for k in sorted(at))
        body = [f"{n.name} = {n.op}({', '.join(i.name for i in n.inputs)}) {{{attr_text(n.attrs)}}} : "
                f"{list(n.shape)}" for n in self.nodes]
        return "\n".join(body + ["return " + ", ".join(o.name for o in self.outputs)]) + "\n"

    def evaluate(self, inputs, observe=None, keep_all: bool = True) -> dict:
        """Float64 activations {node name: torch tensor} on batched inputs (a dict by input name, or a sequence in
        input order). `observe(node, tensor)` is called as each value is computed; with keep_all=False a value is
        dropped once its last reader has run (graph outputs are kept), so a calibration pass that only observes
        holds a few activations at a time."""
        import torch

        if not isinstance(inputs, dict):
            inputs = {n.name: x for n, x in zip(self.inputs, inputs, strict=True)}
        last_read = {}
        if not keep_all:
            for pos, n in enumerate(self.nodes):
                for i in n.inputs:
                    last_read[i.name] = pos
            for o in self.outputs:
                last_read[o.name] = len(self.nodes)
        env = {}
        with torch.no_grad():
            for pos, n in enumerate(self.nodes):
                rule = _FLOAT_RULES.get(n.op)
                if rule is None:
                    raise NotImplementedError(f"no float semantics for frontend op {n.op!r}")
                v = rule(n, [env[i.name] for i in n.inputs], inputs)
                env[n.name] = v
                if observe is not None:
                    observe(n, v)
                if not keep_all:
                    for i in {x.name for x in n.inputs}:
                        if last_read.get(i, -1) <= pos:
                            env.pop(i, None)
                    if last_read.get(n.name, -1) < pos:
                        env.pop(n.name, None)
        return env


# ------------------------------------------------------------------------------------- float semantics
# One function per frontend op: (node, operand tensors, graph inputs) -> float64 result, batched on the leading
# dim. These define what the quantized graph approximates (its activations calibrate the scales, and the
# float-path tolerance is measured against them).

def _t64(a):
    import torch
    return None if a is None else torch.as_tensor(a, dtype=torch.float64)


def _f_input(n, a, inputs):
    import torch
    v = torch.as_tensor(inputs[n.name])
    return v.long() if n.attrs.get("ids") else v.to(torch.float64)


def _f_embed(n, a, inputs):
    ids = a[0]
    v = _t64(n.attrs["wte"])[ids]
    pos = n.attrs["wpe"]
    return v if pos is None else v + _t64(pos)[: ids.shape[-1]]


def _f_layernorm(n, a, inputs):
    import torch.nn.functional as F
    x = a[0]
    return F.layer_norm(x, (x.shape[-1],), _t64(n.attrs["weight"]), _t64(n.attrs["bias"]), n.attrs["eps"])


def _f_rmsnorm(n, a, inputs):
    x = a[0]
    v = x * (x.pow(2).mean(dim=-1, keepdim=True) + n.attrs["eps"]).rsqrt()
    w = n.attrs["weight"]
    return v if w is None else v * _t64(w)


def _f_linear(n, a, inputs):
    import torch.nn.functional as F
    w, b, rows = _t64(n.attrs["weight"]), _t64(n.attrs["bias"]), n.attrs["rows"]
    if rows is not None:
        w = w[rows[0]:rows[1]]
        b = None if b is None else b[rows[0]:rows[1]]
    return F.linear(a[0], w, b)


def _f_matmul(n, a, inputs):
    import torch
    v = torch.matmul(a[0], a[1])
    f = n.attrs["factor"]
    if f is None:
        return v
    return v / math.sqrt(f[1]) if f[0] == "inv_sqrt" else v * f[1]


_CAUSAL_BIAS = {}


def _causal_bias(t1, t2):
    """(t1, t2) float64: 0 where row i keeps column j (j <= i), -inf elsewhere (cached per shape)."""
    import torch
    key = (t1, t2)
    if key not in _CAUSAL_BIAS:
        _CAUSAL_BIAS[key] = torch.zeros(t1, t2, dtype=torch.float64).masked_fill(
            torch.ones(t1, t2, dtype=torch.bool).triu(1), float("-inf"))
    return _CAUSAL_BIAS[key]


def _f_softmax(n, a, inputs):
    import torch.nn.functional as F
    x = a[0]
    if n.attrs["causal"]:
        x = x + _causal_bias(x.shape[-2], x.shape[-1])        # adding 0 leaves kept scores exact
    return F.softmax(x, dim=-1)


def _f_gelu(n, a, inputs):
    import torch.nn.functional as F
    return F.gelu(a[0], approximate=n.attrs["approximate"])


def _f_silu(n, a, inputs):
    import torch.nn.functional as F
    return F.silu(a[0])


def _f_transpose(n, a, inputs):
    x, perm = a[0], n.attrs["perm"]
    lead = x.dim() - len(perm)
    return x.permute(*range(lead), *(lead + p for p in perm))


def _f_reshape(n, a, inputs):
    x = a[0]
    lead = x.dim() - len(n.inputs[0].shape)
    return x.reshape(*x.shape[:lead], *n.shape)


def _f_split_heads(n, a, inputs):
    x, nh = a[0], n.attrs["nh"]
    return x.reshape(*x.shape[:-1], nh, x.shape[-1] // nh).transpose(-3, -2)


def _f_merge_heads(n, a, inputs):
    x = a[0].transpose(-3, -2)
    return x.reshape(*x.shape[:-2], x.shape[-2] * x.shape[-1])


_FLOAT_RULES = {
    "input": _f_input, "embed": _f_embed, "layernorm": _f_layernorm, "rmsnorm": _f_rmsnorm,
    "linear": _f_linear, "matmul": _f_matmul, "softmax": _f_softmax, "gelu": _f_gelu, "silu": _f_silu,
    "mul": lambda n, a, inputs: a[0] * a[1], "add": lambda n, a, inputs: a[0] + a[1],
    "transpose": _f_transpose, "reshape": _f_reshape, "split_heads": _f_split_heads,
    "merge_heads": _f_merge_heads,
}


def _fmt(v):
    import numpy as np
    if isinstance(v, np.ndarray):
        return f"array{list(v.shape)}"
    return repr(v)


# ---------------------------------------------------------------------------------------------- capture

@dataclass(eq=False)
class _V:
    """An exported-graph value: a constant tensor, an activation (an FNode, maybe pending a layout pattern), or a
    tuple from split."""
    kind: str                       # "const" | "act" | "tuple"
    value: object = None            # torch tensor (const) / python scalar
    node: FNode | None = None       # act: the FNode it maps to
    shape: tuple = ()               # act: full shape including the batch dim
    pending: tuple | None = None    # act layout pattern in progress: ("heads", nh) / ("merge", nh) / ("tok", W)
    items: list = field(default_factory=list)


class _Capture:
    def __init__(self, ep, batch):
        self.ep, self.batch = ep, batch
        self.nodes, self.names = [], set()
        self.vals = {}

    def fresh(self, base):
        n, i = base, 1
        while n in self.names:
            i += 1
            n = f"{base}_{i}"
        self.names.add(n)
        return n

    def add(self, op, base, inputs, attrs, shape) -> FNode:
        n = FNode(op, self.fresh(base), list(inputs), dict(attrs), tuple(int(d) for d in shape))
        self.nodes.append(n)
        return n

    def act(self, node, full_shape, pending=None):
        return _V("act", node=node, shape=tuple(int(d) for d in full_shape), pending=pending)

    # -------------------------------------------------------------------------------------------------
    def run(self):
        import torch

        ep = self.ep
        sig = ep.graph_signature
        consts = {}
        consts.update({k: ep.state_dict[v] for k, v in sig.inputs_to_parameters.items()})
        consts.update({k: (ep.state_dict[v] if v in ep.state_dict else ep.constants[v])
                       for k, v in sig.inputs_to_buffers.items()})
        consts.update({k: ep.constants[v] for k, v in sig.inputs_to_lifted_tensor_constants.items()})
        user_inputs = list(sig.user_inputs)
        inputs, outputs = [], []
        for fx in ep.graph.nodes:
            if fx.op == "placeholder":
                if fx.name in consts:
                    self.vals[fx] = _V("const", value=consts[fx.name].detach())
                elif fx.name in user_inputs:
                    val = fx.meta["val"]
                    if val.dim() < 1 or val.shape[0] != self.batch:
                        raise UnsupportedOpError(f"input {fx.name}: leading (batch) dim must be {self.batch}")
                    ids = not val.dtype.is_floating_point
                    n = self.add("input", fx.name, [], {"ids": ids}, val.shape[1:])
                    self.vals[fx] = self.act(n, val.shape)
                    inputs.append(n)
                else:
                    raise UnsupportedOpError(f"placeholder {fx.name} is neither a user input nor a constant")
                continue
            if fx.op == "output":
                for a in fx.args[0]:
                    v = self.vals[a]
                    if v.kind != "act":
                        raise UnsupportedOpError("a graph output must depend on the input")
                    outputs.append(self.settle(v))
                continue
            if fx.op != "call_function":
                raise UnsupportedOpError(f"{fx.op} node {fx.name} ({fx.target})")
            args = [self._arg(a) for a in fx.args]
            kwargs = {k: self._arg(a) for k, a in fx.kwargs.items()}
            if all(not isinstance(a, _V) or a.kind == "const" for a in list(args) + list(kwargs.values())):
                self.vals[fx] = self._fold(fx, args, kwargs)          # constant subgraph
                continue
            self.vals[fx] = self.lower(fx, args, kwargs)
        return FGraph(self.nodes, inputs, outputs, self.batch)

    def _arg(self, a):
        import torch.fx
        if isinstance(a, torch.fx.Node):
            return self.vals[a]
        if isinstance(a, (list, tuple)):
            return type(a)(self._arg(x) for x in a)
        return a

    def _fold(self, fx, args, kwargs):
        import torch
        def unwrap(a):
            if isinstance(a, _V):
                return a.value if a.kind == "const" else a.items
            if isinstance(a, (list, tuple)):
                return type(a)(unwrap(x) for x in a)
            return a
        with torch.no_grad():
            out = fx.target(*unwrap(args), **unwrap(kwargs))
        if isinstance(out, (list, tuple)):
            return _V("tuple", items=[_V("const", value=o) for o in out])
        return _V("const", value=out)

    def settle(self, v: _V) -> FNode:
        """The FNode of an activation, closing a pending layout pattern as a plain reshape/transpose."""
        if v.pending is None:
            return v.node
        kind = v.pending[0]
        if kind == "tok":
            return self.add("embed", "embed", [v.node], {"wte": v.pending[1], "wpe": None}, v.shape[1:])
        if kind == "view_heads":                       # a view (B, T, nh, hd) never transposed
            return self.add("reshape", "reshape", [v.node], {}, v.shape[1:])
        if kind == "merge":                            # transposed back (B, T, nh, hd) but not viewed
            return self.add("transpose", "transpose", [v.node], {"perm": [1, 0, 2]}, v.shape[1:])
        raise UnsupportedOpError(f"unfinished layout pattern {kind}")

    def lower(self, fx, args, kw):
        import torch
        a = torch.ops.aten
        t = fx.target
        name = fx.name
        val = fx.meta.get("val")
        shape = tuple(val.shape) if hasattr(val, "shape") else ()
        A = [x for x in args if isinstance(x, _V) and x.kind == "act"]
        if t == a.embedding.default:
            w, ids = args[0], args[1]
            if w.kind != "const" or ids.kind != "act":
                raise UnsupportedOpError("embedding of a non-constant table")
            return _V("act", node=self.settle(ids), shape=shape, pending=("tok", w.value.detach().double().numpy()))
        if t == a.add.Tensor:
            x, y = args[0], args[1]
            if isinstance(x, _V) and x.kind == "act" and x.pending and x.pending[0] == "tok" and \
                    isinstance(y, _V) and y.kind == "const":
                return self.act(self.add("embed", name, [x.node], {"wte": x.pending[1], "wpe": _pos_table(y.value)},
                                         shape[1:]), shape)
            if isinstance(y, _V) and y.kind == "act" and y.pending and y.pending[0] == "tok" and \
                    isinstance(x, _V) and x.kind == "const":
                return self.act(self.add("embed", name, [y.node], {"wte": y.pending[1], "wpe": _pos_table(x.value)},
                                         shape[1:]), shape)
            if len(A) == 2 and len(args) == 2 and kw.get("alpha", 1) == 1:
                return self.act(self.add("add", name, [self.settle(x), self.settle(y)], {}, shape[1:]), shape)
            raise UnsupportedOpError(f"aten.add.Tensor with a constant operand ({name})")
        if t == a.layer_norm.default:
            x = args[0]
            w = args[2] if len(args) > 2 else kw.get("weight")
            b = args[3] if len(args) > 3 else kw.get("bias")
            eps = args[4] if len(args) > 4 else kw.get("eps", 1e-5)
            if len(args[1]) != 1:
                raise UnsupportedOpError("layer_norm over more than the last axis")
            return self.act(self.add("layernorm", name, [self.settle(x)],
                                     {"weight": _np(w), "bias": _np(b), "eps": float(eps)}, shape[1:]), shape)
        if t == getattr(a, "rms_norm", None) and t is not None and t == a.rms_norm.default:
            x, w = args[0], (args[2] if len(args) > 2 else kw.get("weight"))
            eps = args[3] if len(args) > 3 else kw.get("eps")
            return self.act(self.add("rmsnorm", name, [self.settle(x)],
                                     {"weight": _np(w), "eps": float(eps if eps is not None else 1e-6)},
                                     shape[1:]), shape)
        if t == a.linear.default:
            x, w = args[0], args[1]
            b = args[2] if len(args) > 2 else kw.get("bias")
            if w.kind != "const":
                raise UnsupportedOpError("linear with a non-constant weight")
            return self.act(self.add("linear", name, [self.settle(x)],
                                     {"weight": _np(w), "bias": _np(b), "rows": None}, shape[1:]), shape)
        if t in (a.split.Tensor, a.split_with_sizes.default):
            x = args[0]
            dim = args[2] if len(args) > 2 else kw.get("dim", 0)
            if dim not in (-1, len(x.shape) - 1):
                raise UnsupportedOpError("split along an axis other than the last")
            src = self.settle(x)
            if src.op != "linear" or src.attrs["rows"] is not None:
                raise UnsupportedOpError("split of something other than a linear output")
            c = x.shape[-1]
            sizes = [args[1]] * (c // args[1]) if t == a.split.Tensor else list(args[1])
            items, lo = [], 0
            for i, sz in enumerate(sizes):
                n = self.add("linear", f"{src.name}_{i}", list(src.inputs),
                             {"weight": src.attrs["weight"], "bias": src.attrs["bias"], "rows": (lo, lo + sz)},
                             x.shape[1:-1] + (sz,))
                items.append(self.act(n, x.shape[:-1] + (sz,)))
                lo += sz
            if not self._used_elsewhere(src):
                self.nodes.remove(src)
            return _V("tuple", items=items)
        if t == operator.getitem:
            return args[0].items[args[1]]
        if t in (a.view.default, a.reshape.default, a._unsafe_view.default):
            x = args[0]
            new = tuple(int(d) for d in args[1])
            if -1 in new:
                new = tuple(shape)
            if x.pending and x.pending[0] == "merge" and len(new) == len(x.shape) - 1:
                return self.act(self.add("merge_heads", name, [x.node], {"nh": x.pending[1]}, new[1:]), new)
            if x.pending is None and len(new) == len(x.shape) + 1 and new[:-2] == x.shape[:-1] and \
                    new[-2] * new[-1] == x.shape[-1]:
                return _V("act", node=x.node, shape=new, pending=("view_heads", new[-2]))
            return self.act(self.add("reshape", name, [self.settle(x)], {}, new[1:]), new)
        if t in (a.transpose.int, a.permute.default):
            x = args[0]
            r = len(x.shape)
            if t == a.transpose.int:
                d0, d1 = args[1] % r, args[2] % r
                perm = list(range(r))
                perm[d0], perm[d1] = perm[d1], perm[d0]
            else:
                perm = [p % r for p in args[1]]
            if perm[0] != 0:
                raise UnsupportedOpError("transpose of the batch dim")
            if x.pending and x.pending[0] == "view_heads" and perm == [0, 2, 1, 3]:
                nh = x.pending[1]
                return self.act(self.add("split_heads", name, [x.node], {"nh": nh}, shape[1:]), shape)
            if x.pending is None and x.node.op in ("split_heads", "matmul") and r == 4 and perm == [0, 2, 1, 3]:
                return _V("act", node=x.node, shape=shape, pending=("merge", x.shape[1]))
            return self.act(self.add("transpose", name, [self.settle(x)], {"perm": [p - 1 for p in perm[1:]]},
                                     shape[1:]), shape)
        if t in (a.clone.default, a.contiguous.default, a.alias.default, a.dropout.default, a._to_copy.default,
                 a.to.dtype):
            return args[0]
        if t == a.scaled_dot_product_attention.default:
            q, k, v = args[0], args[1], args[2]
            mask = args[3] if len(args) > 3 else kw.get("attn_mask")
            causal = bool(args[5] if len(args) > 5 else kw.get("is_causal", False))
            scale = args[6] if len(args) > 6 else kw.get("scale")
            if mask is not None:
                raise UnsupportedOpError("scaled_dot_product_attention with an explicit mask")
            qn, kn, vn = self.settle(q), self.settle(k), self.settle(v)
            hd = q.shape[-1]
            kt = self.add("transpose", f"{name}_kT", [kn], {"perm": [0, 2, 1]}, kn.shape[:-2] + kn.shape[-1:] + kn.shape[-2:-1])
            factor = ("inv_sqrt", hd) if scale is None else ("mul", float(scale))
            sc = self.add("matmul", f"{name}_scores", [qn, kt], {"factor": factor}, qn.shape[:-1] + (k.shape[-2],))
            p = self.add("softmax", f"{name}_p", [sc], {"causal": causal}, sc.shape)
            o = self.add("matmul", f"{name}_o", [p, vn], {"factor": None}, sc.shape[:-1] + (hd,))
            return self.act(o, shape)
        if t == a.matmul.default:
            x, y = args
            if x.kind != "act" or y.kind != "act":
                raise UnsupportedOpError("matmul with a constant operand (use nn.Linear)")
            return self.act(self.add("matmul", name, [self.settle(x), self.settle(y)], {"factor": None}, shape[1:]),
                            shape)
        if t in (a.mul.Tensor, a.mul.Scalar, a.div.Tensor, a.div.Scalar):
            x, y = args
            if isinstance(y, (int, float)) or (isinstance(y, _V) and y.kind == "const" and y.value.numel() == 1):
                c = float(y if isinstance(y, (int, float)) else y.value.item())
                if t in (a.div.Tensor, a.div.Scalar):
                    c = 1.0 / c
                n = self.settle(x)
                if n.op == "matmul" and len(self.users_of(n)) == 0:
                    f = n.attrs["factor"]
                    base = 1.0 if f is None else (1 / math.sqrt(f[1]) if f[0] == "inv_sqrt" else f[1])
                    n.attrs["factor"] = ("mul", base * c)
                    return self.act(n, shape)
                raise UnsupportedOpError("a scalar multiply of something other than a matmul")
            if len(A) == 2 and t == a.mul.Tensor:
                return self.act(self.add("mul", name, [self.settle(x), self.settle(y)], {}, shape[1:]), shape)
            raise UnsupportedOpError(f"{t} with a tensor constant")
        if t in (a.softmax.int, a._softmax.default):
            x = args[0]
            n = self.settle(x)
            causal = False
            if n.op == "masked_causal":
                causal, n = True, n.inputs[0]
                self.nodes.remove(self._last_masked)
            return self.act(self.add("softmax", name, [n], {"causal": causal}, shape[1:]), shape)
        if t in (a.masked_fill.Scalar, a.where.self):
            if t == a.masked_fill.Scalar:
                x, mask, fill = args[0], args[1], args[2]
            else:
                mask, fill, x = args[0], args[1], args[2]
                mask = _V("const", value=~mask.value) if isinstance(mask, _V) and mask.kind == "const" else mask
                fill = fill.value.item() if isinstance(fill, _V) else fill
            if not (isinstance(mask, _V) and mask.kind == "const" and fill == float("-inf")):
                raise UnsupportedOpError("masked_fill other than a constant causal mask with -inf")
            m = mask.value.bool()
            tt = m.shape[-1]
            if not bool((m.reshape(-1, m.shape[-2], tt)[0] == ~torch.ones(m.shape[-2], tt, dtype=torch.bool).tril()).all()):
                raise UnsupportedOpError("masked_fill with a mask that is not causal")
            n = self.add("masked_causal", name, [self.settle(x)], {}, shape[1:])
            self._last_masked = n
            return self.act(n, shape)
        if t == a.gelu.default:
            approx = kw.get("approximate", args[1] if len(args) > 1 else "none")
            return self.act(self.add("gelu", name, [self.settle(args[0])], {"approximate": approx}, shape[1:]), shape)
        if t == a.silu.default:
            return self.act(self.add("silu", name, [self.settle(args[0])], {}, shape[1:]), shape)
        raise UnsupportedOpError(f"unsupported ATen op {t} ({name})")

    def users_of(self, n):
        return [m for m in self.nodes if any(i is n for i in m.inputs)]

    def _used_elsewhere(self, n):
        return bool(self.users_of(n))


def _np(v):
    if v is None:
        return None
    if isinstance(v, _V):
        if v.kind != "const":
            raise UnsupportedOpError("a parameter that depends on the input")
        v = v.value
    return v.detach().double().numpy()


def _pos_table(v):
    """The positional rows added to a token embedding: the constant (T, C) result of wpe[arange(T)]."""
    arr = v.detach().double().numpy()
    return arr.reshape(arr.shape[-2], arr.shape[-1])


def capture(module, example_inputs) -> FGraph:
    """torch.export the module (eval mode, float64 not required) and match its graph into an FGraph."""
    import torch

    if not isinstance(example_inputs, (list, tuple)):
        example_inputs = (example_inputs,)
    module = module.eval()
    batch = int(example_inputs[0].shape[0])
    with torch.no_grad():
        ep = torch.export.export(module, tuple(example_inputs))
    fg = _Capture(ep, batch).run()
    bad = [n for n in fg.nodes if n.op == "masked_causal"]
    if bad:
        raise UnsupportedOpError("a causal mask not followed by a softmax")
    return fg
