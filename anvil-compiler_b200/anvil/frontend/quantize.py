"""Quantization: FGraph (anvil.frontend.capture) + calibration inputs -> anvil.graph IR.

    q = quantize(fgraph, calib, headroom=1.5)
    q.module, q.consts                        # anvil.graph module + {const sym: int array}
    q.scales, q.bounds                        # {value sym: scale}, overflow proof {op sym: worst |intermediate|}
    q.reference(x_float)                      # float activations keyed by IR sym

Numeric recipe (the reference's, anvil/frontend/quantize.py:276-493, which the scales and constants must match
exactly): symmetric per-tensor scales; a graph input's scale is max |x| / qmax over the raw calibration data;
every other activation's scale is `headroom` x max |a| / qmax of its float value on the fake-quantized
calibration inputs, where scores feeding a causal softmax count only where the mask keeps them; a weight's scale
is max |w| / 127 over the tensor (over the chunk, for a linear split into chunks); every requant (M, s) comes from
fixed_point against the worst case of its integer operands; the LUTs are built by anvil.frontend.numerics; the
finished graph must pass prove_no_overflow.

How this module is organised (its own design): a calibration pass (`ActStats`) observes every float activation
once, as the graph evaluates, and keeps only the max-abs per node; the lowering (`_Lowering`) walks the FGraph
once and hands each node to the rule for its op (`_Lowering.RULES`), which reads the operands' quantized
descriptions (`QVal`: IR value, scale, integer bound, dtype) and returns the node's own.

Extensions for the nanoGPT family (the reference frontend rejects these, anvil/frontend/capture.py:162-173,
476-478):
  * linear bias: bias_q = round(b / (s_in s_w)) as an i32 const added to the accumulator (qlinear's `bias`
    operand); an all-zero quantized bias is dropped, leaving exactly the reference's qlinear.
  * layernorm: layernorm_int = rmsnorm_int on the mean-centred row, with the constants of the reference's wide
    recipe (rmsnorm_lut_wide: eps folded into the sum as ss_init, an eps-free rsqrt LUT, exact at every
    normalisation shift) for entries up to twice the input magnitude; the LayerNorm bias quantized at the output
    scale as an i8 bias.
  * gelu: a 256-entry int8 LUT (the reference's silu_lut recipe with GELU) as a `lut` op; the cuda target fuses
    it into the producing qlinear's epilogue.
  * embed: wte and wpe each quantized per tensor; (Ma, Mb, s) from fixed_point as for a residual add.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from ..ir import graph as g
from .numerics import (HEADROOM, QMAX, RSQRT_LEN, SOFTMAX_ONE, exp_lut, fixed_point, gelu_lut, maxabs_scale,
                       prove_no_overflow, quantize_array, rmsnorm_lut, rmsnorm_lut_wide, silu_lut)

CALIB_CHUNK = 8192


@dataclass
class Quantized:
    module: object                                  # anvil.graph Module with one func
    consts: dict                                    # const sym -> int64 array
    scales: dict                                    # value sym -> scale (None for i32 LUTs / ids)
    bounds: dict                                    # prove_no_overflow result
    graph: object = None                            # the FGraph
    syms: dict = field(default_factory=dict)        # FGraph node name -> IR sym

    def reference(self, *inputs) -> dict:
        """Float activations {IR sym: numpy array} of the captured graph on batched float inputs."""
        acts = self.graph.evaluate(list(inputs))
        return {self.syms[k]: v.detach().numpy() for k, v in acts.items() if k in self.syms}


# ------------------------------------------------------------------------------------------- calibration

class ActStats:
    """Calibration statistics: the scale of every float graph input and max |activation| of every float node.

    Inputs are fake-quantized first (x -> clip(rint(x / s), -qmax - 1, qmax) * s with s = max |x| / qmax, qmax
    of the input's dtype); token-id inputs pass through. The samples are evaluated `chunk` at a time; max-abs
    does not depend on the chunking."""

    def __init__(self, fg, calib_inputs, wide=(), chunk=CALIB_CHUNK):
        import torch

        arrays = list(calib_inputs) if isinstance(calib_inputs, (list, tuple)) else [calib_inputs]
        if len(arrays) != len(fg.inputs):
            raise ValueError(f"{len(arrays)} calibration arrays for {len(fg.inputs)} graph inputs")
        self.input_scale, feeds = {}, []
        for node, arr in zip(fg.inputs, arrays):
            arr = arr.detach().cpu().numpy() if isinstance(arr, torch.Tensor) else np.asarray(arr)
            if tuple(arr.shape[1:]) != tuple(node.shape):
                raise ValueError(f"calibration input {node.name}: shape {arr.shape[1:]} != {node.shape} "
                                 "(plus a batch dim)")
            if node.attrs.get("ids"):
                self.input_scale[node.name] = None
                feeds.append(arr)
                continue
            qmax = QMAX["i16" if node.name in wide else "i8"]
            s = float(np.abs(arr).max()) / qmax
            self.input_scale[node.name] = s
            feeds.append(np.clip(np.rint(arr / s), -qmax - 1, qmax) * s)
        # scores whose consumer is a causal softmax: only the kept (lower-triangle) entries count
        self._masked = {n.name for n in fg.nodes
                        if any(u.op == "softmax" and u.attrs["causal"] for u in fg.users(n))}
        self.maxabs: dict = {}
        for lo in range(0, len(feeds[0]), chunk):
            fg.evaluate([f[lo:lo + chunk] for f in feeds], observe=self._observe, keep_all=False)

    def _observe(self, node, v):
        import torch
        if not v.dtype.is_floating_point:
            return
        a = torch.tril(v) if node.name in self._masked else v
        m = float(a.abs().max())
        self.maxabs[node.name] = max(self.maxabs.get(node.name, 0.0), m)


def residual_nodes(fg, branches=True) -> set:
    """Names of the residual-stream values that residual="i16" widens (anvil/frontend/quantize.py:320-335): a
    float graph input, add or embedding is on the stream when something reads it or it is a graph output, every
    reader is a norm or an add, and it is not a graph input that is also an output; with `branches`, so is a
    linear (not an output) read only by adds on the stream: the attention and MLP branch outputs."""
    outs = {o.name for o in fg.outputs}

    def on_stream(n):
        readers = fg.users(n)
        if n.op not in ("input", "add", "embed") or n.attrs.get("ids"):
            return False
        if n.op == "input" and n.name in outs:
            return False
        return bool(readers or n.name in outs) and all(u.op in ("rmsnorm", "layernorm", "add") for u in readers)

    stream = {n.name for n in fg.nodes if on_stream(n)}
    if branches:
        for n in fg.nodes:
            readers = fg.users(n)
            if n.op == "linear" and n.name not in outs and readers and \
                    all(u.op == "add" and u.name in stream for u in readers):
                stream.add(n.name)
    return stream


# --------------------------------------------------------------------------------------------- lowering

@dataclass
class QVal:
    """A node's quantized value as its readers see it."""
    ir: object                          # the IR value (None: folded into its reader, e.g. a silu gate)
    scale: float | None                 # real value = integer * scale (None: token ids)
    bound: int | None                   # the largest |integer| the value can hold (None: token ids)
    dtype: str = "i8"
    prob: bool = False                  # a softmax result: probabilities times `one`


class _Lowering:
    def __init__(self, fg, stats: ActStats, *, sym, dtype, headroom, softmax_one, rsqrt_len, inline, sym_name):
        self.fg, self.stats, self.sym, self.dtype = fg, stats, sym, dtype
        self.headroom, self.one, self.rsqrt_len, self.inline = headroom, softmax_one, rsqrt_len, inline
        self.b = g.GraphBuilder(sym_name)
        self.consts, self.scales, self.q = {}, {}, {}
        outs = {id(o) for o in fg.outputs}
        # silu(gate) read only by products becomes the LUT of a lut_mul (the SwiGLU gate)
        self.silu_gates = {n.name for n in fg.nodes if n.op == "silu" and id(n) not in outs and fg.users(n)
                           and all(u.op == "mul" for u in fg.users(n))}

    # ---- helpers
    def const(self, name, data, dtype="i8", scale=None):
        data = np.asarray(data, dtype=np.int64)
        if not self.inline:
            self.consts[name] = data
        self.scales[name] = scale
        return self.b.const(name, list(data.shape), dtype, scale, value=data if self.inline else None)

    def out_scale(self, n) -> float:
        return self.headroom * (self.stats.maxabs[n.name] / QMAX[self.dtype[n.name]])

    @staticmethod
    def weight(w):
        s = maxabs_scale(w)
        return quantize_array(w, s), s

    def stored(self, n, ir, scale) -> QVal:
        """The QVal of a node that stores a fresh requantised result in its own dtype."""
        dt = self.dtype[n.name]
        return QVal(ir, scale, QMAX[dt] + 1, dt)

    # ---- rules: (node, operand QVals) -> QVal
    def r_input(self, n, a):
        name = self.sym[n.name]
        if n.attrs.get("ids"):
            return QVal(self.b.input(name, list(n.shape), "i32"), None, None, "i32")
        s = self.stats.input_scale[n.name]
        dt = self.dtype[n.name]
        return QVal(self.b.input(name, list(n.shape), dt, s), s, QMAX[dt] + 1, dt)

    def r_embed(self, n, a):
        name, so = self.sym[n.name], self.out_scale(n)
        tok_q, s_tok = self.weight(n.attrs["wte"])
        pos = n.attrs["wpe"]
        if pos is not None and np.abs(pos).max() > 0:
            pos_q, s_pos = self.weight(pos)
        else:                                           # no positional table: a zero one at the token scale
            pos_q, s_pos = np.zeros((n.shape[0], n.shape[1]), dtype=np.int64), s_tok
        (ma, mb), s = fixed_point([s_tok / so, s_pos / so], [128, 128])
        ir = self.b.embed(name, a[0].ir, self.const(f"{name}.wte", tok_q, "i8", s_tok),
                          self.const(f"{name}.wpe", pos_q, "i8", s_pos), ma, mb, s, so)
        return self.stored(n, ir, so)

    def _norm(self, n, a, center):
        name, so, x = self.sym[n.name], self.out_scale(n), a[0]
        d = n.shape[-1]
        wq, sw = self.weight(n.attrs["weight"] if n.attrs["weight"] is not None else np.ones(d))
        wmax, eps = int(np.abs(wq).max()), n.attrs["eps"]
        if center or x.dtype != "i8":
            # the wide recipe: eps folded into the sum (ss_init), an eps-free LUT, exact at every shift k; a
            # mean-centred row's entries reach twice the input's magnitude. (The eps-in-the-LUT form of an i8
            # rmsnorm adds 4^k eps at shift k, far too much for the small rows of N(0, 0.02) embeddings.)
            lut, s, c, e = rmsnorm_lut_wide(x.scale, sw, so, wmax, d, eps, (2 if center else 1) * x.bound,
                                            self.rsqrt_len)
        else:
            (lut, s), c, e = rmsnorm_lut(x.scale, sw, so, wmax, d, eps, self.rsqrt_len), 0, 0
        w_c = self.const(f"{name}.w", wq, "i8", sw)
        lut_c = self.const(f"{name}.rsqrt_lut", lut, "i32")
        if not center:
            return self.stored(n, self.b.rmsnorm_int(name, x.ir, w_c, lut_c, 1, s, so, ss_shift=c, ss_init=e), so)
        bias = None
        if n.attrs.get("bias") is not None:
            bq = quantize_array(n.attrs["bias"], so)
            bias = self.const(f"{name}.b", bq, "i8", so) if np.any(bq) else None
        return self.stored(n, self.b.layernorm_int(name, x.ir, w_c, lut_c, 1, s, so, ss_shift=c, ss_init=e,
                                                   bias=bias), so)

    def r_rmsnorm(self, n, a):
        return self._norm(n, a, center=False)

    def r_layernorm(self, n, a):
        return self._norm(n, a, center=True)

    def r_linear(self, n, a):
        name, so, x = self.sym[n.name], self.out_scale(n), a[0]
        w, bias_f, rows = n.attrs["weight"], n.attrs["bias"], n.attrs["rows"]
        if rows is not None:                            # one chunk of a split linear, with its own weight scale
            w = w[rows[0]:rows[1]]
            bias_f = None if bias_f is None else bias_f[rows[0]:rows[1]]
        wq, sw = self.weight(w.T)                        # (in, out)
        bias, bmax = None, 0
        if bias_f is not None:
            bq = np.rint(np.asarray(bias_f) / (x.scale * sw)).astype(np.int64)
            if np.any(bq):
                bias, bmax = self.const(f"{name}.b", bq, "i32", x.scale * sw), int(np.abs(bq).max())
        worst = x.bound * int(np.abs(wq).sum(axis=0).max()) + bmax
        (m,), s = fixed_point([x.scale * sw / so], [worst])
        ir = self.b.qlinear(name, x.ir, self.const(f"{name}.w", wq, "i8", sw), m, s, so,
                            dtype=self.dtype[n.name], bias=bias)
        return self.stored(n, ir, so)

    def r_matmul(self, n, a):
        name, so = self.sym[n.name], self.out_scale(n)
        x, y = a
        if x.prob and y.prob:
            raise NotImplementedError(f"{n.name}: product of two softmax outputs")
        # a probability operand carries p * one in its integers: its real scale is 1 / one
        real = (y.scale / self.one if x.prob else x.scale / self.one) if (x.prob or y.prob) else x.scale * y.scale
        f = n.attrs["factor"]
        if f is not None:
            real = real / math.sqrt(f[1]) if f[0] == "inv_sqrt" else real * f[1]
        if real / so <= 0:
            raise NotImplementedError(f"{n.name}: non-positive matmul scale factor")
        (m,), s = fixed_point([real / so], [n.inputs[0].shape[-1] * x.bound * y.bound])
        return self.stored(n, self.b.qmatmul(name, x.ir, y.ir, m, s, so), so)

    def _relayout(self, n, a, ir):
        # same integers, scale and bound; a relaid softmax result is no longer treated as probabilities (its scale
        # 1 / one then enters a product as it is, as the reference's recipe does)
        x = a[0]
        return QVal(ir, x.scale, x.bound, x.dtype)

    def r_transpose(self, n, a):
        return self._relayout(n, a, self.b.transpose(self.sym[n.name], a[0].ir, n.attrs["perm"], a[0].scale))

    def r_reshape(self, n, a):
        return self._relayout(n, a, self.b.reshape(self.sym[n.name], a[0].ir, list(n.shape), a[0].scale))

    def r_split_heads(self, n, a):                       # (.., T, C) -> (.., T, nh, hd) -> (.., nh, T, hd)
        name, x, nh = self.sym[n.name], a[0], n.attrs["nh"]
        src = n.inputs[0].shape
        r = self.b.reshape(f"{name}.r", x.ir, [*src[:-1], nh, src[-1] // nh], x.scale)
        k = len(src) + 1
        return self._relayout(n, a, self.b.transpose(name, r, list(range(k - 3)) + [k - 2, k - 3, k - 1], x.scale))

    def r_merge_heads(self, n, a):                       # (.., nh, T, hd) -> (.., T, nh, hd) -> (.., T, C)
        name, x = self.sym[n.name], a[0]
        k = len(n.inputs[0].shape)
        t = self.b.transpose(f"{name}.t", x.ir, list(range(k - 3)) + [k - 2, k - 3, k - 1], x.scale)
        return self._relayout(n, a, self.b.reshape(name, t, list(n.shape), x.scale))

    def r_softmax(self, n, a):
        name, x = self.sym[n.name], a[0]
        lut = self.const(f"{name}.exp_lut", exp_lut(x.scale, n.shape[-1], self.one), "i32")
        ir = self.b.softmax_lut(name, x.ir, lut, self.one, n.attrs["causal"], 1 / self.one)
        return QVal(ir, 1 / self.one, self.one, "i8", prob=True)

    def _lut_of(self, n, a, table, tag, so):
        name = self.sym[n.name]
        return self.stored(n, self.b.lut(name, a[0].ir, self.const(f"{name}.{tag}", table, "i8", so), so), so)

    def r_gelu(self, n, a):
        so = self.out_scale(n)
        table, _ = gelu_lut(a[0].scale, so, n.attrs.get("approximate", "none"))
        return self._lut_of(n, a, table, "gelu_lut", so)

    def r_silu(self, n, a):
        if n.name in self.silu_gates:                    # becomes the LUT of the lut_mul that reads it
            return QVal(None, a[0].scale, a[0].bound, a[0].dtype)
        so = self.out_scale(n)
        xs = np.arange(-128, 128) * a[0].scale
        return self._lut_of(n, a, quantize_array(xs / (1 + np.exp(-xs)), so), "silu_lut", so)

    def r_mul(self, n, a):
        name, so = self.sym[n.name], self.out_scale(n)
        gate_i = next((i for i, op in enumerate(n.inputs) if op.name in self.silu_gates), None)
        if gate_i is None:
            raise NotImplementedError(f"{n.name}: anvil.graph has no elementwise product of two activations "
                                      "(only silu(a) * b, as lut_mul)")
        gate_node, up = n.inputs[gate_i], a[1 - gate_i]
        pre = self.q[gate_node.inputs[0].name]            # the silu's own input
        table, s_silu = silu_lut(pre.scale)
        (m,), s = fixed_point([s_silu * up.scale / so], [up.bound * int(np.abs(table).max())])
        ir = self.b.lut_mul(name, pre.ir, up.ir, self.const(f"{name}.silu_lut", table, "i8", s_silu), m, s, so)
        return self.stored(n, ir, so)

    def r_add(self, n, a):
        name, so = self.sym[n.name], self.out_scale(n)
        x, y = a
        (ma, mb), s = fixed_point([x.scale / so, y.scale / so], [x.bound, y.bound])
        return self.stored(n, self.b.add_requant(name, x.ir, y.ir, ma, mb, s, so, dtype=self.dtype[n.name]), so)

    RULES = {"input": r_input, "embed": r_embed, "rmsnorm": r_rmsnorm, "layernorm": r_layernorm,
             "linear": r_linear, "matmul": r_matmul, "transpose": r_transpose, "reshape": r_reshape,
             "split_heads": r_split_heads, "merge_heads": r_merge_heads, "softmax": r_softmax, "gelu": r_gelu,
             "silu": r_silu, "mul": r_mul, "add": r_add}

    def run(self) -> Quantized:
        for n in self.fg.nodes:
            rule = self.RULES.get(n.op)
            if rule is None:
                raise NotImplementedError(f"{n.name}: frontend op {n.op}")
            qv = rule(self, n, [self.q[i.name] for i in n.inputs])
            self.q[n.name] = qv
            if qv.ir is not None:
                self.scales[self.sym[n.name]] = qv.scale
        self.b.output(*(self.q[o.name].ir for o in self.fg.outputs))
        module = self.b.module()
        bounds = prove_no_overflow(module, self.consts)
        syms = {k: self.sym[k] for k, v in self.q.items() if v.ir is not None}
        return Quantized(module, self.consts, self.scales, bounds, self.fg, syms)


def quantize(fg, calib_inputs, headroom=HEADROOM, *, names=None, softmax_one=SOFTMAX_ONE, rsqrt_len=RSQRT_LEN,
             inline=False, sym_name="graph", residual="i8", residual_branches=True) -> Quantized:
    """Calibrate `fg` on `calib_inputs` (one array per graph input, leading batch dim) and lower it to anvil.graph.
    `names` renames FGraph nodes to IR syms (default: the node names); residual="i16" stores the residual stream
    (residual_nodes) as i16 at max-abs / 32767."""
    names = dict(names or {})
    unknown = set(names) - {n.name for n in fg.nodes}
    if unknown:
        raise KeyError(f"names for unknown nodes: {sorted(unknown)}")
    sym = {n.name: names.get(n.name, n.name) for n in fg.nodes}
    if len(set(sym.values())) != len(sym):
        raise ValueError("names map two nodes to one sym")
    if residual not in QMAX:
        raise ValueError(f"residual dtype {residual!r} not in {sorted(QMAX)}")
    wide = residual_nodes(fg, residual_branches) if residual != "i8" else set()
    if any(fg.node(w).op == "embed" for w in wide):
        raise NotImplementedError("an i16 residual stream starting at an embedding")
    dtype = {n: ("i16" if n in wide else "i8") for n in sym}
    stats = ActStats(fg, calib_inputs, wide)
    return _Lowering(fg, stats, sym=sym, dtype=dtype, headroom=headroom, softmax_one=softmax_one,
                     rsqrt_len=rsqrt_len, inline=inline, sym_name=sym_name).run()
