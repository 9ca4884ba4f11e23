"""Quantization: FGraph (anvil.frontend.capture) + calibration inputs -> anvil.graph IR.

    q = quantize(fgraph, calib, headroom=1.5)
    q.module, q.consts                        # anvil.graph module + {const sym: int array}
    q.scales, q.bounds                        # {value sym: scale}, overflow proof {op sym: worst |intermediate|}
    q.reference(x_float)                      # float activations keyed by IR sym

The recipe is the reference's (anvil/frontend/quantize.py:1-21, 338-493): symmetric per-tensor int8; input scales
max-abs / 127 over the calibration inputs; every other activation scale `headroom` x max-abs / 127 of its float
value on the fake-quantized calibration inputs (scores only where a causal softmax keeps them); weights max-abs /
127 per tensor (per chunk for a split linear); every requant (M, s) from fixed_point against the worst case over
all int8 inputs; LUTs as the reference builds them; then prove_no_overflow over the finished graph.

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
        import torch
        with torch.no_grad():
            acts = self.graph.evaluate(list(inputs))
        return {self.syms[k]: v.detach().numpy() for k, v in acts.items() if k in self.syms}


def _calibrate(fg, calib_inputs, chunk=CALIB_CHUNK, wide=()):
    """(input scales, {node name: max |float activation|}) on the fake-quantized calibration inputs
    (anvil/frontend/quantize.py:276-300); token-id inputs pass through unquantized."""
    import torch

    if not isinstance(calib_inputs, (list, tuple)):
        calib_inputs = [calib_inputs]
    if len(calib_inputs) != len(fg.inputs):
        raise ValueError(f"{len(calib_inputs)} calibration arrays for {len(fg.inputs)} graph inputs")
    sin, deq = {}, []
    for n, c in zip(fg.inputs, calib_inputs):
        c = c.detach().cpu().numpy() if isinstance(c, torch.Tensor) else np.asarray(c)
        if tuple(c.shape[1:]) != tuple(n.shape):
            raise ValueError(f"calibration input {n.name}: shape {c.shape[1:]} != {n.shape} (plus a batch dim)")
        if n.attrs.get("ids"):
            sin[n.name] = None
            deq.append(c)
            continue
        qmax = QMAX["i16" if n.name in wide else "i8"]
        sin[n.name] = float(np.abs(c).max()) / qmax
        deq.append(np.clip(np.rint(c / sin[n.name]), -qmax - 1, qmax) * sin[n.name])
    amax = {}
    for lo in range(0, len(deq[0]), chunk):
        with torch.no_grad():
            acts = fg.evaluate([d[lo:lo + chunk] for d in deq])
        for k, v in _act_maxabs(fg, acts).items():
            amax[k] = max(amax.get(k, 0.0), v)
    return sin, amax


def _act_maxabs(fg, acts):
    import torch
    out = {}
    for n in fg.nodes:
        v = acts[n.name]
        if not v.dtype.is_floating_point:
            continue
        if any(u.op == "softmax" and u.attrs["causal"] for u in fg.users(n)):
            keep = torch.ones(v.shape[-2], v.shape[-1], dtype=torch.bool).tril()
            v = v.masked_fill(~keep, 0)
        out[n.name] = float(v.abs().max())
    return out


def residual_nodes(fg, branches=True) -> set:
    """Residual-stream node names (anvil/frontend/quantize.py:320-335): inputs and adds feeding only norms / adds,
    plus (with branches) the linears feeding only such adds."""
    outs = {o.name for o in fg.outputs}
    wide = set()
    norms = ("rmsnorm", "layernorm")
    for n in fg.nodes:
        us = fg.users(n)
        if n.op in ("input", "add", "embed") and (us or n.name in outs) and all(u.op in norms + ("add",) for u in us) \
                and (n.op != "input" or n.name not in outs) and not n.attrs.get("ids"):
            wide.add(n.name)
    if branches:
        wide |= {n.name for n in fg.nodes if n.op == "linear" and n.name not in outs and fg.users(n)
                 and all(u.name in wide and u.op == "add" for u in fg.users(n))}
    return wide


def quantize(fg, calib_inputs, headroom=HEADROOM, *, names=None, softmax_one=SOFTMAX_ONE, rsqrt_len=RSQRT_LEN,
             inline=False, sym_name="graph", residual="i8", residual_branches=True) -> Quantized:
    """Calibrate `fg` on `calib_inputs` (one array per graph input, leading batch dim) and lower it to anvil.graph
    (anvil/frontend/quantize.py:338-493 plus the extensions in the module docstring)."""
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
    dt = {n: ("i16" if n in wide else "i8") for n in sym}
    sin, amax = _calibrate(fg, calib_inputs, wide=wide)

    users = {n.name: fg.users(n) for n in fg.nodes}
    fused_silu = {n.name for n in fg.nodes if n.op == "silu" and users[n.name]
                  and all(u.op == "mul" for u in users[n.name]) and n not in fg.outputs}
    b = g.GraphBuilder(sym_name)
    consts, scales, ir, mag, soft = {}, {}, {}, {}, set()

    def const(name, data, dtype="i8", scale=None):
        data = np.asarray(data, dtype=np.int64)
        if not inline:
            consts[name] = data
        scales[name] = scale
        return b.const(name, list(data.shape), dtype, scale, value=data if inline else None)

    def act_scale(n):
        return headroom * (amax[n.name] / QMAX[dt[n.name]])

    def weight(w_io):
        sw = maxabs_scale(w_io)
        return quantize_array(w_io, sw), sw

    for n in fg.nodes:
        s_name = sym[n.name]
        ins = [ir.get(i.name) for i in n.inputs]
        sc_in = [scales.get(sym[i.name]) for i in n.inputs]
        if n.op == "input":
            if n.attrs.get("ids"):
                so = None
                v = b.input(s_name, list(n.shape), "i32")
                mag[n.name] = None
            else:
                so = sin[n.name]
                v = b.input(s_name, list(n.shape), dt[n.name], so)
        elif n.op == "embed":
            so = act_scale(n)
            wte_q, s_te = weight(n.attrs["wte"])
            wpe = n.attrs["wpe"] if n.attrs["wpe"] is not None else np.zeros((n.shape[0], n.shape[1]))
            if np.abs(wpe).max() > 0:
                wpe_q, s_pe = weight(wpe)
            else:
                wpe_q, s_pe = np.zeros(wpe.shape, dtype=np.int64), s_te
            (ma, mb), s = fixed_point([s_te / so, s_pe / so], [128, 128])
            v = b.embed(s_name, ins[0], const(f"{s_name}.wte", wte_q, "i8", s_te),
                        const(f"{s_name}.wpe", wpe_q, "i8", s_pe), ma, mb, s, so)
        elif n.op in ("rmsnorm", "layernorm"):
            so = act_scale(n)
            d = n.shape[-1]
            wf = n.attrs["weight"] if n.attrs["weight"] is not None else np.ones(d)
            wq, sw = weight(wf)
            wmax = int(np.abs(wq).max())
            center = n.op == "layernorm"
            mx = mag[n.inputs[0].name]
            if dt[n.inputs[0].name] == "i8" and not center:
                lut, s = rmsnorm_lut(sc_in[0], sw, so, wmax, d, n.attrs["eps"], rsqrt_len)
                c = e = 0
            elif center:
                # layernorm: eps folded into the sum (ss_init) with an eps-free LUT, exact at every
                # normalisation shift k; the eps-in-the-LUT form adds 4^k eps at shift k, which is large for
                # the small activations of N(0, 0.02)-initialised embeddings (anvil/frontend/quantize.py:122-128)
                lut, s, c, e = rmsnorm_lut_wide(sc_in[0], sw, so, wmax, d, n.attrs["eps"], 2 * mx, rsqrt_len)
            else:
                lut, s, c, e = rmsnorm_lut_wide(sc_in[0], sw, so, wmax, d, n.attrs["eps"], (2 if center else 1) * mx,
                                                rsqrt_len)
            w_c = const(f"{s_name}.w", wq, "i8", sw)
            l_c = const(f"{s_name}.rsqrt_lut", lut, "i32")
            if center:
                bias = None
                if n.attrs.get("bias") is not None:
                    bq = quantize_array(n.attrs["bias"], so)
                    if np.any(bq):
                        bias = const(f"{s_name}.b", bq, "i8", so)
                v = b.layernorm_int(s_name, ins[0], w_c, l_c, 1, s, so, ss_shift=c, ss_init=e, bias=bias)
            else:
                v = b.rmsnorm_int(s_name, ins[0], w_c, l_c, 1, s, so, ss_shift=c, ss_init=e)
        elif n.op == "linear":
            so = act_scale(n)
            w = n.attrs["weight"]
            bias_f = n.attrs["bias"]
            if n.attrs["rows"] is not None:
                lo, hi = n.attrs["rows"]
                w = w[lo:hi]
                bias_f = None if bias_f is None else bias_f[lo:hi]
            wq, sw = weight(w.T)
            bias = None
            bmax = 0
            if bias_f is not None:
                bq = np.rint(np.asarray(bias_f) / (sc_in[0] * sw)).astype(np.int64)
                if np.any(bq):
                    bias = const(f"{s_name}.b", bq, "i32", sc_in[0] * sw)
                    bmax = int(np.abs(bq).max())
            bound = mag[n.inputs[0].name] * int(np.abs(wq).sum(axis=0).max()) + bmax
            (m,), s = fixed_point([sc_in[0] * sw / so], [bound])
            v = b.qlinear(s_name, ins[0], const(f"{s_name}.w", wq, "i8", sw), m, s, so, dtype=dt[n.name], bias=bias)
        elif n.op == "matmul":
            so = act_scale(n)
            a_, b_ = n.inputs
            if a_.name in soft and b_.name in soft:
                raise NotImplementedError(f"{n.name}: product of two softmax outputs")
            if a_.name in soft:
                base = sc_in[1] / softmax_one
            elif b_.name in soft:
                base = sc_in[0] / softmax_one
            else:
                base = sc_in[0] * sc_in[1]
            f = n.attrs["factor"]
            mult = base / so if f is None else (base / math.sqrt(f[1]) / so if f[0] == "inv_sqrt" else base * f[1] / so)
            if mult <= 0:
                raise NotImplementedError(f"{n.name}: non-positive matmul scale factor")
            bound = n.inputs[0].shape[-1] * mag[a_.name] * mag[b_.name]
            (m,), s = fixed_point([mult], [bound])
            v = b.qmatmul(s_name, ins[0], ins[1], m, s, so)
        elif n.op == "transpose":
            so = sc_in[0]
            v = b.transpose(s_name, ins[0], n.attrs["perm"], so)
        elif n.op == "reshape":
            so = sc_in[0]
            v = b.reshape(s_name, ins[0], list(n.shape), so)
        elif n.op == "softmax":
            so = 1 / softmax_one
            lut = exp_lut(sc_in[0], n.shape[-1], softmax_one)
            v = b.softmax_lut(s_name, ins[0], const(f"{s_name}.exp_lut", lut, "i32"), softmax_one, n.attrs["causal"],
                              so)
            soft.add(n.name)
        elif n.op == "gelu":
            so = act_scale(n)
            lut, _ = gelu_lut(sc_in[0], so, n.attrs.get("approximate", "none"))
            v = b.lut(s_name, ins[0], const(f"{s_name}.gelu_lut", lut, "i8", so), so)
        elif n.op == "silu":
            if n.name in fused_silu:
                continue
            so = act_scale(n)
            x = np.arange(-128, 128) * sc_in[0]
            lut = quantize_array(x / (1 + np.exp(-x)), so)
            v = b.lut(s_name, ins[0], const(f"{s_name}.silu_lut", lut, "i8", so), so)
        elif n.op == "mul":
            a_, b_ = n.inputs
            if a_.name in fused_silu:
                gate, up = a_, b_
            elif b_.name in fused_silu:
                gate, up = b_, a_
            else:
                raise NotImplementedError(f"{n.name}: anvil.graph has no elementwise product of two activations "
                                          "(only silu(a) * b, as lut_mul)")
            so = act_scale(n)
            s_gate, s_up = scales[sym[gate.inputs[0].name]], scales[sym[up.name]]
            lut, s_silu = silu_lut(s_gate)
            (m,), s = fixed_point([s_silu * s_up / so], [mag[up.name] * int(np.abs(lut).max())])
            v = b.lut_mul(s_name, ir[gate.inputs[0].name], ir[up.name],
                          const(f"{s_name}.silu_lut", lut, "i8", s_silu), m, s, so)
        elif n.op == "add":
            so = act_scale(n)
            (ma, mb), s = fixed_point([sc_in[0] / so, sc_in[1] / so], [mag[n.inputs[0].name], mag[n.inputs[1].name]])
            v = b.add_requant(s_name, ins[0], ins[1], ma, mb, s, so, dtype=dt[n.name])
        elif n.op == "split_heads":
            so, nh = sc_in[0], n.attrs["nh"]
            r = b.reshape(f"{s_name}.r", ins[0], [*n.inputs[0].shape[:-1], nh, n.inputs[0].shape[-1] // nh], so)
            rank = len(n.inputs[0].shape) + 1
            v = b.transpose(s_name, r, list(range(rank - 3)) + [rank - 2, rank - 3, rank - 1], so)
        elif n.op == "merge_heads":
            so, rank = sc_in[0], len(n.inputs[0].shape)
            tr = b.transpose(f"{s_name}.t", ins[0], list(range(rank - 3)) + [rank - 2, rank - 3, rank - 1], so)
            v = b.reshape(s_name, tr, list(n.shape), so)
        else:
            raise NotImplementedError(f"{n.name}: frontend op {n.op}")
        ir[n.name] = v
        scales[s_name] = so
        if n.op == "input" and n.attrs.get("ids"):
            continue
        mag[n.name] = softmax_one if n.op == "softmax" else (
            mag[n.inputs[0].name] if n.op in ("transpose", "reshape", "split_heads", "merge_heads")
            else QMAX[dt[n.name]] + 1)
    b.output(*(ir[o.name] for o in fg.outputs))
    module = b.module()
    bounds = prove_no_overflow(module, consts)
    syms = {k: v for k, v in sym.items() if k in ir}
    return Quantized(module, consts, scales, bounds, fg, syms)
