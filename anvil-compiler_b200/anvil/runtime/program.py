"""Lower an anvil.graph module to the `cuda` target's launch list (anvil_op records) for one batch size.

This is the cuda target's counterpart of the reference's lowering + codegen + memory plan chain
(anvil/lower/graph_to_tensor.py:409, anvil/codegen/__init__.py:117-214, anvil/memplan.py:190-198), built for a
B200 instead of a 4-thread toy core:

* Values are device buffers with a leading batch dim (the oracle's batch=True semantics,
  anvil/interp/graph.py:43-51); consts carry none and live in one read-only const region, packed once.
* Layout ops (reshape, transpose) are views (shape, element strides, offset) over a root buffer; a kernel that
  needs a contiguous operand gets one through a strided-copy (TRANSPOSE) launch, so most head split / merge
  transposes cost nothing unless someone reads them.
* qmatmul / qlinear become one int8 GEMM launch with the requant epilogue. The right operand is consumed as B^T
  ([.., N, K], K contiguous): a const weight is transposed once when the const region is packed; a
  `transpose(x, swap last two)` operand is read in place; anything else is materialised.
* Fusions (only when keep="outputs", so every fused-away value is unobservable): a `lut` whose input is a GEMM
  result used nowhere else becomes the GEMM's LUT epilogue (bit-identical: qmatmul with lut =
  lut_i8(requant(.)), anvil/semantics.py:95-103); the head-batched qk^T -> softmax_lut -> p@v chain becomes one
  fused attention launch when the shapes allow (hd 64 or 128, T2 <= 1024), its V projection writing V^T
  head-major so the P @ V MMA reads it K-major, and its output landing in the merged-heads layout.
* Activation buffers are placed by anvil.memplan (liveness, 256-byte aligned offsets).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from ..ir import graph as g
from .. import memplan
from . import cuda as C

NP = {"i8": np.int8, "i16": np.int16, "i32": np.int32}
ISZ = {"i8": 1, "i16": 2, "i32": 4}
CONST_ALIGN = 256
SIMT_MAX_WORK = 1 << 21            # GEMMs with M*N*K below this run on the CUDA-core kernel (launch-bound anyway)


def row_major(shape) -> tuple:
    st, acc = [], 1
    for d in reversed(shape):
        st.append(acc)
        acc *= d
    return tuple(reversed(st))


@dataclass
class View:
    """A tensor as (root buffer, shape, element strides, element offset, dtype)."""
    root: str                   # arena buffer name, or const key
    const: bool
    shape: tuple
    strides: tuple
    offset: int
    dtype: str

    @property
    def contiguous(self) -> bool:
        return self.offset == 0 and all(s == r or d == 1 for s, r, d in
                                        zip(self.strides, row_major(self.shape), self.shape))

    @property
    def numel(self) -> int:
        return math.prod(self.shape)

    def permute(self, perm) -> "View":
        return View(self.root, self.const, tuple(self.shape[p] for p in perm),
                    tuple(self.strides[p] for p in perm), self.offset, self.dtype)


def view_reshape(v: "View", new_shape) -> "View | None":
    """v reshaped to new_shape without moving data, or None when the strides do not allow it (numpy's no-copy
    reshape rule: each group of old dims that maps onto a group of new dims must be contiguous within itself)."""
    new_shape = tuple(int(d) for d in new_shape)
    if math.prod(new_shape) != v.numel:
        return None
    old = [(d, s) for d, s in zip(v.shape, v.strides) if d != 1]
    new = [d for d in new_shape if d != 1]
    out, i, j = [], 0, 0
    while i < len(old) or j < len(new):
        if i >= len(old) or j >= len(new):
            return None
        gi, gj = [old[i]], [new[j]]
        po, pn = old[i][0], new[j]
        i += 1
        j += 1
        while po != pn:
            if po < pn:
                if i >= len(old):
                    return None
                gi.append(old[i])
                po *= old[i][0]
                i += 1
            else:
                if j >= len(new):
                    return None
                gj.append(new[j])
                pn *= new[j]
                j += 1
        for (d0, s0), (d1, s1) in zip(gi, gi[1:]):
            if s0 != s1 * d1:
                return None
        st = gi[-1][1]
        strides = []
        for d in reversed(gj):
            strides.append(st)
            st *= d
        out.extend(reversed(strides))
    it = iter(out)
    full = []
    for d in new_shape:
        full.append(next(it) if d != 1 else 0)
    full = tuple(full)
    # size-1 dims: any stride; give them the next dim's extent for a tidy view
    return View(v.root, v.const, new_shape, full, v.offset, v.dtype)


@dataclass
class DevOp:
    """One launch before the arena is planned: buffer slots hold ("act", name) / ("const", offset) / None."""
    kind: int
    slots: list
    fields: dict
    reads: list
    writes: list
    label: str
    work: dict = field(default_factory=dict)      # algorithmic ops / bytes (summary, roofline)


class ConstPool:
    """The const region: host arrays in device layout, 256-byte aligned, deduplicated by key."""

    def __init__(self):
        self.chunks, self.index, self.size = [], {}, 0

    def add(self, key, arr: np.ndarray) -> int:
        if key in self.index:
            return self.index[key]
        arr = np.ascontiguousarray(arr)
        off = -(-self.size // CONST_ALIGN) * CONST_ALIGN
        self.chunks.append((off, arr.view(np.uint8).ravel()))
        self.index[key] = off
        self.size = off + arr.nbytes
        return off

    def blob(self) -> np.ndarray:
        out = np.zeros(max(self.size, 1), dtype=np.uint8)
        for off, b in self.chunks:
            out[off:off + b.size] = b
        return out


@dataclass
class DeviceProgram:
    ops: list                       # [AnvilOp]
    devops: list                    # [DevOp] (labels, work, for summary)
    plan: memplan.MemPlan
    inputs: dict                    # input sym -> (arena offset, shape, dtype)
    outputs: list                   # [(sym or None, View)] graph outputs in order
    views: dict                     # sym -> View of every readable value
    buffers: dict                   # buffer name -> bytes
    batch: int
    keep: str
    fused: list                     # names of fusions applied

    def arena_offset(self, view: View) -> int:
        return self.plan.addresses[view.root]


class LoweringError(NotImplementedError):
    pass


class Lowering:
    def __init__(self, module, consts: dict, pool: ConstPool, batch: int, keep: str = "outputs",
                 checked: bool = False, fuse: bool = True, gemm: str = "auto"):
        self.func = g.func_of(module)
        self.consts = consts
        self.pool = pool
        self.B = int(batch)
        self.keep = keep
        self.checked = checked
        self.fuse = fuse and keep == "outputs"
        self.gemm_mode = gemm
        self.views: dict[int, View] = {}
        self.const_vals: dict[str, np.ndarray] = {}
        self.devops: list[DevOp] = []
        self.bufs: dict[str, int] = {}
        self.inputs: dict[str, str] = {}
        self.nbuf = 0
        self.fused: list[str] = []
        self.skip: set[int] = set()
        self.uses: dict[int, list] = {}
        for op in self.func.ops:
            for v in op.operands:
                self.uses.setdefault(id(v), []).append(op)
        self.out_ids = set()
        for op in self.func.ops:
            if isinstance(op, g.OutputOp):
                self.out_ids |= {id(v) for v in op.values}

    # ------------------------------------------------------------------------------------------ helpers
    def new_buf(self, name_hint: str, nbytes: int) -> str:
        self.nbuf += 1
        name = f"{name_hint}#{self.nbuf}"
        self.bufs[name] = int(nbytes)
        return name

    def new_view(self, hint, shape, dtype) -> View:
        shape = tuple(int(d) for d in shape)
        name = self.new_buf(hint, math.prod(shape) * ISZ[dtype])
        return View(name, False, shape, row_major(shape), 0, dtype)

    def const_array(self, v: View) -> np.ndarray:
        base = self.const_vals[v.root]
        flat = base.ravel()
        itemsz = flat.itemsize
        return np.lib.stride_tricks.as_strided(flat[v.offset:], v.shape, [s * itemsz for s in v.strides]).copy()

    def const_slot(self, v: View, np_dtype, layout="raw") -> tuple:
        arr = self.const_array(v)
        if layout == "T":
            arr = np.swapaxes(arr, -1, -2)
        key = (v.root, v.shape, v.strides, v.offset, layout, np.dtype(np_dtype).str)
        return ("const", self.pool.add(key, np.ascontiguousarray(arr, dtype=np_dtype)))

    def act_slot(self, v: View, elem_off: int = 0) -> tuple:
        return ("act", v.root, (v.offset + elem_off) * ISZ[v.dtype])

    def emit(self, kind, slots, fields, label, reads, writes, work=None):
        self.devops.append(DevOp(kind, slots, fields, [r for r in reads], [w for w in writes], label, work or {}))

    def contig(self, v: View, label: str) -> View:
        """v itself if contiguous, else a TRANSPOSE (strided copy) into a fresh buffer."""
        if v.const:
            raise LoweringError(f"{label}: a constant where the device needs an activation")
        if v.contiguous:
            return v
        out = self.new_view(f"{label}.c", v.shape, v.dtype)
        shape, strides = list(v.shape), list(v.strides)
        # merge dims that are contiguous in both input and output order, to stay within rank 6
        ms, mt = [shape[0]], [strides[0]]
        for d, s in zip(shape[1:], strides[1:]):
            if mt[-1] == s * d:
                ms[-1] *= d
                mt[-1] = s
            else:
                ms.append(d)
                mt.append(s)
        ms2, mt2 = [d for d in ms if d != 1] or [1], [s for d, s in zip(ms, mt) if d != 1] or [1]
        if len(ms2) > 6:
            raise LoweringError(f"{label}: strided copy of rank {len(ms2)} > 6")
        self.emit(C.OP_TRANSPOSE, [self.act_slot(v), self.act_slot(out)],
                  {"dims": [len(ms2)] + ms2, "strides": mt2, "in_bytes": ISZ[v.dtype]}, f"{label}.copy",
                  [v.root], [out.root], {"bytes": 2 * v.numel * ISZ[v.dtype]})
        return out

    def flags(self, extra=0):
        return extra | (C.F_CHECKED if self.checked else 0)

    # ------------------------------------------------------------------------------------------- lowering
    def run(self):
        self.detect_fusions()
        for idx, op in enumerate(self.func.ops):          # consts first: a fused epilogue may need a later table
            if isinstance(op, g.ConstOp):
                self.idx = idx
                self._ConstOp(op)
        for idx, op in enumerate(self.func.ops):
            if idx in self.skip or isinstance(op, g.ConstOp):
                continue
            self.idx = idx
            handler = getattr(self, "_" + type(op).__name__)
            handler(op)
        return self

    def _InputOp(self, op):
        t = g.qt(op.result)
        v = self.new_view(op.sym_str, (self.B,) + tuple(t.dims), t.dtype)
        self.inputs[op.sym_str] = v.root
        self.views[id(op.result)] = v

    def _ConstOp(self, op):
        t = g.qt(op.result)
        arr = op.value if op.value is not None else self.consts.get(op.sym_str)
        if arr is None:
            raise ValueError(f"no value for graph const {op.sym_str!r}")
        arr = np.asarray(arr, dtype=np.int64).reshape(t.dims)
        key = op.sym_str or f"inline#{self.idx}"
        self.const_vals[key] = arr
        self.views[id(op.result)] = View(key, True, tuple(t.dims), row_major(t.dims), 0, t.dtype)

    def _ReshapeOp(self, op):
        x = self.views[id(op.x)]
        t = g.qt(op.result)
        if x.const:
            if not x.contiguous:
                key = f"{x.root}@{self.idx}"
                self.const_vals[key] = self.const_array(x)
                x = View(key, True, x.shape, row_major(x.shape), 0, x.dtype)
            self.views[id(op.result)] = View(x.root, True, tuple(t.dims), row_major(t.dims), x.offset, x.dtype)
            return
        shape = (self.B,) + tuple(t.dims)
        rv = view_reshape(x, shape)
        if rv is None:
            x = self.contig(x, op.sym_str or "reshape")
            rv = View(x.root, False, shape, row_major(shape), x.offset, x.dtype)
        self.views[id(op.result)] = rv

    def _TransposeOp(self, op):
        x = self.views[id(op.x)]
        perm = op.perm_list
        if not x.const:
            perm = [0] + [p + 1 for p in perm]
        self.views[id(op.result)] = x.permute(perm)

    def _OutputOp(self, op):
        pass

    # ---- GEMM
    def _gemm(self, op):
        if id(op) in self.attn:            # the scores matmul: emitted with the p@v matmul, once V exists
            return
        if id(op) in self.attn_o:
            return self._attention(*self.attn_o[id(op)])
        if id(op) in self.qkv:             # one launch for the three projections, at the first of them
            if id(op.result) not in self.views:
                self._qkv_gemm(self.qkv[id(op)])
            return
        a = self.views[id(op.a)]
        b = self.views[id(op.b)]
        t = g.qt(op.result)
        label = op.sym_str or "qmatmul"
        if a.const:
            raise LoweringError(f"{label}: constant left operand")
        a = self.contig(a, f"{label}.a")
        K, N = b.shape[-2], b.shape[-1]
        M = a.shape[-2]
        lut_op = None
        if self.fuse and op.lut is None and t.dtype == "i8" and id(op.result) not in self.out_ids:
            us = self.uses.get(id(op.result), [])
            if len(us) == 1 and isinstance(us[0], g.LutOp) and us[0].x is op.result:
                lut_op = us[0]
        out_val = lut_op.result if lut_op is not None else op.result
        out_label = (lut_op.sym_str or label) if lut_op is not None else label
        flags = self.flags()
        lut_slot = None
        if op.lut is not None or lut_op is not None:
            tv = self.views[id(op.lut if op.lut is not None else lut_op.table)]
            if not tv.const:
                raise LoweringError(f"{label}: LUT is not a constant")
            lut_slot = self.const_slot(tv, np.int8)
            flags |= C.F_LUT
        bias_slot = None
        if op.bias is not None:
            bv = self.views[id(op.bias)]
            if self.checked:
                bias_slot = self.const_slot(bv, np.int32)
            else:                   # proven: fold the bias into the rounding term, bias*M + 2^(s-1)
                folded = self.const_array(bv) * int(op.M) + ((1 << (op.s - 1)) if op.s else 0)
                bias_slot = ("const", self.pool.add((bv.root, "bias_rnd", int(op.M), int(op.s)),
                                                    np.ascontiguousarray(folded, dtype=np.int32)))
                flags |= C.F_BIAS_RND
            flags |= C.F_BIAS
        reads = [a.root]
        if b.const and len(b.shape) == 2:
            bt_slot = self.const_slot(b, np.int8, "T")
            batch, Mt = 1, math.prod(a.shape[:-1])
            a_bs = bt_bs = 0
            outs_shape = a.shape[:-1] + (N,)
            per_sample = [(0, 0)]
        elif b.const:                                  # head-batched const weight: one launch per sample
            bt_slot = self.const_slot(b, np.int8, "T")
            batch, Mt = math.prod(b.shape[:-2]), M
            a_bs, bt_bs = M * K, N * K
            outs_shape = a.shape[:-1] + (N,)
            per_sample = [(s, s) for s in range(self.B)]
        else:
            bt = b.permute(list(range(len(b.shape) - 2)) + [len(b.shape) - 1, len(b.shape) - 2])
            bt = self.contig(bt, f"{label}.bT")
            reads.append(bt.root)
            bt_slot = None
            batch, Mt = math.prod(a.shape[:-2]), M
            a_bs, bt_bs = M * K, N * K
            outs_shape = a.shape[:-1] + (N,)
            per_sample = [(0, 0)]
        # fused residual add: add_requant(other, y) (either order) where y = this GEMM's result used only there
        res_add = None
        if (self.fuse and not self.checked and lut_op is None and id(op) not in self.vt_gemm and batch == 1
                and len(per_sample) == 1 and id(op.result) not in self.out_ids):
            us = self.uses.get(id(op.result), [])
            if len(us) == 1 and isinstance(us[0], g.AddRequantOp) and us[0].a is not us[0].b:
                add = us[0]
                other = add.b if add.a is op.result else add.a
                ov = self.views.get(id(other))
                if ov is not None and not ov.const and ov.contiguous and ov.shape == tuple(outs_shape):
                    res_add = (add, ov, add.a is op.result)
        odtype = t.dtype if res_add is None else g.qt(res_add[0].result).dtype
        out = self.new_view(out_label if res_add is None else (res_add[0].sym_str or out_label), outs_shape, odtype)
        ostrides = [Mt * N, N, 0, 0, 1]
        if id(op) in self.vt_gemm and batch == 1 and len(per_sample) == 1 and lut_slot is None:
            # head-major transposed output for a fused attention's V: element (b, t, c) at b*C*T + c*T + t
            T = self.vt_gemm[id(op)]
            ostrides = [Mt * N, 1, T, N * T, T]
            out = View(out.root, False, out.shape, (N * T, 1, T), 0, out.dtype)
            self.fused.append(f"{label}:vT_epilogue")
        if self.gemm_mode == "simt" or (self.gemm_mode == "auto" and Mt * N * K * batch < SIMT_MAX_WORK):
            flags |= C.F_SIMT
        extra, res_slot = {}, None
        if res_add is not None:
            add, ov, y_is_a = res_add
            flags |= C.F_RESIDUAL
            res_slot = self.act_slot(ov)
            reads = reads + [ov.root]
            extra = {"in_bytes": ISZ[t.dtype], "in2_bytes": ISZ[ov.dtype], "shift2": add.s,
                     "ma": add.Mb if y_is_a else add.Ma, "mb": add.Ma if y_is_a else add.Mb}
            out_label = add.sym_str or out_label
        for s_a, _ in per_sample:
            a_elem = s_a * batch * M * K if len(per_sample) > 1 else 0
            o_elem = s_a * batch * M * N if len(per_sample) > 1 else 0
            slots = [self.act_slot(a, a_elem), bt_slot if bt_slot is not None else self.act_slot(bt),
                     self.act_slot(out, o_elem), lut_slot, bias_slot, res_slot]
            self.emit(C.OP_GEMM, slots,
                      {"dims": [batch, Mt, N, K], "strides": [a_bs, bt_bs] + ostrides[:2] + ostrides[2:],
                       "mult": op.M, "shift": op.s,
                       "out_bytes": ISZ[odtype], "flags": flags, **extra}, out_label, reads, [out.root],
                      {"ops": 2 * batch * Mt * N * K, "bytes": batch * Mt * K + N * K * (batch if bt_bs else 1)
                       + batch * Mt * N * ISZ[odtype]})
        if res_add is not None:
            self.views[id(res_add[0].result)] = out
            self.skip.add(self.func.ops.index(res_add[0]))
            self.fused.append(f"{label}+{res_add[0].sym_str}:residual_epilogue")
        else:
            self.views[id(out_val)] = out
        if lut_op is not None:
            self.skip.add(self.func.ops.index(lut_op))
            self.fused.append(f"{label}+{out_label}:lut_epilogue")

    _QMatmulOp = _gemm
    _QLinearOp = _gemm

    def _qkv_gemm(self, group):
        """q, k, v = x @ Wq, x @ Wk, x @ Wv (each with its own requant and bias) as one GEMM over the concatenated
        weights, reading x once: q and k land side by side in one row-major buffer (row stride 2C, read in place by
        the fused attention), v head-major transposed (the attention's V^T operand)."""
        q, k, v = group
        a = self.contig(self.views[id(q.a)], f"{q.sym_str}.a")
        K, Cw = g.qt(q.b).dims
        Mt = math.prod(a.shape[:-1])
        T = self.vt_gemm[id(v)]
        ws = [self.const_array(self.views[id(o.b)]) for o in group]
        bt = np.ascontiguousarray(np.concatenate([w.T for w in ws]), dtype=np.int8)
        bt_slot = ("const", self.pool.add(("qkv_w",) + tuple(self.views[id(o.b)].root for o in group), bt))
        flags = C.F_SPLIT
        bias_slot = None
        if any(o.bias is not None for o in group):
            parts = []
            for o in group:
                bq = self.const_array(self.views[id(o.bias)]) if o.bias is not None else np.zeros(Cw, np.int64)
                parts.append(bq * int(o.M) + ((1 << (o.s - 1)) if o.s else 0))
            bias_slot = ("const", self.pool.add(("qkv_b",) + tuple(
                (self.views[id(o.bias)].root if o.bias is not None else None, int(o.M), int(o.s)) for o in group),
                np.ascontiguousarray(np.concatenate(parts), dtype=np.int32)))
            flags |= C.F_BIAS | C.F_BIAS_RND
        lead = a.shape[:-1]
        label = "+".join(o.sym_str or "qlinear" for o in group)
        qk = self.new_view(f"{q.sym_str}+{k.sym_str}", lead + (2 * Cw,), "i8")
        vb = self.new_view(v.sym_str or "v", lead + (Cw,), "i8")
        self.emit(C.OP_GEMM, [self.act_slot(a), bt_slot, self.act_slot(qk), None, bias_slot, None,
                              self.act_slot(vb)],
                  {"dims": [1, Mt, 3 * Cw, K, Cw, 2 * Cw, T], "strides": [0, 0, Mt * 2 * Cw, 2 * Cw, 0, 0, 1],
                   "mult": q.M, "shift": q.s, "out_bytes": 1, "flags": flags,
                   "aux": [(int(o.M) << 8) | int(o.s) for o in group]}, label, [a.root], [qk.root, vb.root],
                  {"ops": 2 * Mt * 3 * Cw * K, "bytes": Mt * K + 3 * Cw * K + Mt * 3 * Cw})
        qs = qk.strides[:-1] + (1,)
        self.views[id(q.result)] = View(qk.root, False, lead + (Cw,), qs, 0, "i8")
        self.views[id(k.result)] = View(qk.root, False, lead + (Cw,), qs, Cw, "i8")
        self.views[id(v.result)] = View(vb.root, False, vb.shape, (Cw * T, 1, T), 0, "i8")
        self.fused.append(f"{label}:qkv_split")

    # ---- fused attention
    def _attention(self, sop, pop, oop):
        label = oop.sym_str or "attention"
        q = self.views[id(sop.a)]                       # (B, H, T1, hd)
        kT = self.views[id(sop.b)]                      # (B, H, hd, T2)
        vh = self.views[id(oop.b)]                      # (B, H, T2, hd)
        B, H, T1, hd = q.shape
        T2 = kT.shape[-1]
        k = kT.permute([0, 1, 3, 2])

        def tma_ok(v):
            return v.strides[-1] == 1 and all(st % 16 == 0 for st in v.strides[:-1]) and v.offset % 16 == 0

        if not tma_ok(q):
            q = self.contig(q, f"{label}.q")
        if not tma_ok(k):
            k = self.contig(k, f"{label}.k")
        vt = vh.permute([0, 1, 3, 2])                   # (B, H, hd, T2), must be dense
        if not vt.contiguous:
            vt = self.contig(vt, f"{label}.vT")
        out = self.new_view(label, (B, T1, H * hd), "i8")
        flags = C.F_CAUSAL if pop.causal_bool else 0
        kept = sum(min(i + 1, T2) for i in range(T1)) if pop.causal_bool else T1 * T2
        self.emit(C.OP_ATTENTION,
                  [self.act_slot(q), self.act_slot(k), self.act_slot(vt), self.act_slot(out),
                   self._const(pop.lut, label, np.int32)],
                  {"dims": [B, H, T1, T2, hd],
                   "strides": [q.strides[0], q.strides[1], q.strides[2], k.strides[0], k.strides[1], k.strides[2],
                               T1 * H * hd, H * hd],
                   "mult": sop.M, "shift": sop.s, "mult2": oop.M, "shift2": oop.s, "one": pop.one, "flags": flags},
                  label, [q.root, k.root, vt.root], [out.root], {"ops": 4 * hd * kept * B * H})
        self.views[id(oop.result)] = View(out.root, False, (B, H, T1, hd), (T1 * H * hd, hd, H * hd, 1), 0, "i8")
        self.fused.append(f"{sop.sym_str}+{pop.sym_str}+{label}:attention")

    def detect_fusions(self):
        """Find head-batched qk^T -> softmax_lut -> p@v chains the fused attention kernel can run, and the V
        projections that can write V^T for them."""
        self.attn, self.attn_o, self.vt_gemm, self.qkv = {}, {}, {}, {}
        if not self.fuse or self.checked:
            return
        uses = self.uses
        single = lambda v, op: uses.get(id(v), []) == [op] and id(v) not in self.out_ids  # noqa: E731
        for op in self.func.ops:
            if not isinstance(op, g.SoftmaxLutOp) or g.qt(op.result).dtype != "i8" or op.one > 127:
                continue
            sop = op.x.owner
            if not isinstance(sop, g.QMatmulOp) or sop.lut is not None or g.qt(sop.result).dtype != "i8":
                continue
            if not single(op.x, op):
                continue
            us = uses.get(id(op.result), [])
            if len(us) != 1 or id(op.result) in self.out_ids:
                continue
            oop = us[0]
            if not isinstance(oop, g.QMatmulOp) or oop.a is not op.result or oop.lut is not None or \
                    g.qt(oop.result).dtype != "i8":
                continue
            qd, kd, vd = g.qt(sop.a).dims, g.qt(sop.b).dims, g.qt(oop.b).dims
            if len(qd) != 3 or len(kd) != 3 or len(vd) != 3:
                continue
            H, T1, hd = qd
            T2 = kd[-1]
            if hd not in (64, 128) or T2 > 1024 or T2 % 16 or vd != (H, T2, hd) or kd != (H, hd, T2):
                continue
            self.attn[id(sop)] = (op, oop)
            self.attn_o[id(oop)] = (sop, op, oop)
            self.skip.add(self.func.ops.index(op))
            # V^T straight from the V projection: vh = transpose(reshape(v, [T2, H, hd]), [1, 0, 2])
            tr = oop.b.owner
            if isinstance(tr, g.TransposeOp) and tr.perm_list == [1, 0, 2] and single(oop.b, oop):
                rs = tr.x.owner
                if isinstance(rs, g.ReshapeOp) and single(tr.x, tr) and g.qt(rs.result).dims == (T2, H, hd):
                    vop = rs.x.owner
                    if isinstance(vop, (g.QLinearOp, g.QMatmulOp)) and single(rs.x, rs) and vop.lut is None \
                            and len(g.qt(vop.b).dims) == 2 and g.qt(vop.result).dims == (T2, H * hd) \
                            and g.qt(vop.result).dtype == "i8":
                        self.vt_gemm[id(vop)] = T2
        # the q, k and v projections of one attention, linears of one input, as one split-output GEMM
        for sop, pop, oop in list(self.attn_o.values()):
            group = (self._layout_source(sop.a), self._layout_source(sop.b), self._layout_source(oop.b))
            if self._splittable(group):
                for op in group:
                    self.qkv[id(op)] = group

    @staticmethod
    def _layout_source(v):
        """The op producing value v, looking through reshapes and transposes."""
        op = v.owner
        while isinstance(op, (g.ReshapeOp, g.TransposeOp)):
            op = op.x.owner
        return op

    def _splittable(self, group) -> bool:
        """q, k, v: linears of one input with constant 2-D weights, equal widths that are whole 256-column tiles,
        i8 results that are no graph outputs, v feeding the attention transposed (its V^T epilogue), on the
        tcgen05 path."""
        q, k, v = group
        if len({id(o) for o in group}) != 3 or id(v) not in self.vt_gemm or id(q) in self.vt_gemm or \
                id(k) in self.vt_gemm or self.gemm_mode == "simt":
            return False
        for o in group:
            if not isinstance(o, (g.QLinearOp, g.QMatmulOp)) or o.lut is not None or o.a is not q.a or \
                    not isinstance(o.b.owner, g.ConstOp) or len(g.qt(o.b).dims) != 2 or \
                    g.qt(o.result).dtype != "i8" or id(o.result) in self.out_ids:
                return False
        dims = [g.qt(o.b).dims for o in group]
        K, C = dims[0]
        # the transposed part leaves through 32-row tile stores inside one sequence: T a multiple of 32
        return all(d == (K, C) for d in dims) and C % 256 == 0 and K % 16 == 0 and self.vt_gemm[id(v)] % 32 == 0

    # ---- memory-bound ops
    def _act(self, value, label):
        v = self.views[id(value)]
        return self.contig(v, label)

    def _const(self, value, label, np_dtype):
        v = self.views[id(value)]
        if not v.const:
            raise LoweringError(f"{label}: operand must be a constant on the cuda target")
        return self.const_slot(v, np_dtype)

    def _LutOp(self, op):
        label = op.sym_str or "lut"
        x = self._act(op.x, label)
        out = self.new_view(label, x.shape, "i8")
        self.emit(C.OP_LUT, [self.act_slot(x), self._const(op.table, label, np.int8), self.act_slot(out)],
                  {"dims": [x.numel]}, label, [x.root], [out.root], {"bytes": 2 * x.numel})
        self.views[id(op.result)] = out

    def _LutMulOp(self, op):
        label = op.sym_str or "lut_mul"
        x, y = self._act(op.x, label), self._act(op.y, label)
        out = self.new_view(label, x.shape, "i8")
        self.emit(C.OP_LUT_MUL, [self.act_slot(x), self.act_slot(y), self._const(op.table, label, np.int8),
                                 self.act_slot(out)],
                  {"dims": [x.numel], "mult": op.M, "shift": op.s, "flags": self.flags()}, label,
                  [x.root, y.root], [out.root], {"bytes": 3 * x.numel})
        self.views[id(op.result)] = out

    def _AddRequantOp(self, op):
        label = op.sym_str or "add_requant"
        a, b = self._act(op.a, label), self._act(op.b, label)
        t = g.qt(op.result)
        out = self.new_view(label, a.shape, t.dtype)
        self.emit(C.OP_ADD_REQUANT, [self.act_slot(a), self.act_slot(b), self.act_slot(out)],
                  {"dims": [a.numel], "in_bytes": ISZ[a.dtype], "in2_bytes": ISZ[b.dtype], "out_bytes": ISZ[t.dtype],
                   "ma": op.Ma, "mb": op.Mb, "shift": op.s, "flags": self.flags()}, label, [a.root, b.root],
                  [out.root], {"bytes": a.numel * (ISZ[a.dtype] + ISZ[b.dtype] + ISZ[t.dtype])})
        self.views[id(op.result)] = out

    def _norm(self, op, center):
        label = op.sym_str or ("layernorm_int" if center else "rmsnorm_int")
        x = self._act(op.x, label)
        d = x.shape[-1]
        lutv = self.views[id(op.lut)]
        out = self.new_view(label, x.shape, "i8")
        flags = self.flags(C.F_CENTER if center else 0)
        bias_slot = None
        if center and op.bias is not None:
            bias_slot = self._const(op.bias, label, np.int8)
            flags |= C.F_BIAS
        self.emit(C.OP_NORM, [self.act_slot(x), self._const(op.w, label, np.int8),
                              self._const(op.lut, label, np.int32), self.act_slot(out), bias_slot],
                  {"dims": [x.numel // d, d, lutv.shape[0]], "in_bytes": ISZ[x.dtype], "mult": op.M, "shift": op.s,
                   "ss_shift": op.ss_shift_int, "ss_init": op.ss_init_int, "flags": flags}, label, [x.root],
                  [out.root], {"bytes": x.numel * (ISZ[x.dtype] + 1)})
        self.views[id(op.result)] = out

    def _RmsNormIntOp(self, op):
        self._norm(op, False)

    def _LayerNormIntOp(self, op):
        self._norm(op, True)

    def _SoftmaxLutOp(self, op):
        label = op.sym_str or "softmax_lut"
        x = self._act(op.x, label)
        t = g.qt(op.result)
        t1, t2 = x.shape[-2], x.shape[-1]
        out = self.new_view(label, x.shape, t.dtype)
        self.emit(C.OP_SOFTMAX, [self.act_slot(x), self._const(op.lut, label, np.int32), self.act_slot(out)],
                  {"dims": [x.numel // (t1 * t2), t1, t2], "one": op.one, "out_bytes": ISZ[t.dtype],
                   "flags": self.flags(C.F_CAUSAL if op.causal_bool else 0)}, label, [x.root], [out.root],
                  {"bytes": x.numel * (1 + ISZ[t.dtype])})
        self.views[id(op.result)] = out

    def _EmbedOp(self, op):
        label = op.sym_str or "embed"
        ids = self._act(op.ids, label)
        wte, wpe = self.views[id(op.wte)], self.views[id(op.wpe)]
        T = ids.shape[-1]
        d = wte.shape[1]
        out = self.new_view(label, ids.shape + (d,), "i8")
        self.emit(C.OP_EMBED, [self.act_slot(ids), self._const(op.wte, label, np.int8),
                               self._const(op.wpe, label, np.int8), self.act_slot(out)],
                  {"dims": [ids.numel // T, T, d, wte.shape[0]], "ma": op.Ma, "mb": op.Mb, "shift": op.s,
                   "flags": self.flags()}, label, [ids.root], [out.root], {"bytes": ids.numel * (4 + 3 * d)})
        self.views[id(op.result)] = out


def lower_program(module, consts: dict, pool: ConstPool, batch: int, keep="outputs", checked=False, fuse=True,
                  gemm="auto", guard: int = 0) -> DeviceProgram:
    L = Lowering(module, consts, pool, batch, keep, checked, fuse, gemm)
    L.run()
    func = L.func
    outs = []
    for op in func.ops:
        if isinstance(op, g.OutputOp):
            outs = [(v.owner.sym_str, L.views[id(v)]) for v in op.values]
    views = {}
    for op in func.ops:
        if op.result is not None and op.sym_str is not None and id(op.result) in L.views:
            v = L.views[id(op.result)]
            if not v.const:
                views[op.sym_str] = v
    # liveness over the emitted launches
    defs, uses = {}, {}
    for i, d in enumerate(L.devops):
        for r in d.reads:
            uses.setdefault(r, []).append(i)
        for w in d.writes:
            defs.setdefault(w, i)
    input_bufs = set(L.inputs.values())
    # the graph inputs stay live through the whole chain (never reused), so a device-resident replay of the
    # chain (anvil_model_run_device, graph replays) reads the same inputs every time
    keep_roots = {v.root for _, v in outs if not v.const} | input_bufs
    if keep == "all":
        keep_roots |= {v.root for v in views.values()}
    sizes = {b: n for b, n in L.bufs.items() if b in defs or b in input_bufs}
    for b in list(sizes):
        if b not in defs and b not in input_bufs:
            del sizes[b]
    plan = memplan.plan(len(L.devops), sizes, defs, uses, input_bufs, keep_roots, "outputs",
                        const_bytes=pool.size, guard=guard)
    ops = []
    for i, d in enumerate(L.devops):
        o = C.AnvilOp()
        o.kind = d.kind
        o.op_index = i
        f = d.fields
        o.flags = int(f.get("flags", 0))
        o.in_bytes = int(f.get("in_bytes", 1))
        o.in2_bytes = int(f.get("in2_bytes", 1))
        o.out_bytes = int(f.get("out_bytes", 1))
        for j, v in enumerate(f.get("dims", [])):
            o.dims[j] = int(v)
        for j, v in enumerate(f.get("strides", [])):
            o.strides[j] = int(v)
        for j in range(8):
            o.off[j] = C.LOC_NONE
        for j, s in enumerate(d.slots):
            if s is None:
                continue
            if s[0] == "const":
                o.off[j] = C.LOC_CONST | int(s[1])
            else:
                o.off[j] = plan.addresses[s[1]] + int(s[2])
        for k in ("mult", "shift", "ma", "mb", "one", "ss_shift", "ss_init", "mult2", "shift2"):
            setattr(o, k, int(f.get(k, 0)))
        for j, v in enumerate(f.get("aux", [])):
            o.aux[j] = int(v)
        ops.append(o)
    inputs = {}
    for op in func.ops:
        if isinstance(op, g.InputOp):
            v = L.views[id(op.result)]
            inputs[op.sym_str] = (plan.addresses[v.root], v.shape, v.dtype)
    return DeviceProgram(ops, L.devops, plan, inputs, outs, views, dict(L.bufs), L.B, keep, L.fused)
