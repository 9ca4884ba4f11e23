"""Generate the golden fixtures in tests/golden/ by EXECUTING the reference's own Python sources.

Run where a checkout of the reference exists, with $ANVIL_REFERENCE naming its directory:

    ANVIL_REFERENCE=<reference checkout> python tests/golden/make_golden.py

The reference's anvil package cannot be imported whole here (it needs xdsl and the missing xf submodule), but two
of its modules run on numpy alone once their imports are satisfied:

  * anvil/semantics.py         imports `xf.golden` for the base ops; it is given the restated base ops of
                               oracle.semantics. Its generalized ops (the i16 paths of requant_dtype,
                               add_requant and rmsnorm_wide, sq_shift, requant_var, lut_i8, qmatmul) then run as
                               the reference wrote them, so their outputs pin oracle.semantics' restatement.
  * anvil/frontend/quantize.py the numeric primitives (fixed_point, rmsnorm_lut, rmsnorm_lut_wide, silu_lut,
                               exp_bits, exp_lut, rsqrt_kmax, ss_shift_for) pin the host constant builders of
                               anvil.frontend.quantize.

It also evaluates the reference's frozen 2-layer model graph (data/codesign/model_graph.json.gz: graph text,
consts, one held-out input) with the reference semantics module above swapped into the oracle interpreter, and
stores every value, so the oracle and the CUDA target are pinned against the reference's code on its own model.
Nothing at test time reads the reference checkout: only the fixtures written here.
"""
from __future__ import annotations

import gzip
import importlib.util
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if not os.environ.get("ANVIL_REFERENCE"):
    sys.exit("make_golden.py: set ANVIL_REFERENCE to the reference checkout's directory")
REF = Path(os.environ["ANVIL_REFERENCE"])
sys.path[:0] = [str(ROOT / "anvil-compiler_b200"), str(ROOT)]

from oracle import semantics as osem  # noqa: E402


def _load(name, path, package=None):
    spec = importlib.util.spec_from_file_location(name, path, submodule_search_locations=None)
    mod = importlib.util.module_from_spec(spec)
    if package:
        mod.__package__ = package
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def reference_modules():
    """(reference semantics module, reference quantize module), executed from the reference sources over the
    restated xf.golden base."""
    golden = types.ModuleType("xf.golden")
    for n in ("I8", "I32", "clamp_i8", "matmul_i8", "requant", "residual_add", "rmsnorm_int", "rsqrt_index",
              "softmax_lut", "swiglu_lut"):
        setattr(golden, n, getattr(osem, n))
    golden.relu = lambda x: np.maximum(np.asarray(x, dtype=np.int64), 0)
    golden._i32 = osem.check_i32
    golden._i8 = osem.check_i8
    xf = types.ModuleType("xf")
    xf.golden = golden
    sys.modules["xf"], sys.modules["xf.golden"] = xf, golden
    pkg = types.ModuleType("refanvil")
    pkg.__path__ = []
    sys.modules["refanvil"] = pkg
    sem = _load("refanvil.semantics", REF / "anvil" / "semantics.py", "refanvil")
    pkg.semantics = sem
    ir = types.ModuleType("refanvil.ir")
    ir.__path__ = []
    ir.graph = types.ModuleType("refanvil.ir.graph")       # quantize() needs the real dialect; the primitives do not
    sys.modules["refanvil.ir"], sys.modules["refanvil.ir.graph"] = ir, ir.graph
    fe = types.ModuleType("refanvil.frontend")
    fe.__path__ = []
    sys.modules["refanvil.frontend"] = fe
    q = _load("refanvil.frontend.quantize", REF / "anvil" / "frontend" / "quantize.py", "refanvil.frontend")
    return sem, q


def _ints(a):
    return np.asarray(a, dtype=np.int64).tolist()


def semantics_cases(sem, rng):
    cases = []
    for _ in range(40):
        acc = rng.integers(-(1 << 22), 1 << 22, 64)
        m, s = int(rng.integers(1, 1 << 8)), int(rng.integers(0, 20))
        cases.append({"fn": "requant_dtype", "args": [_ints(acc), m, s, "i16"],
                      "out": _ints(sem.requant_dtype(acc, m, s, "i16"))})
        a = rng.integers(-(1 << 15), 1 << 15, 64)
        b = rng.integers(-128, 128, 64) if rng.random() < 0.5 else rng.integers(-(1 << 15), 1 << 15, 64)
        ma, mb = int(rng.integers(1, 1 << 15)), int(rng.integers(1, 1 << 15))
        s2 = int(rng.integers(14, 24))
        dt = "i16" if rng.random() < 0.5 else "i8"
        try:
            out = sem.add_requant(a, b, ma, mb, s2, dt)
            cases.append({"fn": "add_requant", "args": [_ints(a), _ints(b), ma, mb, s2, dt], "out": _ints(out)})
        except (OverflowError, ValueError) as e:
            cases.append({"fn": "add_requant", "args": [_ints(a), _ints(b), ma, mb, s2, dt],
                          "raises": type(e).__name__})
        t, d = int(rng.integers(1, 5)), int(rng.integers(4, 40))
        x = rng.integers(-(1 << 15), 1 << 15, (t, d))
        w = rng.integers(-128, 128, d)
        c, e = int(rng.integers(4, 9)), int(rng.integers(0, 64))
        lut = np.round((1 << 15) / np.sqrt(np.arange(1024) + 1)).astype(np.int64)
        s3 = int(rng.integers(0, 12))
        try:
            out = sem.rmsnorm_wide(x, w, lut, 1, s3, c, e, "i16")
            cases.append({"fn": "rmsnorm_wide", "args": [_ints(x), _ints(w), _ints(lut), 1, s3, c, e, "i16"],
                          "out": _ints(out)})
        except (OverflowError, ValueError) as err:
            cases.append({"fn": "rmsnorm_wide", "args": [_ints(x), _ints(w), _ints(lut), 1, s3, c, e, "i16"],
                          "raises": type(err).__name__})
        xs = rng.integers(-(1 << 15), 1 << 15, 32)
        cases.append({"fn": "sq_shift", "args": [_ints(xs), c], "out": _ints(sem.sq_shift(xs, c))})
        a8, b8 = rng.integers(-128, 128, (6, 5)), rng.integers(-128, 128, (5, 7))
        ms, ss = int(rng.integers(1, 300)), int(rng.integers(6, 14))
        cases.append({"fn": "qmatmul", "args": [_ints(a8), _ints(b8), ms, ss, None, "i16"],
                      "out": _ints(sem.qmatmul(a8, b8, ms, ss, None, "i16"))})
        accv = rng.integers(-(1 << 20), 1 << 20, (3, 8))
        sv = rng.integers(4, 14, (3, 1))
        cases.append({"fn": "requant_var", "args": [_ints(accv), 5, _ints(sv)],
                      "out": _ints(sem.requant_var(accv, 5, sv))})
    return cases


def quantize_cases(q, rng):
    cases = []
    for _ in range(60):
        n = int(rng.integers(1, 4))
        ms = [float(v) for v in rng.uniform(1e-6, 2.0, n)]
        bounds = [int(v) for v in rng.integers(1, 1 << 24, n)]
        k = int(rng.integers(0, 4))
        try:
            mi, s = q.fixed_point(ms, bounds, k)
            cases.append({"fn": "fixed_point", "args": [ms, bounds, k], "out": [mi, s]})
        except (ValueError, OverflowError) as e:
            cases.append({"fn": "fixed_point", "args": [ms, bounds, k], "raises": type(e).__name__})
    for t in (8, 16, 64, 1024):
        for sc in (0.01, 0.03, 0.1):
            cases.append({"fn": "exp_lut", "args": [sc, t], "out": _ints(q.exp_lut(sc, t))})
            cases.append({"fn": "exp_bits", "args": [t], "out": int(q.exp_bits(t))})
    for d in (8, 32, 64, 768):
        cases.append({"fn": "rsqrt_kmax", "args": [d], "out": int(q.rsqrt_kmax(d))})
        sx, sw, sh = float(rng.uniform(0.01, 0.05)), float(rng.uniform(0.005, 0.02)), float(rng.uniform(0.01, 0.05))
        wmax = int(rng.integers(64, 128))
        lut, s = q.rmsnorm_lut(sx, sw, sh, wmax, d, 1e-5)
        cases.append({"fn": "rmsnorm_lut", "args": [sx, sw, sh, wmax, d, 1e-5], "out": [_ints(lut), int(s)]})
        sxw = float(rng.uniform(2e-4, 8e-4))
        lut, s, c, e = q.rmsnorm_lut_wide(sxw, sw, sh, wmax, d, 1e-6, 1 << 15)
        cases.append({"fn": "rmsnorm_lut_wide", "args": [sxw, sw, sh, wmax, d, 1e-6, 1 << 15],
                      "out": [_ints(lut), int(s), int(c), int(e)]})
        cases.append({"fn": "ss_shift_for", "args": [d, 1 << 15], "out": int(q.ss_shift_for(d, 1 << 15))})
    for s_in in (0.01, 0.05, 0.2):
        lut, s = q.silu_lut(s_in)
        cases.append({"fn": "silu_lut", "args": [s_in], "out": [_ints(lut), float(s)]})
    return cases


def frozen_model_values(sem):
    """Every value of the reference's frozen model on its stored input, evaluated by the oracle interpreter with
    the reference's own semantics module in place of oracle.semantics."""
    from anvil.ir import parse_ir
    from oracle import interp

    with gzip.open(REF / "data" / "codesign" / "model_graph.json.gz", "rt") as f:
        body = json.load(f)
    module = parse_ir(body["ir"])
    consts = {k: np.asarray(v, dtype=np.int64).reshape(body["shapes"][k]) for k, v in body["consts"].items()}
    x = np.asarray(body["x"], dtype=np.int64)
    saved = interp.sem
    proxy = types.SimpleNamespace(**{n: getattr(osem, n) for n in dir(osem) if not n.startswith("__")})
    for n in ("qmatmul", "lut_i8", "swiglu_lut", "rmsnorm_wide", "softmax_lut", "add_requant", "check_dtype"):
        setattr(proxy, n, getattr(sem, n))
    base_qmatmul = sem.qmatmul
    proxy.qmatmul = lambda a, b, m, s, lut=None, dtype="i8", bias=None: base_qmatmul(a, b, m, s, lut, dtype)
    interp.sem = proxy
    try:
        vals = interp.run(module, {"x": x}, consts).values
    finally:
        interp.sem = saved
    return {"ir": body["ir"], "consts": body["consts"], "shapes": body["shapes"], "x": body["x"],
            "values": {k: _ints(v) for k, v in vals.items()}}


def write(name, obj):
    with gzip.open(HERE / name, "wt") as f:
        json.dump(obj, f, sort_keys=True, separators=(",", ":"))
    print("wrote", HERE / name)


def main():
    sem, q = reference_modules()
    rng = np.random.default_rng(20261201)
    write("reference_semantics.json.gz", {"source": "anvil/semantics.py (reference), base ops restated",
                                          "cases": semantics_cases(sem, rng)})
    write("reference_quantize.json.gz", {"source": "anvil/frontend/quantize.py (reference) primitives",
                                         "cases": quantize_cases(q, rng)})
    write("frozen_model.json.gz", {"source": "data/codesign/model_graph.json.gz (reference), values by the "
                                   "reference semantics module", **frozen_model_values(sem)})
    with gzip.open(REF / "data" / "cost" / "model_graph.json.gz", "rt") as f:
        body = json.load(f)
    write("frozen_model_i8.json.gz", {"source": "data/cost/model_graph.json.gz (reference), no stored input",
                                      "ir": body["ir"], "consts": body["consts"], "shapes": body["shapes"]})


if __name__ == "__main__":
    main()
