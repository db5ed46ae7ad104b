"""End to end on the host: random elementwise forall bodies written as MLIR
text go through the shim's parser and program compiler, the oracle runs the
programs, and numpy evaluates the generator's own op list (independently of
the shim) op by op in float32.  Bit-exact, NaN matching NaN."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import spmd_mod
from test_forall_program import bits_equal_nan

BIN = {"addf": np.add, "subf": np.subtract, "mulf": np.multiply, "divf": np.divide}
PREDS = ["oeq", "ogt", "oge", "olt", "ole", "one", "ord", "ueq", "ugt", "uge", "ult", "ule", "une", "uno"]


def _maximum(x, y, take_max):
    nan = np.isnan(x) | np.isnan(y)
    if take_max:
        m = np.where(x == y, np.where(np.signbit(x), y, x), np.where(x > y, x, y))
    else:
        m = np.where(x == y, np.where(np.signbit(x), x, y), np.where(x < y, x, y))
    return np.where(nan, np.float32(np.nan), m).astype(np.float32)


def _cmp(pred, x, y):
    u = np.isnan(x) | np.isnan(y)
    return {"oeq": x == y, "ogt": x > y, "oge": x >= y, "olt": x < y, "ole": x <= y, "one": ~u & (x != y),
            "ord": ~u, "ueq": u | (x == y), "ugt": u | (x > y), "uge": u | (x >= y), "ult": u | (x < y),
            "ule": u | (x <= y), "une": x != y, "uno": u}[pred]


def random_body(rs, n_in: int, n_ops: int):
    """(MLIR body lines, numpy evaluator) of a random f32 DAG ending in a store to %Out."""
    lines, evals = [], []
    vals = []
    for k in range(n_in):
        lines.append(f"    %x{k} = memref.load %In{k}[%i] : memref<?xf32>")
        vals.append((f"%x{k}", ("in", k)))
    c = float(np.float32(rs.uniform(-2, 2)))
    lines.append(f"    %k0 = arith.constant {c!r} : f32")
    vals.append(("%k0", ("const", np.float32(c))))
    bools = []
    for j in range(n_ops):
        r = rs.random_sample()
        name = f"%t{j}"
        pick = lambda: vals[rs.randint(len(vals))]  # noqa: E731
        if r < 0.45:
            op = list(BIN)[rs.randint(4)]
            a, b = pick(), pick()
            lines.append(f"    {name} = arith.{op} {a[0]}, {b[0]} : f32")
            vals.append((name, (op, a[0], b[0])))
        elif r < 0.6:
            op = ["maximumf", "minimumf"][rs.randint(2)]
            a, b = pick(), pick()
            lines.append(f"    {name} = arith.{op} {a[0]}, {b[0]} : f32")
            vals.append((name, (op, a[0], b[0])))
        elif r < 0.75:
            op = ["arith.negf", "math.absf", "math.sqrt"][rs.randint(3)]
            a = pick()
            lines.append(f"    {name} = {op} {a[0]} : f32")
            vals.append((name, (op, a[0])))
        elif r < 0.88:
            pred = PREDS[rs.randint(len(PREDS))]
            a, b = pick(), pick()
            lines.append(f"    {name} = arith.cmpf {pred}, {a[0]}, {b[0]} : f32")
            bools.append((name, ("cmp", pred, a[0], b[0])))
        elif bools:
            cnd = bools[rs.randint(len(bools))]
            a, b = pick(), pick()
            lines.append(f"    {name} = arith.select {cnd[0]}, {a[0]}, {b[0]} : f32")
            vals.append((name, ("select", cnd[0], a[0], b[0])))
    root = vals[-1][0]
    table0 = dict(vals + bools)

    def loads_something(v, seen=None):
        seen = set() if seen is None else seen
        if v in seen:
            return False
        seen.add(v)
        d = table0[v]
        if d[0] == "in":
            return True
        return any(loads_something(o, seen) for o in d[1:] if isinstance(o, str) and o.startswith("%"))

    if root.startswith("%x") or not loads_something(root):  # compute something, from a load
        lines.append(f"    %tz = arith.addf {root}, %x0 : f32")
        vals.append(("%tz", ("addf", root, "%x0")))
        root = "%tz"
    lines.append(f"    memref.store {root}, %Out[%i] : memref<?xf32>")
    table = dict(vals + bools)

    def evaluate(inputs):
        memo = {}

        def ev(v):
            if v in memo:
                return memo[v]
            d = table[v]
            with np.errstate(all="ignore"):
                if d[0] == "in":
                    r = inputs[d[1]]
                elif d[0] == "const":
                    r = np.full(inputs[0].shape, d[1], np.float32)
                elif d[0] in BIN:
                    r = BIN[d[0]](ev(d[1]), ev(d[2])).astype(np.float32)
                elif d[0] in ("maximumf", "minimumf"):
                    r = _maximum(ev(d[1]), ev(d[2]), d[0] == "maximumf")
                elif d[0] == "arith.negf":
                    r = np.negative(ev(d[1]))
                elif d[0] == "math.absf":
                    r = np.abs(ev(d[1]))
                elif d[0] == "math.sqrt":
                    r = np.sqrt(ev(d[1])).astype(np.float32)
                elif d[0] == "cmp":
                    r = _cmp(d[1], ev(d[2]), ev(d[3]))
                else:  # select
                    r = np.where(ev(d[1]), ev(d[2]), ev(d[3])).astype(np.float32)
            memo[v] = r
            return r

        return ev(root)

    return lines, evaluate


@pytest.mark.parametrize("seed", range(64))
def test_random_mlir_bodies(seed, oracle_mod):
    rs = np.random.RandomState(900 + seed)
    n_in = 1 + seed % 4
    lines, evaluate = random_body(rs, n_in, 3 + seed % 9)
    args = ", ".join([f"%In{k}: memref<?xf32>" for k in range(n_in)] + ["%Out: memref<?xf32>", "%N: index"])
    text = (f"func.func @k({args}) attributes {{spmd.kernel}} {{\n"
            "  %c0 = arith.constant 0 : index\n  %c1 = arith.constant 1 : index\n"
            "  \"spmd.forall\"(%c0, %N, %c1) ({\n  ^bb0(%i: index):\n" + "\n".join(lines) +
            "\n    \"spmd.yield\"() : () -> ()\n  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : "
            "(index, index, index) -> ()\n  func.return\n}\n")
    shim = spmd_mod("mlir_shim")
    (d,) = shim.describe(text)
    assert d["pattern"] in ("map", "ewise", "axpy", "stencil"), d
    ins = [rs.uniform(-3, 3, 257).astype(np.float32) for _ in range(n_in)]
    ins[0][:4] = [0.0, -0.0, np.inf, -np.inf]
    want = evaluate(ins)
    if d["pattern"] != "map":
        pytest.skip(f"mapped to the fixed {d['pattern']} entry (covered by its own tests)")
    views = [ins[int(name[3:])] for name in d["inputs"]]
    consts = [float(c) for c in d["consts"]]
    got = oracle_mod.forall_map(views, (257,), d["code"], consts)
    assert bits_equal_nan(got, want)


@pytest.mark.parametrize("seed", range(24))
def test_random_2d_stencil_bodies(seed, oracle_mod):
    """2-D interior domains whose loads read neighbours at offsets in
    {-1, 0, 1}: each (memref, offset) pair becomes a shifted view."""
    rs = np.random.RandomState(1900 + seed)
    n_in = 1 + seed % 2
    N, M = 23, 37
    offs = [(int(rs.randint(-1, 2)), int(rs.randint(-1, 2))) for _ in range(2 + seed % 3)]
    lines = ["    %im = arith.subi %i, %c1 : index", "    %ip = arith.addi %i, %c1 : index",
             "    %jm = arith.subi %j, %c1 : index", "    %jp = arith.addi %j, %c1 : index"]
    idx = {-1: ("%im", "%jm"), 0: ("%i", "%j"), 1: ("%ip", "%jp")}
    loads = []
    for q, (di, dj) in enumerate(offs):
        k = q % n_in
        lines.append(f"    %l{q} = memref.load %In{k}[{idx[di][0]}, {idx[dj][1]}] : memref<?x?xf32>")
        loads.append((k, di, dj))
    # a non-linear fold: t = max(l0, l1) - l2 ..., alternating ops
    ops = ["arith.maximumf", "arith.subf", "arith.mulf", "arith.minimumf", "arith.addf"]
    acc = "%l0"
    chosen = []
    for q in range(1, len(offs)):
        op = ops[int(rs.randint(len(ops)))]
        lines.append(f"    %a{q} = {op} {acc}, %l{q} : f32")
        chosen.append(op)
        acc = f"%a{q}"
    if len(offs) == 1 or all(o == "arith.addf" for o in chosen):
        lines.append(f"    %sq = arith.mulf {acc}, {acc} : f32")
        chosen.append("square")
        acc = "%sq"
    lines.append(f"    memref.store {acc}, %Out[%i, %j] : memref<?x?xf32>")
    args = ", ".join([f"%In{k}: memref<?x?xf32>" for k in range(n_in)] +
                     ["%Out: memref<?x?xf32>", "%Nm1: index", "%Mm1: index"])
    text = (f"func.func @k({args}) attributes {{spmd.kernel}} {{\n"
            "  %c1 = arith.constant 1 : index\n"
            "  \"spmd.forall\"(%c1, %c1, %Nm1, %Mm1, %c1, %c1) ({\n  ^bb0(%i: index, %j: index):\n" +
            "\n".join(lines) + "\n    \"spmd.yield\"() : () -> ()\n  }) {operandSegmentSizes = array<i32: 2, 2, 2>} : "
            "(index, index, index, index, index, index) -> ()\n  func.return\n}\n")
    shim = spmd_mod("mlir_shim")
    (d,) = shim.describe(text)
    ins = [rs.uniform(-2, 2, (N, M)).astype(np.float32) for _ in range(n_in)]
    sl = lambda k, di, dj: ins[k][1 + di:N - 1 + di, 1 + dj:M - 1 + dj]  # noqa: E731
    vals = [sl(*ld) for ld in loads]
    with np.errstate(all="ignore"):
        acc_v = vals[0]
        for q, op in enumerate(chosen, start=1):
            if op == "square":
                acc_v = (acc_v * acc_v).astype(np.float32)
                continue
            x, y = acc_v, vals[q]
            if op == "arith.maximumf":
                acc_v = _maximum(x, y, True)
            elif op == "arith.minimumf":
                acc_v = _maximum(x, y, False)
            else:
                acc_v = {"arith.subf": np.subtract, "arith.mulf": np.multiply, "arith.addf": np.add}[op](x, y)
                acc_v = acc_v.astype(np.float32)
    if d["pattern"] == "stencil":
        pytest.skip("a linear fold: the promoted-stencil entry (covered by its own tests)")
    assert d["pattern"] == "map", d
    views = [ins[int(name[3:])][1 + o[0]:N - 1 + o[0], 1 + o[1]:M - 1 + o[1]]
             for name, o in zip(d["inputs"], d["input_offsets"])]
    got = oracle_mod.forall_map(views, (N - 2, M - 2), d["code"], [float(c) for c in d["consts"]])
    assert bits_equal_nan(got, acc_v)


@pytest.mark.parametrize("seed", range(16))
def test_random_guarded_and_multi_output_bodies(seed, oracle_mod):
    """`if (a <pred> b) Out[i] = v` (in place, or with an else store) and
    bodies with two outputs, the second reading the first after its store."""
    rs = np.random.RandomState(2900 + seed)
    pred = PREDS[seed % len(PREDS)]
    n = 301
    a = rs.uniform(-2, 2, n).astype(np.float32)
    b = rs.uniform(-2, 2, n).astype(np.float32)
    out0 = rs.uniform(-2, 2, n).astype(np.float32)
    shim = spmd_mod("mlir_shim")
    with_else = bool(seed % 2)
    else_region = ("      %w = arith.subf %a, %b : f32\n      memref.store %w, %Out[%i] : memref<?xf32>\n"
                   if with_else else "")
    text = f"""
func.func @g(%A: memref<?xf32>, %B: memref<?xf32>, %Out: memref<?xf32>, %N: index) attributes {{spmd.kernel}} {{
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({{
  ^bb0(%i: index):
    %a = memref.load %A[%i] : memref<?xf32>
    %b = memref.load %B[%i] : memref<?xf32>
    %c = arith.cmpf {pred}, %a, %b : f32
    %v = arith.mulf %a, %b : f32
    "spmd.if"(%c) ({{
      memref.store %v, %Out[%i] : memref<?xf32>
      "spmd.yield"() : () -> ()
    }}, {{
{else_region}      "spmd.yield"() : () -> ()
    }}) : (i1) -> ()
    "spmd.yield"() : () -> ()
  }}) {{operandSegmentSizes = array<i32: 1, 1, 1>}} : (index, index, index) -> ()
  func.return
}}

func.func @two(%A: memref<?xf32>, %B: memref<?xf32>, %Out: memref<?xf32>, %N: index) attributes {{spmd.kernel}} {{
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({{
  ^bb0(%i: index):
    %a = memref.load %A[%i] : memref<?xf32>
    %s = arith.maximumf %a, %a : f32
    memref.store %s, %B[%i] : memref<?xf32>
    %bb = memref.load %B[%i] : memref<?xf32>
    %q = arith.divf %bb, %a : f32
    memref.store %q, %Out[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }}) {{operandSegmentSizes = array<i32: 1, 1, 1>}} : (index, index, index) -> ()
  func.return
}}
"""
    d = {x["function"]: x for x in shim.describe(text)}
    g = d["g"]
    assert g["pattern"] == "map", g
    env = {"%A": a, "%B": b, "%Out": out0}
    got = oracle_mod.forall_map([env[x] for x in g["inputs"]], (n,), g["code"], [float(c) for c in g["consts"]])
    with np.errstate(all="ignore"):
        cond = _cmp(pred, a, b)
        want = np.where(cond, a * b, (a - b) if with_else else out0).astype(np.float32)
    assert bits_equal_nan(got, want)
    two = d["two"]
    assert two["pattern"] == "maps"
    env = {"%A": a, "%B": b.copy(), "%Out": out0.copy()}
    for m in two["maps"]:
        env[m["output"]] = oracle_mod.forall_map([env[x] for x in m["inputs"]], (n,), m["code"],
                                                 [float(c) for c in m["consts"]])
    with np.errstate(all="ignore"):
        assert bits_equal_nan(env["%B"], a) and bits_equal_nan(env["%Out"], (a / a).astype(np.float32))
