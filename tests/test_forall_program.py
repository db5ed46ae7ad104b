"""The body program of the general elementwise forall on the host: the
compiler from an expression DAG, the C oracle that evaluates programs
(checked against numpy float32 arithmetic, op by op, as an independent
restatement), the opcode table against include/spmd_b200.h, and the C entry's
argument checks (which return before any CUDA call)."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT, spmd_mod

fp = spmd_mod("forall_program")


def _np_eval(root, nodes, inputs, consts):
    """Direct numpy float32 evaluation of a DAG (each op rounded on its own)."""
    memo = {}

    def ev(v):
        if v in memo:
            return memo[v]
        n = nodes[v]
        k = n[0]
        with np.errstate(all="ignore"):
            if k == "load":
                r = inputs[n[1]].astype(np.float32)
            elif k == "const":
                r = np.full(inputs[0].shape, consts[n[1]], np.float32)
            elif k == "cmp":
                x, y = ev(n[1]), ev(n[2])
                u = np.isnan(x) | np.isnan(y)
                r = {1: x == y, 2: x > y, 3: x >= y, 4: x < y, 5: x <= y, 6: ~u & (x != y), 7: ~u,
                     8: u | (x == y), 9: u | (x > y), 10: u | (x >= y), 11: u | (x < y), 12: u | (x <= y),
                     13: x != y, 14: u, 15: np.ones_like(u), 0: np.zeros_like(u)}[n[3]].astype(np.float32)
            elif k == "select":
                r = np.where(ev(n[1]) != 0, ev(n[2]), ev(n[3])).astype(np.float32)
            elif k in ("neg", "abs", "sqrt"):
                x = ev(n[1])
                r = {"neg": np.negative, "abs": np.abs, "sqrt": np.sqrt}[k](x).astype(np.float32)
            else:
                x, y = ev(n[1]), ev(n[2])
                if k in ("maximum", "minimum"):
                    nan = np.isnan(x) | np.isnan(y)
                    if k == "maximum":
                        m = np.where(x == y, np.where(np.signbit(x), y, x), np.where(x > y, x, y))
                    else:
                        m = np.where(x == y, np.where(np.signbit(x), x, y), np.where(x < y, x, y))
                    r = np.where(nan, np.float32(np.nan), m).astype(np.float32)
                elif k in ("and", "or", "xor"):
                    a, b = x != 0, y != 0
                    r = {"and": a & b, "or": a | b, "xor": a ^ b}[k].astype(np.float32)
                else:
                    r = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide}[k](x, y)
                    r = r.astype(np.float32)
        memo[v] = r
        return r

    return ev(root)


def random_dag(rs, n_inputs: int, n_ops: int):
    """A random DAG over every opcode; returns (root, nodes, consts)."""
    nodes = {f"x{k}": ("load", k) for k in range(n_inputs)}
    consts = [float(np.float32(c)) for c in rs.uniform(-2, 2, size=3)] + [0.0, -0.0]
    for j in range(len(consts)):
        nodes[f"c{j}"] = ("const", j)
    vals = list(nodes)
    bools = []
    arith = ["add", "sub", "mul", "div", "maximum", "minimum", "neg", "abs", "sqrt"]
    for i in range(n_ops):
        r = rs.random_sample()
        v = f"t{i}"
        if r < 0.15:
            nodes[v] = ("cmp", vals[rs.randint(len(vals))], vals[rs.randint(len(vals))], int(rs.randint(16)))
            bools.append(v)
            continue
        if r < 0.25 and bools:
            nodes[v] = ("select", bools[rs.randint(len(bools))], vals[rs.randint(len(vals))],
                        vals[rs.randint(len(vals))])
        elif r < 0.3 and len(bools) >= 2:
            nodes[v] = (["and", "or", "xor"][rs.randint(3)], bools[rs.randint(len(bools))],
                        bools[rs.randint(len(bools))])
            bools.append(v)
            continue
        else:
            op = arith[rs.randint(len(arith))]
            a = vals[rs.randint(len(vals))]
            nodes[v] = (op, a) if op in fp.UNARY else (op, a, vals[rs.randint(len(vals))])
        vals.append(v)
    # the root: a fold of the last few values, so most of the DAG is live
    root = vals[-1]
    for j, v in enumerate(vals[-4:-1]):
        nodes[f"r{j}"] = ("add", root, v)
        root = f"r{j}"
    if all(nodes[v][0] != "load" for v in _reachable(root, nodes)):
        nodes["rl"] = ("add", root, "x0")
        root = "rl"
    return root, nodes, consts


def _reachable(root, nodes):
    out, todo = set(), [root]
    while todo:
        v = todo.pop()
        if v in out:
            continue
        out.add(v)
        todo.extend(fp._operands(nodes[v]))
    return out


def bits_equal_nan(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit-equal, except that any NaN matches any NaN (payloads are not specified)."""
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and np.array_equal(a.view(np.uint32)[~na], b.view(np.uint32)[~nb]))


def test_opcodes_match_the_header():
    text = (ROOT / "include" / "spmd_b200.h").read_text()
    got = {m.group(1).lower(): int(m.group(2)) for m in re.finditer(r"SPMDB200_MAP_([A-Z]+) = (\d+)", text)}
    assert got == fp.OPS
    for name, val in [("INPUTS", fp.MAX_INPUTS), ("REGS", fp.MAX_REGS), ("INSNS", fp.MAX_INSNS),
                      ("CONSTS", fp.MAX_CONSTS)]:
        assert re.search(rf"#define SPMDB200_MAP_MAX_{name} {val}\b", text)


@pytest.mark.parametrize("seed", range(12))
def test_oracle_runs_compiled_dags_like_numpy(seed, oracle_mod):
    rs = np.random.RandomState(100 + seed)
    n_in = 1 + seed % 4
    root, nodes, consts = random_dag(rs, n_in, 4 + seed)
    code, n_regs, loads, _ = fp.compile_dag(root, nodes)
    assert n_regs <= fp.MAX_REGS and code[-1][0] & 255 == fp.OPS["store"]
    shape = [(37,), (9, 13), (3, 5, 7)][seed % 3]
    ins = [rs.uniform(-3, 3, size=shape).astype(np.float32) for _ in range(n_in)]
    ins[0].reshape(-1)[:3] = [0.0, -0.0, np.inf]
    got = oracle_mod.forall_map(ins, shape, code, consts)
    want = _np_eval(root, nodes, ins, consts)
    assert bits_equal_nan(got, want)


def test_register_reuse_and_copy():
    nodes = {"a": ("load", 0), "b": ("load", 1), "s": ("add", "a", "b"), "m": ("mul", "s", "s"),
             "q": ("sqrt", "m")}
    code, n_regs, _, _ = fp.compile_dag("q", nodes)
    assert n_regs == 2 and len(code) == 6
    code, n_regs, _, _ = fp.compile_dag("a", {"a": ("load", 0)})
    assert code == [fp.insn("load", 0, aux=0), fp.insn("store", 0, 0)] and n_regs == 1


def _map_call(lib, rank=1, sizes=(8,), n_in=1, code=None, n_regs=2, consts=(1.0,)):
    i64 = lambda v: (ctypes.c_int64 * max(len(v), 1))(*v)
    code = code or [fp.insn("load", 0, aux=0), fp.insn("store", 0, 0)]
    words = (ctypes.c_int32 * (2 * len(code)))(*[w for c in code for w in c])
    ptrs = (ctypes.c_void_p * 1)(0x1000)
    cs = (ctypes.c_float * max(len(consts), 1))(*consts)
    return lib.spmdb200_forall_map(rank, i64(sizes), n_in, ptrs, i64([1] * rank * max(n_in, 1)),
                                   ctypes.c_void_p(0x2000), i64([1] * rank), words, len(code), cs, len(consts),
                                   n_regs, None)


@pytest.mark.parametrize("case", ["rank", "opcode", "reg_field", "read_before_write", "store_not_last",
                                  "load_after_op", "bad_input", "no_load", "bad_const", "too_many_regs",
                                  "too_many_insns", "select_cond_unwritten", "bad_predicate", "negative_size"])
def test_forall_map_rejects_bad_programs_before_launch(case):
    lib = spmd_mod("_lib").lib()
    I = fp.insn
    kw = {}
    if case == "rank":
        kw = dict(rank=4, sizes=(1, 1, 1, 1))
    elif case == "opcode":
        kw = dict(code=[I("load", 0, aux=0), (0x11, 0), I("store", 0, 0)])
    elif case == "reg_field":
        kw = dict(code=[I("load", 0, aux=0), I("add", 1, 0, 5), I("store", 0, 1)])
    elif case == "read_before_write":
        kw = dict(code=[I("load", 0, aux=0), I("add", 0, 0, 1), I("store", 0, 0)])
    elif case == "store_not_last":
        kw = dict(code=[I("load", 0, aux=0), I("store", 0, 0), I("neg", 0, 0)])
    elif case == "load_after_op":
        kw = dict(code=[I("load", 0, aux=0), I("neg", 1, 0), I("load", 0, aux=0), I("store", 0, 1)])
    elif case == "bad_input":
        kw = dict(code=[I("load", 0, aux=3), I("store", 0, 0)])
    elif case == "no_load":
        kw = dict(code=[I("const", 0, aux=0), I("store", 0, 0)])
    elif case == "bad_const":
        kw = dict(code=[I("load", 0, aux=0), I("const", 1, aux=4), I("store", 0, 1)])
    elif case == "too_many_regs":
        kw = dict(n_regs=fp.MAX_REGS + 1)
    elif case == "too_many_insns":
        kw = dict(code=[I("load", 0, aux=0)] + [I("neg", 0, 0)] * (fp.MAX_INSNS - 1) + [I("store", 0, 0)])
    elif case == "select_cond_unwritten":
        kw = dict(code=[I("load", 0, aux=0), I("select", 0, 0, 0, aux=1), I("store", 0, 0)])
    elif case == "bad_predicate":
        kw = dict(code=[I("load", 0, aux=0), I("cmp", 1, 0, 0, aux=16), I("store", 0, 1)])
    elif case == "negative_size":
        kw = dict(sizes=(-1,))
    st = _map_call(lib, **kw)
    assert st in (-1, -4), st  # invalid argument / unsupported, before any CUDA call
    assert lib.spmdb200_last_error_message().decode()


def test_compiled_programs_pass_the_library_validator():
    """Every program compile_dag emits satisfies spmdb200_forall_map's checks
    (LOAD prefix, one final STORE, fields in range, registers written before
    they are read).  An empty domain makes the entry validate the program
    and return without any CUDA call."""
    lib = spmd_mod("_lib").lib()
    rs = np.random.RandomState(77)
    for trial in range(200):
        n_in = 1 + trial % 6
        root, nodes, consts = random_dag(rs, n_in, 2 + trial % 15)
        try:
            code, n_regs, _, _ = fp.compile_dag(root, nodes)
        except ValueError:
            continue  # over the register / instruction limits: the shim reports these
        words = (ctypes.c_int32 * (2 * len(code)))(*[w for c in code for w in c])
        i64 = lambda v: (ctypes.c_int64 * max(len(v), 1))(*v)  # noqa: E731
        ptrs = (ctypes.c_void_p * n_in)(*([0x1000] * n_in))
        cs = (ctypes.c_float * len(consts))(*consts)
        st = lib.spmdb200_forall_map(1, i64([0]), n_in, ptrs, i64([1] * n_in), ctypes.c_void_p(0x2000), i64([1]),
                                     words, len(code), cs, len(consts), n_regs, None)
        assert st == 0, (trial, lib.spmdb200_last_error_message().decode())
