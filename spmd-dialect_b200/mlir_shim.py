"""Textual-MLIR shim: maps `spmd.kernel` functions written with `spmd.forall` /
`spmd.reduce` onto this library's C entries, so code (and orchestration)
written against the dialect runs here without MLIR, LLVM or a PTX toolchain.

It reads the generic operation form the dialect's tests use
("spmd.forall"(lbs, ubs, steps) ({ ^bb0(ivs): ... }) {attrs}), evaluates the
index arithmetic symbolically, and recognises the lowered shapes of the hot
path:

* elementwise foralls: C[i] = A[i] + B[i] (the ewise kernel,
  test/SPMD/lower-to-gpu-nvptx.mlir:54-71) and Y[i] = a * X[i] + Y[i];
* linear stencils: B[p] = s * (w0 A[p + o0] + w1 A[p + o1] + ...) in source
  order (a left fold of arith.addf), any rank 1-3, with the group forall's
  `spmd.tile_sizes`, the lane step and `spmd.memory_policy` handed to the
  promotion plan (lib/Analysis/PromotionPlanAnalysis.cpp:53-164) -- e.g. the
  promoted 3-point stencil (test/SPMD/lower-to-gpu-nvptx-promoted.mlir:32-67);
* any other per-point body -- a DAG of arith / math f32 ops over loads at the
  store's index plus constant offsets, f32 constants and scalar arguments,
  `spmd.if` values and guarded stores, several stores per point -- as the
  straight-line programs of the general forall entry (spmdb200_forall_map);
* reductions: an `spmd.reduce` (any kind, include/spmd/IR/SPMDAttrs.td:74-80)
  of one memref, combined into a rank-0 memref with memref.atomic_rmw of the
  same kind (the hierarchical sum, SPMDToGPU.cpp:249-415) or one atomic per
  element (the atomic baseline), and a top-level `spmd.reduce` whose value
  the function returns or stores.

`load(text)` returns callables taking the function's own arguments (CUDA
tensors for memrefs, ints for index, floats for f32).  The command line adds
stand-ins for the two build steps of the reference's differential script
(scripts/run-differential.sh:108-140 `_compile_so`, scripts/gen-ptx.sh):

    python mlir_shim.py describe kernels.mlir
    python mlir_shim.py so  kernels.mlir scf|omp out.so     # host entries (ewise, stencil_cpu, ...)
    python mlir_shim.py ptx kernels.mlir ewise|promoted|hierarchical out.ptx [sm]

`so` and `ptx` check that every kernel in the file has an entry of the same
name and calling convention in this library, then write the library (or the
kernel module, loadable by cuModuleLoadData like PTX) to the output path;
anything the shim does not recognise is reported, not guessed.
"""
from __future__ import annotations

import json
import re
import shutil
import struct
import sys
from dataclasses import dataclass, field
from pathlib import Path

HERE = Path(__file__).resolve().parent

if __package__:
    from . import forall_program as _fp
else:  # run as a script from its own directory
    import forall_program as _fp


class ShimError(ValueError):
    """The MLIR text uses a form or pattern the shim does not map."""


# ----------------------------------------------------------------------------- parsing
@dataclass
class Op:
    name: str                  # e.g. "arith.addf", "spmd.forall"
    result: str | None
    operands: list
    attrs: str = ""            # raw attribute text
    extra: str = ""            # predicate / reduction kind / memref index list
    region: list = field(default_factory=list)
    block_args: list = field(default_factory=list)
    type: str = ""
    more_regions: list = field(default_factory=list)  # regions after the first (spmd.if's else)


@dataclass
class Arg:
    name: str
    kind: str                  # "memref", "index", "f32", "i32"
    rank: int = 0
    elem: str = ""


@dataclass
class Func:
    name: str
    args: list
    ops: list
    kernel: bool


_REGION_OP = re.compile(r'(?:(%[\w.#]+)\s*=\s*)?"(spmd\.\w+)"\(([^)]*)\)\s*\(\{')
_SIG = re.compile(r'\s*:\s*\(([^)]*)\)\s*->\s*(\(\)|[^\s,}]+)')
_FUNC = re.compile(r'func\.func\s+(?:private\s+)?@([\w.]+)\s*\(([^)]*)\)\s*(?:->\s*[^{]*?)?\s*(attributes\s*\{[^}]*\})?\s*\{')


def _strip_comments(text: str) -> str:
    return "\n".join(line.split("//", 1)[0] for line in text.splitlines())


def _match_brace(s: str, i: int) -> int:
    """Index of the brace closing the one at s[i]."""
    depth = 0
    for j in range(i, len(s)):
        if s[j] == "{":
            depth += 1
        elif s[j] == "}":
            depth -= 1
            if depth == 0:
                return j
    raise ShimError("unbalanced braces")


def _vals(s: str) -> list:
    """Comma-separated items of s, splitting only outside <>, (), [] and {}
    (a memref type such as memref<?xf32, #spmd.addr_space<global>> is one item)."""
    out, depth, cur = [], 0, []
    for ch in s:
        if ch in "<([{":
            depth += 1
        elif ch in ">)]}":
            depth -= 1
        if ch == "," and depth == 0:
            out.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    out.append("".join(cur))
    return [v.strip() for v in out if v.strip()]


def _const_value(text: str, typ: str):
    """An arith.constant literal: decimal, or a hexadecimal bit pattern (MLIR
    prints f32 infinities and NaNs as 0x7F800000-style literals)."""
    text = text.strip()
    if typ in ("f32", "f64"):
        if text.lower().startswith("0x"):
            bits = int(text, 16)
            fmt, width = ("<f", 4) if typ == "f32" else ("<d", 8)
            return struct.unpack(fmt, bits.to_bytes(width, "little"))[0]
        return float(text)
    if text in ("true", "false"):
        return int(text == "true")
    v = int(text, 16) if text.lower().startswith("0x") else int(text)
    if typ == "i32" and v >= 2 ** 31:
        v -= 2 ** 32  # a hexadecimal i32 literal is a bit pattern
    return v


def _parse_simple(line: str) -> Op:
    m = re.match(r'(?:(%[\w.#]+)\s*=\s*)?([\w.]+|"[\w.]+")\s*(.*)$', line)
    if not m:
        return Op("unknown", None, [], extra=line)
    res, name, rest = m.group(1), m.group(2).strip('"'), m.group(3)
    if name == "arith.constant":
        v, t = rest.rsplit(":", 1)
        return Op(name, res, [], extra=v.strip(), type=t.strip())
    if name in ("arith.cmpi", "arith.cmpf"):
        pred, rest2 = rest.split(",", 1)
        ops, t = rest2.rsplit(":", 1)
        return Op(name, res, _vals(ops), extra=pred.strip(), type=t.strip())
    if name == "memref.load":
        mm = re.match(r'(%[\w.#]+)\[([^\]]*)\]\s*:\s*(.*)$', rest)
        return Op(name, res, [mm.group(1)], extra=mm.group(2), type=mm.group(3).strip())
    if name == "memref.store":
        mm = re.match(r'(%[\w.#]+)\s*,\s*(%[\w.#]+)\[([^\]]*)\]\s*:\s*(.*)$', rest)
        return Op(name, None, [mm.group(1), mm.group(2)], extra=mm.group(3), type=mm.group(4).strip())
    if name == "memref.atomic_rmw":
        mm = re.match(r'(\w+)\s+(%[\w.#]+)\s*,\s*(%[\w.#]+)\[([^\]]*)\]', rest)
        return Op(name, res, [mm.group(2), mm.group(3)], extra=mm.group(1), attrs=mm.group(4))
    if name in ("spmd.yield", "spmd.barrier"):
        mm = re.match(r'\(([^)]*)\)', rest)
        return Op(name, None, _vals(mm.group(1)) if mm else [])
    if name in ("func.return", "return"):
        return Op("func.return", None, _vals(rest.split(":", 1)[0]))
    if name.startswith("arith.") or name.startswith("math."):
        ops, t = rest.rsplit(":", 1)
        return Op(name, res, _vals(ops), type=t.strip())
    return Op("unknown", res, [], extra=line)


def _parse_ops(s: str) -> list:
    ops, pos = [], 0
    while pos < len(s):
        while pos < len(s) and s[pos].isspace():
            pos += 1
        if pos >= len(s):
            break
        m = _REGION_OP.match(s, pos)
        if m:
            brace = m.end() - 1
            close = _match_brace(s, brace)
            inner = s[brace + 1:close]
            bb = re.match(r'\s*\^bb\d+\(([^)]*)\)\s*:', inner)
            block_args = [a.split(":")[0].strip() for a in _vals(bb.group(1))] if bb else []
            region = _parse_ops(inner[bb.end():] if bb else inner)
            pos = close + 1
            more = []  # further regions: spmd.if carries a then and an else region
            while True:
                while s[pos].isspace():
                    pos += 1
                if s[pos] != ",":
                    break
                pos += 1
                while s[pos].isspace():
                    pos += 1
                if s[pos] != "{":
                    raise ShimError(f"{m.group(2)}: expected a region after ','")
                close = _match_brace(s, pos)
                more.append(_parse_ops(s[pos + 1:close]))
                pos = close + 1
            if s[pos] != ")":
                raise ShimError(f"{m.group(2)}: expected ')' after its region")
            pos += 1
            while pos < len(s) and s[pos].isspace():
                pos += 1
            attrs = ""
            if pos < len(s) and s[pos] == "{":
                aend = _match_brace(s, pos)
                attrs = s[pos + 1:aend]
                pos = aend + 1
            sig = _SIG.match(s, pos)
            if sig:
                pos = sig.end()
            ops.append(Op(m.group(2), m.group(1), _vals(m.group(3)), attrs=attrs, region=region,
                          block_args=block_args, more_regions=more))
            continue
        eol = s.find("\n", pos)
        eol = len(s) if eol < 0 else eol
        line = s[pos:eol].strip()
        pos = eol + 1
        if line:
            ops.append(_parse_simple(line))
    return ops


def _parse_arg(a: str) -> Arg:
    name, t = [x.strip() for x in a.split(":", 1)]
    mm = re.match(r'memref<(.*)>$', t)
    if mm:
        dims = mm.group(1).split("x")
        elem = dims[-1].split(",")[0].strip()
        return Arg(name, "memref", len(dims) - 1, elem)
    return Arg(name, t if t in ("index", "f32", "i32") else t)


def parse_module(text: str) -> list:
    """Every func.func of the module (kernels marked by `spmd.kernel`)."""
    text = _strip_comments(text)
    funcs = []
    for m in _FUNC.finditer(text):
        start = m.end() - 1
        body = text[start + 1:_match_brace(text, start)]
        args = [_parse_arg(a) for a in _vals(m.group(2))]
        funcs.append(Func(m.group(1), args, _parse_ops(body), bool(m.group(3) and "spmd.kernel" in m.group(3))))
    return funcs


# ----------------------------------------------------------------------------- analysis
class _Aff:
    """An index value: sum of coeff * symbol + const (symbols: ivs and index args)."""

    def __init__(self, terms=None, const=0):
        self.terms = dict(terms or {})
        self.const = const

    def __add__(self, o):
        t = dict(self.terms)
        for k, v in o.terms.items():
            t[k] = t.get(k, 0) + v
        return _Aff({k: v for k, v in t.items() if v}, self.const + o.const)

    def __sub__(self, o):
        return self + o.scale(-1)

    def scale(self, c):
        return _Aff({k: v * c for k, v in self.terms.items()}, self.const * c)


def _attr_ints(attrs: str, key: str) -> list | None:
    m = re.search(r'"?' + re.escape(key) + r'"?\s*=\s*array<i64:\s*([^>]*)>', attrs)
    return [int(x) for x in _vals(m.group(1))] if m else None


def _attr_enum(attrs: str, key: str) -> str | None:
    m = re.search(r'"?' + re.escape(key) + r'"?\s*=\s*#spmd\.\w+<(\w+)>', attrs)
    return m.group(1) if m else None


def _segments(op: Op) -> tuple:
    seg = re.search(r'operandSegmentSizes\s*=\s*array<i32:\s*([^>]*)>', op.attrs)
    if seg:
        n = [int(x) for x in _vals(seg.group(1))]
    else:
        r = len(op.operands) // 3
        n = [r, r, r]
    o = op.operands
    return o[:n[0]], o[n[0]:n[0] + n[1]], o[n[0] + n[1]:n[0] + n[1] + n[2]]


@dataclass
class Mapping:
    """How one spmd.kernel function maps onto the library."""
    name: str
    pattern: str               # "ewise" | "axpy" | "stencil" | "reduce"
    entry: str                 # C entry called
    detail: dict

    def to_json(self) -> dict:
        return {"function": self.name, "pattern": self.pattern, "entry": self.entry, **self.detail}


class _Env:
    def __init__(self, func: Func):
        self.func = func
        self.idx: dict = {}      # ssa -> _Aff
        self.consts: dict = {}   # ssa -> python number
        self.defs: dict = {}     # ssa -> Op
        for a in func.args:
            if a.kind == "index":
                self.idx[a.name] = _Aff({a.name: 1})

    def index(self, v: str) -> _Aff:
        if v in self.idx:
            return self.idx[v]
        raise ShimError(f"{self.func.name}: index value {v} is not an affine function of the loop indices")

    def visit(self, op: Op) -> None:
        if op.result:
            self.defs[op.result] = op
        if op.name == "arith.constant":
            val = _const_value(op.extra, op.type)
            self.consts[op.result] = val
            if op.type == "index":
                self.idx[op.result] = _Aff({}, val)
        elif op.name in ("arith.addi", "arith.subi", "arith.muli") and op.type == "index":
            try:
                a, b = self.index(op.operands[0]), self.index(op.operands[1])
            except ShimError:
                return  # not affine: any load through it makes the function unmappable
            if op.name == "arith.addi":
                self.idx[op.result] = a + b
            elif op.name == "arith.subi":
                self.idx[op.result] = a - b
            elif not a.terms:
                self.idx[op.result] = b.scale(a.const)
            elif not b.terms:
                self.idx[op.result] = a.scale(b.const)


def _walk(ops, env: _Env, path=()):
    """Yields (op, enclosing spmd ops) depth first, feeding env."""
    for op in ops:
        env.visit(op)
        yield op, path
        if op.region:
            for a in op.block_args:
                env.idx[a] = _Aff({a: 1})
            yield from _walk(op.region, env, path + (op,))
        for r in op.more_regions:
            yield from _walk(r, env, path + (op,))


def _fold(env: _Env, v: str, loads: list) -> tuple:
    """(taps, scale): v as a left fold t = w0 x0; t = t + wk xk; then t * s."""
    op = env.defs.get(v)
    if op is None:
        raise ShimError(f"{env.func.name}: value {v} has no definition the shim understands")
    if op.name == "memref.load":
        loads.append(op)
        return [(None, op)], None
    if op.name == "arith.mulf":
        a, b = op.operands
        const, other = (a, b) if a in env.consts else (b, a) if b in env.consts else (None, None)
        if const is None:
            raise ShimError(f"{env.func.name}: product of two non-constant values")
        inner = env.defs.get(other)
        if inner is not None and inner.name == "memref.load":
            loads.append(inner)
            return [(env.consts[const], inner)], None
        taps, scale = _fold(env, other, loads)
        if scale is not None:
            raise ShimError(f"{env.func.name}: more than one final scale")
        return taps, env.consts[const]
    if op.name == "arith.addf":
        a, b = op.operands
        left, ls = _fold(env, a, loads)
        right, rs = _fold(env, b, loads)
        if ls is not None or rs is not None or len(right) != 1:
            raise ShimError(f"{env.func.name}: the sum is not a left fold in source order")
        return left + right, None
    raise ShimError(f"{env.func.name}: {op.name} is not part of a linear stencil")


def analyse(func: Func) -> Mapping:
    """Recognises the function's pattern; raises ShimError when it maps to nothing."""
    env = _Env(func)
    nodes = list(_walk(func.ops, env))
    unknown = [op.extra for op, _ in nodes if op.name == "unknown"]
    if unknown:
        raise ShimError(f"{func.name}: unsupported operation: {unknown[0]}")
    args = {a.name: a for a in func.args}
    foralls = [op for op, _ in nodes if op.name == "spmd.forall"]
    reduces = [(op, p) for op, p in nodes if op.name == "spmd.reduce"]
    atomics = [(op, p) for op, p in nodes if op.name == "memref.atomic_rmw"]
    stores = [(op, p) for op, p in nodes if op.name == "memref.store"]
    ifs = [op for op, _ in nodes if op.name == "spmd.if" and not op.result]  # guarded stores
    if [op for op, _ in nodes if op.name == "spmd.if"] and (reduces or atomics or not foralls):
        raise ShimError(f"{func.name}: spmd.if (a guarded store or a select) is not mapped here "
                        f"(only as the guarded store of an elementwise forall)")
    if not foralls:
        return _analyse_returned_reduce(func, env, args, reduces)
    group = foralls[0]
    lbs, ubs, steps = _segments(group)
    tile = _attr_ints(group.attrs, "spmd.tile_sizes")
    policy = _attr_enum(group.attrs, "spmd.memory_policy")
    if ifs:
        return _analyse_guarded(func, env, args, ifs, stores, foralls, lbs, ubs, steps)

    if atomics:  # ---------------------------------------------------------- reductions
        at, _ = atomics[0]
        val, out = at.operands
        if args.get(out) is None or args[out].rank != 0:
            raise ShimError(f"{func.name}: atomic_rmw target must be a rank-0 memref argument")
        if reduces:
            red, _ = reduces[0]
            kind = _attr_enum(red.attrs, "spmd.kind") or "add"
            src = _reduce_source(func, env, red)
            if at.extra not in _COMBINES[kind]:
                # Each tile's `kind` result is folded into out by a different
                # operation: out = out (+) r_0 (+) r_1 ..., not one reduction.
                raise ShimError(f"{func.name}: per-tile {kind} results combined by atomic_rmw {at.extra}: "
                                f"not a single {kind} reduction")
            init = env.consts.get(red.operands[3]) if len(red.operands) > 3 else None
            if init is None or not _is_identity(kind, init):
                raise ShimError(f"{func.name}: the spmd.reduce init must be the identity of {kind} "
                                f"(each tile folds it in once)")
        else:
            kind = {"addf": "add", "addi": "add"}.get(at.extra)
            v = env.defs.get(val)
            if kind is None or v is None or v.name != "memref.load":
                raise ShimError(f"{func.name}: atomic_rmw of a loaded element expected")
            src = v.operands[0]
        if at.extra not in ("addf", "addi") and not reduces:
            raise ShimError(f"{func.name}: unsupported atomic kind {at.extra}")
        n_arg = ubs[0] if ubs and ubs[0] in args else None
        elem = args[src].elem
        if elem == "f32" and kind == "add":
            entry = "spmdb200_hierarchical_sum" if reduces else "spmdb200_sum_f32"
        else:
            entry = f"spmdb200_reduce_{elem}"
        return Mapping(func.name, "reduce", entry, {"kind": kind, "input": src, "output": out, "n": n_arg,
                                                    "combine": at.extra, "elem": elem})

    if not stores and not reduces and all(op.name in ("spmd.forall", "spmd.yield", "arith.constant", "func.return")
                                          for op, _ in nodes):
        # A forall whose body does nothing (test/SPMD/normalize.mlir): no effect to run.
        return Mapping(func.name, "empty", None, {})
    if len(stores) > 1 and not reduces and not atomics:
        return _analyse_multi_store(func, env, args, nodes, stores, foralls, lbs, ubs, steps)
    if len(stores) != 1:
        raise ShimError(f"{func.name}: expected exactly one memref.store, found {len(stores)}")
    st, _ = stores[0]
    try:
        return _analyse_linear(func, env, args, st, foralls, lbs, ubs, tile, policy)
    except ShimError as linear_err:
        try:
            return _analyse_map(func, env, args, st, foralls, lbs, ubs, steps)
        except ShimError as map_err:
            raise ShimError(f"{linear_err}; as an elementwise map: {str(map_err).split(': ', 1)[-1]}") from None


def _analyse_linear(func: Func, env: _Env, args: dict, st: Op, foralls: list, lbs, ubs, tile, policy) -> Mapping:
    """ewise add / axpy / a linear stencil (a left fold of weighted loads)."""
    val, dst = st.operands
    dst_idx = [env.index(v) for v in _vals(st.extra)]
    rank = len(dst_idx)
    loads: list = []
    taps, scale = _fold(env, val, loads)
    srcs = {ld.operands[0] for _, ld in taps}
    # offsets of every load relative to the store's index
    offsets = []
    for w, ld in taps:
        li = [env.index(v) for v in _vals(ld.extra)]
        if len(li) != rank:
            raise ShimError(f"{func.name}: load rank differs from the store's")
        off = []
        for a, b in zip(li, dst_idx):
            d = a - b
            if d.terms:
                raise ShimError(f"{func.name}: load index is not the store index plus a constant")
            off.append(d.const)
        offsets.append(off)
    # iteration domain: the group forall's upper bounds; lane step from the store index
    ub = [u for u in ubs[:rank]]
    lane_steps = []
    inner = foralls[1] if len(foralls) > 1 else None
    for d in range(rank):
        coeffs = sorted(v for k, v in dst_idx[d].terms.items() if inner is None or k in inner.block_args)
        lane_steps.append(coeffs[0] if coeffs else 1)
    lower = []
    for v in lbs[:rank]:
        a = env.index(v)
        if len(a.terms) > 1 or any(c != 1 for c in a.terms.values()) or (a.terms and a.const):
            raise ShimError(f"{func.name}: lower bound {v} must be a constant or an index argument")
        lower.append(next(iter(a.terms)) if a.terms else a.const)
    if rank == 1 and lower == [0] and len(srcs) >= 1 and all(o == [0] for o in offsets):
        ws = [w for w, _ in taps]
        if len(taps) == 2 and ws == [None, None] and scale is None and len(srcs) == 2:
            a, b = [ld.operands[0] for _, ld in taps]
            return Mapping(func.name, "ewise", "spmdb200_ewise", {"a": a, "b": b, "c": dst, "n": ub[0]})
        if len(taps) == 2 and ws[0] is not None and ws[1] is None and scale is None:
            x, y = [ld.operands[0] for _, ld in taps]
            if y == dst:
                return Mapping(func.name, "axpy", "spmdb200_axpy", {"alpha": ws[0], "x": x, "y": dst, "n": ub[0]})
    if len(srcs) != 1:
        raise ShimError(f"{func.name}: a stencil reads exactly one memref (found {sorted(srcs)})")
    (src,) = srcs
    if src == dst:
        raise ShimError(f"{func.name}: the stencil's input is also its output (not read-only)")
    weights = None if all(w is None for w, _ in taps) else [1.0 if w is None else w for w, _ in taps]
    return Mapping(func.name, "stencil", "spmdb200_stencil_nd", {
        "rank": rank, "input": src, "output": dst, "domain": ub, "offsets": offsets, "weights": weights,
        "scale": scale, "tile_sizes": tile or [1] * rank, "steps": lane_steps, "lower": lower,
        "memory_policy": policy or "none"})


# arith / math ops of an elementwise body and their forall_map opcodes.
_MAP_ARITH = {"arith.addf": "add", "arith.subf": "sub", "arith.mulf": "mul", "arith.divf": "div",
              "arith.maximumf": "maximum", "arith.minimumf": "minimum", "arith.negf": "neg", "math.absf": "abs",
              "math.sqrt": "sqrt", "arith.cmpf": "cmp", "arith.select": "select", "arith.andi": "and",
              "arith.ori": "or", "arith.xori": "xor"}


def _analyse_map(func: Func, env: _Env, args: dict, st: Op, foralls: list, lbs, ubs, steps) -> Mapping:
    """A forall with a general f32 body: out[p] = f(in_0[p + o_0], ...) where
    every load reads its memref at the store's index plus a constant offset
    (each (memref, offset) pair becomes a view shifted by the offset, so a
    non-linear stencil -- a max filter, an upwind select -- maps too) and f is
    any DAG of the ops in _MAP_ARITH, f32 constants and f32 scalar arguments:
    the per-point body SPMDToGPU.cpp:491-580 lowers, run by
    spmdb200_forall_map.  The stored memref may be read only at the store's
    own index."""
    val, dst = st.operands
    if args.get(dst) is None or args[dst].kind != "memref" or args[dst].elem != "f32":
        raise ShimError(f"{func.name}: the stored memref must be an f32 memref argument")
    dst_idx = [env.index(v) for v in _vals(st.extra)]
    rank = len(dst_idx)
    if not 1 <= rank <= 3 or args[dst].rank != rank:
        raise ShimError(f"{func.name}: rank 1-3 stores of the memref's full rank only")
    if len(foralls) > 2:
        raise ShimError(f"{func.name}: at most a group and a lane forall")
    group, inner = foralls[0], (foralls[1] if len(foralls) > 1 else None)
    if len(group.block_args) < rank or (inner is not None and len(inner.block_args) < rank):
        raise ShimError(f"{func.name}: the forall's rank is below the store's")
    lower, upper, dom_step = [], [], []
    for d in range(rank):
        want = {group.block_args[d]: 1}
        g_step = env.index(steps[d])
        if inner is not None:
            want[inner.block_args[d]] = 1
            i_lb, i_ub, i_st = (env.index(x[d]) for x in _segments(inner))
            if (i_lb.terms or i_lb.const != 0 or i_st.terms or i_st.const != 1 or i_ub.terms or g_step.terms
                    or i_ub.const != g_step.const):
                raise ShimError(f"{func.name}: the lane forall must cover [0, group step) with step 1")
        elif g_step.terms or g_step.const < 1:
            raise ShimError(f"{func.name}: the forall step must be a positive constant")
        if dst_idx[d].terms != want or dst_idx[d].const != 0:
            raise ShimError(f"{func.name}: the store index is not the loop index in dimension {d}")
        a = env.index(lbs[d])
        if len(a.terms) > 1 or any(c != 1 for c in a.terms.values()) or (a.terms and a.const):
            raise ShimError(f"{func.name}: lower bound {lbs[d]} must be a constant or an index argument")
        lower.append(next(iter(a.terms)) if a.terms else a.const)
        u = env.index(ubs[d])
        if len(u.terms) > 1 or any(c != 1 for c in u.terms.values()) or (u.terms and u.const):
            raise ShimError(f"{func.name}: upper bound {ubs[d]} must be a constant or an index argument")
        upper.append(next(iter(u.terms)) if u.terms else u.const)
        dom_step.append(1 if inner is not None else g_step.const)

    inputs: list = []
    consts: list = []
    nodes: dict = {}

    def visit(v):
        if v in nodes:
            return
        op = env.defs.get(v)
        if op is None:
            a = args.get(v)
            if a is None or a.kind != "f32":
                raise ShimError(f"{func.name}: value {v} is neither an op result nor an f32 argument")
            consts.append(v)
            nodes[v] = ("const", len(consts) - 1)
            return
        if op.name == "memref.load":
            src = op.operands[0]
            if args.get(src) is None or args[src].kind != "memref" or args[src].elem != "f32" \
                    or args[src].rank != rank:
                raise ShimError(f"{func.name}: {src} is not an f32 memref argument of rank {rank}")
            idx = [env.index(x) for x in _vals(op.extra)]
            off = []
            for i, j in zip(idx, dst_idx):
                d = i - j
                if d.terms:
                    raise ShimError(f"{func.name}: {src} is read off the store's index plus a constant")
                off.append(d.const)
            if src == dst and any(off):
                # every point would read values other points overwrite
                raise ShimError(f"{func.name}: the stored memref is also read at another point")
            key = (src, tuple(off))  # a constant offset is a shifted view of the memref
            if key not in inputs:
                inputs.append(key)
            nodes[v] = ("load", inputs.index(key))
            return
        if op.name == "arith.constant":
            if op.type not in ("f32", "i1"):
                raise ShimError(f"{func.name}: constant of type {op.type} in an elementwise body")
            consts.append(float(env.consts[v]))
            nodes[v] = ("const", len(consts) - 1)
            return
        if op.name == "spmd.if":
            # %r = spmd.if(%c) {yield %x} else {yield %y}: select(c, x, y); both
            # regions are side-effect free here (the forall's only store is outside)
            ys = [[o for o in r if o.name == "spmd.yield"] for r in [op.region, *op.more_regions]]
            if len(ys) != 2 or any(len(y) != 1 or len(y[0].operands) != 1 for y in ys):
                raise ShimError(f"{func.name}: an spmd.if value needs one yielded value per region")
            x, y = ys[0][0].operands[0], ys[1][0].operands[0]
            for o in (op.operands[0], x, y):
                visit(o)
            nodes[v] = ("select", op.operands[0], x, y)
            return
        kind = _MAP_ARITH.get(op.name)
        if kind is None:
            raise ShimError(f"{func.name}: {op.name} in an elementwise body is not mapped")
        want_t = "i1" if kind in ("and", "or", "xor") else "f32"
        if kind == "select":
            if op.type != "f32":
                raise ShimError(f"{func.name}: select of type {op.type}")
        elif op.type != want_t:
            raise ShimError(f"{func.name}: {op.name} of type {op.type} (f32 bodies only)")
        for o in op.operands:
            visit(o)
        if kind == "cmp":
            pred = op.extra.strip()
            if pred not in _fp.CMPF:
                raise ShimError(f"{func.name}: arith.cmpf predicate {pred}")
            nodes[v] = ("cmp", op.operands[0], op.operands[1], _fp.CMPF[pred])
        else:
            nodes[v] = (kind, *op.operands)

    visit(val)
    if not inputs:
        raise ShimError(f"{func.name}: a body that loads nothing (a fill) is not mapped")
    if len(consts) > _fp.MAX_CONSTS:
        raise ShimError(f"{func.name}: more than {_fp.MAX_CONSTS} constants")
    try:
        code, n_regs, _, _ = _fp.compile_dag(val, nodes)
    except ValueError as e:
        raise ShimError(f"{func.name}: {e}") from None
    return Mapping(func.name, "map", "spmdb200_forall_map", {
        "rank": rank, "inputs": [m for m, _ in inputs], "input_offsets": [list(o) for _, o in inputs],
        "output": dst, "lower": lower, "domain": upper, "steps": dom_step,
        "code": [list(c) for c in code], "consts": consts, "n_regs": n_regs})


def _analyse_multi_store(func: Func, env: _Env, args: dict, nodes: list, stores: list, foralls: list, lbs, ubs,
                         steps) -> Mapping:
    """A forall body with several stores (several outputs per point) runs as
    one general map per store, in store order.  That order reproduces the
    body's own program order when (1) a memref that is stored anywhere in the
    body is read only at the store's own index, and (2) no store to a memref
    lies between a load of it and the store that load feeds (so each load
    sees the same value -- the old one, or the one an earlier store left --
    in both orders).  Anything else is reported."""
    pos = {id(op): i for i, (op, _) in enumerate(nodes)}
    if len({tuple(id(o) for o in p) for _, p in stores}) != 1:
        raise ShimError(f"{func.name}: the stores sit in different regions")
    stored: dict = {}
    for st, _ in stores:
        stored.setdefault(st.operands[1], []).append(pos[id(st)])
    maps = []
    for st, _ in stores:
        m = _analyse_map(func, env, args, st, foralls, lbs, ubs, steps)
        for name, off in zip(m.detail["inputs"], m.detail["input_offsets"]):
            if name in stored and any(off):
                raise ShimError(f"{func.name}: {name} is stored in the body and read at offset {off}")
        for ld in _dag_loads(env, st.operands[0]):
            src = ld.operands[0]
            if any(pos[id(ld)] < q < pos[id(st)] for q in stored.get(src, [])):
                raise ShimError(f"{func.name}: {src} is stored between a load of it and the store that uses it")
        maps.append(m.detail)
    return Mapping(func.name, "maps", "spmdb200_forall_map", {"maps": maps, "outputs": [d["output"] for d in maps]})


def _dag_loads(env: _Env, root: str) -> list:
    """The memref.load ops an SSA value depends on."""
    out, seen, todo = [], set(), [root]
    while todo:
        v = todo.pop()
        if v in seen:
            continue
        seen.add(v)
        op = env.defs.get(v)
        if op is None:
            continue
        if op.name == "memref.load":
            out.append(op)
            continue
        todo.extend(op.operands)
        if op.name == "spmd.if":  # a value spmd.if depends on what its regions yield
            for r in [op.region, *op.more_regions]:
                todo.extend(o for y in r if y.name == "spmd.yield" for o in y.operands)
    return out


def _analyse_guarded(func: Func, env: _Env, args: dict, ifs: list, stores: list, foralls: list, lbs, ubs,
                     steps) -> Mapping:
    """A forall whose only store sits in an spmd.if: `if (c) A[p] = v`, with
    an empty else region or `else A[p] = w`, is the elementwise map
    A[p] = select(c, v, w) -- with A[p] itself for the missing else (an
    in-place map: each point is read before it is written).  The guarded-store
    form of test/SPMD/lower-to-gpu.mlir:200-213, run by spmdb200_forall_map."""
    if len(ifs) != 1 or ifs[0].result:
        raise ShimError(f"{func.name}: one spmd.if without results (a guarded store) is mapped, not {len(ifs)}")
    op_if = ifs[0]
    then_st = [o for o in _iter_ops(op_if.region) if o.name == "memref.store"]
    else_st = [o for r in op_if.more_regions for o in _iter_ops(r) if o.name == "memref.store"]
    if len(then_st) != 1 or len(else_st) > 1 or len(stores) != len(then_st) + len(else_st):
        raise ShimError(f"{func.name}: the spmd.if must hold the forall's only store (one per region)")
    st = then_st[0]
    if else_st:
        a = [env.index(v) for v in _vals(st.extra)]
        b = [env.index(v) for v in _vals(else_st[0].extra)]
        if else_st[0].operands[1] != st.operands[1] or any(x.terms != y.terms or x.const != y.const
                                                           for x, y in zip(a, b)):
            raise ShimError(f"{func.name}: the two regions store to different places")
        other = else_st[0].operands[0]
    else:
        other = "%__guarded_old"
        env.defs[other] = Op("memref.load", other, [st.operands[1]], extra=st.extra, type=st.type)
    sel = "%__guarded_select"
    env.defs[sel] = Op("arith.select", sel, [op_if.operands[0], st.operands[0], other], type="f32")
    synth = Op("memref.store", None, [sel, st.operands[1]], extra=st.extra, type=st.type)
    return _analyse_map(func, env, args, synth, foralls, lbs, ubs, steps)


# memref.atomic_rmw kinds that combine per-tile results of each reduction kind
# into the output with the same operation (signed i32 max/min; f32 max/min
# with arith.maximumf/minimumf's NaN and signed-zero rules).
_COMBINES = {"add": ("addf", "addi"), "mul": ("mulf", "muli"), "max": ("maximumf", "maxs"),
             "min": ("minimumf", "mins"), "and": ("andi",), "or": ("ori",), "xor": ("xori",)}


def _is_identity(kind: str, v) -> bool:
    if kind in ("add", "or", "xor"):
        return v == 0
    if kind == "mul":
        return v == 1
    if kind == "and":
        return v == -1
    if kind == "max":
        return v == float("-inf") or v == -2 ** 31
    return v == float("inf") or v == 2 ** 31 - 1  # min


def _reduce_source(func: Func, env: _Env, red: Op) -> str:
    """The memref an spmd.reduce body loads and yields (through masking selects)."""
    yields = [o for o in red.region if o.name == "spmd.yield"]
    y = env.defs.get(yields[-1].operands[0]) if yields and yields[-1].operands else None
    while y is not None and y.name == "arith.select":
        y = env.defs.get(y.operands[1])
    if y is None or y.name != "memref.load":
        raise ShimError(f"{func.name}: spmd.reduce body must yield one (masked) load")
    return y.operands[0]


def _analyse_returned_reduce(func: Func, env: _Env, args: dict, reduces: list) -> Mapping:
    """A top-level spmd.reduce over [0, N) whose value the function returns
    (the host-level reduction the SCF and OpenMP lowerings take, e.g.
    test/SPMD/sum.mlir @sum): the value is init (+) A[0] (+) ... (+) A[N-1]."""
    rets = [op for op in func.ops if op.name == "func.return"]
    top = [op for op in func.ops if op.name == "spmd.reduce"]
    if len(reduces) != 1 or len(top) != 1:
        raise ShimError(f"{func.name}: no spmd.forall")
    red = top[0]
    stored = [op for op in func.ops if op.name == "memref.store" and op.operands[0] == red.result]
    target = None
    if stored and len([op for op in func.ops if op.name == "memref.store"]) == 1:
        # memref.store %r, %out[c] (test/SPMD/ops.mlir @sum): out[c] = the value
        st = stored[0]
        at = [env.index(v) for v in _vals(st.extra)]
        if args.get(st.operands[1]) is None or any(a.terms for a in at):
            raise ShimError(f"{func.name}: the reduce's value is stored to a non-argument or a varying index")
        target = (st.operands[1], [a.const for a in at])
    elif not rets or rets[-1].operands != [red.result]:
        raise ShimError(f"{func.name}: no spmd.forall")
    lb, ub, step = (env.index(v) for v in red.operands[:3])
    if lb.terms or lb.const != 0 or step.terms or step.const != 1:
        raise ShimError(f"{func.name}: the returned spmd.reduce must run over [0, N) with step 1")
    src = _reduce_source(func, env, red)
    ld = next(op for op in _iter_ops(red.region) if op.name == "memref.load" and op.operands[0] == src)
    idx = [env.index(v) for v in _vals(ld.extra)]
    if len(idx) != 1 or idx[0].const != 0 or idx[0].terms != {red.block_args[0]: 1}:
        raise ShimError(f"{func.name}: the reduce must load {src}[iv]")
    kind = _attr_enum(red.attrs, "spmd.kind") or "add"
    init = env.consts.get(red.operands[3]) if len(red.operands) > 3 else None
    if init is None:
        raise ShimError(f"{func.name}: the spmd.reduce init must be a constant")
    n_arg = red.operands[1] if red.operands[1] in args else ub.const
    elem = args[src].elem
    return Mapping(func.name, "reduce", f"spmdb200_reduce_{elem}", {
        "kind": kind, "input": src, "output": target[0] if target else None, "at": target[1] if target else None,
        "n": n_arg, "combine": "store" if target else "return", "elem": elem, "init": init})


# ----------------------------------------------------------------------------- binding
class BoundKernel:
    """Calls the mapped entry with the MLIR function's own argument list."""

    def __init__(self, func: Func, mapping: Mapping):
        self.func, self.mapping = func, mapping
        self.names = [a.name for a in func.args]

    def __repr__(self) -> str:
        return f"BoundKernel({self.mapping.name} -> {self.mapping.entry})"

    def __call__(self, *vals, stream=None):
        import importlib
        k = importlib.import_module(__package__ + ".kernels") if __package__ else importlib.import_module("kernels")
        if len(vals) != len(self.names):
            raise TypeError(f"{self.func.name} takes {len(self.names)} arguments")
        env = dict(zip(self.names, vals))
        m, d = self.mapping, self.mapping.detail

        def num(v):
            return int(env[v]) if v in env else int(v) if str(v).lstrip("-").isdigit() else None

        if m.pattern == "ewise":
            n = num(d["n"])
            return k.ewise(env[d["a"]][:n], env[d["b"]][:n], out=env[d["c"]][:n], stream=stream)
        if m.pattern == "axpy":
            n = num(d["n"])
            return k.axpy(d["alpha"], env[d["x"]][:n], env[d["y"]][:n], stream=stream)
        if m.pattern == "stencil":
            dom = [num(u) if u in env else self._const(u) for u in d["domain"]]
            lo = [int(env[v]) if isinstance(v, str) else int(v) for v in d["lower"]]
            # Output point q of the view is global point lo + q: shift the reads by lo.
            out = env[d["output"]][tuple(slice(a, max(a, b)) for a, b in zip(lo, dom))]
            offs = [[o + a for o, a in zip(off, lo)] for off in d["offsets"]]
            policy = 0 if d["memory_policy"] == "prefer_group" else 1
            return k.stencil_nd(env[d["input"]], out, offs, weights=d["weights"],
                                scale=1.0 if d["scale"] is None else d["scale"], tile_sizes=d["tile_sizes"],
                                steps=d["steps"], policy=policy, stream=stream)
        if m.pattern == "empty":
            return None
        if m.pattern == "maps":  # several outputs per point: one map per store, in store order
            for sub in d["maps"]:
                self._run_map(k, sub, env, num, stream)
            return None
        if m.pattern == "map":
            return self._run_map(k, d, env, num, stream)
        if m.pattern == "reduce" and d["combine"] in ("return", "store"):
            n = num(d["n"]) if isinstance(d["n"], str) else int(d["n"])
            a = env[d["input"]][:n]
            if d["combine"] == "store":  # out[c] = init (+) a[0] (+) ...
                target = env[d["output"]][tuple(d["at"])].reshape(1)
                k.reduce(d["kind"], a, d["init"], out=target, stream=stream)
                return None
            out = a.new_empty(1)
            k.reduce(d["kind"], a, d["init"], out=out, stream=stream)
            return out.item()
        if m.pattern == "reduce":
            n = num(d["n"]) if d["n"] else env[d["input"]].shape[0]
            a, out = env[d["input"]][:n], env[d["output"]].reshape(1)
            if m.entry == "spmdb200_hierarchical_sum":
                return k.hierarchical_sum(a, out, stream=stream)
            if m.entry == "spmdb200_sum_f32":
                return k.sum_f32(a, out, stream=stream)
            init = out.item()  # the combine folds the old value in, as atomic_rmw does
            return k.reduce(d["kind"], a, init, out=out, stream=stream)
        raise ShimError(f"unbound pattern {m.pattern}")

    def _run_map(self, k, d: dict, env: dict, num, stream):
        """One general forall map: views of the domain box (shifted by each
        load's offset), checked against the tensors' sizes on the host."""
        lo = [int(env[v]) if isinstance(v, str) else int(v) for v in d["lower"]]
        hi = [num(u) if u in env else self._const(u) if isinstance(u, str) else int(u) for u in d["domain"]]
        box = tuple(slice(a, max(a, b), s) for a, b, s in zip(lo, hi, d["steps"]))
        ot = env[d["output"]]
        if any(b > a and (a < 0 or b > ot.shape[k]) for k, (a, b) in enumerate(zip(lo, hi))):
            raise ShimError(f"{self.func.name}: the domain {lo}..{hi} is outside {d['output']}'s sizes "
                            f"{tuple(ot.shape)}")
        out = ot[box]
        views = []
        for x, off in zip(d["inputs"], d["input_offsets"]):
            t = env[x]
            if out.numel() and any(a + o < 0 or max(a, b) + o > t.shape[k]
                                   for k, (a, b, o) in enumerate(zip(lo, hi, off))):
                raise ShimError(f"{self.func.name}: {x} read at offset {off} outside its sizes {tuple(t.shape)}")
            views.append(t[tuple(slice(a + o, max(a, b) + o, s) for a, b, o, s in zip(lo, hi, off, d["steps"]))])
        if out.numel() == 0:
            return out
        consts = [float(env[c]) if isinstance(c, str) else c for c in d["consts"]]
        return k.forall_map(views, out, [tuple(c) for c in d["code"]], consts, n_regs=d["n_regs"],
                            stream=stream)

    def _const(self, v):
        for op in _iter_ops(self.func.ops):
            if op.result == v and op.name == "arith.constant":
                return int(op.extra)
        raise ShimError(f"{self.func.name}: domain bound {v} is neither an argument nor a constant")


def _iter_ops(ops):
    for op in ops:
        yield op
        yield from _iter_ops(op.region)
        for r in op.more_regions:
            yield from _iter_ops(r)


def load(text: str, skip_unmapped: bool = False) -> dict:
    """name -> BoundKernel for the module's spmd.kernel functions; a function
    the shim cannot map raises ShimError unless skip_unmapped."""
    out = {}
    for f in parse_module(text):
        if not f.kernel:
            continue
        try:
            out[f.name] = BoundKernel(f, analyse(f))
        except ShimError:
            if not skip_unmapped:
                raise
    return out


def describe(text: str) -> list:
    res = []
    for f in parse_module(text):
        if not f.kernel:
            continue
        try:
            res.append(analyse(f).to_json())
        except ShimError as e:
            res.append({"function": f.name, "pattern": None, "error": str(e)})
    return res


# ----------------------------------------------------------------------------- build stand-ins
# Host entries with the reference's names and signatures (harness/run_host.py)
# and the kernel names a reference PTX module carries (func name + "_kernel").
HOST_ENTRIES = {"ewise", "stencil_cpu", "atomic_sum", "hierarchical_sum"}
MODULE_KERNELS = {"ewise": "ewise_kernel", "promoted_stencil": "promoted_stencil_kernel",
                  "atomic_sum": "atomic_sum_kernel", "hierarchical_sum": "hierarchical_sum_kernel"}


def build_so(text: str, out: str) -> list:
    names = [f.name for f in parse_module(text) if f.kernel]
    missing = [n for n in names if n not in HOST_ENTRIES]
    if not names or missing:
        raise ShimError(f"no host entry of this name in the library: {missing or '(no spmd.kernel function)'}")
    lib = HERE / "libspmdb200.so"
    if not lib.exists():
        raise ShimError("libspmdb200.so is not built (run spmd-dialect_b200/build.py)")
    shutil.copyfile(lib, out)
    return names


def build_module(text: str, out: str) -> list:
    names = [f.name for f in parse_module(text) if f.kernel]
    missing = [n for n in names if n not in MODULE_KERNELS]
    if not names or missing:
        raise ShimError(f"no kernel of this name in the module: {missing or '(no spmd.kernel function)'}")
    mod = HERE / "spmdb200_kernels.cubin"
    if not mod.exists():
        raise ShimError("spmdb200_kernels.cubin is not built (run spmd-dialect_b200/build.py)")
    shutil.copyfile(mod, out)
    return [MODULE_KERNELS[n] for n in names]


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) < 2 or argv[0] not in ("describe", "so", "ptx"):
        print(__doc__.split("\n\n")[-2], file=sys.stderr)
        return 2
    text = Path(argv[1]).read_text()
    try:
        if argv[0] == "describe":
            print(json.dumps(describe(text), indent=1))
        elif argv[0] == "so":
            if len(argv) != 4 or argv[2] not in ("scf", "omp"):
                raise ShimError("usage: so FILE scf|omp OUT.so")
            print("host entries:", ", ".join(build_so(text, argv[3])))
        else:
            if len(argv) < 4 or argv[2] not in ("ewise", "promoted", "hierarchical"):
                raise ShimError("usage: ptx FILE ewise|promoted|hierarchical OUT [sm]")
            print("kernels:", ", ".join(build_module(text, argv[3])))
    except ShimError as e:
        print(f"ERROR: {e}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
