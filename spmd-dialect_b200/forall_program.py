"""The straight-line body program of spmdb200_forall_map (include/spmd_b200.h):
opcodes, arith.cmpf predicate numbers, instruction encoding, and a compiler
from an SSA expression DAG to instructions with registers allocated.

An instruction is two int32 words, w0 = op | dst << 8 | a << 16 | b << 24 and
w1 = aux.  No torch, no library: the textual-MLIR shim and the device wrapper
both build programs with it.
"""
from __future__ import annotations

# SPMDB200_MAP_* of include/spmd_b200.h.
OPS = {"load": 0, "const": 1, "add": 2, "sub": 3, "mul": 4, "div": 5, "maximum": 6, "minimum": 7, "neg": 8,
       "abs": 9, "sqrt": 10, "cmp": 11, "select": 12, "and": 13, "or": 14, "xor": 15, "store": 16}
# arith.cmpf predicates, numbered as the dialect's CmpFPredicate enum.
CMPF = {"false": 0, "oeq": 1, "ogt": 2, "oge": 3, "olt": 4, "ole": 5, "one": 6, "ord": 7, "ueq": 8, "ugt": 9,
        "uge": 10, "ult": 11, "ule": 12, "une": 13, "uno": 14, "true": 15}
UNARY = {"neg", "abs", "sqrt"}
MAX_INPUTS, MAX_REGS, MAX_INSNS, MAX_CONSTS = 8, 16, 64, 32


def insn(op: str, dst: int = 0, a: int = 0, b: int = 0, aux: int = 0) -> tuple[int, int]:
    """One instruction as its two int32 words."""
    w0 = OPS[op] | (dst << 8) | (a << 16) | (b << 24)
    return (w0 - (1 << 32) if w0 >= 1 << 31 else w0, aux)


def compile_dag(root: str, nodes: dict) -> tuple[list, int, list, list]:
    """Compiles the value `root` of an expression DAG to a program.

    nodes maps a value name to ("load", input_index) | ("const", const_index)
    | (op, operand names..., aux) with op one of OPS (cmp: aux = predicate;
    select: operands (cond, a, b)).  Returns (code, n_regs, load order, the
    node order): LOADs first (one per input), then the other nodes in
    dependency order, then the STORE; registers are reused after a value's
    last use.
    """
    order: list = []
    seen: set = set()

    def visit(v):
        if v in seen:
            return
        seen.add(v)
        n = nodes[v]
        if n[0] not in ("load", "const"):
            for o in _operands(n):
                visit(o)
        order.append(v)

    visit(root)
    loads = sorted((v for v in order if nodes[v][0] == "load"), key=lambda v: nodes[v][1])
    rest = [v for v in order if nodes[v][0] != "load"]
    seq = loads + rest
    last = {}
    for i, v in enumerate(seq):
        for o in _operands(nodes[v]):
            last[o] = i
    last[root] = len(seq)  # read by the STORE
    reg: dict = {}
    free: list = []
    top = 0
    code = []
    for i, v in enumerate(seq):
        n = nodes[v]
        ops = _operands(n)
        src = [reg[o] for o in ops]
        for o in set(ops):
            if last[o] == i:
                free.append(reg[o])
        free.sort()
        if free:
            d = free.pop(0)
        else:
            d, top = top, top + 1
        reg[v] = d
        if n[0] == "load":
            code.append(insn("load", d, aux=n[1]))
        elif n[0] == "const":
            code.append(insn("const", d, aux=n[1]))
        elif n[0] == "select":
            code.append(insn("select", d, src[1], src[2], aux=src[0]))
        elif n[0] == "cmp":
            code.append(insn("cmp", d, src[0], src[1], aux=n[3]))
        elif n[0] in UNARY:
            code.append(insn(n[0], d, src[0]))
        else:
            code.append(insn(n[0], d, src[0], src[1]))
    code.append(insn("store", 0, reg[root]))
    if top > MAX_REGS or len(code) > MAX_INSNS or len(loads) > MAX_INPUTS:
        raise ValueError(f"body too large: {top} registers, {len(code)} instructions, {len(loads)} inputs "
                         f"(limits {MAX_REGS}, {MAX_INSNS}, {MAX_INPUTS})")
    return code, top, loads, seq


def _operands(n: tuple) -> list:
    if n[0] in ("load", "const"):
        return []
    if n[0] == "cmp":
        return [n[1], n[2]]
    if n[0] == "select":
        return [n[1], n[2], n[3]]
    if n[0] in UNARY:
        return [n[1]]
    return [n[1], n[2]]
