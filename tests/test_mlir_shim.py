"""The textual-MLIR shim on the host: parsing the dialect's generic form,
recognising the hot-path patterns, reporting what it cannot map, and the
build stand-ins of the differential script.  When SPMD_REFERENCE_DIR names a
checkout of the reference, its own kernel files (test/SPMD/*.mlir) are mapped
too."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

from conftest import ROOT, spmd_mod

MLIR = ROOT / "tests" / "mlir" / "kernels.mlir"
_REF_DIR = os.environ.get("SPMD_REFERENCE_DIR", "")
REFERENCE = Path(_REF_DIR) / "test" / "SPMD" if _REF_DIR else None


def _by_name():
    shim = spmd_mod("mlir_shim")
    return {d["function"]: d for d in shim.describe(MLIR.read_text())}


def test_patterns_recognised():
    d = _by_name()
    assert d["ewise"]["entry"] == "spmdb200_ewise"
    assert d["axpy"]["pattern"] == "axpy" and d["axpy"]["alpha"] == 2.5
    ps = d["promoted_stencil"]
    assert ps["offsets"] == [[0, 0], [0, 1], [1, 0]] and ps["tile_sizes"] == [32, 8]
    assert ps["memory_policy"] == "prefer_group" and ps["scale"] is None and ps["weights"] is None
    jac = d["jacobi_interior"]
    assert jac["offsets"] == [[0, 0], [-1, 0], [1, 0], [0, 1], [0, -1]] and jac["scale"] == pytest.approx(0.2)
    assert d["pairs_stepped"]["steps"] == [2] and d["pairs_stepped"]["offsets"] == [[0], [1]]
    assert d["smooth_interior"]["lower"] == [1] and d["smooth_interior"]["weights"] == [0.5, 0.5]
    assert d["hierarchical_sum"]["entry"] == "spmdb200_hierarchical_sum"
    assert d["max_i32"]["entry"] == "spmdb200_reduce_i32" and d["max_i32"]["kind"] == "max"


def test_unmappable_functions_are_reported_not_guessed():
    d = _by_name()
    assert d["gather_unsupported"]["pattern"] is None
    assert "affine" in d["gather_unsupported"]["error"]
    shim = spmd_mod("mlir_shim")
    with pytest.raises(shim.ShimError):
        shim.load(MLIR.read_text())  # load() maps every kernel or fails


def test_plan_of_mapped_stencils():
    """The mapped tile sizes / offsets drive the same promotion plan."""
    k = spmd_mod("kernels")
    ps = _by_name()["promoted_stencil"]
    mn = [min(o[d] for o in ps["offsets"]) for d in range(2)]
    mx = [max(o[d] for o in ps["offsets"]) for d in range(2)]
    assert k.promotion_plan(ps["tile_sizes"], mn, mx, steps=ps["steps"])[:2] == (0, (33, 9))


def test_build_stand_ins(tmp_path):
    shim = spmd_mod("mlir_shim")
    one = tmp_path / "ewise.mlir"
    text = MLIR.read_text()
    one.write_text(text[:text.index("func.func @axpy")])
    so = tmp_path / "ewise_scf.so"
    r = subprocess.run([sys.executable, str(ROOT / "spmd-dialect_b200" / "mlir_shim.py"), "so", str(one), "scf",
                        str(so)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    import ctypes
    assert hasattr(ctypes.CDLL(str(so)), "ewise")  # the reference's host entry name
    mod = tmp_path / "ewise.ptx"
    r = subprocess.run([sys.executable, str(ROOT / "spmd-dialect_b200" / "mlir_shim.py"), "ptx", str(one), "ewise",
                        str(mod), "sm_100"], capture_output=True, text=True)
    assert r.returncode == 0 and "ewise_kernel" in r.stdout and mod.stat().st_size > 0
    with pytest.raises(shim.ShimError):
        shim.build_so(text, str(tmp_path / "all.so"))  # axpy etc. have no reference host entry


@pytest.mark.skipif(REFERENCE is None or not REFERENCE.exists(),
                    reason="SPMD_REFERENCE_DIR does not name a reference checkout")
def test_reference_kernel_files_map():
    shim = spmd_mod("mlir_shim")
    want = {
        "lower-to-gpu-nvptx.mlir": {"ewise": "spmdb200_ewise"},
        "lower-to-gpu-nvptx-promoted.mlir": {"promoted_stencil": "spmdb200_stencil_nd"},
        "lower-to-gpu-nvptx-reduction.mlir": {"atomic_sum": "spmdb200_sum_f32"},
        "lower-to-gpu-nvptx-hierarchical-reduction.mlir": {"hierarchical_sum": "spmdb200_hierarchical_sum"},
        "differential-stencil.mlir": {"stencil_cpu": "spmdb200_stencil_nd"},
    }
    for f, names in want.items():
        got = {d["function"]: d.get("entry") for d in shim.describe((REFERENCE / f).read_text())}
        for n, e in names.items():
            assert got.get(n) == e, (f, n, got)
    maps = {"ewise.mlir": ["ewise2d"], "ops.mlir": ["ewise_square"],
            "cross-pipeline-regression.mlir": ["ewise_regression", "ewise_nonzero_lb"],
            "subset_positive.mlir": ["legal_kernel"]}
    for f, names in maps.items():
        got = {d["function"]: d for d in shim.describe((REFERENCE / f).read_text())}
        for n in names:
            assert got[n]["entry"] == "spmdb200_forall_map", (f, n, got[n])
    kinds = {d["function"]: d for d in shim.describe((REFERENCE / "reduction-hierarchical-f32-kinds.mlir").read_text())}
    assert kinds["reduce_add"]["entry"] == "spmdb200_hierarchical_sum"
    assert all(kinds[k]["pattern"] is None for k in ("reduce_mul", "reduce_max", "reduce_min"))
    steps = {d["function"]: (d["offsets"], d["steps"]) for d in shim.describe((REFERENCE / "promotion.mlir").read_text())}
    assert steps["stencil1d_stepped"] == ([[0], [1]], [2])
    assert steps["stencil_pos_halo"][0] == [[1], [2]] and steps["stencil_neg_halo"][0] == [[-1], [-2]]


_FORMS = r'''
func.func @sum_returned(%A: memref<?xf32, #spmd.addr_space<global>>, %N: index) -> f32 attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %z = arith.constant 0.0 : f32
  %r = "spmd.reduce"(%c0, %N, %c1, %z) ({
  ^bb0(%k: index):
    %v = memref.load %A[%k] : memref<?xf32, #spmd.addr_space<global>>
    "spmd.yield"(%v) : (f32) -> ()
  }) {"spmd.kind" = #spmd.reduction_kind<add>} : (index, index, index, f32) -> f32
  func.return %r : f32
}

func.func @max_then_add(%A: memref<?xf32>, %out: memref<f32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c64 = arith.constant 64 : index
  "spmd.forall"(%c0, %N, %c64) ({
  ^bb0(%t: index):
    %lo = arith.constant 0xFF800000 : f32
    %m = "spmd.reduce"(%c0, %c64, %c1, %lo) ({
    ^bb1(%l: index):
      %g = arith.addi %t, %l : index
      %v = memref.load %A[%g] : memref<?xf32>
      "spmd.yield"(%v) : (f32) -> ()
    }) {"spmd.kind" = #spmd.reduction_kind<max>} : (index, index, index, f32) -> f32
    memref.atomic_rmw addf %m, %out[] : (f32, memref<f32>) -> f32
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>} : (index, index, index) -> ()
  func.return
}

func.func @max_f32(%A: memref<?xf32>, %out: memref<f32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c64 = arith.constant 64 : index
  "spmd.forall"(%c0, %N, %c64) ({
  ^bb0(%t: index):
    %lo = arith.constant 0xFF800000 : f32
    %m = "spmd.reduce"(%c0, %c64, %c1, %lo) ({
    ^bb1(%l: index):
      %g = arith.addi %t, %l : index
      %v = memref.load %A[%g] : memref<?xf32>
      "spmd.yield"(%v) : (f32) -> ()
    }) {"spmd.kind" = #spmd.reduction_kind<max>} : (index, index, index, f32) -> f32
    memref.atomic_rmw maximumf %m, %out[] : (f32, memref<f32>) -> f32
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>} : (index, index, index) -> ()
  func.return
}

func.func @guarded(%A: memref<?xf32>, %N: index, %t: f32) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %v = memref.load %A[%i] : memref<?xf32>
    %c = arith.cmpf ogt, %v, %t : f32
    "spmd.if"(%c) ({
      memref.store %t, %A[%i] : memref<?xf32>
      "spmd.yield"() : () -> ()
    }, {
      "spmd.yield"() : () -> ()
    }) : (i1) -> ()
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}
'''


def test_forms_beyond_the_kernel_file():
    """Hexadecimal f32 literals, memref types with attributes, multi-region
    spmd.if (a guarded store), a returned top-level reduce, and per-tile
    results combined by an operation other than the reduction's own kind
    (reported, not mapped)."""
    shim = spmd_mod("mlir_shim")
    d = {x["function"]: x for x in shim.describe(_FORMS)}
    r = d["sum_returned"]
    assert r["pattern"] == "reduce" and r["output"] is None and r["combine"] == "return" and r["init"] == 0.0
    assert "not a single max reduction" in d["max_then_add"]["error"]
    assert d["max_f32"]["entry"] == "spmdb200_reduce_f32" and d["max_f32"]["kind"] == "max"
    assert d["guarded"]["pattern"] == "map" and d["guarded"]["output"] == "%A"  # a guarded store: a select
    assert shim._const_value("0xFF800000", "f32") == float("-inf")
    assert shim._const_value("0x7FC00000", "f32") != shim._const_value("0x7FC00000", "f32")  # NaN
    assert shim._const_value("0xFFFFFFFF", "i32") == -1
    assert shim._vals("%A: memref<?xf32, #spmd.addr_space<global>>, %N: index") == [
        "%A: memref<?xf32, #spmd.addr_space<global>>", "%N: index"]


def test_general_elementwise_bodies(oracle_mod):
    """Bodies beyond add / axpy map to the forall-map program; running the
    program through the oracle equals numpy evaluating the MLIR ops one by one."""
    import numpy as np
    d = _by_name()
    m = d["mul2d"]
    assert m["pattern"] == "map" and m["inputs"] == ["%A", "%B"] and m["n_regs"] == 2
    assert d["plus_one_from4"]["lower"] == [4] and d["plus_one_from4"]["consts"] == [1.0]
    assert d["clamp_tiled"]["consts"] == ["%lim"] and d["clamp_tiled"]["steps"] == [1]
    assert d["hypot3d"]["steps"] == [1, 1, 2] and d["hypot3d"]["rank"] == 3
    assert d["scale_in_place"]["inputs"] == ["%B"] and d["scale_in_place"]["output"] == "%B"
    rs = np.random.RandomState(3)
    x, y = rs.randn(4, 6, 10).astype(np.float32), rs.randn(4, 6, 10).astype(np.float32)
    h = d["hypot3d"]
    got = oracle_mod.forall_map([x[:, :, ::2], y[:, :, ::2]], (4, 6, 5), h["code"], h["consts"])
    xs, ys = x[:, :, ::2], y[:, :, ::2]
    r = np.sqrt(xs * xs + ys * ys)
    want = (np.maximum(r, np.abs(xs)) / r).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    c = d["clamp_tiled"]
    a = rs.uniform(-3, 3, 300).astype(np.float32)
    got = oracle_mod.forall_map([a], a.shape, c["code"], [1.5])
    assert np.array_equal(got, np.clip(a, np.float32(-1.5), np.float32(1.5)))


def test_empty_forall_maps_to_nothing():
    shim = spmd_mod("mlir_shim")
    text = """
func.func @nothing(%N: index) attributes {spmd.kernel} {
  %c2 = arith.constant 2 : index
  %c3 = arith.constant 3 : index
  "spmd.forall"(%c2, %N, %c3) ({
  ^bb0(%i: index):
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}
"""
    (d,) = shim.describe(text)
    assert d["pattern"] == "empty" and d["entry"] is None
    assert shim.load(text)["nothing"](10) is None


def test_guarded_stores_map_to_selects(oracle_mod):
    """`if (c) A[i] = t` is the in-place map A[i] = select(c, t, A[i]); an
    if / else pair storing to one place is select(c, then, else)."""
    import numpy as np
    d = _by_name()
    g = d["clamp_guarded"]
    assert g["pattern"] == "map" and g["inputs"] == ["%A"] and g["output"] == "%A" and g["consts"] == ["%t"]
    a = np.random.RandomState(31).uniform(-2, 2, 777).astype(np.float32)
    got = oracle_mod.forall_map([a], a.shape, g["code"], [0.5])
    assert np.array_equal(got, np.where(a > np.float32(0.5), np.float32(0.5), a))
    e = d["abs_if_else"]
    assert e["pattern"] == "map" and e["inputs"] == ["%A"] and e["output"] == "%B"
    m = np.random.RandomState(32).uniform(-2, 2, (9, 13)).astype(np.float32)
    got = oracle_mod.forall_map([m], m.shape, e["code"], e["consts"])
    assert np.array_equal(got.view(np.uint32), np.where(m >= 0, m, -m).astype(np.float32).view(np.uint32))


def test_spmd_if_value_is_a_select(oracle_mod):
    import numpy as np
    d = _by_name()["select_by_if"]
    assert d["pattern"] == "map" and d["inputs"] == ["%A", "%B"] and d["output"] == "%C"
    rs = np.random.RandomState(34)
    a, b = rs.randn(501).astype(np.float32), rs.randn(501).astype(np.float32)
    got = oracle_mod.forall_map([a, b], a.shape, d["code"], d["consts"])
    assert np.array_equal(got, np.where(a < b, b - a, a - b).astype(np.float32))


def test_nonlinear_stencils_map_as_shifted_views(oracle_mod):
    import numpy as np
    d = _by_name()
    mf = d["max_filter_interior"]
    assert mf["pattern"] == "map" and mf["inputs"] == ["%A"] * 3
    assert sorted(mf["input_offsets"]) == [[-1], [0], [1]] and mf["lower"] == [1]
    a = np.random.RandomState(36).randn(600).astype(np.float32)
    views = [a[1 + o[0]:599 + o[0]] for o in mf["input_offsets"]]
    got = oracle_mod.forall_map(views, (598,), mf["code"], mf["consts"])
    assert np.array_equal(got, np.maximum(a[:598], a[2:]) - a[1:599])
    up = d["upwind2d"]
    assert up["pattern"] == "map" and sorted(up["input_offsets"]) == [[-1, 0], [0, 0], [1, 0]]
    m = np.random.RandomState(37).randn(20, 30).astype(np.float32)
    views = [m[1 + o[0]:19 + o[0], o[1]:30 + o[1]] for o in up["input_offsets"]]
    got = oracle_mod.forall_map(views, (18, 30), up["code"], up["consts"])
    c = m[1:19]
    assert np.array_equal(got, np.where(c > 0, c - m[:18], m[2:] - c).astype(np.float32))
    bad = d["in_place_neighbour_unsupported"]
    assert bad["pattern"] is None and "also read at another point" in bad["error"]


def _one(body: str, args: str = "%A: memref<?xf32>, %B: memref<?xf32>, %N: index") -> dict:
    shim = spmd_mod("mlir_shim")
    text = f"""
func.func @k({args}) attributes {{spmd.kernel}} {{
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({{
  ^bb0(%i: index):
{body}
    "spmd.yield"() : () -> ()
  }}) {{operandSegmentSizes = array<i32: 1, 1, 1>}} : (index, index, index) -> ()
  func.return
}}
"""
    (d,) = shim.describe(text)
    return d


def test_map_bodies_the_shim_reports():
    fill = _one("""    %z = arith.constant 2.0 : f32
    memref.store %z, %B[%i] : memref<?xf32>""")
    assert fill["pattern"] is None and "fill" in fill["error"]
    f64 = _one("""    %a = memref.load %A[%i] : memref<?xf64>
    %b = arith.mulf %a, %a : f64
    memref.store %b, %B[%i] : memref<?xf64>""", "%A: memref<?xf64>, %B: memref<?xf64>, %N: index")
    assert f64["pattern"] is None
    i32 = _one("""    %a = memref.load %A[%i] : memref<?xi32>
    %b = arith.muli %a, %a : i32
    memref.store %b, %B[%i] : memref<?xi32>""", "%A: memref<?xi32>, %B: memref<?xi32>, %N: index")
    assert i32["pattern"] is None
    # 17 values live at once exceed the 16 registers of a body program
    loads = "\n".join(f"    %x{k} = memref.load %A{k}[%i] : memref<?xf32>" for k in range(8))
    muls = "\n".join(f"    %y{k} = arith.mulf %x{k}, %x{k} : f32" for k in range(8))
    tree = ["%y0"]
    chain = []
    for k in range(1, 8):
        chain.append(f"    %s{k} = arith.addf {tree[-1]}, %y{k} : f32")
        tree.append(f"%s{k}")
    big = _one(loads + "\n" + muls + "\n" + "\n".join(chain) + f"\n    memref.store {tree[-1]}, %B[%i] : memref<?xf32>",
               ", ".join(f"%A{k}: memref<?xf32>" for k in range(8)) + ", %B: memref<?xf32>, %N: index")
    assert big["pattern"] == "map" and big["n_regs"] <= 16  # the allocator reuses registers
    nine = "\n".join(f"    %x{k} = memref.load %A{k}[%i] : memref<?xf32>" for k in range(9))
    sums = ["%x0"]
    for k in range(1, 9):
        nine += f"\n    %t{k} = arith.addf {sums[-1]}, %x{k} : f32"
        sums.append(f"%t{k}")
    too_many = _one(nine + f"\n    memref.store {sums[-1]}, %B[%i] : memref<?xf32>",
                    ", ".join(f"%A{k}: memref<?xf32>" for k in range(9)) + ", %B: memref<?xf32>, %N: index")
    assert too_many["pattern"] is None and "inputs" in too_many["error"]


_TWO_OUTPUTS = r"""
func.func @two_outputs(%A: memref<?xf32>, %B: memref<?xf32>, %C: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %two = arith.constant 2.0 : f32
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %a = memref.load %A[%i] : memref<?xf32>
    %b = arith.mulf %a, %two : f32
    memref.store %b, %B[%i] : memref<?xf32>
    %bb = memref.load %B[%i] : memref<?xf32>
    %c = arith.addf %bb, %a : f32
    memref.store %c, %C[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}

func.func @stale_read(%A: memref<?xf32>, %B: memref<?xf32>, %C: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %old = memref.load %B[%i] : memref<?xf32>
    %a = memref.load %A[%i] : memref<?xf32>
    memref.store %a, %B[%i] : memref<?xf32>
    %c = arith.addf %old, %a : f32
    memref.store %c, %C[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}
"""


def test_several_outputs_run_as_maps_in_store_order(oracle_mod):
    """B = 2a; C = B + a (reading B after its store) runs as two maps in order;
    a load of B before B's store, used after it, is reported."""
    import numpy as np
    shim = spmd_mod("mlir_shim")
    d = {x["function"]: x for x in shim.describe(_TWO_OUTPUTS)}
    two = d["two_outputs"]
    assert two["pattern"] == "maps" and two["outputs"] == ["%B", "%C"]
    a = np.random.RandomState(39).randn(300).astype(np.float32)
    b = oracle_mod.forall_map([a], a.shape, two["maps"][0]["code"], two["maps"][0]["consts"])
    env = {"%A": a, "%B": b}
    m1 = two["maps"][1]
    c = oracle_mod.forall_map([env[x] for x in m1["inputs"]], a.shape, m1["code"], m1["consts"])
    assert np.array_equal(b, a * np.float32(2)) and np.array_equal(c, b + a)
    assert d["stale_read"]["pattern"] is None and "between a load" in d["stale_read"]["error"]


def test_map_binding_builds_views_before_the_device_call():
    """On the host the bound maps slice their views (offsets, lower bounds,
    several outputs) and check ranges; the device wrapper then refuses CPU
    tensors, so nothing runs without a GPU."""
    import torch
    shim = spmd_mod("mlir_shim")
    fns = shim.load((ROOT / "tests" / "mlir" / "kernels.mlir").read_text(), skip_unmapped=True)
    a, b = torch.zeros(600), torch.zeros(600)
    with pytest.raises(ValueError, match="CUDA"):
        fns["max_filter_interior"](a, b, 599)
    with pytest.raises(shim.ShimError, match="outside"):
        fns["max_filter_interior"](a, b, 601)
    with pytest.raises(ValueError, match="CUDA"):
        fns["mul2d"](torch.zeros(4, 5), torch.zeros(4, 5), torch.zeros(4, 5), 4, 5)
    two = shim.load(_TWO_OUTPUTS, skip_unmapped=True)["two_outputs"]
    with pytest.raises(ValueError, match="CUDA"):
        two(torch.zeros(8), torch.zeros(8), torch.zeros(8), 8)
