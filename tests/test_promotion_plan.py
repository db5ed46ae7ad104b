"""The promotion plan (spmdb200_promotion_plan) against the reference's own
lit-test expectations for PromoteGroupMemory / PromotionPlanAnalysis.  Host
only: the plan needs no GPU."""
from __future__ import annotations

import pytest

from conftest import spmd_mod

BIG = 2 ** 62  # an offset the access analysis could not bound (INT64_MAX / 4 and up)


@pytest.mark.parametrize("tile,steps,mn,mx,ro,code,dims,nbytes,src", [
    # 3-point stencil, 32x8 tile, reads (0,0),(0,1),(1,0): memref<33x9xf32, group>
    ([32, 8], None, [0, 0], [1, 1], True, 0, (33, 9), 1188, "test/SPMD/promotion.mlir:59; promoted_e2e.mlir:29-38"),
    # stepped 1-D: tile 4, step 2, offsets 0 and 1 -> memref<8xf32, group>
    ([4], [2], [0], [1], True, 0, (8,), 32, "test/SPMD/promotion.mlir:163"),
    # positive-only halo A[i+1], A[i+2] -> memref<5xf32, group>
    ([4], None, [1], [2], True, 0, (5,), 20, "test/SPMD/promotion.mlir:215"),
    # negative-only halo A[i-2], A[i-1] -> memref<5xf32, group>
    ([4], None, [-2], [-1], True, 0, (5,), 20, "test/SPMD/promotion.mlir:260"),
    # oversized 2-D: 129 x 129 x 4 = 66,564 B > 49,152 B -> skipped
    ([128, 128], None, [0, 0], [1, 1], True, 3, (129, 129), 66564, "test/SPMD/promotion.mlir:296-301"),
    # oversized 1-D: tile 4096, offsets 0 and 12288 -> 16,384 x 4 = 65,536 B
    ([4096], None, [0], [12288], True, 3, (16384,), 65536, "test/SPMD/promote-group-memory-negative.mlir:147-170"),
    # no reuse: every lane reads its own element
    ([32, 8], None, [0, 0], [0, 0], True, 4, (32, 8), 1024, "test/SPMD/promotion.mlir:103"),
    # write conflict: the operand is also stored to
    ([32, 8], None, [0, 0], [1, 1], False, 2, None, None, "test/SPMD/promote-group-memory-negative.mlir:54-63"),
    # non-affine index: the analysis cannot bound the offsets
    ([32], None, [0], [BIG], True, 1, None, None, "test/SPMD/promote-group-memory-negative.mlir:15-23"),
])
def test_plan_matches_reference_lit_expectations(tile, steps, mn, mx, ro, code, dims, nbytes, src):
    k = spmd_mod("kernels")
    got, gdims, gbytes = k.promotion_plan(tile, mn, mx, steps=steps, read_only=ro)
    assert got == code, f"{src}: plan {k.PLAN_REASONS[got]}, expected {k.PLAN_REASONS[code]}"
    if dims is not None:
        assert gdims == dims and gbytes == nbytes, src


def test_plan_group_memory_limit_and_element_size():
    k = spmd_mod("kernels")
    assert k.promotion_plan([128, 128], [0, 0], [1, 1], max_group_bytes=96 * 1024)[0] == 0
    code, dims, nbytes = k.promotion_plan([32, 8], [0, 0], [1, 1], elem_bytes=8)
    assert (code, dims, nbytes) == (0, (33, 9), 2376)
    code, dims, _ = k.promotion_plan([8, 8, 4], [-1, -1, -1], [1, 1, 1])
    assert code == 0 and dims == (10, 10, 6)


def test_plan_rejects_bad_arguments():
    k = spmd_mod("kernels")
    L = spmd_mod("_lib")
    with pytest.raises(L.SpmdError):
        k.promotion_plan([1, 2, 3, 4], [0] * 4, [1] * 4)
