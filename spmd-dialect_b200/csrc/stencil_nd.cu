// stencil_nd.cu -- the general promoted-tile stencil: any rank 1-3, any tile
// sizes and steps, any list of read offsets, driven by the same promotion plan
// the reference's PromotionPlanAnalysis computes
// (lib/Analysis/PromotionPlanAnalysis.cpp:53-164):
//
//   footprint[d] = (tile[d] - 1) * step[d] + max_off[d] - min_off[d] + 1
//
// promoted when the offsets are bounded, the operand is read-only, the
// footprint fits the group-memory limit and some dimension has reuse
// (max_off > min_off).  A promoted launch stages each tile's footprint into
// shared memory (cooperative guarded copy, barrier, compute from the tile --
// PromoteGroupMemory.cpp:113-314); otherwise every lane reads global memory.
//
// The body is a linear stencil in source order:
//   t = w0 * A[p + off0];  t = t + wk * A[p + offk] (k = 1..);  B[p] = t * scale
// with the multiplies left out when the weights are all 1 (weights == NULL)
// or the scale is 1, so e.g. the 3-point promoted stencil and the Jacobi
// interiors are reproduced bit for bit.  Output points are p = k * step per
// dimension inside B's extents; reads outside A's extents are 0 (the
// reference leaves those tile slots unwritten).
#include "internal.h"

namespace spmdb200 {
namespace {

constexpr int kNdThreads = 256;
constexpr int kNdWarps = kNdThreads / 32;
// Footprint budget of one staged tile chosen by the kernel (a block holds two):
// three blocks of 256 threads fit one SM's shared memory.
constexpr int kNdTileBytes = 36 * 1024;

// Launch parameters.  Dimensions are outermost first and padded to 3 with
// extent-1 dimensions in front; the last dimension is the contiguous one.
// A kernel tile is kt[0] x kt[1] rows of kt[2] output points; each row is cut
// into segments of 32 * CPL points, and a "unit" (one row segment) is what a
// warp computes at once: CPL points per lane, 32 apart.
struct NdStencil {
  int ntaps, has_w, has_scale;
  float scale;
  long long a_size[3], a_stride[3], b_stride[3];
  long long npts[3];  // output points per dimension (ceil(b_size / step))
  long long tiles[3], ntiles;
  int step[3];
  int kt[3];    // output points per dimension of one kernel tile
  int fdim[3];  // footprint extent per dimension of one kernel tile
  int min_off[3], max_off[3];
  int vsplit;   // segments per tile row
  // Staged footprint layout (promoted): cell (i0, i1, c) at pad + i0 * pitch0
  // + i1 * pitch1 + c of a buffer of buf_cells floats.  With unit contiguous
  // strides the pitches are congruent to A's strides mod 4 and pad is the
  // element address of cell (0, 0, 0) mod 4, so every 16-byte chunk of A
  // lands on a 16-byte boundary of shared memory; otherwise the pitches are
  // dense and pad is 0.
  int pitch0, pitch1, buf_cells;
  // Promoted: offsets inside one tile fit 32 bits (checked on the host).
  int as0, as1;  // A strides of the two outer dimensions
  int bs0, bs1;  // B distance between neighbouring point rows (step * stride)
  int gstep[3];  // the grid size as tile coordinates (mixed radix tiles[0..2])
  // Rank-3 z-streaming (promoted, unit strides, z step 1): a work item is
  // kt[1] x kt[2] points of kz consecutive planes; its input planes pass
  // through a ring of `ring` slots of slot_cells floats, slot_cells
  // congruent to A's plane stride mod 4 and ring a multiple of 4, so the
  // 16-byte phase of every staged cell again matches A's.
  int kz, ring, slot_cells;
  float *b_base;       // B, and the elements it covers (1 + its largest offset): checked builds
  long long b_span;
  int tap_dz[kNdMaxTaps];  // off_j[0] - min_off[0]
  int tap_in[kNdMaxTaps];  // (off_j[1] - min_off[1]) * pitch1 + off_j[2] - min_off[2]
  int off[kNdMaxTaps][3];
  int tap_lin[kNdMaxTaps];         // (off_j - min_off) . (pitch0, pitch1, 1)
  long long tap_goff[kNdMaxTaps];  // off_j . a_stride
  float w[kNdMaxTaps];
};

__device__ __forceinline__ void cp_async4(uint32_t dst, const float *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const float *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// A block's current tile: its index t and coordinates (the contiguous
// dimension fastest).  Blocks step through the tiles by the grid size, added
// as a mixed-radix number so no division runs per tile; tile counts fit 32
// bits (checked on the host).
struct TileIter {
  unsigned t;
  int c[3];
  __device__ __forceinline__ void start(const NdStencil &k, unsigned t0) {
    const unsigned n2 = (unsigned)k.tiles[2], n1 = (unsigned)k.tiles[1];
    const unsigned q = t0 / n2;
    t = t0;
    c[2] = (int)(t0 - q * n2);
    c[1] = (int)(q % n1);
    c[0] = (int)(q / n1);
  }
  __device__ __forceinline__ void advance(const NdStencil &k) {
    t += gridDim.x;
    c[2] += k.gstep[2];
    int carry = c[2] >= (int)k.tiles[2];
    c[2] -= carry ? (int)k.tiles[2] : 0;
    c[1] += k.gstep[1] + carry;
    carry = c[1] >= (int)k.tiles[1];
    c[1] -= carry ? (int)k.tiles[1] : 0;
    c[0] += k.gstep[0] + carry;
  }
};

// A warp's contiguous share of a tile's units, as (i0, i1, seg) of its first
// unit and a count; the same for every tile, so decoded once per launch.
struct UnitRange {
  int i0, i1, seg, n;
};
__device__ __forceinline__ UnitRange warp_units(const NdStencil &k, int warp) {
  const int units = k.kt[0] * k.kt[1] * k.vsplit;
  const int per = (units + kNdWarps - 1) / kNdWarps;
  const int u0 = warp * per;
  UnitRange r;
  r.n = units - u0 < per ? (units - u0 > 0 ? units - u0 : 0) : per;
  const int row = u0 / k.vsplit;
  r.seg = u0 - row * k.vsplit;
  r.i0 = row / k.kt[1];
  r.i1 = row - r.i0 * k.kt[1];
  return r;
}
__device__ __forceinline__ void next_unit(const NdStencil &k, int &i0, int &i1, int &seg) {
  if (++seg == k.vsplit) {
    seg = 0;
    if (++i1 == k.kt[1]) {
      i1 = 0;
      ++i0;
    }
  }
}

// [lo, hi): the footprint cells of one dimension that lie inside A.
__device__ __forceinline__ void inside_range(long long base, long long size, int f, int &lo, int &hi) {
  lo = base >= 0 ? 0 : (int)(-base < f ? -base : f);
  const long long h = size - base;
  hi = h < 0 ? 0 : (h > f ? f : (int)h);
}

// One footprint row into shared memory, 4 bytes per copy (any contiguous
// stride): cp.async for the cells inside A (columns [c_lo, c_hi) of a row
// inside A), a plain 0 store for the rest.
__device__ __forceinline__ void stage_row(float *srow, const float *__restrict__ A, long long arow, long long s2a,
                                          int f2, int c_lo, int c_hi, bool row_in, int c0, int cstep) {
  if (!row_in) {
    for (int c = c0; c < f2; c += cstep) srow[c] = 0.0f;
  } else if (c_lo == 0 && c_hi == f2) {
    uint32_t dst = smem_u32(srow + c0);
    const float *src = A + (arow + c0 * s2a);
    for (int c = c0; c < f2; c += cstep, dst += 4u * cstep, src += cstep * s2a) cp_async4(dst, src);
  } else {
    for (int c = c0; c < f2; c += cstep) {
      if (c >= c_lo && c < c_hi)
        cp_async4(smem_u32(srow + c), A + (arow + c * s2a));
      else
        srow[c] = 0.0f;
    }
  }
}

// The same with unit stride, in 16-byte chunks: the cells before A's first
// 16-byte boundary in the row and after its last one go 4 bytes at a time
// (at most 3 each).  phase = element address of the row's cell 0, mod 4;
// srow + c and A + arow + c share their 16-byte phase.
__device__ __forceinline__ void stage_row16(float *srow, const float *__restrict__ A, long long arow, int phase,
                                            int f2, int c_lo, int c_hi, bool row_in, int c0, int cstep) {
  if (!row_in || c_hi <= c_lo) {
    for (int c = c0; c < f2; c += cstep) srow[c] = 0.0f;
    return;
  }
  for (int c = c0; c < c_lo; c += cstep) srow[c] = 0.0f;
  for (int c = c_hi + c0; c < f2; c += cstep) srow[c] = 0.0f;
  int h1 = c_lo + ((4 - ((phase + c_lo) & 3)) & 3);
  h1 = h1 < c_hi ? h1 : c_hi;
  const int nch = (c_hi - h1) >> 2, b1 = h1 + 4 * nch;
  if (c0 < h1 - c_lo) cp_async4(smem_u32(srow + c_lo + c0), A + (arow + c_lo + c0));
  if (c0 < c_hi - b1) cp_async4(smem_u32(srow + b1 + c0), A + (arow + b1 + c0));
  uint32_t dst = smem_u32(srow + h1) + 16u * c0;
  const float *src = A + (arow + h1 + 4 * c0);
#pragma unroll 2
  for (int q = c0; q < nch; q += cstep, dst += 16u * cstep, src += 4 * cstep) cp_async16(dst, src);
}

// Left fold of the taps in source order for CPL points 32 apart; `live`
// masks the points past the tile's last column (their slots are not read).
template <int CPL, bool GUARD, typename Load>
__device__ __forceinline__ void fold_taps(const NdStencil &k, Load ld, int nlive, float *acc) {
  for (int j = 0; j < k.ntaps; ++j) {
    float v[CPL];
#pragma unroll
    for (int u = 0; u < CPL; ++u) v[u] = (!GUARD || u < nlive) ? ld(j, u) : 0.0f;
    if (k.has_w) {
      const float w = k.w[j];
#pragma unroll
      for (int u = 0; u < CPL; ++u) v[u] = __fmul_rn(w, v[u]);
    }
    if (j == 0) {
#pragma unroll
      for (int u = 0; u < CPL; ++u) acc[u] = v[u];
    } else {
#pragma unroll
      for (int u = 0; u < CPL; ++u) acc[u] = __fadd_rn(acc[u], v[u]);
    }
  }
}

#ifdef SPMDB200_CHECKED
__device__ unsigned long long g_check_first;  // first out-of-range access (see common.cuh)
#endif

// One output store; a checked build skips (and records) a store outside B.
__device__ __forceinline__ void st_out(const NdStencil &k, float *p, float v) {
#ifdef SPMDB200_CHECKED
  const long long o = p - k.b_base;
  if (!record_check(&g_check_first, o >= 0 && o < k.b_span, 2, o)) return;
#endif
  *p = v;
}

template <int CPL, bool GUARD>
__device__ __forceinline__ void store_points(const NdStencil &k, float *bp, long long bstep, int nlive,
                                             const float *acc) {
#pragma unroll
  for (int u = 0; u < CPL; ++u)
    if (!GUARD || u < nlive) st_out(k, bp + u * bstep, k.has_scale ? __fmul_rn(acc[u], k.scale) : acc[u]);
}

__device__ __forceinline__ void tile_base(const NdStencil &k, const TileIter &it, long long *base) {
#pragma unroll
  for (int d = 0; d < 3; ++d) base[d] = (long long)it.c[d] * k.kt[d] * k.step[d] + k.min_off[d];
}

// Stages a tile's footprint into buf (cooperative, bounds-guarded copy) and
// returns the tile's pad.  Footprint rows go to warps (warp w: rows w, w + 8,
// ...; (r0, r1) is the warp's first row as (i0, i1)); a single row is spread
// over the whole block.
template <bool UNIT>
__device__ __forceinline__ int stage_tile(const NdStencil &k, const float *__restrict__ A, const TileIter &it,
                                          float *buf, int r0, int r1) {
  const int f0 = k.fdim[0], f1 = k.fdim[1], f2 = k.fdim[2];
#ifdef SPMDB200_CHECKED
  // Checked builds: every cell of the buffer starts as a NaN, so a read of a
  // cell that the staging below does not write shows up in the output.  The
  // caller's barrier released the buffer; all threads get here together.
  for (int i = threadIdx.x; i < k.buf_cells; i += kNdThreads) buf[i] = __int_as_float(0x7fc0dead);
  __syncthreads();
#endif
  const long long s2a = UNIT ? 1 : k.a_stride[2];
  long long base[3];  // A index of footprint cell (0, 0, 0)
  tile_base(k, it, base);
  int lo0, hi0, lo1, hi1, c_lo, c_hi;
  inside_range(base[0], k.a_size[0], f0, lo0, hi0);
  inside_range(base[1], k.a_size[1], f1, lo1, hi1);
  inside_range(base[2], k.a_size[2], f2, c_lo, c_hi);
  const long long a_cell0 = base[0] * k.a_stride[0] + base[1] * k.a_stride[1] + base[2] * s2a;
  const int pad = UNIT ? (int)(((long long)(reinterpret_cast<uintptr_t>(A) >> 2) + a_cell0) & 3) : 0;
  buf += pad;
  const bool flat = f0 * f1 == 1;
  const int c0 = flat ? (int)threadIdx.x : (int)(threadIdx.x & 31), cstep = flat ? kNdThreads : 32;
  for (int i0 = flat ? 0 : r0, i1 = flat ? 0 : r1; i0 < f0;) {
    const bool in = i0 >= lo0 && i0 < hi0 && i1 >= lo1 && i1 < hi1;
    const int roff = i0 * k.as0 + i1 * k.as1;
    float *srow = buf + i0 * k.pitch0 + i1 * k.pitch1;
    if (UNIT)
      stage_row16(srow, A, a_cell0 + roff, (pad + roff) & 3, f2, c_lo, c_hi, in, c0, cstep);
    else
      stage_row(srow, A, a_cell0 + roff, s2a, f2, c_lo, c_hi, in, c0, cstep);
    if (flat) break;
    for (i1 += kNdWarps; i1 >= f1; i1 -= f1) ++i0;
  }
  return pad;
}

// CPL points 32 apart from the staged tile: a left fold of the taps in
// source order per point, then the optional scale.
struct ParamTaps {  // tap offsets of the tiled kernels (kernel parameters)
  const NdStencil &k;
  __device__ __forceinline__ int operator()(int j) const { return k.tap_lin[j]; }
};
// NT > 0: the tap count as a compile-time constant (the tap loop unrolls and
// the offsets stay in registers); 0: k.ntaps at run time.
template <int CPL, int ST2, bool GUARD, typename Taps = ParamTaps, int NT = 0>
__device__ __forceinline__ void fold_staged(const NdStencil &k, const float *sp, int st2, int nlive, float *acc,
                                            Taps taps) {
  const int cs = 32 * (ST2 > 0 ? ST2 : st2);
  const int nt = NT > 0 ? NT : k.ntaps;
  const float *q = sp + taps(0);
  if (!k.has_w) {
#pragma unroll
    for (int u = 0; u < CPL; ++u) acc[u] = (!GUARD || u < nlive) ? q[u * cs] : 0.0f;
#pragma unroll (NT > 0 ? NT : 1)
    for (int j = 1; j < nt; ++j) {
      q = sp + taps(j);
#pragma unroll
      for (int u = 0; u < CPL; ++u) acc[u] = __fadd_rn(acc[u], (!GUARD || u < nlive) ? q[u * cs] : 0.0f);
    }
  } else {
    float w = k.w[0];
#pragma unroll
    for (int u = 0; u < CPL; ++u) acc[u] = __fmul_rn(w, (!GUARD || u < nlive) ? q[u * cs] : 0.0f);
#pragma unroll (NT > 0 ? NT : 1)
    for (int j = 1; j < nt; ++j) {
      q = sp + taps(j);
      w = k.w[j];
#pragma unroll
      for (int u = 0; u < CPL; ++u)
        acc[u] = __fadd_rn(acc[u], __fmul_rn(w, (!GUARD || u < nlive) ? q[u * cs] : 0.0f));
    }
  }
  if (k.has_scale) {
#pragma unroll
    for (int u = 0; u < CPL; ++u) acc[u] = __fmul_rn(acc[u], k.scale);
  }
}

// Promoted: a block stages its tiles' footprints in shared memory and
// computes each tile's points from there.  Two buffers: the next tile's copy
// is in flight while the current tile is computed.  UNIT: unit contiguous
// strides of A and B and step 1 along the contiguous dimension.
template <bool UNIT, int CPL>
__global__ void __launch_bounds__(kNdThreads, 3) stencil_nd_promoted_kernel(const float *__restrict__ A,
                                                                            float *__restrict__ B,
                                                                            const __grid_constant__ NdStencil k) {
  extern __shared__ __align__(16) float tile_buf[];
  constexpr int SEG = 32 * CPL;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kcols = k.kt[2];
  const int st2 = UNIT ? 1 : k.step[2];
  const int bcol = UNIT ? 1 : (int)(k.step[2] * k.b_stride[2]);  // B distance between neighbouring points
  const int ss0 = k.step[0] * k.pitch0, ss1 = k.step[1] * k.pitch1;  // tile_buf distance between point rows
  const UnitRange ur = warp_units(k, warp);
  const int r0 = warp / k.fdim[1], r1 = warp - r0 * k.fdim[1];  // this warp's first footprint row
  const unsigned ntiles = (unsigned)k.ntiles;
  TileIter cur, next;  // the tile computed in this iteration; the one staged during it
  cur.start(k, blockIdx.x);
  int pad = 0, pad_next = 0;
  if (cur.t < ntiles) pad = stage_tile<UNIT>(k, A, cur, tile_buf, r0, r1);
  asm volatile("cp.async.commit_group;" ::: "memory");
  next = cur;
  next.advance(k);
  for (int b = 0; cur.t < ntiles; b ^= 1) {
    if (next.t < ntiles) pad_next = stage_tile<UNIT>(k, A, next, tile_buf + (b ^ 1) * k.buf_cells, r0, r1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // cur's copies (all but the newest group)
    __syncthreads();
    const float *buf = tile_buf + b * k.buf_cells + pad;
    const long long pc0 = (long long)cur.c[2] * kcols;  // first output column of the tile
    const int ncols = k.npts[2] - pc0 < kcols ? (int)(k.npts[2] - pc0) : kcols;
    const long long p0t = (long long)cur.c[0] * k.kt[0], p1t = (long long)cur.c[1] * k.kt[1];
    const int rows0 = k.npts[0] - p0t < k.kt[0] ? (int)(k.npts[0] - p0t) : k.kt[0];  // point rows in the tile
    const int rows1 = k.npts[1] - p1t < k.kt[1] ? (int)(k.npts[1] - p1t) : k.kt[1];
    float *btile = B + (p0t * k.bs0 + p1t * k.bs1 + pc0 * bcol);
    int i0 = ur.i0, i1 = ur.i1, seg = ur.seg;
    for (int n = 0; n < ur.n; ++n, next_unit(k, i0, i1, seg)) {
      if (i0 >= rows0 || i1 >= rows1) continue;
      const int cb = seg * SEG + lane;  // this lane's first column in the tile
      const float *sp = buf + i0 * ss0 + i1 * ss1 + cb * st2;
      float *bp = btile + (i0 * k.bs0 + i1 * k.bs1 + cb * bcol);
      float acc[CPL];
      if (ncols - seg * SEG >= SEG) {
        fold_staged<CPL, UNIT ? 1 : 0, false>(k, sp, st2, CPL, acc, ParamTaps{k});
#pragma unroll
        for (int u = 0; u < CPL; ++u) st_out(k, bp + u * 32 * bcol, acc[u]);
      } else {
        // points of this lane before the tile's last column: lane + 32u < ncols - seg*SEG
        const int rem = ncols - seg * SEG - lane;
        const int nlive = rem <= 0 ? 0 : (rem + 31) / 32;
        if (nlive == 0) continue;
        fold_staged<CPL, UNIT ? 1 : 0, true>(k, sp, st2, nlive, acc, ParamTaps{k});
#pragma unroll
        for (int u = 0; u < CPL; ++u)
          if (u < nlive) st_out(k, bp + u * 32 * bcol, acc[u]);
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
    cur = next;
    pad = pad_next;
    next.advance(k);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Rank 3, promoted, unit strides, z step 1: each work item streams its
// input planes through a ring of shared-memory slots (cp.async 16-byte
// staging, one commit group per plane, PF planes in flight while one output
// plane is computed from the span0 + 1 planes in the ring).  A plane's
// halo rows and columns are staged once per plane rather than once per
// z-extent of a tile, so the staged cells per point drop from ~1.9 (tiles of
// 4 x 8 x 128) to ~1.16.
// NT > 0: the tap count at compile time (offsets of a plane's taps held in
// registers, the tap loop unrolled); 0: any tap count.
template <int CPL, int PF, int NT>
__global__ void __launch_bounds__(kNdThreads, 4) stencil_nd_stream3_kernel(const float *__restrict__ A,
                                                                           float *__restrict__ B,
                                                                           const __grid_constant__ NdStencil k) {
  extern __shared__ __align__(16) float ring[];
  // Tap offsets for each ring position of the output plane: s_toff[r][j] =
  // ((r + dz_j) mod ring) * slot_cells + in-plane offset of tap j.
  __shared__ int s_toff[16][kNdMaxTaps];
  constexpr int SEG = 32 * CPL;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int fy = k.fdim[1], fx = k.fdim[2], kcols = k.kt[2];
  const int R1 = k.ring - 1, S = k.slot_cells, span0 = k.max_off[0] - k.min_off[0];
  for (int i = threadIdx.x; i < k.ring * k.ntaps; i += kNdThreads) {
    const int r = i / k.ntaps, j = i - r * k.ntaps;
    s_toff[r][j] = ((r + k.tap_dz[j]) & R1) * S + k.tap_in[j];
  }
  const int ss1 = k.step[1] * k.pitch1;
  const long long bs0 = k.b_stride[0];
  // This warp's contiguous share of a plane's units (rows x segments).
  const int units = k.kt[1] * k.vsplit, per = (units + kNdWarps - 1) / kNdWarps, u0 = warp * per;
  const int nu = units - u0 < per ? (units - u0 > 0 ? units - u0 : 0) : per;
  const int row0 = u0 / k.vsplit, seg0 = u0 - row0 * k.vsplit;
  const int a0m4 = (int)(k.a_stride[0] & 3);
  TileIter it;
  it.start(k, blockIdx.x);
  for (; it.t < (unsigned)k.ntiles; it.advance(k)) {
    const long long z0 = (long long)it.c[0] * k.kz;  // first output plane of the item
    const int nz = k.npts[0] - z0 < k.kz ? (int)(k.npts[0] - z0) : k.kz;
    const long long gz0 = z0 + k.min_off[0];
    const long long gy0 = (long long)it.c[1] * k.kt[1] * k.step[1] + k.min_off[1];
    const long long gx0 = (long long)it.c[2] * kcols + k.min_off[2];
    int lo1, hi1, c_lo, c_hi;
    inside_range(gy0, k.a_size[1], fy, lo1, hi1);
    inside_range(gx0, k.a_size[2], fx, c_lo, c_hi);
    const long long a_cell0 = gz0 * k.a_stride[0] + gy0 * k.a_stride[1] + gx0;
    const int pad = (int)(((long long)(reinterpret_cast<uintptr_t>(A) >> 2) + a_cell0) & 3);
    const int np = nz + span0;  // input planes of the item
    auto stage_plane = [&](int p) {
      const long long gz = gz0 + p;
      const bool pin = gz >= 0 && gz < k.a_size[0];
      float *slot = ring + (p & R1) * S + pad;
      const long long aplane = a_cell0 + p * k.a_stride[0];
      const int pphase = pad + ((p * a0m4) & 3);
      for (int r = warp; r < fy; r += kNdWarps) {
        const bool in = pin && r >= lo1 && r < hi1;
        const int roff = r * k.as1;
        stage_row16(slot + r * k.pitch1, A, aplane + roff, (pphase + roff) & 3, fx, c_lo, c_hi, in, lane, 32);
      }
    };
    for (int p = 0; p < span0 + PF; ++p) {  // one commit group per plane, empty past the item
      if (p < np) stage_plane(p);
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    const long long p1t = (long long)it.c[1] * k.kt[1], pc0 = (long long)it.c[2] * kcols;
    const int rows1 = k.npts[1] - p1t < k.kt[1] ? (int)(k.npts[1] - p1t) : k.kt[1];
    const int ncols = k.npts[2] - pc0 < kcols ? (int)(k.npts[2] - pc0) : kcols;
    float *bplane = B + (z0 * bs0 + p1t * k.bs1 + pc0);
    for (int zo = 0; zo < nz; ++zo, bplane += bs0) {
      if (zo + span0 + PF < np) stage_plane(zo + span0 + PF);
      asm volatile("cp.async.commit_group;" ::: "memory");
      asm volatile("cp.async.wait_group %0;" ::"n"(PF) : "memory");  // planes up to zo + span0 have landed
      __syncthreads();
      const int *toff = s_toff[zo & R1];
      int toffr[NT > 0 ? NT : 1];
      if constexpr (NT > 0) {
#pragma unroll
        for (int j = 0; j < NT; ++j) toffr[j] = toff[j];
      }
      auto taps = [&](int j) {
        if constexpr (NT > 0)
          return toffr[j];
        else
          return toff[j];
      };
      int i1 = row0, seg = seg0;
      for (int n = 0; n < nu; ++n) {
        if (i1 < rows1) {
          const int cb = seg * SEG + lane;
          const float *sp = ring + pad + i1 * ss1 + cb;
          float *bp = bplane + (i1 * k.bs1 + cb);
          float acc[CPL];
          if (ncols - seg * SEG >= SEG) {
            fold_staged<CPL, 1, false, decltype(taps), NT>(k, sp, 1, CPL, acc, taps);
#pragma unroll
            for (int u = 0; u < CPL; ++u) st_out(k, bp + u * 32, acc[u]);
          } else {
            const int rem = ncols - seg * SEG - lane;
            const int nlive = rem <= 0 ? 0 : ((rem + 31) >> 5);
            if (nlive > 0) {
              fold_staged<CPL, 1, true, decltype(taps), NT>(k, sp, 1, nlive, acc, taps);
#pragma unroll
              for (int u = 0; u < CPL; ++u)
                if (u < nlive) st_out(k, bp + u * 32, acc[u]);
            }
          }
        }
        if (++seg == k.vsplit) {
          seg = 0;
          ++i1;
        }
      }
      __syncthreads();  // plane zo's slot is refilled in the next iteration
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
  }
}

// Not promoted: the same tiles, units and fold, every tap read from global
// memory (the caches catch the neighbours' reuse).  Units whose taps all land
// inside A read without per-point bounds checks.
template <bool UNIT, int CPL>
__global__ void __launch_bounds__(kNdThreads, 4) stencil_nd_direct_kernel(const float *__restrict__ A,
                                                                          float *__restrict__ B,
                                                                          const __grid_constant__ NdStencil k) {
  constexpr int SEG = 32 * CPL;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kcols = k.kt[2];
  const long long s2a = UNIT ? 1 : k.a_stride[2], s2b = UNIT ? 1 : k.b_stride[2];
  const int st2 = UNIT ? 1 : k.step[2];
  const long long bcol = (long long)st2 * s2b, acol = (long long)st2 * s2a;
  const UnitRange ur = warp_units(k, warp);
  TileIter it;
  it.start(k, blockIdx.x);
  for (; it.t < (unsigned)k.ntiles; it.advance(k)) {
    const long long pc0 = (long long)it.c[2] * kcols;
    const int ncols = k.npts[2] - pc0 < kcols ? (int)(k.npts[2] - pc0) : kcols;
    int i0 = ur.i0, i1 = ur.i1, seg = ur.seg;
    for (int n = 0; n < ur.n; ++n, next_unit(k, i0, i1, seg)) {
      const long long p0 = (long long)it.c[0] * k.kt[0] + i0, p1 = (long long)it.c[1] * k.kt[1] + i1;
      if (p0 >= k.npts[0] || p1 >= k.npts[1]) continue;
      const long long o0 = p0 * k.step[0], o1 = p1 * k.step[1];
      const long long c_first = pc0 + seg * SEG;  // the unit's first output column
      const int rem = ncols - seg * SEG - lane;
      const int nlive = rem <= 0 ? 0 : (rem + 31) / 32;
      if (nlive == 0) continue;
      const long long o2 = (c_first + lane) * st2;
      float *bp = B + o0 * k.b_stride[0] + o1 * k.b_stride[1] + o2 * s2b;
      const long long c_last = (c_first + (ncols - seg * SEG < SEG ? ncols - seg * SEG : SEG) - 1) * st2;
      const bool inside = o0 + k.min_off[0] >= 0 && o0 + k.max_off[0] < k.a_size[0] && o1 + k.min_off[1] >= 0 &&
                          o1 + k.max_off[1] < k.a_size[1] && c_first * st2 + k.min_off[2] >= 0 &&
                          c_last + k.max_off[2] < k.a_size[2];
      float acc[CPL];
      if (inside) {
        const float *ap = A + (o0 * k.a_stride[0] + o1 * k.a_stride[1] + o2 * s2a);
        auto ld = [&](int j, int u) { return __ldg(ap + k.tap_goff[j] + u * 32 * acol); };
        fold_taps<CPL, true>(k, ld, nlive, acc);
      } else {
        auto ld = [&](int j, int u) {
          const long long g0 = o0 + k.off[j][0], g1 = o1 + k.off[j][1], g2 = o2 + u * 32 * st2 + k.off[j][2];
          const bool in = g0 >= 0 && g0 < k.a_size[0] && g1 >= 0 && g1 < k.a_size[1] && g2 >= 0 && g2 < k.a_size[2];
          return in ? __ldg(A + (g0 * k.a_stride[0] + g1 * k.a_stride[1] + g2 * s2a)) : 0.0f;
        };
        fold_taps<CPL, true>(k, ld, nlive, acc);
      }
      store_points<CPL, true>(k, bp, 32 * bcol, nlive, acc);
    }
  }
}

template <typename K>
cudaError_t launch_grid(K kern, const NdStencil &k, size_t smem, const float *a, float *b, cudaStream_t s) {
  int dev = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (smem > 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
  }
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kNdThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const long long cap = (long long)per_sm * num_sms(dev);
  const long long g = k.ntiles < cap ? (k.ntiles > 0 ? k.ntiles : 1) : cap;
  NdStencil kl = k;
  kl.gstep[2] = (int)(g % kl.tiles[2]);
  kl.gstep[1] = (int)((g / kl.tiles[2]) % kl.tiles[1]);
  kl.gstep[0] = (int)(g / (kl.tiles[2] * kl.tiles[1]));
  kern<<<(unsigned)g, kNdThreads, smem, s>>>(a, b, kl);
  return cudaGetLastError();
}

long long footprint_cells(const int *kt, const int *step, const int *span) {
  long long n = 1;
  for (int d = 0; d < 3; ++d) n *= (long long)(kt[d] - 1) * step[d] + span[d] + 1;
  return n;
}

// Rank-3 z-streaming launch (see stencil_nd_stream3_kernel); returns
// cudaErrorNotSupported when the problem does not fit it.
#ifndef SPMDB200_STREAM3_PREFETCH
#define SPMDB200_STREAM3_PREFETCH 1  // planes in flight per block (2-4 measured slower: a larger ring costs blocks)
#endif
#ifndef SPMDB200_STREAM3_ROWS
#define SPMDB200_STREAM3_ROWS 16  // output rows of a work item
#endif
cudaError_t launch_stream3(NdStencil k, const int *span, const float *a, float *b, cudaStream_t s) {
  // Row segments of 128 or 256 points (4 or 8 per lane): the wider one when
  // it wastes no more of the last column tile (512^3 7-point: 2.9 vs
  // 2.4 TB/s; 320^3: 1.4 vs 1.8 TB/s, whose 320-point rows fill 128-point
  // tiles better).
  const long long nx = k.npts[2];
  const long long waste4 = ((nx + 127) / 128) * 128 - nx, waste8 = ((nx + 255) / 256) * 256 - nx;
  const int kCpl = waste8 <= waste4 ? 8 : 4;
  constexpr int kPf = SPMDB200_STREAM3_PREFETCH;
  // span0 + 1 planes read + kPf in flight, rounded up to a power of two >= 4
  // (slot indices are masked; a multiple of 4 keeps the 16-byte phase).
  const int need = span[0] + 1 + kPf;
  k.ring = need <= 4 ? 4 : (need <= 8 ? 8 : 16);
  k.kt[1] = (int)(k.npts[1] < SPMDB200_STREAM3_ROWS ? k.npts[1] : SPMDB200_STREAM3_ROWS);
  k.kt[2] = (int)(k.npts[2] < 32 * kCpl ? k.npts[2] : 32 * kCpl);
  for (;;) {
    k.fdim[1] = (k.kt[1] - 1) * k.step[1] + span[1] + 1;
    k.fdim[2] = k.kt[2] + span[2];
    k.pitch1 = k.fdim[2] + (int)((((k.a_stride[1] - k.fdim[2]) % 4) + 4) % 4);
    long long cells = (long long)k.fdim[1] * k.pitch1 + 3;
    cells += (((k.a_stride[0] - cells) % 4) + 4) % 4;
    k.slot_cells = (int)cells;
    if (cells * k.ring * 4 <= 64 * 1024) break;
    if (k.kt[1] > 1)
      k.kt[1] = (k.kt[1] + 1) / 2;
    else if (k.kt[2] > 1)
      k.kt[2] = (k.kt[2] + 1) / 2;
    else
      return cudaErrorNotSupported;
  }
  const long long a_ext = (long long)k.fdim[1] * k.a_stride[1] + k.pitch1;
  const long long b_ext = (long long)k.kt[1] * k.step[1] * k.b_stride[1] + k.kt[2];
  if (a_ext >= 0x7fffffffLL || b_ext >= 0x7fffffffLL) return cudaErrorNotSupported;
  k.as1 = (int)k.a_stride[1];
  k.bs1 = (int)(k.step[1] * k.b_stride[1]);
  k.fdim[0] = 1;
  k.kt[0] = 1;
  k.vsplit = (k.kt[2] + 32 * kCpl - 1) / (32 * kCpl);
  for (int j = 0; j < k.ntaps; ++j) {
    k.tap_dz[j] = k.off[j][0] - k.min_off[0];
    k.tap_in[j] = (k.off[j][1] - k.min_off[1]) * k.pitch1 + (k.off[j][2] - k.min_off[2]);
  }
  // Planes per item: long enough to amortise the span0-plane prologue, short
  // enough for about two items per resident block.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const long long tiles_yx = ((k.npts[1] + k.kt[1] - 1) / k.kt[1]) * ((k.npts[2] + k.kt[2] - 1) / k.kt[2]);
  const long long want_items = 2LL * 4 * num_sms(dev);
  long long kz = (k.npts[0] * tiles_yx + want_items - 1) / want_items;
  if (kz < 4LL * (span[0] + 1)) kz = 4LL * (span[0] + 1);
  if (kz > 64) kz = 64;
  if (kz > k.npts[0]) kz = k.npts[0];
  k.kz = (int)(kz > 0 ? kz : 1);
  k.tiles[0] = (k.npts[0] + k.kz - 1) / k.kz;
  k.tiles[1] = (k.npts[1] + k.kt[1] - 1) / k.kt[1];
  k.tiles[2] = (k.npts[2] + k.kt[2] - 1) / k.kt[2];
  k.ntiles = k.tiles[0] * k.tiles[1] * k.tiles[2];
  if (k.ntiles == 0) return cudaSuccess;
  if (k.ntiles > 0x7fffffffLL) return cudaErrorNotSupported;
  const size_t smem = (size_t)k.slot_cells * k.ring * sizeof(float);
  if (k.ntaps == 7)  // the 3-D star
    return kCpl == 8 ? launch_grid(stencil_nd_stream3_kernel<8, kPf, 7>, k, smem, a, b, s)
                     : launch_grid(stencil_nd_stream3_kernel<4, kPf, 7>, k, smem, a, b, s);
  return kCpl == 8 ? launch_grid(stencil_nd_stream3_kernel<8, kPf, 0>, k, smem, a, b, s)
                   : launch_grid(stencil_nd_stream3_kernel<4, kPf, 0>, k, smem, a, b, s);
}

}  // namespace

int promotion_plan(int rank, const int64_t *tile_sizes, const int64_t *steps, const int64_t *min_off,
                   const int64_t *max_off, int64_t elem_bytes, int64_t max_group_bytes, int read_only,
                   int64_t *tile_dims_out, int64_t *footprint_bytes_out) {
  if (rank < 1 || rank > 3 || !tile_sizes || !min_off || !max_off || elem_bytes < 1 || max_group_bytes < 0)
    return -1;
  const int64_t big = INT64_MAX / 4;
  for (int d = 0; d < rank; ++d)  // 1. bounded (statically decomposable) accesses
    if (max_off[d] >= big || min_off[d] <= -big || min_off[d] > max_off[d]) return kPlanSkipUnbounded;
  if (!read_only) return kPlanSkipReadWrite;  // 2. read-only operand
  int64_t bytes = elem_bytes;                 // 3. footprint per dimension
  for (int d = 0; d < rank; ++d) {
    const int64_t t = tile_sizes[d] > 0 ? tile_sizes[d] : 1;
    const int64_t s = (steps && steps[d] > 0) ? steps[d] : 1;
    const int64_t dim = (t - 1) * s + max_off[d] - min_off[d] + 1;
    if (tile_dims_out) tile_dims_out[d] = dim;
    bytes = (bytes > INT64_MAX / dim) ? INT64_MAX : bytes * dim;
  }
  if (footprint_bytes_out) *footprint_bytes_out = bytes;
  if (bytes > max_group_bytes) return kPlanSkipFootprint;  // 4. fits group memory
  for (int d = 0; d < rank; ++d)                           // 5. reuse across lanes
    if (max_off[d] > min_off[d]) return kPlanPromote;
  return kPlanSkipNoReuse;
}

int check_read_stencil_nd(unsigned long long *first) {
#ifdef SPMDB200_CHECKED
  if (!first) return 1;  // only asks whether this is a checked build
  unsigned long long v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_check_first, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_check_first, &z, sizeof(z)) != cudaSuccess)
    return -1;
  *first = v;
  return 1;
#else
  if (first) *first = 0;
  return 0;
#endif
}

cudaError_t launch_stencil_nd(const StencilNdProblem &p, int promote, cudaStream_t s) {
  // The plan decides whether to stage (on the caller's tile); the kernel then
  // stages its own, larger tiles -- staging changes where values are read
  // from, never the values.  Dimensions are right-aligned into 3 slots.
  NdStencil k{};
  k.b_base = p.b;
  k.b_span = 1;
  for (int q = 0; q < p.rank; ++q) k.b_span += (p.b_size[q] > 0 ? p.b_size[q] - 1 : 0) * p.b_stride[q];
  k.ntaps = p.ntaps;
  k.has_w = p.weights != nullptr;
  k.has_scale = p.scale != 1.0f;
  k.scale = p.scale;
  const int pad = 3 - p.rank;
  int span[3] = {0, 0, 0};
  for (int d = 0; d < 3; ++d) {
    const int q = d - pad;  // problem dimension, or < 0 for a padding dimension
    k.a_size[d] = q >= 0 ? p.a_size[q] : 1;
    k.a_stride[d] = q >= 0 ? p.a_stride[q] : 0;
    k.b_stride[d] = q >= 0 ? p.b_stride[q] : 0;
    k.step[d] = q >= 0 ? (int)p.step[q] : 1;
    k.npts[d] = q >= 0 ? (p.b_size[q] + p.step[q] - 1) / p.step[q] : 1;
    int mn = 0, mx = 0;
    for (int j = 0; j < p.ntaps; ++j) {
      const int o = q >= 0 ? (int)p.offsets[j * p.rank + q] : 0;
      k.off[j][d] = o;
      mn = (j == 0 || o < mn) ? o : mn;
      mx = (j == 0 || o > mx) ? o : mx;
    }
    k.min_off[d] = mn;
    k.max_off[d] = mx;
    span[d] = mx - mn;
  }
  for (int j = 0; j < p.ntaps; ++j) {
    k.w[j] = p.weights ? p.weights[j] : 1.0f;
    k.tap_goff[j] = k.off[j][0] * k.a_stride[0] + k.off[j][1] * k.a_stride[1] + k.off[j][2] * k.a_stride[2];
  }
  const bool unit = k.a_stride[2] == 1 && k.b_stride[2] == 1 && k.step[2] == 1;
  if (promote && p.rank == 3 && unit && k.step[0] == 1 && span[0] <= 6) {
    const cudaError_t e = launch_stream3(k, span, p.a, p.b, s);
    if (e != cudaErrorNotSupported) return e;
  }
  // Kernel tile: ~8K points per promoted tile (rows of 512 points, 16 per
  // lane; rank 3: 4 x 8 rows of 128), ~4K per direct one; never larger than
  // the grid of output points.  A promoted tile shrinks, outer dimensions
  // first, until its footprint fits the budget.
  static const int kPromoted[3][3] = {{1, 1, 8192}, {1, 16, 512}, {4, 8, 128}};
  static const int kDirect[3][3] = {{1, 1, 4096}, {1, 16, 256}, {4, 8, 128}};
  const int cpl = p.rank == 3 ? 4 : (promote ? 16 : 8);
  for (int d = 0; d < 3; ++d) {
    const long long want = (promote ? kPromoted : kDirect)[p.rank - 1][d];
    k.kt[d] = (int)(k.npts[d] < want ? (k.npts[d] > 0 ? k.npts[d] : 1) : want);
  }
  if (promote) {
    // A promoted plan's footprint fits group memory on the caller's tile, so
    // the footprint of a one-point tile (the shrinking's floor) fits too.
    int one[3] = {1, 1, 1};
    const long long floor_cells = footprint_cells(one, k.step, span);
    const long long budget_cells = floor_cells * 4 > kNdTileBytes ? floor_cells : kNdTileBytes / 4;
    while (footprint_cells(k.kt, k.step, span) > budget_cells) {
      int d = 0;
      while (d < 3 && k.kt[d] == 1) ++d;
      if (d == 3) break;
      k.kt[d] = d < 2 ? k.kt[d] - 1 : (k.kt[d] + 1) / 2;
    }
    for (int d = 0; d < 3; ++d) k.fdim[d] = (int)((long long)(k.kt[d] - 1) * k.step[d] + span[d] + 1);
    // Offsets inside a tile must fit 32 bits; otherwise read A directly
    // (identical values, no staging).
    const long long a_ext = (k.fdim[0] - 1) * k.a_stride[0] + (k.fdim[1] - 1) * k.a_stride[1] +
                            (long long)k.fdim[2] * k.a_stride[2];
    const long long b_ext = (long long)(k.kt[0] - 1) * k.step[0] * k.b_stride[0] +
                            (long long)(k.kt[1] - 1) * k.step[1] * k.b_stride[1] +
                            (long long)k.kt[2] * k.step[2] * k.b_stride[2];
    if (a_ext >= 0x7fffffffLL || b_ext >= 0x7fffffffLL) return launch_stencil_nd(p, 0, s);
    k.as0 = (int)k.a_stride[0];
    k.as1 = (int)k.a_stride[1];
    k.bs0 = (int)(k.step[0] * k.b_stride[0]);
    k.bs1 = (int)(k.step[1] * k.b_stride[1]);
    if (unit) {  // pitches congruent to A's strides mod 4 (see NdStencil); 3 cells of pad slack
      k.pitch1 = k.fdim[2] + (int)((((k.a_stride[1] - k.fdim[2]) % 4) + 4) % 4);
      const long long rows = (long long)k.fdim[1] * k.pitch1;
      k.pitch0 = (int)(rows + (((k.a_stride[0] - rows) % 4) + 4) % 4);
      k.buf_cells = (k.fdim[0] * k.pitch0 + 3 + 3) & ~3;
    } else {
      k.pitch1 = k.fdim[2];
      k.pitch0 = k.fdim[1] * k.fdim[2];
      k.buf_cells = (k.fdim[0] * k.pitch0 + 3) & ~3;
    }
    for (int j = 0; j < p.ntaps; ++j)
      k.tap_lin[j] = (k.off[j][0] - k.min_off[0]) * k.pitch0 + (k.off[j][1] - k.min_off[1]) * k.pitch1 +
                     (k.off[j][2] - k.min_off[2]);
  }
  k.vsplit = (k.kt[2] + 32 * cpl - 1) / (32 * cpl);
  k.ntiles = 1;
  for (int d = 0; d < 3; ++d) {
    k.tiles[d] = (k.npts[d] + k.kt[d] - 1) / k.kt[d];
    k.ntiles *= k.tiles[d];
  }
  if (k.ntiles == 0) return cudaSuccess;
  if (k.ntiles > 0x7fffffffLL) return cudaErrorInvalidValue;  // tile indices are 32-bit in the kernels
  if (promote) {
    const size_t smem = 2 * (size_t)k.buf_cells * sizeof(float);  // two buffers
    if (cpl == 16)
      return unit ? launch_grid(stencil_nd_promoted_kernel<true, 16>, k, smem, p.a, p.b, s)
                  : launch_grid(stencil_nd_promoted_kernel<false, 16>, k, smem, p.a, p.b, s);
    return unit ? launch_grid(stencil_nd_promoted_kernel<true, 4>, k, smem, p.a, p.b, s)
                : launch_grid(stencil_nd_promoted_kernel<false, 4>, k, smem, p.a, p.b, s);
  }
  if (cpl == 8)
    return unit ? launch_grid(stencil_nd_direct_kernel<true, 8>, k, 0, p.a, p.b, s)
                : launch_grid(stencil_nd_direct_kernel<false, 8>, k, 0, p.a, p.b, s);
  return unit ? launch_grid(stencil_nd_direct_kernel<true, 4>, k, 0, p.a, p.b, s)
              : launch_grid(stencil_nd_direct_kernel<false, 4>, k, 0, p.a, p.b, s);
}

}  // namespace spmdb200
