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
// Footprint budget of one staged tile chosen by the kernel: the six blocks of
// 256 threads the register file holds per SM fit its shared memory.
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
  int off[kNdMaxTaps][3];
  int tap_lin[kNdMaxTaps];         // (off_j - min_off) flattened over the footprint's extents
  long long tap_goff[kNdMaxTaps];  // off_j . a_stride
  float w[kNdMaxTaps];
};

__device__ __forceinline__ void cp_async4(uint32_t dst, const float *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Tile t -> tile coordinates (the contiguous dimension fastest); tile counts
// fit 32 bits (checked on the host).
__device__ __forceinline__ void tile_coords(const NdStencil &k, unsigned t, long long *tc) {
  const unsigned n2 = (unsigned)k.tiles[2], n1 = (unsigned)k.tiles[1];
  const unsigned q = t / n2;
  tc[2] = t - q * n2;
  tc[1] = q % n1;
  tc[0] = q / n1;
}

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

// One footprint row into shared memory: cp.async for the cells inside A
// (columns [c_lo, c_hi) of a row inside A), a plain 0 store for the rest.
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

template <int CPL, bool GUARD>
__device__ __forceinline__ void store_points(const NdStencil &k, float *bp, long long bstep, int nlive,
                                             const float *acc) {
#pragma unroll
  for (int u = 0; u < CPL; ++u)
    if (!GUARD || u < nlive) bp[u * bstep] = k.has_scale ? __fmul_rn(acc[u], k.scale) : acc[u];
}

// Promoted: each block iteration stages one kernel tile's footprint in shared
// memory (cooperative guarded copy, wait, barrier) and computes the tile's
// points from it.  UNIT: unit contiguous strides of A and B and step 1 along
// the contiguous dimension.
template <bool UNIT, int CPL>
__global__ void __launch_bounds__(kNdThreads, 5) stencil_nd_promoted_kernel(const float *__restrict__ A,
                                                                         float *__restrict__ B,
                                                                         const __grid_constant__ NdStencil k) {
  extern __shared__ float tile_buf[];
  constexpr int SEG = 32 * CPL;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f1 = k.fdim[1], f2 = k.fdim[2];
  const int frows = k.fdim[0] * f1, kcols = k.kt[2];
  const long long s2a = UNIT ? 1 : k.a_stride[2], s2b = UNIT ? 1 : k.b_stride[2];
  const int st2 = UNIT ? 1 : k.step[2];
  const long long bs0 = (long long)k.step[0] * k.b_stride[0], bs1 = (long long)k.step[1] * k.b_stride[1];
  const long long bcol = (long long)st2 * s2b;              // B distance between neighbouring points
  const int ss0 = k.step[0] * f1 * f2, ss1 = k.step[1] * f2;  // tile_buf distance between point rows
  const UnitRange ur = warp_units(k, warp);
  for (unsigned t = blockIdx.x; t < (unsigned)k.ntiles; t += gridDim.x) {
    long long tc[3];
    tile_coords(k, t, tc);
    long long base[3];  // A index of footprint cell 0
#pragma unroll
    for (int d = 0; d < 3; ++d) base[d] = tc[d] * k.kt[d] * k.step[d] + k.min_off[d];
    const long long gc0 = base[2];
    const int c_lo = gc0 >= 0 ? 0 : (int)(-gc0 < f2 ? -gc0 : f2);  // first column inside A
    const long long c_hi_l = k.a_size[2] - gc0;
    const int c_hi = c_hi_l < 0 ? 0 : (c_hi_l > f2 ? f2 : (int)c_hi_l);  // one past the last
    if (frows == 1) {  // one footprint row: the whole block spreads over it
      const bool in = base[0] >= 0 && base[0] < k.a_size[0] && base[1] >= 0 && base[1] < k.a_size[1];
      stage_row(tile_buf, A, base[0] * k.a_stride[0] + base[1] * k.a_stride[1] + gc0 * s2a, s2a, f2, c_lo, c_hi,
                in, threadIdx.x, kNdThreads);
    } else {
      for (int fr = warp; fr < frows; fr += kNdWarps) {
        const int i0 = fr / f1, i1 = fr - i0 * f1;
        const long long g0 = base[0] + i0, g1 = base[1] + i1;
        const bool in = g0 >= 0 && g0 < k.a_size[0] && g1 >= 0 && g1 < k.a_size[1];
        stage_row(tile_buf + fr * f2, A, g0 * k.a_stride[0] + g1 * k.a_stride[1] + gc0 * s2a, s2a, f2, c_lo, c_hi,
                  in, lane, 32);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const long long pc0 = tc[2] * kcols;  // first output column of the tile
    const int ncols = k.npts[2] - pc0 < kcols ? (int)(k.npts[2] - pc0) : kcols;
    const long long p0t = tc[0] * k.kt[0], p1t = tc[1] * k.kt[1];
    float *btile = B + p0t * bs0 + p1t * bs1 + pc0 * bcol;
    int i0 = ur.i0, i1 = ur.i1, seg = ur.seg;
    for (int n = 0; n < ur.n; ++n, next_unit(k, i0, i1, seg)) {
      if (p0t + i0 >= k.npts[0] || p1t + i1 >= k.npts[1]) continue;
      const int cb = seg * SEG + lane;  // this lane's first column in the tile
      const float *sp = tile_buf + i0 * ss0 + i1 * ss1 + cb * st2;
      float *bp = btile + i0 * bs0 + i1 * bs1 + cb * bcol;
      // points of this lane before the tile's last column: lane + 32u < ncols - seg*SEG
      const int rem = ncols - seg * SEG - lane;
      const int nlive = rem <= 0 ? 0 : (rem + 31) / 32;
      auto ld = [&](int j, int u) { return sp[k.tap_lin[j] + u * 32 * st2]; };
      float acc[CPL];
      if (ncols - seg * SEG >= SEG) {
        fold_taps<CPL, false>(k, ld, CPL, acc);
        store_points<CPL, false>(k, bp, 32 * bcol, CPL, acc);
      } else if (nlive > 0) {
        fold_taps<CPL, true>(k, ld, nlive, acc);
        store_points<CPL, true>(k, bp, 32 * bcol, nlive, acc);
      }
    }
    __syncthreads();
  }
}

// Not promoted: the same tiles, units and fold, every tap read from global
// memory (the caches catch the neighbours' reuse).  Units whose taps all land
// inside A read without per-point bounds checks.
template <bool UNIT, int CPL>
__global__ void __launch_bounds__(kNdThreads) stencil_nd_direct_kernel(const float *__restrict__ A,
                                                                       float *__restrict__ B,
                                                                       const __grid_constant__ NdStencil k) {
  constexpr int SEG = 32 * CPL;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kcols = k.kt[2];
  const long long s2a = UNIT ? 1 : k.a_stride[2], s2b = UNIT ? 1 : k.b_stride[2];
  const int st2 = UNIT ? 1 : k.step[2];
  const long long bcol = (long long)st2 * s2b, acol = (long long)st2 * s2a;
  const UnitRange ur = warp_units(k, warp);
  for (unsigned t = blockIdx.x; t < (unsigned)k.ntiles; t += gridDim.x) {
    long long tc[3];
    tile_coords(k, t, tc);
    const long long pc0 = tc[2] * kcols;
    const int ncols = k.npts[2] - pc0 < kcols ? (int)(k.npts[2] - pc0) : kcols;
    int i0 = ur.i0, i1 = ur.i1, seg = ur.seg;
    for (int n = 0; n < ur.n; ++n, next_unit(k, i0, i1, seg)) {
      const long long p0 = tc[0] * k.kt[0] + i0, p1 = tc[1] * k.kt[1] + i1;
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
  kern<<<(unsigned)g, kNdThreads, smem, s>>>(a, b, k);
  return cudaGetLastError();
}

long long footprint_cells(const int *kt, const int *step, const int *span) {
  long long n = 1;
  for (int d = 0; d < 3; ++d) n *= (long long)(kt[d] - 1) * step[d] + span[d] + 1;
  return n;
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

cudaError_t launch_stencil_nd(const StencilNdProblem &p, int promote, cudaStream_t s) {
  // The plan decides whether to stage (on the caller's tile); the kernel then
  // stages its own, larger tiles -- staging changes where values are read
  // from, never the values.  Dimensions are right-aligned into 3 slots.
  NdStencil k{};
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
  // Kernel tile: rows of 256 contiguous points (128 for rank 3) and ~4K points
  // per tile; halved, outer dimensions first, while the footprint exceeds the
  // budget (promoted only), and never larger than the grid of output points.
  const int cpl = p.rank == 3 ? 4 : 8;
  static const int kDefault[3][3] = {{1, 1, 4096}, {1, 16, 256}, {4, 8, 128}};
  for (int d = 0; d < 3; ++d) {
    const long long want = kDefault[p.rank - 1][d];
    k.kt[d] = (int)(k.npts[d] < want ? (k.npts[d] > 0 ? k.npts[d] : 1) : want);
  }
  if (promote) {
    // A promoted plan's footprint fits group memory on the caller's tile, so
    // the footprint of a one-point tile (the halving's floor) fits too.
    int one[3] = {1, 1, 1};
    const long long floor_cells = footprint_cells(one, k.step, span);
    const long long budget_cells = floor_cells * 4 > kNdTileBytes ? floor_cells : kNdTileBytes / 4;
    while (footprint_cells(k.kt, k.step, span) > budget_cells) {
      int d = 0;
      while (d < 3 && k.kt[d] == 1) ++d;
      if (d == 3) break;
      k.kt[d] = (k.kt[d] + 1) / 2;
    }
    for (int d = 0; d < 3; ++d) k.fdim[d] = (int)((long long)(k.kt[d] - 1) * k.step[d] + span[d] + 1);
    for (int j = 0; j < p.ntaps; ++j)
      k.tap_lin[j] = ((k.off[j][0] - k.min_off[0]) * k.fdim[1] + (k.off[j][1] - k.min_off[1])) * k.fdim[2] +
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
  const bool unit = k.a_stride[2] == 1 && k.b_stride[2] == 1 && k.step[2] == 1;
  const size_t smem = promote ? (size_t)footprint_cells(k.kt, k.step, span) * sizeof(float) : 0;
#define SPMD_ND_LAUNCH(KERN)                                                                     \
  (cpl == 8 ? (unit ? launch_grid(KERN<true, 8>, k, smem, p.a, p.b, s)                           \
                    : launch_grid(KERN<false, 8>, k, smem, p.a, p.b, s))                         \
            : (unit ? launch_grid(KERN<true, 4>, k, smem, p.a, p.b, s)                           \
                    : launch_grid(KERN<false, 4>, k, smem, p.a, p.b, s)))
  const cudaError_t e = promote ? SPMD_ND_LAUNCH(stencil_nd_promoted_kernel) : SPMD_ND_LAUNCH(stencil_nd_direct_kernel);
#undef SPMD_ND_LAUNCH
  return e;
}

}  // namespace spmdb200
