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

struct NdStencil {
  int rank, ntaps, promoted, has_w, has_scale;
  float scale;
  long long a_size[3], a_stride[3], b_size[3], b_stride[3];
  long long step[3], npts[3];  // output points per dimension
  long long tiles[3], ntiles;  // tiles per dimension (row-major, last fastest)
  int tile[3], fdim[3], min_off[3];
  long long fcount, tcount;    // footprint cells, lanes per tile
  int off[kNdMaxTaps][3];
  float w[kNdMaxTaps];
};

__device__ __forceinline__ float nd_tap(const NdStencil &k, int j, float a) {
  return k.has_w ? __fmul_rn(k.w[j], a) : a;
}

// Promoted: one tile per block iteration, footprint staged in shared memory.
__global__ void __launch_bounds__(kNdThreads) stencil_nd_promoted_kernel(const float *__restrict__ A,
                                                                         float *__restrict__ B,
                                                                         const __grid_constant__ NdStencil k) {
  extern __shared__ float tile_buf[];
  for (long long t = blockIdx.x; t < k.ntiles; t += gridDim.x) {
    long long tc[3] = {0, 0, 0}, rem = t;
    for (int d = k.rank - 1; d >= 0; --d) {
      tc[d] = rem % k.tiles[d];
      rem /= k.tiles[d];
    }
    long long origin[3] = {0, 0, 0}, base[3] = {0, 0, 0};
    for (int d = 0; d < k.rank; ++d) {
      origin[d] = tc[d] * k.tile[d] * k.step[d];  // output index of lane 0
      base[d] = origin[d] + k.min_off[d];         // A index of footprint cell 0
    }
    // Cooperative guarded copy of the footprint.
    for (long long e = threadIdx.x; e < k.fcount; e += blockDim.x) {
      long long r = e, aoff = 0;
      bool in = true;
      for (int d = k.rank - 1; d >= 0; --d) {
        const long long f = r % k.fdim[d];
        r /= k.fdim[d];
        const long long g = base[d] + f;
        in = in && g >= 0 && g < k.a_size[d];
        aoff += g * k.a_stride[d];
      }
      tile_buf[e] = in ? A[aoff] : 0.0f;
    }
    __syncthreads();
    // Compute from the tile.
    for (long long l = threadIdx.x; l < k.tcount; l += blockDim.x) {
      long long r = l, li[3] = {0, 0, 0}, boff = 0;
      bool in = true;
      for (int d = k.rank - 1; d >= 0; --d) {
        li[d] = r % k.tile[d];
        r /= k.tile[d];
        const long long o = origin[d] + li[d] * k.step[d];
        in = in && o < k.b_size[d];
        boff += o * k.b_stride[d];
      }
      if (!in) continue;
      float acc = 0.0f;
      for (int j = 0; j < k.ntaps; ++j) {
        long long s = 0;
        for (int d = 0; d < k.rank; ++d) s = s * k.fdim[d] + (li[d] * k.step[d] + k.off[j][d] - k.min_off[d]);
        const float v = nd_tap(k, j, tile_buf[s]);
        acc = j == 0 ? v : __fadd_rn(acc, v);
      }
      B[boff] = k.has_scale ? __fmul_rn(acc, k.scale) : acc;
    }
    __syncthreads();
  }
}

// Not promoted: every output point reads global memory directly.
__global__ void __launch_bounds__(kNdThreads) stencil_nd_direct_kernel(const float *__restrict__ A,
                                                                       float *__restrict__ B,
                                                                       const __grid_constant__ NdStencil k) {
  const long long total = k.npts[0] * k.npts[1] * k.npts[2];
  for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < total;
       p += (long long)gridDim.x * blockDim.x) {
    long long r = p, o[3] = {0, 0, 0}, boff = 0;
    for (int d = k.rank - 1; d >= 0; --d) {
      o[d] = (r % k.npts[d]) * k.step[d];
      r /= k.npts[d];
      boff += o[d] * k.b_stride[d];
    }
    float acc = 0.0f;
    for (int j = 0; j < k.ntaps; ++j) {
      long long aoff = 0;
      bool in = true;
      for (int d = 0; d < k.rank; ++d) {
        const long long g = o[d] + k.off[j][d];
        in = in && g >= 0 && g < k.a_size[d];
        aoff += g * k.a_stride[d];
      }
      const float v = nd_tap(k, j, in ? A[aoff] : 0.0f);
      acc = j == 0 ? v : __fadd_rn(acc, v);
    }
    B[boff] = k.has_scale ? __fmul_rn(acc, k.scale) : acc;
  }
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
  NdStencil k{};
  k.rank = p.rank;
  k.ntaps = p.ntaps;
  k.has_w = p.weights != nullptr;
  k.has_scale = p.scale != 1.0f;
  k.scale = p.scale;
  int64_t mn[3] = {0, 0, 0}, mx[3] = {0, 0, 0};
  for (int d = 0; d < 3; ++d) {
    const bool live = d < p.rank;
    k.a_size[d] = live ? p.a_size[d] : 1;
    k.a_stride[d] = live ? p.a_stride[d] : 0;
    k.b_size[d] = live ? p.b_size[d] : 1;
    k.b_stride[d] = live ? p.b_stride[d] : 0;
    k.step[d] = live ? p.step[d] : 1;
    k.npts[d] = live ? (p.b_size[d] + p.step[d] - 1) / p.step[d] : 1;
    k.tile[d] = live ? (int)p.tile[d] : 1;
    mn[d] = mx[d] = live ? p.offsets[d] : 0;
  }
  for (int j = 0; j < p.ntaps; ++j)
    for (int d = 0; d < 3; ++d) {
      k.off[j][d] = d < p.rank ? (int)p.offsets[j * p.rank + d] : 0;
      if (d < p.rank) {
        mn[d] = k.off[j][d] < mn[d] ? k.off[j][d] : mn[d];
        mx[d] = k.off[j][d] > mx[d] ? k.off[j][d] : mx[d];
      }
    }
  for (int j = 0; j < p.ntaps; ++j) k.w[j] = p.weights ? p.weights[j] : 1.0f;
  k.fcount = 1;
  k.tcount = 1;
  k.ntiles = 1;
  for (int d = 0; d < 3; ++d) {
    k.min_off[d] = (int)mn[d];
    k.fdim[d] = (int)((k.tile[d] - 1) * k.step[d] + mx[d] - mn[d] + 1);
    k.tiles[d] = (k.npts[d] + k.tile[d] - 1) / k.tile[d];
    k.fcount *= k.fdim[d];
    k.tcount *= k.tile[d];
    k.ntiles *= k.tiles[d];
  }
  k.promoted = promote;
  int dev = 0;
  cudaGetDevice(&dev);
  const long long cap = (long long)num_sms(dev) * 8;
  if (promote) {
    const size_t smem = (size_t)k.fcount * 4;
    cudaError_t e = cudaFuncSetAttribute(stencil_nd_promoted_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    long long g = k.ntiles < cap ? k.ntiles : cap;
    if (g < 1) g = 1;
    stencil_nd_promoted_kernel<<<(unsigned)g, kNdThreads, smem, s>>>(p.a, p.b, k);
  } else {
    const long long total = k.npts[0] * k.npts[1] * k.npts[2];
    long long g = (total + kNdThreads - 1) / kNdThreads;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    stencil_nd_direct_kernel<<<(unsigned)g, kNdThreads, 0, s>>>(p.a, p.b, k);
  }
  return cudaGetLastError();
}

}  // namespace spmdb200
