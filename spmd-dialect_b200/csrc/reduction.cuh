// reduction.cuh -- device bodies of the hierarchical spmd.reduce (add).
//
// ReduceToHierarchicalGPU (lib/Conversion/SPMDToGPU/SPMDToGPU.cpp:249-415)
// builds: a thread-strided local accumulation (:336-367), a blockDim-slot
// shared-memory scatter + barrier (:370-371), a log2(blockDim) halving tree
// with one barrier per level (:378-394) and one tx==0 atomic into the rank-0
// output (:397-408).  The B200 version keeps the three levels but replaces the
// tree with register shuffles: per-thread f64 accumulation over 128-bit loads,
// a 5-step __shfl_xor tree per warp, one shared-memory slot per warp, and a
// final warp combine -- one __syncthreads instead of nine.
#pragma once

#include "common.cuh"

namespace spmdb200 {

// Per-thread f64 sum of a[0..n) (stride sa) over the grid-stride slice of this
// thread.  Unit stride + 16-byte alignment takes the float4 path.
__device__ __forceinline__ double thread_sum_f64(const float *a, int64_t sa, int64_t n) {
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  double acc0 = 0.0, acc1 = 0.0;
  if (sa == 1 && ((uintptr_t)a & 15u) == 0) {
    const int64_t n4 = n >> 2;
    int64_t i = tid;
    for (; i + nth < n4; i += 2 * nth) {
      const float4 v0 = ld_stream_f4(a + 4 * i);
      const float4 v1 = ld_stream_f4(a + 4 * (i + nth));
      acc0 = __dadd_rn(acc0, (double)v0.x);
      acc1 = __dadd_rn(acc1, (double)v1.x);
      acc0 = __dadd_rn(acc0, (double)v0.y);
      acc1 = __dadd_rn(acc1, (double)v1.y);
      acc0 = __dadd_rn(acc0, (double)v0.z);
      acc1 = __dadd_rn(acc1, (double)v1.z);
      acc0 = __dadd_rn(acc0, (double)v0.w);
      acc1 = __dadd_rn(acc1, (double)v1.w);
    }
    if (i < n4) {
      const float4 v0 = ld_stream_f4(a + 4 * i);
      acc0 = __dadd_rn(acc0, (double)v0.x);
      acc0 = __dadd_rn(acc0, (double)v0.y);
      acc0 = __dadd_rn(acc0, (double)v0.z);
      acc0 = __dadd_rn(acc0, (double)v0.w);
    }
    const int64_t t = (n4 << 2) + tid;
    if (t < n) acc1 = __dadd_rn(acc1, (double)a[t]);
  } else {
    for (int64_t i = tid; i < n; i += nth) acc0 = __dadd_rn(acc0, (double)a[i * sa]);
  }
  return __dadd_rn(acc0, acc1);
}

// Block sum in a fixed order (deterministic for a fixed blockDim).  Any
// blockDim <= 1024; `sh` holds >= 32 doubles.  The total is valid in thread 0.
__device__ __forceinline__ double block_sum_f64(double v, double *sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  if ((blockDim.x & 31) == 0) {
    v = warp_sum_f64(v);
  } else {
    // Partial last warp: shuffle only among the lanes that exist.
    const int wlanes = (warp == nwarps - 1) ? (int)(blockDim.x - 32 * warp) : 32;
    const unsigned mask = (wlanes == 32) ? 0xffffffffu : ((1u << wlanes) - 1u);
    for (int o = 16; o > 0; o >>= 1) {
      const double other = __shfl_down_sync(mask, v, o);
      if (lane + o < wlanes) v = __dadd_rn(v, other);
    }
  }
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < nwarps; ++w) t = __dadd_rn(t, sh[w]);
  __syncthreads();  // sh may be reused by the caller
  return t;
}

// int32 (wrapping) per-thread + block sum; result valid in thread 0.
__device__ __forceinline__ uint32_t thread_sum_u32(const int32_t *a, int64_t sa, int64_t n) {
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t acc = 0;
  if (sa == 1 && ((uintptr_t)a & 15u) == 0) {
    const int64_t n4 = n >> 2;
    const int4 *a4 = reinterpret_cast<const int4 *>(a);
    int64_t i = tid;
    for (; i + nth < n4; i += 2 * nth) {
      const int4 v0 = __ldcs(a4 + i);
      const int4 v1 = __ldcs(a4 + i + nth);
      acc += (uint32_t)v0.x + (uint32_t)v0.y + (uint32_t)v0.z + (uint32_t)v0.w;
      acc += (uint32_t)v1.x + (uint32_t)v1.y + (uint32_t)v1.z + (uint32_t)v1.w;
    }
    if (i < n4) {
      const int4 v0 = __ldcs(a4 + i);
      acc += (uint32_t)v0.x + (uint32_t)v0.y + (uint32_t)v0.z + (uint32_t)v0.w;
    }
    const int64_t t = (n4 << 2) + tid;
    if (t < n) acc += (uint32_t)a[t];
  } else {
    for (int64_t i = tid; i < n; i += nth) acc += (uint32_t)a[i * sa];
  }
  return acc;
}

__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, uint32_t *sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  const int wlanes = (warp == nwarps - 1) ? (int)(blockDim.x - 32 * warp) : 32;
  const unsigned mask = (wlanes == 32) ? 0xffffffffu : ((1u << wlanes) - 1u);
  v = __reduce_add_sync(mask, v);  // redux.sync.add.u32
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  uint32_t t = 0;
  if (threadIdx.x == 0)
    for (int w = 0; w < nwarps; ++w) t += sh[w];
  __syncthreads();
  return t;
}

}  // namespace spmdb200
