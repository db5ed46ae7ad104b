// reduce_kinds.cu -- spmd.reduce for every reduction kind of the dialect
// (add, mul, max, min, and, or, xor; include/spmd/IR/SPMDAttrs.td:74-80).
//
// The reference lowers only f32 add hierarchically; every other kind or type
// goes through ReduceToSCFForGPU (lib/Conversion/SPMDToGPU/SPMDToGPU.cpp:
// 422-477), a serial scf.for with the combine of :425-449.  Here every kind
// gets the hierarchical shape: per-thread combine over a grid-stride slice,
// a warp shuffle tree, a block tree through shared memory, and a grid
// combine by the last block to finish (ticket), in block order -- so the
// result is deterministic for a given device.  Integer kinds and f32
// max/min are exact in any order; f32 add and mul accumulate in f64 and round
// once (reassociated, which the dialect allows for floating-point add/mul,
// include/spmd/IR/SPMDAttrs.td:94-97).
//
// f32 max/min follow arith.maximumf / arith.minimumf: a NaN operand gives NaN,
// and -0 orders below +0.  i32 max/min are signed (arith.maxsi / minsi); i32
// add/mul wrap like arith.addi / muli.
#include <cmath>

#include "internal.h"
#include "reduction.cuh"

namespace spmdb200 {
namespace {

constexpr int kKindThreads = 256;

__device__ __forceinline__ float f_maximum(float a, float b) {
  if (isnan(a) || isnan(b)) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
__device__ __forceinline__ float f_minimum(float a, float b) {
  if (isnan(a) || isnan(b)) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

// Accumulator type and combine for each (element type, kind).
template <typename T, int K>
struct KindOp;
template <>
struct KindOp<float, 0> {  // add: f64 accumulation
  using A = double;
  static __device__ A id() { return -0.0; }
  static __device__ A in(float x) { return (double)x; }
  static __device__ A op(A a, A b) { return __dadd_rn(a, b); }
  static __device__ float fin(float init, A t) { return __double2float_rn(__dadd_rn((double)init, t)); }
};
template <>
struct KindOp<float, 1> {  // mul: f64 accumulation, one rounding (an f32 chain drifts ~sqrt(N) ulps)
  using A = double;
  static __device__ A id() { return 1.0; }
  static __device__ A in(float x) { return (double)x; }
  static __device__ A op(A a, A b) { return __dmul_rn(a, b); }
  static __device__ float fin(float init, A t) { return __double2float_rn(__dmul_rn((double)init, t)); }
};
template <>
struct KindOp<float, 2> {
  using A = float;
  static __device__ A id() { return -INFINITY; }
  static __device__ A in(float x) { return x; }
  static __device__ A op(A a, A b) { return f_maximum(a, b); }
  static __device__ float fin(float init, A t) { return f_maximum(init, t); }
};
template <>
struct KindOp<float, 3> {
  using A = float;
  static __device__ A id() { return INFINITY; }
  static __device__ A in(float x) { return x; }
  static __device__ A op(A a, A b) { return f_minimum(a, b); }
  static __device__ float fin(float init, A t) { return f_minimum(init, t); }
};
template <int K>
struct KindOp<int32_t, K> {
  using A = uint32_t;  // two's-complement arithmetic without signed-overflow UB
  static __device__ A id() {
    return K == 1 ? 1u : K == 2 ? 0x80000000u : K == 3 ? 0x7fffffffu : K == 4 ? 0xffffffffu : 0u;
  }
  static __device__ A in(int32_t x) { return (uint32_t)x; }
  static __device__ A op(A a, A b) {
    switch (K) {
      case 0: return a + b;
      case 1: return a * b;
      case 2: return (int32_t)a >= (int32_t)b ? a : b;
      case 3: return (int32_t)a <= (int32_t)b ? a : b;
      case 4: return a & b;
      case 5: return a | b;
      default: return a ^ b;
    }
  }
  static __device__ int32_t fin(int32_t init, A t) { return (int32_t)op((uint32_t)init, t); }
};

template <typename A>
__device__ __forceinline__ A shfl_xor(A v, int o) {
  return __shfl_xor_sync(0xffffffffu, v, o);
}

template <typename T, int K>
__global__ void __launch_bounds__(kKindThreads) reduce_kind_kernel(const T *__restrict__ a, int64_t sa, int64_t n,
                                                                   T *out, T init, unsigned *ticket, void *partials_raw) {
  using O = KindOp<T, K>;
  using A = typename O::A;
  __shared__ A sh[32];
  __shared__ int last;
  A *partials = static_cast<A *>(partials_raw);
  pdl_wait();  // launched with programmatic dependent launch: nothing global before this
  if (threadIdx.x == 0) pdl_trigger();
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  A acc = O::id();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += nth) acc = O::op(acc, O::in(a[i * sa]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = O::op(acc, shfl_xor(acc, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    A b = O::id();
    for (int w = 0; w < kKindThreads / 32; ++w) b = O::op(b, sh[w]);
    partials[blockIdx.x] = b;
    __threadfence();
    last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (warp == 0) {
    A p = O::id();
    for (int i = lane; i < (int)gridDim.x; i += 32) {
      p = O::op(p, __ldcg(partials + i));
      partials[i] = A(0);  // the workspace is shared with the sums, which read a non-zero word as written
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) p = O::op(p, shfl_xor(p, o));
    if (lane == 0) {
      *out = O::fin(init, p);
      *ticket = 0u;
    }
  }
}

template <typename T, int K>
cudaError_t launch_kind(const T *a, int64_t sa, int64_t n, T *out, T init, void *ws, cudaStream_t s) {
  static int cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int cap = num_sms(dev) * 4;
  if (dev >= 0 && dev < 64) {
    if (cache[dev] == 0) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reduce_kind_kernel<T, K>, kKindThreads, 0) !=
              cudaSuccess ||
          per_sm < 1)
        per_sm = 4;
      cache[dev] = per_sm * num_sms(dev);
    }
    cap = cache[dev];
  }
  int64_t g = (n + kKindThreads * 8 - 1) / (kKindThreads * 8);
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  if (g > kMaxCtas) g = kMaxCtas;
  unsigned *ticket = static_cast<unsigned *>(ws);
  void *partials = static_cast<char *>(ws) + 256;
  return launch_pdl(reduce_kind_kernel<T, K>, (unsigned)g, kKindThreads, 0, s, a, sa, n, out, init, ticket, partials);
}

}  // namespace

cudaError_t launch_reduce_f32(int kind, const float *a, int64_t sa, int64_t n, float *out, float init, void *ws,
                              cudaStream_t s) {
  switch (kind) {
    case 0: return launch_kind<float, 0>(a, sa, n, out, init, ws, s);
    case 1: return launch_kind<float, 1>(a, sa, n, out, init, ws, s);
    case 2: return launch_kind<float, 2>(a, sa, n, out, init, ws, s);
    case 3: return launch_kind<float, 3>(a, sa, n, out, init, ws, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_reduce_i32(int kind, const int32_t *a, int64_t sa, int64_t n, int32_t *out, int32_t init,
                              void *ws, cudaStream_t s) {
  switch (kind) {
    case 0: return launch_kind<int32_t, 0>(a, sa, n, out, init, ws, s);
    case 1: return launch_kind<int32_t, 1>(a, sa, n, out, init, ws, s);
    case 2: return launch_kind<int32_t, 2>(a, sa, n, out, init, ws, s);
    case 3: return launch_kind<int32_t, 3>(a, sa, n, out, init, ws, s);
    case 4: return launch_kind<int32_t, 4>(a, sa, n, out, init, ws, s);
    case 5: return launch_kind<int32_t, 5>(a, sa, n, out, init, ws, s);
    case 6: return launch_kind<int32_t, 6>(a, sa, n, out, init, ws, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace spmdb200
