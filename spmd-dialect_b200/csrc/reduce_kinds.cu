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
#include <type_traits>

#include "internal.h"
#include "reduce_bulk.cuh"
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

// Set when a bounded wait of a staged kind reduction expires (read with the
// sums' flag by spmdb200_reduction_status).
__device__ int g_kind_timeout;

__device__ __forceinline__ float elem_as(float, uint32_t u) { return __uint_as_float(u); }

// Order-preserving integer key of an f32 (an involution): keys of non-NaN
// values compare like the values, with -0 below +0 (arith.maximumf /
// minimumf order).  NaNs of either sign fall outside [key(-inf), key(+inf)].
__device__ __forceinline__ int32_t f32_key(uint32_t bits) {
  const int32_t s = (int32_t)bits;
  return s ^ ((s >> 31) & 0x7fffffff);
}
__device__ __forceinline__ float f32_from_key(int32_t k) { return __int_as_float(k ^ ((k >> 31) & 0x7fffffff)); }
__device__ __forceinline__ int32_t elem_as(int32_t, uint32_t u) { return (int32_t)u; }

// Unit stride, 16-byte aligned input: the sums' shared-memory staging (each
// CTA, one per SM, pulls one contiguous range through the cp.async.bulk ring)
// with this kind's combine per thread, then the same warp / block / last-block
// tree as reduce_kind_kernel.  Each thread combines a fixed subset in a fixed
// order, so the result is deterministic for a given device.
template <typename T, int K>
__global__ void __launch_bounds__(kBulkThreads) reduce_kind_bulk_kernel(const T *__restrict__ a, int64_t n, T *out,
                                                                       T init, unsigned *ticket, void *partials_raw) {
  using O = KindOp<T, K>;
  using A = typename O::A;
  extern __shared__ __align__(128) unsigned char bulk_raw[];
  unsigned char *smem = bulk_raw + ((128u - (smem_u32(bulk_raw) & 127u)) & 127u);
  __shared__ uint64_t full[kBulkStages];
  __shared__ A sh[32];
  __shared__ A own;
  __shared__ int last, abort_flag;
  unsigned long long *words = static_cast<unsigned long long *>(partials_raw);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages; ++s) mbar_init(&full[s], 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  const int64_t units = n >> 2;
  int64_t lo, hi;
  cta_range(units, lo, hi);
  const uint4 *base = reinterpret_cast<const uint4 *>(a);
  if (threadIdx.x == 0) bulk_prefetch_head(base, lo, hi);
  __syncthreads();
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  // Start ticket: the block that starts last combines (see the staged sum).
  unsigned start = 0;
  if (threadIdx.x == 0) start = atomicAdd(ticket, 1u);
  // Four independent chains (one per element of a 16-byte unit): the f32
  // max/min combine is a long dependent sequence, and a single chain held
  // each stage long enough to slow the stream.  Combined in a fixed order.
  A acc;
  bool ok;
  if constexpr (std::is_same<T, float>::value && (K == 2 || K == 3)) {
    // f32 max / min as integer max and min over keys: the largest key (max)
    // or smallest (min) is the result unless a NaN was seen, which shows as
    // a key above key(+inf) or below key(-inf).
    int32_t hi_k = f32_key(0xff800000u), lo_k = f32_key(0x7f800000u);  // key(-inf), key(+inf)
    ok = bulk_stream(base, lo, hi, smem, full, &abort_flag, [&](uint4 v) {
      const int32_t a0 = f32_key(v.x), a1 = f32_key(v.y), a2 = f32_key(v.z), a3 = f32_key(v.w);
      hi_k = max(hi_k, max(max(a0, a1), max(a2, a3)));
      lo_k = min(lo_k, min(min(a0, a1), min(a2, a3)));
    });
    const bool nan = hi_k > f32_key(0x7f800000u) || lo_k < f32_key(0xff800000u);
    acc = nan ? __int_as_float(0x7fc00000) : f32_from_key(K == 2 ? hi_k : lo_k);
  } else {
    A acc0 = O::id(), acc1 = O::id(), acc2 = O::id(), acc3 = O::id();
    ok = bulk_stream(base, lo, hi, smem, full, &abort_flag, [&](uint4 v) {
      acc0 = O::op(acc0, O::in(elem_as(T(), v.x)));
      acc1 = O::op(acc1, O::in(elem_as(T(), v.y)));
      acc2 = O::op(acc2, O::in(elem_as(T(), v.z)));
      acc3 = O::op(acc3, O::in(elem_as(T(), v.w)));
    });
    acc = O::op(O::op(acc0, acc1), O::op(acc2, acc3));
  }
  if (!ok && threadIdx.x == 0) atomicExch(&g_kind_timeout, 1);
  if (blockIdx.x == gridDim.x - 1) {  // the n % 4 elements past the last 16-byte unit
    const int64_t t = (units << 2) + threadIdx.x;
    if (t < n) acc = O::op(acc, O::in(a[t]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = O::op(acc, shfl_xor(acc, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    A b = O::id();
    for (int w = 0; w < kBulkThreads / 32; ++w) b = O::op(b, sh[w]);
    last = (start == gridDim.x - 1);
    if (last)
      own = b;
    else
      st_relaxed_u64(words + blockIdx.x, partial_word(b));  // value and presence in one word: no fence
  }
  __syncthreads();
  if (!last) return;
  // The combiner: one thread per block partial polls its word, then the same
  // fixed tree (per-thread order, warp shuffles, warps in order); every word
  // read is cleared, so the workspace stays all-zero.
  A p = O::id();
  bool lost = false;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += kBulkThreads) {
    A v = own;
    if (i != (int)blockIdx.x) {
      const unsigned long long w = poll_partial(words + i);
      lost |= (w == 0ull);
      if (w)
        partial_value(w, v);
      else
        v = O::id();
      st_relaxed_u64(words + i, 0ull);
    }
    p = O::op(p, v);
  }
  if (lost) atomicExch(&g_kind_timeout, 1);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) p = O::op(p, shfl_xor(p, o));
  __syncthreads();  // thread 0 has finished reading sh[] above
  if (lane == 0) sh[warp] = p;
  __syncthreads();
  if (threadIdx.x == 0) {
    A t = O::id();
    for (int w = 0; w < kBulkThreads / 32; ++w) t = O::op(t, sh[w]);
    *out = O::fin(init, t);
    *ticket = 0u;
  }
}

template <typename T, int K>
cudaError_t launch_kind_bulk(const T *a, int64_t n, T *out, T init, void *ws, cudaStream_t s) {
  static int cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (cache[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(reduce_kind_bulk_kernel<T, K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kBulkSmem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reduce_kind_bulk_kernel<T, K>, kBulkThreads,
                                                      kBulkSmem) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    cache[dev] = per_sm * num_sms(dev);
  }
  const int64_t chunks = ((n >> 2) * 16 + kBulkChunk - 1) / kBulkChunk;  // at least one chunk per CTA
  int64_t g = chunks < 1 ? 1 : chunks;
  if (g > cache[dev]) g = cache[dev];
  if (g > kMaxCtas) g = kMaxCtas;
  unsigned *ticket = static_cast<unsigned *>(ws);
  void *partials = static_cast<char *>(ws) + 256;
  return launch_pdl(reduce_kind_bulk_kernel<T, K>, (unsigned)g, kBulkThreads, kBulkSmem, s, a, n, out, init, ticket,
                    partials);
}

template <typename T, int K>
cudaError_t launch_kind(const T *a, int64_t sa, int64_t n, T *out, T init, void *ws, cudaStream_t s) {
  if (sa == 1 && (reinterpret_cast<uintptr_t>(a) & 15u) == 0) return launch_kind_bulk<T, K>(a, n, out, init, ws, s);
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

int kind_timeout_flag(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kind_timeout, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_kind_timeout, &zero, sizeof(int));
  }
  return v;
}

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
