// reduce.cu -- library launches of spmd.reduce add (f32 deterministic, i32
// exact, and the reference's one-atomic-per-block form).
#include "internal.h"
#include "reduce_bulk.cuh"
#include "reduction.cuh"

namespace spmdb200 {

constexpr int kSumThreads = 256;
constexpr size_t kSumWsHeader = 256;  // ticket + padding, partials follow

// Resident blocks of `kernel` on the device (blocks per SM x SM count), so a
// reduction grid is exactly one wave: no half-empty second wave at the tail.
template <class K>
static int resident_blocks(K kernel, int dev, int *cache) {
  if (dev < 0 || dev >= 64) return num_sms(dev) * 4;
  if (cache[dev] == 0) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kSumThreads, 0) != cudaSuccess || per_sm < 1)
      per_sm = 4;
    cache[dev] = per_sm * num_sms(dev);
  }
  return cache[dev];
}

template <class K>
static int reduce_grid(K kernel, int *cache, int64_t n) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t cap = resident_blocks(kernel, dev, cache);
  int64_t want = (n + kSumThreads * 16 - 1) / (kSumThreads * 16);
  if (want < 1) want = 1;
  if (want > cap) want = cap;
  if (want > kMaxCtas) want = kMaxCtas;
  return (int)want;
}

size_t sum_f32_workspace_bytes(int64_t n) {
  (void)n;
  // Sized for the largest grid any device can ask for, so one workspace fits every N.
  return kSumWsHeader + sizeof(double) * (size_t)kMaxCtas;
}

// Deterministic f32 sum: per-block f64 partials, last block (ticket) combines
// them in index order and performs the single f32 rounding of
// out = out + total -- or, when f64_out is set, stores the f64 total there
// unrounded (a rank's share of a sum across GPUs).  The ticket and every
// partial read are reset to 0, so the workspace is all-zero again for the
// next call (the staged sum below relies on that).
__global__ void __launch_bounds__(kSumThreads, 8) sum_f32_kernel(const float *__restrict__ a, int64_t sa,
                                                              int64_t n, float *out,
                                                              unsigned *ticket, double *partials,
                                                              double *f64_out) {
  __shared__ double sh[32];
  __shared__ int last;
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const double b = block_sum_f64(thread_sum_f64(a, sa, n), sh);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = b;
    __threadfence();
    const unsigned t = atomicAdd(ticket, 1u);
    last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  double p = 0.0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
    p = __dadd_rn(p, __ldcg(partials + i));
    partials[i] = 0.0;  // the staged sum reads a non-zero word as a written partial
  }
  const double tot = block_sum_f64(p, sh);
  if (threadIdx.x == 0) {
    if (f64_out) {
      *f64_out = tot;
    } else {
      const float o = *out;
      *out = __double2float_rn(__dadd_rn((double)o, tot));
    }
    *ticket = 0u;
  }
}

__global__ void __launch_bounds__(kSumThreads) sum_i32_kernel(const int32_t *__restrict__ a, int64_t sa,
                                                              int64_t n, int32_t *out) {
  __shared__ uint32_t sh[32];
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const uint32_t b = block_sum_u32(thread_sum_u32(a, sa, n), sh);
  if (threadIdx.x == 0 && b != 0u) atomicAdd(reinterpret_cast<unsigned *>(out), b);
}

__global__ void __launch_bounds__(kSumThreads, 8) hier_sum_f32_kernel(const float *__restrict__ a, int64_t sa,
                                                                   int64_t n, float *out) {
  __shared__ double sh[32];
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const double b = block_sum_f64(thread_sum_f64(a, sa, n), sh);
  if (threadIdx.x == 0) atomicAdd(out, __double2float_rn(b));
}

// ---- shared-memory-staged kernels (unit stride, 16-byte aligned input) --------
// Set when a bounded wait of a staged reduction expires (read by
// spmdb200_reduction_status).
__device__ int g_reduce_timeout;

enum class BulkMode { kF32Det, kI32, kF32Atomic };

template <BulkMode M>
__global__ void __launch_bounds__(kBulkThreads) sum_bulk_kernel(const void *__restrict__ a, int64_t n, void *out,
                                                               unsigned *ticket, double *partials,
                                                               double *f64_out) {
  extern __shared__ __align__(128) unsigned char bulk_raw[];
  // Aligned by pointer arithmetic on the shared array, so the stage reads
  // stay shared-space (LDS) accesses.
  unsigned char *smem = bulk_raw + ((128u - (smem_u32(bulk_raw) & 127u)) & 127u);
  __shared__ uint64_t full[kBulkStages];
  __shared__ double shd[32];
  __shared__ uint32_t shu[32];
  __shared__ int last, abort_flag;
  __shared__ double own;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages; ++s) mbar_init(&full[s], 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  const int64_t units = n >> 2;  // 16-byte units; the last n % 4 elements are the tail
  int64_t lo, hi;
  cta_range(units, lo, hi);
  const uint4 *base = reinterpret_cast<const uint4 *>(a);
  // While the previous kernel finishes, warm L2 with this CTA's first chunks.
  if (threadIdx.x == 0) bulk_prefetch_head(base, lo, hi);
  __syncthreads();
  pdl_wait();  // the previous kernel of the stream is complete (it may have written the input)
  if (threadIdx.x == 0) pdl_trigger();
  // The value the sum adds to, read now so the last block's final store does
  // not wait on it (nothing else writes *out while this kernel runs).
  double init = 0.0;
  // Start ticket: the block that takes the last one combines the partials.
  // Every other block has started by then, so its polls wait only on blocks
  // that are already running.  The atomic's result is first needed after the
  // stream loop, so its round trip overlaps the loads.
  unsigned start = 0;
  if constexpr (M == BulkMode::kF32Det) {
    if (threadIdx.x == 0) {
      start = atomicAdd(ticket, 1u);
      if (!f64_out) init = (double)*static_cast<const float *>(out);
    }
  }
  if constexpr (M == BulkMode::kI32) {
    uint32_t acc = 0;
    const bool ok = bulk_stream(base, lo, hi, smem, full, &abort_flag,
                                [&](uint4 v) { acc += v.x + v.y + v.z + v.w; });
    if (!ok && threadIdx.x == 0) atomicExch(&g_reduce_timeout, 1);
    if (blockIdx.x == gridDim.x - 1) {
      const int64_t t = (units << 2) + threadIdx.x;
      if (t < n) acc += (uint32_t) static_cast<const int32_t *>(a)[t];
    }
    const uint32_t b = block_sum_u32(acc, shu);
    if (threadIdx.x == 0 && b != 0u) atomicAdd(static_cast<unsigned *>(out), b);
  } else {
    double acc0 = 0.0, acc1 = 0.0;
    const bool ok = bulk_stream(base, lo, hi, smem, full, &abort_flag, [&](uint4 v) {
      acc0 = __dadd_rn(acc0, (double)__uint_as_float(v.x));
      acc1 = __dadd_rn(acc1, (double)__uint_as_float(v.y));
      acc0 = __dadd_rn(acc0, (double)__uint_as_float(v.z));
      acc1 = __dadd_rn(acc1, (double)__uint_as_float(v.w));
    });
    if (!ok && threadIdx.x == 0) atomicExch(&g_reduce_timeout, 1);
    if (blockIdx.x == gridDim.x - 1) {
      const int64_t t = (units << 2) + threadIdx.x;
      if (t < n) acc0 = __dadd_rn(acc0, (double)static_cast<const float *>(a)[t]);
    }
    const double b = block_sum_f64(__dadd_rn(acc0, acc1), shd);
    if constexpr (M == BulkMode::kF32Atomic) {
      if (threadIdx.x == 0) atomicAdd(static_cast<float *>(out), __double2float_rn(b));
    } else {
      unsigned long long *words = reinterpret_cast<unsigned long long *>(partials);
      if (threadIdx.x == 0) {
        last = (start == gridDim.x - 1);
        if (last)
          own = b;
        else
          st_relaxed_u64(words + blockIdx.x, (unsigned long long)__double_as_longlong(b) ^ kPartialKey);
      }
      __syncthreads();
      if (!last) return;
      // Combine in block-index order (the same fixed tree for every call);
      // each word read is cleared again, so the workspace stays all-zero.
      double p = 0.0;
      bool lost = false;
      for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
        double v = own;
        if (i != (int)blockIdx.x) {
          const unsigned long long w = poll_partial(words + i);
          lost |= (w == 0ull);
          v = w ? __longlong_as_double((long long)(w ^ kPartialKey)) : 0.0;
          st_relaxed_u64(words + i, 0ull);
        }
        p = __dadd_rn(p, v);
      }
      if (lost) atomicExch(&g_reduce_timeout, 1);
      const double tot = block_sum_f64(p, shd);
      if (threadIdx.x == 0) {
        if (f64_out)
          *f64_out = tot;
        else
          *static_cast<float *>(out) = __double2float_rn(__dadd_rn(init, tot));
        *ticket = 0u;
      }
    }
  }
}

template <BulkMode M>
static int bulk_grid(int64_t n) {
  static int cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 1;
  if (cache[dev] == 0) {
    cudaFuncSetAttribute(sum_bulk_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBulkSmem);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sum_bulk_kernel<M>, kBulkThreads, kBulkSmem) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    cache[dev] = per_sm * num_sms(dev);
  }
  const int64_t chunks = ((n >> 2) * 16 + kBulkChunk - 1) / kBulkChunk;  // at least one chunk per CTA
  int64_t g = chunks < 1 ? 1 : chunks;
  if (g > cache[dev]) g = cache[dev];
  if (g > kMaxCtas) g = kMaxCtas;
  return (int)g;
}

static bool bulk_ok(const void *p, int64_t stride) {
  return stride == 1 && (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

static int g_f32_cache[64], g_i32_cache[64], g_hier_cache[64];

int sum_f32_grid(int64_t n) {
  // The larger of the two paths' grids (both write one partial per block).
  const int a = reduce_grid(sum_f32_kernel, g_f32_cache, n), b = bulk_grid<BulkMode::kF32Det>(n);
  return a > b ? a : b;
}

cudaError_t launch_sum_f32(View1 a, float *out, int64_t n, void *ws, cudaStream_t s, double *f64_out) {
  unsigned *ticket = static_cast<unsigned *>(ws);
  double *partials = reinterpret_cast<double *>(static_cast<char *>(ws) + kSumWsHeader);
  // Launched with programmatic dependent launch: back-to-back reductions
  // overlap each launch and prologue with the previous kernel's tail.
  if (bulk_ok(a.p, a.s))
    return launch_pdl(sum_bulk_kernel<BulkMode::kF32Det>, bulk_grid<BulkMode::kF32Det>(n), kBulkThreads, kBulkSmem,
                      s, a.p, n, out, ticket, partials, f64_out);
  return launch_pdl(sum_f32_kernel, reduce_grid(sum_f32_kernel, g_f32_cache, n), kSumThreads, 0, s, a.p, a.s, n, out,
                    ticket, partials, f64_out);
}

cudaError_t launch_sum_i32(const int32_t *a, int64_t stride, int32_t *out, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (bulk_ok(a, stride))
    return launch_pdl(sum_bulk_kernel<BulkMode::kI32>, bulk_grid<BulkMode::kI32>(n), kBulkThreads, kBulkSmem, s, a,
                      n, out, nullptr, nullptr, nullptr);
  return launch_pdl(sum_i32_kernel, reduce_grid(sum_i32_kernel, g_i32_cache, n), kSumThreads, 0, s, a, stride, n,
                    out);
}

cudaError_t launch_hier_sum_f32(View1 a, float *out, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (bulk_ok(a.p, a.s))
    return launch_pdl(sum_bulk_kernel<BulkMode::kF32Atomic>, bulk_grid<BulkMode::kF32Atomic>(n), kBulkThreads,
                      kBulkSmem, s, a.p, n, out, nullptr, nullptr, nullptr);
  return launch_pdl(hier_sum_f32_kernel, reduce_grid(hier_sum_f32_kernel, g_hier_cache, n), kSumThreads, 0, s, a.p,
                    a.s, n, out);
}

}  // namespace spmdb200

namespace spmdb200 {
int reduction_timeout_flag(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_reduce_timeout, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_reduce_timeout, &zero, sizeof(int));
  }
  return v;
}
}  // namespace spmdb200
