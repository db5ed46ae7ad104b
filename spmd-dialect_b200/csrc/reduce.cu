// reduce.cu -- library launches of spmd.reduce add (f32 deterministic, i32
// exact, and the reference's one-atomic-per-block form).
#include "internal.h"
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
// out = out + total.  The ticket is reset to 0 so the workspace stays reusable.
__global__ void __launch_bounds__(kSumThreads, 8) sum_f32_kernel(const float *__restrict__ a, int64_t sa,
                                                              int64_t n, float *out,
                                                              unsigned *ticket, double *partials) {
  __shared__ double sh[32];
  __shared__ int last;
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
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) p = __dadd_rn(p, __ldcg(partials + i));
  const double tot = block_sum_f64(p, sh);
  if (threadIdx.x == 0) {
    const float o = *out;
    *out = __double2float_rn(__dadd_rn((double)o, tot));
    *ticket = 0u;
  }
}

__global__ void __launch_bounds__(kSumThreads) sum_i32_kernel(const int32_t *__restrict__ a, int64_t sa,
                                                              int64_t n, int32_t *out) {
  __shared__ uint32_t sh[32];
  const uint32_t b = block_sum_u32(thread_sum_u32(a, sa, n), sh);
  if (threadIdx.x == 0 && b != 0u) atomicAdd(reinterpret_cast<unsigned *>(out), b);
}

__global__ void __launch_bounds__(kSumThreads, 8) hier_sum_f32_kernel(const float *__restrict__ a, int64_t sa,
                                                                   int64_t n, float *out) {
  __shared__ double sh[32];
  const double b = block_sum_f64(thread_sum_f64(a, sa, n), sh);
  if (threadIdx.x == 0) atomicAdd(out, __double2float_rn(b));
}

static int g_f32_cache[64], g_i32_cache[64], g_hier_cache[64];

int sum_f32_grid(int64_t n) { return reduce_grid(sum_f32_kernel, g_f32_cache, n); }

cudaError_t launch_sum_f32(View1 a, float *out, int64_t n, void *ws, cudaStream_t s) {
  const int g = sum_f32_grid(n);
  unsigned *ticket = static_cast<unsigned *>(ws);
  double *partials = reinterpret_cast<double *>(static_cast<char *>(ws) + kSumWsHeader);
  sum_f32_kernel<<<g, kSumThreads, 0, s>>>(a.p, a.s, n, out, ticket, partials);
  return cudaGetLastError();
}

cudaError_t launch_sum_i32(const int32_t *a, int64_t stride, int32_t *out, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  sum_i32_kernel<<<reduce_grid(sum_i32_kernel, g_i32_cache, n), kSumThreads, 0, s>>>(a, stride, n, out);
  return cudaGetLastError();
}

cudaError_t launch_hier_sum_f32(View1 a, float *out, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  hier_sum_f32_kernel<<<reduce_grid(hier_sum_f32_kernel, g_hier_cache, n), kSumThreads, 0, s>>>(a.p, a.s, n, out);
  return cudaGetLastError();
}

}  // namespace spmdb200
