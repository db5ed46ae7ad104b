// jacobi3d.cu -- Jacobi-3D 7-point sweeps: the generic per-sweep path, the
// seeded 3-D input fill and the layout check of the temporally blocked kernel
// (jacobi3d_tb.cu, which runs every x-contiguous, 16-byte aligned layout, on
// one GPU and in z-slabs).
//
// Generic path: one launch per sweep, one thread per cell (x fastest), any
// strides; residual partials combined by the last block in block order.
#include <cuda.h>

#include "internal.h"

namespace spmdb200 {
namespace {

__device__ __forceinline__ double sq_diff3(float a, float b) {
  const double d = __dsub_rn((double)a, (double)b);
  return __dmul_rn(d, d);
}

__global__ void __launch_bounds__(256) jacobi3d_sweep_generic_kernel(
    const float *__restrict__ u, float *__restrict__ v, long long sz, long long sy, long long sx,
    long long d, long long h, long long w, int want, double *partials, unsigned *ticket, double *res_slot) {
  __shared__ double sh[32];
  __shared__ int last;
  const float k7 = 1.0f / 7.0f;
  const long long nth = (long long)gridDim.x * blockDim.x;
  const long long total = d * h * w;
  double acc = 0.0;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += nth) {
    const long long z = idx / (h * w), rem = idx - z * h * w;
    const long long y = rem / w, x = rem - y * w;
    const long long o0 = z * sz + y * sy + x * sx;
    const float c = u[o0];
    float o = c;
    if (z > 0 && z < d - 1 && y > 0 && y < h - 1 && x > 0 && x < w - 1) {
      float t = __fadd_rn(c, u[o0 - sx]);
      t = __fadd_rn(t, u[o0 + sx]);
      t = __fadd_rn(t, u[o0 - sy]);
      t = __fadd_rn(t, u[o0 + sy]);
      t = __fadd_rn(t, u[o0 - sz]);
      t = __fadd_rn(t, u[o0 + sz]);
      o = __fmul_rn(t, k7);
      if (want) acc = __dadd_rn(acc, sq_diff3(o, c));
    }
    v[o0] = o;
  }
  if (!want) return;
  acc = warp_sum_f64(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double b = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) b = __dadd_rn(b, sh[i]);
    partials[blockIdx.x] = b;
    __threadfence();
    last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x < 32) {
    double p = 0.0;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += 32) p = __dadd_rn(p, __ldcg(partials + i));
    p = warp_sum_f64(p);
    if (threadIdx.x == 0) {
      *res_slot = p;
      *ticket = 0u;
    }
  }
}

// Seeded synthetic 3-D input: cell (gz, y, x) of the global g_d x h x w grid
// is uniform [0, 1) from the counter hash of (seed, gz * h + y, x); global
// boundary cells and planes outside [0, g_d) are 0.
__global__ void __launch_bounds__(256) fill_jacobi3d_input_kernel(float *p, long long sz, long long sy,
                                                                  long long planes, long long h, long long w,
                                                                  long long g_z0, long long g_d, uint64_t seed) {
  const long long nth = (long long)gridDim.x * blockDim.x;
  const long long total = planes * h * w;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += nth) {
    const long long z = idx / (h * w), rem = idx - z * h * w;
    const long long y = rem / w, x = rem - y * w;
    const long long gz = g_z0 + z;
    const bool interior = gz > 0 && gz < g_d - 1 && y > 0 && y < h - 1 && x > 0 && x < w - 1;
    p[z * sz + y * sy + x] = interior ? hash_uniform(seed, (uint64_t)(gz * h + y), (uint64_t)x) : 0.0f;
  }
}

}  // namespace

cudaError_t launch_fill_jacobi3d_input(float *p, int64_t sz, int64_t sy, int64_t planes, int64_t h, int64_t w,
                                       int64_t g_z0, int64_t g_d, uint64_t seed, cudaStream_t s) {
  if (planes <= 0 || h <= 0 || w <= 0) return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  long long g = (planes * h * w + 255) / 256;
  const long long cap = (long long)num_sms(dev) * 8;
  if (g > cap) g = cap;
  fill_jacobi3d_input_kernel<<<(unsigned)g, 256, 0, s>>>(p, sz, sy, planes, h, w, g_z0, g_d, seed);
  return cudaGetLastError();
}

cudaError_t launch_jacobi3d_generic(const Jacobi3dProblem &p, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  const long long cells = p.d * p.h * p.w;
  long long g = (cells + 255) / 256;
  const long long cap = (long long)num_sms(dev) * 8;
  if (g > cap) g = cap;
  if (g > kMaxCtas) g = kMaxCtas;
  if (g < 1) g = 1;
  float *a = p.u, *b = p.v;
  for (long long sw = 1; sw <= p.sweeps; ++sw) {
    const int want = p.res_every > 0 && sw % p.res_every == 0;
    double *slot = want ? p.res_out + (sw / p.res_every - 1) : nullptr;
    jacobi3d_sweep_generic_kernel<<<(unsigned)g, 256, 0, s>>>(a, b, p.sz, p.sy, p.sx, p.d, p.h, p.w, want,
                                                               p.ws->partial[0], &p.ws->ticket, slot);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    float *t = a;
    a = b;
    b = t;
  }
  return cudaSuccess;
}


bool jacobi3d_tma_ok(const Jacobi3dProblem &p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p.u), b = reinterpret_cast<uintptr_t>(p.v);
  return p.sx == 1 && ((a | b) & 15u) == 0 && (p.sy * 4) % 16 == 0 && (p.sz * 4) % 16 == 0 && p.w >= 1 &&
         p.h >= 1 && p.d >= 1 && p.sy >= p.w && p.sz >= p.sy * p.h && p.w < (1ll << 30) && p.h < (1ll << 30) &&
         p.d < (1ll << 30) && p.sz < (1ll << 37) && p.sweeps <= (1ll << 30);
}

}  // namespace spmdb200
