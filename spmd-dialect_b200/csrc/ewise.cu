// ewise.cu -- library launches of the elementwise maps (ewise add, axpy).
#include "elementwise.cuh"
#include "internal.h"

namespace spmdb200 {

template <class Op>
__global__ void __launch_bounds__(256, 4) ewise_map_kernel(Op op, const float *a, int64_t sa,
                                                        const float *b, int64_t sb, float *c,
                                                        int64_t sc, int64_t n) {
  ewise_body(op, a, sa, b, sb, c, sc, n);
}

// Grid: enough 256-thread blocks for one float4 per thread, capped at 8
// resident blocks per SM (2048 threads) -- the grid-stride loop covers the rest.
static int ewise_grid(int64_t n) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t cap = (int64_t)num_sms(dev) * 8;
  int64_t want = ((n + 3) / 4 + 255) / 256;
  if (want < 1) want = 1;
  return (int)(want < cap ? want : cap);
}

cudaError_t launch_ewise_add(View1 a, View1 b, View1 c, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  ewise_map_kernel<AddOp><<<ewise_grid(n), 256, 0, s>>>(AddOp{}, a.p, a.s, b.p, b.s, c.p, c.s, n);
  return cudaGetLastError();
}

cudaError_t launch_axpy(float alpha, View1 x, View1 y, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  ewise_map_kernel<AxpyOp><<<ewise_grid(n), 256, 0, s>>>(AxpyOp{alpha}, x.p, x.s, y.p, y.s, y.p, y.s, n);
  return cudaGetLastError();
}

}  // namespace spmdb200
