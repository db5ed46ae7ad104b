// stencil3.cu -- library launch of the promoted 3-point stencil
//   B[i,j] = (A[i,j] + A[i,j+1]) + A[i+1,j],  0 <= i < n, 0 <= j < m
// (test/SPMD/lower-to-gpu-nvptx-promoted.mlir:32-67).  It is the general
// promoted-tile stencil with the offsets (0,0), (0,1), (1,0) in that order:
// footprint cells outside A read as 0 and stores stay inside n x m, exactly
// as the reference-signature promoted_stencil_kernel of the kernel module does.
#include "internal.h"

namespace spmdb200 {

cudaError_t launch_stencil3(View2 a, View2 b, int64_t n, int64_t m, cudaStream_t s) {
  if (n <= 0 || m <= 0) return cudaSuccess;
  static const int64_t kOffsets[6] = {0, 0, 0, 1, 1, 0};
  StencilNdProblem p{};
  p.rank = 2;
  p.ntaps = 3;
  p.a = a.p;
  p.b = b.p;
  p.a_size[0] = a.n0;
  p.a_size[1] = a.n1;
  p.a_stride[0] = a.s0;
  p.a_stride[1] = a.s1;
  p.b_size[0] = n;
  p.b_size[1] = m;
  p.b_stride[0] = b.s0;
  p.b_stride[1] = b.s1;
  p.step[0] = p.step[1] = 1;
  p.tile[0] = 32;  // the reference's group tile; the kernel stages larger ones
  p.tile[1] = 8;
  p.offsets = kOffsets;
  p.weights = nullptr;
  p.scale = 1.0f;
  return launch_stencil_nd(p, 1, s);
}

}  // namespace spmdb200
