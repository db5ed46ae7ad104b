// refabi.cu -- device kernels with the entry names and .param layouts of the
// PTX the reference's gen-ptx.sh pipeline writes, so a cuModuleLoadData caller
// (harness/cuda_driver.py:124-140) can load spmdb200_kernels.cubin in place of
// the reference's .ptx and launch with unchanged argument lists.
//
// Parameter lists (i64 = long long, ptr = float*):
//   ewise_kernel            (i64 tile, i64 N, A x5, B x5, C x5)         harness/run_ewise.py:31-70
//   promoted_stencil_kernel (i64 TR, i64 TC, A x7, i64 c1, B x7)        harness/run_promoted_stencil.py:28-65
//   promoted_stencil_kernel_square (i64 T, A x7, i64 c1, B x7)          the TR == TC (CSE-merged) form
//   atomic_sum_kernel       (i64 tile, i64 N, A x5, out x3)             harness/run_reduction.py:32-49
//   hierarchical_sum_kernel (i64 tile, i64 N, ptr A.aligned, ptr out)   scripts/gen-ptx.sh:116-130
//
// Every kernel is correct for any grid/block shape (grid-stride bodies), so
// the reference launches (grid=ceil(N/tile), block=tile; grid=(N/TR, M/TC),
// block=(TR+1)(TC+1)) work unchanged.  Memref offsets and strides are honoured.
#include "elementwise.cuh"
#include "reduction.cuh"
#include "stencil3.cuh"

using spmdb200::View2;

extern "C" __global__ void __launch_bounds__(1024) ewise_kernel(long long tile, long long N,
                                        float *A_base, float *A, long long A_off, long long A_size, long long A_st,
                                        float *B_base, float *B, long long B_off, long long B_size, long long B_st,
                                        float *C_base, float *C, long long C_off, long long C_size, long long C_st) {
  (void)tile; (void)A_base; (void)B_base; (void)C_base; (void)A_size; (void)B_size; (void)C_size;
  spmdb200::ewise_body(spmdb200::AddOp{}, A + A_off, A_st, B + B_off, B_st, C + C_off, C_st, N);
}

// Output extent = B's sizes (the reference kernel's loop bounds come from the
// host-side grid; the copy guard uses A's sizes via memref.dim).
extern "C" __global__ void __launch_bounds__(1024) promoted_stencil_kernel(long long TR, long long TC,
                                                   float *A_base, float *A, long long A_off, long long A_n0,
                                                   long long A_n1, long long A_s0, long long A_s1,
                                                   long long c1,
                                                   float *B_base, float *B, long long B_off, long long B_n0,
                                                   long long B_n1, long long B_s0, long long B_s1) {
  (void)A_base; (void)B_base;
  __shared__ spmdb200::Stencil3Smem sm;
  const View2 a{A + A_off, A_n0, A_n1, A_s0, A_s1};
  const View2 b{B + B_off, B_n0, B_n1, B_s0, B_s1};
  spmdb200::stencil3_body(a, b, B_n0, B_n1, c1, TR, TC, sm);
}

extern "C" __global__ void __launch_bounds__(1024) promoted_stencil_kernel_square(long long T,
                                                          float *A_base, float *A, long long A_off, long long A_n0,
                                                          long long A_n1, long long A_s0, long long A_s1,
                                                          long long c1,
                                                          float *B_base, float *B, long long B_off, long long B_n0,
                                                          long long B_n1, long long B_s0, long long B_s1) {
  (void)A_base; (void)B_base;
  __shared__ spmdb200::Stencil3Smem sm;
  const View2 a{A + A_off, A_n0, A_n1, A_s0, A_s1};
  const View2 b{B + B_off, B_n0, B_n1, B_s0, B_s1};
  spmdb200::stencil3_body(a, b, B_n0, B_n1, c1, T, T, sm);
}

// out += sum(A[0..N)) with one f32 atomic per block (the reference does one per
// element; the sum it produces is the same up to f32 rounding order).
extern "C" __global__ void __launch_bounds__(1024) atomic_sum_kernel(long long tile, long long N,
                                             float *A_base, float *A, long long A_off, long long A_size,
                                             long long A_st,
                                             float *out_base, float *out, long long out_off) {
  (void)tile; (void)A_base; (void)A_size; (void)out_base;
  __shared__ double sh[32];
  const double b = spmdb200::block_sum_f64(spmdb200::thread_sum_f64(A + A_off, A_st, N), sh);
  if (threadIdx.x == 0) atomicAdd(out + out_off, __double2float_rn(b));
}

extern "C" __global__ void __launch_bounds__(1024) hierarchical_sum_kernel(long long tile, long long N, float *A, float *out) {
  (void)tile;
  __shared__ double sh[32];
  const double b = spmdb200::block_sum_f64(spmdb200::thread_sum_f64(A, 1, N), sh);
  if (threadIdx.x == 0) atomicAdd(out, __double2float_rn(b));
}
