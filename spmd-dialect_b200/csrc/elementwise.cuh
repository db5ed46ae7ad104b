// elementwise.cuh -- device bodies of the elementwise spmd.forall maps.
//
// The reference lowers `spmd.forall (i) in [0,N)` with tile T to one block of
// T lanes per tile, each lane doing one scalar load/op/store guarded by i < N
// (lib/Conversion/SPMDToGPU/SPMDToGPU.cpp:491-580,
// lib/Transforms/MaterializeTilingAndMapping.cpp:153-173).  Here each thread
// walks the iteration space grid-stride with 128-bit loads and stores, so the
// body is correct for ANY launch shape (including the reference's
// grid=ceil(N/32), block=32) and saturates HBM for the library's own launches.
// Arithmetic is spelled with __fadd_rn/__fmul_rn so nothing is contracted.
#pragma once

#include "common.cuh"

namespace spmdb200 {

struct AddOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return __fadd_rn(a, b); }
};
struct AxpyOp {
  float alpha;
  __device__ __forceinline__ float operator()(float x, float y) const {
    return __fadd_rn(__fmul_rn(alpha, x), y);
  }
};

template <class Op>
__device__ __forceinline__ float4 apply4(Op op, float4 a, float4 b) {
  return make_float4(op(a.x, b.x), op(a.y, b.y), op(a.z, b.z), op(a.w, b.w));
}

// c[i] = op(a[i], b[i]) for i < n; unit strides, 16-byte aligned pointers.
// 2 float4 per operand in flight per thread per iteration (64 B/thread: at
// 1024 resident threads per SM that is ~9.7 MB in flight over 148 SMs, above
// the ~6.5 MB the HBM latency-bandwidth product asks for).
template <class Op>
__device__ __forceinline__ void ewise_vec_body(Op op, const float *a, const float *b, float *c,
                                               int64_t n) {
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n4 = n >> 2;
  int64_t i = tid;
  for (; i + nth < n4; i += 2 * nth) {
    const float4 a0 = ld_f4(a + 4 * i), a1 = ld_f4(a + 4 * (i + nth));
    const float4 b0 = ld_f4(b + 4 * i), b1 = ld_f4(b + 4 * (i + nth));
    st_f4(c + 4 * i, apply4(op, a0, b0));
    st_f4(c + 4 * (i + nth), apply4(op, a1, b1));
  }
  for (; i < n4; i += nth) st_f4(c + 4 * i, apply4(op, ld_f4(a + 4 * i), ld_f4(b + 4 * i)));
  const int64_t t = (n4 << 2) + tid;  // at most 3 tail elements
  if (t < n) c[t] = op(a[t], b[t]);
}

// Any strides, any alignment.
template <class Op>
__device__ __forceinline__ void ewise_strided_body(Op op, const float *a, int64_t sa, const float *b,
                                                   int64_t sb, float *c, int64_t sc, int64_t n) {
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += nth)
    c[i * sc] = op(a[i * sa], b[i * sb]);
}

template <class Op>
__device__ __forceinline__ void ewise_body(Op op, const float *a, int64_t sa, const float *b,
                                           int64_t sb, float *c, int64_t sc, int64_t n) {
  const bool vec = sa == 1 && sb == 1 && sc == 1 &&
                   (((uintptr_t)a | (uintptr_t)b | (uintptr_t)c) & 15u) == 0;
  if (vec)
    ewise_vec_body(op, a, b, c, n);
  else
    ewise_strided_body(op, a, sa, b, sb, c, sc, n);
}

}  // namespace spmdb200
