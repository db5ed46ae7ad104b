/*
 * spmd_b200.h -- C ABI of libspmdb200.so, the B200 (sm_100a) implementation of
 * the kernels that spmd-dialect's SPMDToGPU lowering emits:
 *
 *   (1) elementwise spmd.forall maps            (ewise, axpy, any f32 body:
 *                                                forall_map)
 *   (2) PromoteGroupMemory-tiled stencil sweeps (3-point promoted stencil,
 *       Jacobi-2D 5-point, Jacobi-3D 7-point)
 *   (3) ReduceToHierarchicalGPU spmd.reduce     (f32 sum, i32 sum)
 *
 * Memref descriptors follow MLIR's unpacked memref-to-LLVM convention
 * (harness/run_host.py:8-11,41-65 in the reference):
 *   rank-0 memref : (T* base, T* aligned, int64 offset)
 *   rank-1 memref : (T* base, T* aligned, int64 offset, int64 size, int64 stride)
 *   rank-2 memref : (base, aligned, offset, size0, size1, stride0, stride1)
 *   rank-3 memref : (base, aligned, offset, size0, size1, size2,
 *                    stride0, stride1, stride2)
 * Element (i,j) of a rank-2 memref lives at aligned[offset + i*stride0 + j*stride1].
 * `base` is carried for ABI compatibility and never dereferenced.
 *
 * Three families of entry points:
 *
 *  A. Reference-named HOST entries (`ewise`, `stencil_cpu`, `atomic_sum`,
 *     `hierarchical_sum`).  Same names and unpacked signatures as the
 *     SPMDToSCF / SPMDToOpenMP shared libraries that harness/run_host.py loads
 *     with ctypes (restype=None).  Buffers are HOST memory; the entry copies
 *     them to the current CUDA device, runs the B200 kernel, copies the result
 *     back and synchronises.  Errors cannot be returned through `void`; they are
 *     printed to stderr and kept for spmdb200_last_error().
 *
 *  B. `spmdb200_*` DEVICE entries.  Same descriptor convention, device
 *     pointers, an explicit cudaStream_t (passed as void*; NULL = legacy default
 *     stream), asynchronous, returning an int status (SPMDB200_OK = 0).
 *
 *  C. `spmdb200_*_host` END-TO-END entries for the configurations the
 *     reference has no kernel for (axpy, Jacobi-2D/3D): host buffers in, host
 *     buffers out, synchronous, int status.
 *
 * The device kernels with the reference's PTX entry names and .param layouts
 * (ewise_kernel, promoted_stencil_kernel, atomic_sum_kernel,
 * hierarchical_sum_kernel) ship in spmdb200_kernels.cubin for
 * cuModuleLoadData-based callers (harness/cuda_driver.py:124-140); they are
 * not C functions and are documented in INTEGRATION.md.
 */
#ifndef SPMD_B200_H
#define SPMD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------- */
#define SPMDB200_OK               0
#define SPMDB200_ERR_INVALID_ARG (-1) /* bad descriptor: null data, negative size/stride, bound > size */
#define SPMDB200_ERR_CUDA        (-2) /* a CUDA runtime call or a launch failed */
#define SPMDB200_ERR_TIMEOUT     (-3) /* a bounded device-side wait expired (grid barrier / peer flag) */
#define SPMDB200_ERR_UNSUPPORTED (-4) /* layout outside what the entry accepts */
#define SPMDB200_ERR_WORKSPACE   (-5) /* workspace null, too small or misaligned */
#define SPMDB200_ERR_NO_DEVICE   (-6) /* no CUDA device visible */
#define SPMDB200_ERR_BOUNDS      (-7) /* a checked build recorded an out-of-range access */

const char *spmdb200_status_string(int status);
/* Last status recorded by any entry on this host thread (0 after success). */
int spmdb200_last_error(void);
const char *spmdb200_last_error_message(void);
/* Library version string and the device architecture it was built for. */
const char *spmdb200_version(void);
/* Frees the device staging buffers cached by the family-A/C host entries. */
int spmdb200_release_cache(void);

/* =========================================================================
 * A. Reference-named host entries (drop-in for the SCF/OpenMP .so files).
 * ========================================================================= */

/* C[i] = A[i] + B[i], i < N.
 * Replaces `ewise` from test/SPMD/lower-to-gpu-nvptx.mlir:54-71 as loaded by
 * harness/run_host.py:84-101 (_EWISE_ARGTYPES). */
void ewise(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
           float *B_base, float *B_aligned, int64_t B_offset, int64_t B_size, int64_t B_stride,
           float *C_base, float *C_aligned, int64_t C_offset, int64_t C_size, int64_t C_stride,
           int64_t N);

/* B[i,j] = (A[i,j] + A[i,j+1]) + A[i+1,j] for i < N, j < M.  A is normally
 * (N+1)x(M+1); reads outside A's sizes contribute 0.
 * Replaces `stencil_cpu` from test/SPMD/differential-stencil.mlir:19-37 as
 * loaded by harness/run_host.py:119-137 (_STENCIL_ARGTYPES). */
void stencil_cpu(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size0, int64_t A_size1,
                 int64_t A_stride0, int64_t A_stride1,
                 float *B_base, float *B_aligned, int64_t B_offset, int64_t B_size0, int64_t B_size1,
                 int64_t B_stride0, int64_t B_stride1,
                 int64_t N, int64_t M);

/* out[] += sum(A[0..N)).  Caller zero-initialises out for a plain sum.
 * Replaces `atomic_sum` from test/SPMD/lower-to-gpu-nvptx-reduction.mlir:30-44
 * as loaded by harness/run_host.py:160-175 (_REDUCTION_ARGTYPES). */
void atomic_sum(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                float *out_base, float *out_aligned, int64_t out_offset,
                int64_t N);

/* Same contract as atomic_sum.
 * Replaces `hierarchical_sum` from
 * test/SPMD/lower-to-gpu-nvptx-hierarchical-reduction.mlir:58-88 as loaded by
 * harness/run_host.py:195-203. */
void hierarchical_sum(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                      float *out_base, float *out_aligned, int64_t out_offset,
                      int64_t N);

/* =========================================================================
 * B. Device entries (device pointers, stream-ordered, int status).
 * ========================================================================= */

/* C = A + B (f32), the device-pointer form of the launch in
 * harness/run_ewise.py:53-70 (ewise_kernel). */
int spmdb200_ewise(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                   float *B_base, float *B_aligned, int64_t B_offset, int64_t B_size, int64_t B_stride,
                   float *C_base, float *C_aligned, int64_t C_offset, int64_t C_size, int64_t C_stride,
                   int64_t N, void *stream);

/* Y[i] = fadd(fmul(a, X[i]), Y[i]) with no FMA contraction: the elementwise
 * spmd.forall y = a*x + y lowered the way lane foralls are lowered in
 * lib/Conversion/SPMDToGPU/SPMDToGPU.cpp:491-580.  No reference entry. */
int spmdb200_axpy(float a,
                  float *X_base, float *X_aligned, int64_t X_offset, int64_t X_size, int64_t X_stride,
                  float *Y_base, float *Y_aligned, int64_t Y_offset, int64_t Y_size, int64_t Y_stride,
                  int64_t N, void *stream);

/* Elementwise spmd.forall with a general f32 body, y[p] = f(x0[p], x1[p], ...)
 * over a rank 1-3 domain (the lane lowering of SPMDToGPU.cpp:491-580 applied
 * to any body of arith ops, not only C = A + B).  The body is a straight-line
 * program of `n_insns` instructions, two int32 words each:
 *   w0 = op | dst << 8 | a << 16 | b << 24,  w1 = aux
 * over `n_regs` f32 registers (<= SPMDB200_MAP_MAX_REGS):
 *   LOAD     r[dst] = inputs[aux][p]        (all LOADs come first)
 *   CONST    r[dst] = consts[aux]
 *   ADD SUB MUL DIV   r[dst] = r[a] op r[b], IEEE round-to-nearest, each
 *                     rounded on its own (never contracted to an FMA)
 *   MAXIMUM MINIMUM   arith.maximumf / minimumf (NaN in, NaN out; -0 < +0)
 *   NEG ABS SQRT      r[dst] = f(r[a]) (sign flip, sign clear, IEEE sqrt)
 *   CMP      r[dst] = cmpf(aux, r[a], r[b]) ? 1 : 0, aux = arith.cmpf's
 *            predicate number (0 false, 1 oeq, 2 ogt, 3 oge, 4 olt, 5 ole,
 *            6 one, 7 ord, 8 ueq, 9 ugt, 10 uge, 11 ult, 12 ule, 13 une,
 *            14 uno, 15 true)
 *   SELECT   r[dst] = r[aux] != 0 ? r[a] : r[b]
 *   AND OR XOR        booleans (nonzero = true) -> 1 / 0
 *   STORE    out[p] = r[a]                  (exactly one, the last)
 * Every register is written before it is read.  sizes[d] is the domain;
 * input_strides holds rank strides (in elements) per input, row after row;
 * out_strides likewise.  The output may be one of the inputs (same view: each
 * point is read before it is written); other overlaps are undefined.  NaN
 * results are NaN (the payload is not specified).  No reference entry. */
enum {
  SPMDB200_MAP_LOAD = 0, SPMDB200_MAP_CONST = 1, SPMDB200_MAP_ADD = 2, SPMDB200_MAP_SUB = 3,
  SPMDB200_MAP_MUL = 4, SPMDB200_MAP_DIV = 5, SPMDB200_MAP_MAXIMUM = 6, SPMDB200_MAP_MINIMUM = 7,
  SPMDB200_MAP_NEG = 8, SPMDB200_MAP_ABS = 9, SPMDB200_MAP_SQRT = 10, SPMDB200_MAP_CMP = 11,
  SPMDB200_MAP_SELECT = 12, SPMDB200_MAP_AND = 13, SPMDB200_MAP_OR = 14, SPMDB200_MAP_XOR = 15,
  SPMDB200_MAP_STORE = 16
};
#define SPMDB200_MAP_MAX_INPUTS 8
#define SPMDB200_MAP_MAX_REGS 16
#define SPMDB200_MAP_MAX_INSNS 64
#define SPMDB200_MAP_MAX_CONSTS 32
int spmdb200_forall_map(int rank, const int64_t *sizes, int n_inputs, const float *const *inputs,
                        const int64_t *input_strides, float *out, const int64_t *out_strides,
                        const int32_t *code, int n_insns, const float *consts, int n_consts, int n_regs,
                        void *stream);

/* Checked builds (libspmdb200_checked.so, from `build.py --checked`): the
 * general kernels (spmdb200_forall_map, spmdb200_stencil_nd and the stencils
 * on it) test every global index against its view's extent and every shared
 * register index against the program's, skip a failing access and record the
 * first one; the promoted stencil also fills each shared tile with NaN before
 * staging it, so a read of a cell the staging did not write comes out NaN.
 * Synchronises the device and returns SPMDB200_OK, or SPMDB200_ERR_BOUNDS
 * with *first_out = the first record (bit 63 set, site in bits 48-62: 1 input
 * load, 2 output store, 3 shared register; low 48 bits: the index) and
 * clears it; SPMDB200_ERR_UNSUPPORTED in a release build.  No counterpart in
 * the reference (its checks are static, lib/Conversion/SPMDToGPU/
 * SPMDToGPU.cpp:771-780). */
int spmdb200_check_status(unsigned long long *first_out);

/* 3-point promoted stencil B[i,j] = (A[i,j] + A[i,j+1]) + A[i+1,j] over
 * i < N, j < M with a shared-memory tile plus 1-cell halo; reads outside A's
 * sizes contribute 0.  Device-pointer form of promoted_stencil_kernel
 * (test/SPMD/lower-to-gpu-nvptx-promoted.mlir:32-67,
 * harness/run_promoted_stencil.py:68-108). */
int spmdb200_stencil3pt(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size0, int64_t A_size1,
                        int64_t A_stride0, int64_t A_stride1,
                        float *B_base, float *B_aligned, int64_t B_offset, int64_t B_size0, int64_t B_size1,
                        int64_t B_stride0, int64_t B_stride1,
                        int64_t N, int64_t M, void *stream);

/* ---- general promoted-tile stencil (rank 1-3) ------------------------------ */
/* Promotion decision for one operand, restating computePromotionPlan
 * (lib/Analysis/PromotionPlanAnalysis.cpp:53-164) on explicit inputs: per
 * dimension d < rank the tile size, the original loop step (NULL: 1) and the
 * min / max constant read offset.  footprint[d] = (tile - 1) * step + max - min
 * + 1 (tile_dims_out[d], when the offsets are bounded), footprint bytes =
 * elem_bytes * prod(footprint).  Returns SPMDB200_PLAN_PROMOTE, a
 * SPMDB200_PLAN_SKIP_* reason (in the reference's check order: unbounded
 * offsets, read-write operand, footprint above max_group_bytes, no reuse
 * because every offset is equal), or a negative status.  Host only. */
#define SPMDB200_PLAN_PROMOTE 0
#define SPMDB200_PLAN_SKIP_UNBOUNDED 1
#define SPMDB200_PLAN_SKIP_READ_WRITE 2
#define SPMDB200_PLAN_SKIP_FOOTPRINT 3
#define SPMDB200_PLAN_SKIP_NO_REUSE 4
#define SPMDB200_DEFAULT_GROUP_MEM_BYTES 49152 /* TargetDescriptor.h:26-37 maxGroupMemBytes */
int spmdb200_promotion_plan(int rank, const int64_t *tile_sizes, const int64_t *steps,
                            const int64_t *min_offsets, const int64_t *max_offsets, int64_t elem_bytes,
                            int64_t max_group_bytes, int read_only, int64_t *tile_dims_out,
                            int64_t *footprint_bytes_out);

/* B[p] = s * (((w0 * A[p + off0]) + w1 * A[p + off1]) + ...) for every output
 * point p = (k0 * step0, ...) inside B's sizes (rank 1-3; sizes / strides /
 * steps / tile sizes are host arrays of `rank` entries, strides in elements;
 * offsets is ntaps x rank, 1 <= ntaps <= 64).  weights NULL means every w = 1
 * and no multiply; scale 1.0f means no final multiply; arithmetic in the
 * given order with no contraction.  Reads outside A's sizes are 0.  With
 * policy 0 (prefer_group) the promotion plan above decides whether each
 * tile's footprint is staged in shared memory (max_group_bytes <= 0: the
 * reference's 48 KB; at most 227 KB); policy 1 (no_promotion) reads global
 * memory directly.  A and B must not overlap.  *promoted_out (optional)
 * reports the path taken.  The general form of the promoted stencil behind
 * PromoteGroupMemory.cpp:113-314. */
int spmdb200_stencil_nd(int rank, const float *A, const int64_t *A_sizes, const int64_t *A_strides,
                        float *B, const int64_t *B_sizes, const int64_t *B_strides,
                        int ntaps, const int64_t *offsets, const float *weights, float scale,
                        const int64_t *tile_sizes, const int64_t *steps, int64_t max_group_bytes,
                        int policy, int *promoted_out, void *stream);

/* Bytes of device workspace spmdb200_sum_f32 needs for N elements. */
size_t spmdb200_sum_workspace_bytes(int64_t N);

/* out[] = (float)((double)out[] + sum(A[0..N))), the hierarchical reduction of
 * lib/Conversion/SPMDToGPU/SPMDToGPU.cpp:249-415 (strided per-thread sum,
 * block tree, grid combine) redone as f64 per-thread accumulation, warp
 * shuffles, a block tree and a deterministic last-block grid combine in f64:
 * one rounding to f32, identical bits on every call.
 * `ws` is device memory of at least spmdb200_sum_workspace_bytes(N) bytes,
 * 256-byte aligned, ZERO-FILLED before its first use; every call leaves it
 * zero-filled again.  Calls that share `ws` must not overlap on the GPU. */
int spmdb200_sum_f32(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                     float *out_base, float *out_aligned, int64_t out_offset,
                     int64_t N, void *ws, size_t ws_bytes, void *stream);

/* *partial (device f64) = the unrounded f64 total of A[0..N) in the same
 * deterministic order as spmdb200_sum_f32: one rank's share of a sum split
 * across GPUs, combined by the caller in rank order before the single f32
 * rounding.  Same workspace as spmdb200_sum_f32.  No reference entry. */
int spmdb200_sum_f32_partial(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                             int64_t N, double *partial, void *ws, size_t ws_bytes, void *stream);

/* The same deterministic sum as spmdb200_sum_f32 for callers that cannot
 * allocate device memory: code inside a stream capture that must not
 * allocate, a plugin whose host application owns every device allocation, or
 * a path with no workspace to hand out.  No counterpart in the reference.
 * The scratch (ticket + one f64 partial per block) lives in a file-scope
 * __device__ array of 256 + 2048*8 = 16,640 bytes that every GPU loading the
 * library holds until exit; a launch needing more than 2048 block partials is
 * rejected with SPMDB200_ERR_WORKSPACE (the reduction never launches more, so
 * every N >= 0 fits).  The array has one instance per CUDA context: the
 * first call in each context (the primary context, or one the caller made
 * current) looks up its device address (cudaGetSymbolAddress) and should come
 * before any stream capture; after destroying a context that used this entry,
 * do not call it again in the process (a new context may reuse the handle).
 * Allocates nothing.  All calls share the array; each clears the header and
 * the partial words it will use before its launch.  Calls that overlap on the
 * GPU race on the array and must be serialised by the caller. */
int spmdb200_sum_f32_noalloc(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                             float *out_base, float *out_aligned, int64_t out_offset,
                             int64_t N, void *stream);

/* out[] += sum(A[0..N)) in int32 two's-complement arithmetic (wraps like
 * arith.addi), exact in any order.  The int32 spmd.reduce add that the
 * reference lowers through ReduceToSCFForGPU (SPMDToGPU.cpp:422-477). */
int spmdb200_sum_i32(int32_t *A_base, int32_t *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                     int32_t *out_base, int32_t *out_aligned, int64_t out_offset,
                     int64_t N, void *stream);

/* spmd.reduce of every reduction kind (include/spmd/IR/SPMDAttrs.td:74-80):
 * kind 0 add, 1 mul, 2 max, 3 min, 4 and, 5 or, 6 xor (f32 takes 0-3).
 * out[] = init (+) A[0] (+) ... (+) A[N-1].  The reference lowers these through
 * the serial ReduceToSCFForGPU fallback (lib/Conversion/SPMDToGPU/SPMDToGPU.cpp:
 * 422-477, combine :425-449); here they get the hierarchical shape with a
 * deterministic grid combine.  i32 kinds and f32 max/min are exact in any
 * order (max/min follow arith.maximumf/minimumf: NaN in, NaN out; -0 < +0;
 * i32 max/min are signed; i32 add/mul wrap).  f32 add and mul accumulate in
 * f64 and round once.  `ws` as for spmdb200_sum_f32
 * (spmdb200_sum_workspace_bytes(N), 256-byte aligned, zero-filled before its
 * first use, left zero-filled by every call). */
int spmdb200_reduce_f32(int kind, float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size,
                        int64_t A_stride, float *out_base, float *out_aligned, int64_t out_offset, int64_t N,
                        float init, void *ws, size_t ws_bytes, void *stream);
int spmdb200_reduce_i32(int kind, int32_t *A_base, int32_t *A_aligned, int64_t A_offset, int64_t A_size,
                        int64_t A_stride, int32_t *out_base, int32_t *out_aligned, int64_t out_offset, int64_t N,
                        int32_t init, void *ws, size_t ws_bytes, void *stream);

/* Synchronises the current device and reports whether any reduction launched
 * since the last call hit a bounded-wait timeout in its shared-memory staging
 * (SPMDB200_ERR_TIMEOUT; the affected result is invalid) -- clears the flag. */
int spmdb200_reduction_status(void);

/* out[] += sum(A) with one f32 atomic per block: the exact semantics of the
 * reference's hierarchical_sum_kernel (SPMDToGPU.cpp:397-408), order of the
 * block atomics unspecified. */
int spmdb200_hierarchical_sum(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                              float *out_base, float *out_aligned, int64_t out_offset,
                              int64_t N, void *stream);

/* ---- Jacobi-2D 5-point --------------------------------------------------- */
/* One sweep: for every cell (i,j) of the H x W grid
 *   boundary (i==0 || i==H-1 || j==0 || j==W-1):  V[i,j] = U[i,j]
 *   interior: V[i,j] = fmul(0.2f, ((((U[i,j] + U[i-1,j]) + U[i+1,j]) + U[i,j+1]) + U[i,j-1]))
 * `sweeps` sweeps ping-pong U -> V -> U ...; the final grid is in U when
 * `sweeps` is even and in V when it is odd.  When res_every > 0, after every
 * sweep k with k % res_every == 0 (k = 1-based), res_out[k/res_every - 1] =
 * sum over cells of ((double)new - (double)old)^2 (device memory, f64).
 * U and V must have the same shape and strides.  Pitch-aligned grids
 * (stride1 == 1, 16-byte aligned rows) run one persistent kernel that stages
 * tiles with TMA and separates sweeps with a bounded grid barrier; other
 * layouts run one launch per sweep.  `ws`: >= spmdb200_jacobi_workspace_bytes()
 * bytes of device memory, 256-byte aligned, contents irrelevant.
 * The promoted-stencil semantics follow lib/Transforms/PromoteGroupMemory.cpp:
 * 113-314; the per-cell order of operations is MLIR source order. */
size_t spmdb200_jacobi_workspace_bytes(void);
int spmdb200_jacobi2d(float *U_base, float *U_aligned, int64_t U_offset, int64_t U_size0, int64_t U_size1,
                      int64_t U_stride0, int64_t U_stride1,
                      float *V_base, float *V_aligned, int64_t V_offset, int64_t V_size0, int64_t V_size1,
                      int64_t V_stride0, int64_t V_stride1,
                      int64_t sweeps, int64_t res_every, double *res_out,
                      void *ws, size_t ws_bytes, void *stream);

/* Process-wide limits of the persistent kernels' bounded waits: `grid_ms` for
 * waits inside one GPU (grid barrier, TMA stages), `peer_ms` for waits on a
 * neighbouring GPU's halo delivery.  Defaults 4000 and 20000 ms.  A wait that
 * runs out makes the run end with SPMDB200_ERR_TIMEOUT instead of hanging. */
int spmdb200_set_wait_budget_ms(int64_t grid_ms, int64_t peer_ms);

/* Reads the device status word a Jacobi run left in `ws` (synchronises
 * `stream`): SPMDB200_OK or SPMDB200_ERR_TIMEOUT. */
int spmdb200_workspace_status(void *ws, void *stream);

/* End-to-end Jacobi-2D on HOST buffers: copies U (H x W, row pitch stride0
 * elements, stride1 must be 1) to the device, runs `sweeps` sweeps, copies the
 * final grid back into U and the residuals into res_out (host, f64, may be
 * NULL when res_every == 0).  Synchronous. */
int spmdb200_jacobi2d_host(float *U_base, float *U_aligned, int64_t U_offset, int64_t U_size0, int64_t U_size1,
                           int64_t U_stride0, int64_t U_stride1,
                           int64_t sweeps, int64_t res_every, double *res_out);

/* The same job on a batch of `count` independent HOST grids that share one
 * shape and row pitch: grid k is U_aligned[k] + U_offset (H x W, row pitch
 * stride0 elements, stride1 == 1); its residuals go to res_out[k] (res_out may
 * be NULL when res_every == 0).  Each grid is swept in place exactly as
 * spmdb200_jacobi2d_host would sweep it.  The grids run one after another on
 * the GPU through two device slots.  Grid k+1's upload and grid k-1's download
 * run on their own streams while grid k is swept, so the PCIe copies overlap
 * the sweeps.  With pinned host grids, the batch costs the sweeps plus one
 * upload and one download.  Pageable grids give the same results, but their
 * copies do not overlap.  The grids must not overlap one another in host
 * memory.  Synchronous.  No reference counterpart (the reference has no
 * Jacobi entry); it serves a stream of independent grids. */
int spmdb200_jacobi2d_host_batch(int64_t count, float *const *U_aligned, int64_t U_offset, int64_t U_size0,
                                 int64_t U_size1, int64_t U_stride0, int64_t U_stride1,
                                 int64_t sweeps, int64_t res_every, double *const *res_out);

/* ---- Jacobi-2D over row slabs on several GPUs (one process per GPU) ------ */
/* No reference counterpart: the reference runs on one GPU.  The global grid
 * has G rows; this rank owns global rows [g_first, g_first + R), R >= 8.  U
 * and V are (R + 16) x W local arrays (descriptor sizes (R+16, W), stride1 ==
 * 1, 16-byte aligned rows): local rows 0-7 are the eight halo rows above
 * (global g_first - 8 .. g_first - 1), rows 8..R+7 are owned, rows
 * R+8..R+15 are the halo rows below.  The kernel fuses up to eight sweeps per
 * pass and keeps every halo current over NVLink: before its first pass each
 * run stores its first / last eight owned rows of U into the neighbours' halo
 * rows, and every pass does the same with the rows it writes (halo rows of
 * U need not hold anything on entry).  up_* / dn_* are the neighbours' U, V
 * and workspace as mapped in this process (spmdb200_ipc_open), NULL at the
 * global top / bottom; up_rows is the number of rows the neighbour above owns
 * (our first owned rows land in its local rows up_rows + 8 .. up_rows + 15).
 * all_ws[q] is rank q's workspace as mapped here (all_ws[rank] is `ws`); the
 * residual of every residual sweep is all-gathered into each rank's
 * workspace.  *deliveries (host, in/out) counts the halo deliveries this rank
 * has received from each neighbour since the workspaces were cleared: 0 for
 * the first run after every rank cleared its workspace
 * (spmdb200_jacobi_ws_reset) and all ranks waited for one another, then
 * whatever the previous call left in it.  The kernel waits on these
 * monotonic counters, so back-to-back runs need no host synchronisation
 * between them.  res_out (device, optional) receives this rank's local
 * residual contributions.  Sweep semantics and ping-pong are those of
 * spmdb200_jacobi2d; global rows 0 and G-1 and columns 0 and W-1 are
 * fixed. */
int spmdb200_jacobi2d_slab(float *U_base, float *U_aligned, int64_t U_offset, int64_t U_size0, int64_t U_size1,
                           int64_t U_stride0, int64_t U_stride1,
                           float *V_base, float *V_aligned, int64_t V_offset, int64_t V_size0, int64_t V_size1,
                           int64_t V_stride0, int64_t V_stride1,
                           int64_t g_first, int64_t G, int64_t sweeps, int64_t res_every, double *res_out,
                           void *ws, float *up_u, float *up_v, void *up_ws, int64_t up_rows,
                           float *dn_u, float *dn_v, void *dn_ws,
                           int rank, int nranks, void *const *all_ws, int64_t *deliveries, void *stream);
/* Jacobi-3D over z-slabs on several GPUs (one process per GPU).  No reference
 * counterpart.  The global grid has D planes of H x W; this rank owns global
 * planes [z_first, z_first + Z), Z >= 2.  U and V are (Z + 4) x H x W local
 * arrays (descriptor sizes (Z+4, H, W), x contiguous, 16-byte aligned rows and
 * planes): local planes 0..1 are the halo planes above (global z_first - 2 ..
 * z_first - 1), planes 2..Z+1 are owned, planes Z+2..Z+3 are the halo planes
 * below.  A run advances up to two sweeps per pass; the kernel stores the
 * first / last owned planes of each pass straight into the neighbour's halo
 * planes over NVLink, and before its first pass it delivers its input's edge
 * planes the same way.  up_planes is the number of planes the neighbour
 * above owns (>= 2; our first owned plane lands in its local plane
 * up_planes + 2).  All ranks' arrays share H, W and the row and plane
 * strides.  Neighbour, workspace, delivery-count, residual and ping-pong
 * semantics are those of spmdb200_jacobi2d_slab
 * (spmdb200_jacobi2d_slab_residuals reads the all-gathered residuals);
 * global planes 0 and D-1, rows 0 and H-1 and columns 0 and W-1 are fixed. */
int spmdb200_jacobi3d_slab(float *U_base, float *U_aligned, int64_t U_offset, int64_t U_size0, int64_t U_size1,
                           int64_t U_size2, int64_t U_stride0, int64_t U_stride1, int64_t U_stride2,
                           float *V_base, float *V_aligned, int64_t V_offset, int64_t V_size0, int64_t V_size1,
                           int64_t V_size2, int64_t V_stride0, int64_t V_stride1, int64_t V_stride2,
                           int64_t z_first, int64_t D, int64_t sweeps, int64_t res_every, double *res_out,
                           void *ws, float *up_u, float *up_v, void *up_ws, int64_t up_planes,
                           float *dn_u, float *dn_v, void *dn_ws,
                           int rank, int nranks, void *const *all_ws, int64_t *deliveries, void *stream);
/* Halo depth of the slab layouts: rows on each side of a Jacobi-2D row slab
 * (dims == 2: 8) or planes on each side of a Jacobi-3D z-slab (dims == 3: 2);
 * -1 for other dims.  No reference counterpart. */
int spmdb200_jacobi_slab_halo(int dims);
/* Clears the 256-byte header of a Jacobi workspace on `stream`. */
int spmdb200_jacobi_ws_reset(void *ws, void *stream);
/* After every rank's slab run has finished: res_host[r] = sum over ranks q
 * (in rank order) of rank q's residual contribution r, r < nres.  Synchronous. */
int spmdb200_jacobi2d_slab_residuals(void *ws, int nranks, int64_t nres, double *res_host);

/* Device memory and CUDA IPC for the slab path (cudaMalloc'd, so IPC-able). */
int spmdb200_dev_alloc(size_t bytes, void **out);
int spmdb200_dev_free(void *p);
/* Copies `bytes` between any two addresses (host or device; direction from
 * unified addressing) on `stream`, then synchronises it. */
int spmdb200_memcpy(void *dst, const void *src, size_t bytes, void *stream);
/* The same copy, asynchronous on `stream` (pinned host memory for overlap;
 * the caller orders it with events).  No reference counterpart. */
int spmdb200_memcpy_async(void *dst, const void *src, size_t bytes, void *stream);
/* 64-byte IPC handle of a spmdb200_dev_alloc pointer. */
int spmdb200_ipc_handle(void *dev_ptr, void *handle64_out);
int spmdb200_ipc_open(const void *handle64, void **dev_ptr_out);
int spmdb200_ipc_close(void *dev_ptr);
/* Fills a rows x W block of a row-major f32 grid (row pitch `pitch`) with the
 * seeded synthetic Jacobi input: cell (g, c) of the global G x W grid, g =
 * g_row0 + local row, is uniform [0,1) from a counter-based hash of
 * (seed, g, c); global boundary rows/columns and rows outside [0, G) are 0.
 * Every rank computes the same value for a global cell, so halos need no
 * exchange at start-up. */
int spmdb200_fill_jacobi_input(float *p, int64_t pitch, int64_t rows, int64_t W, int64_t g_row0, int64_t G,
                               uint64_t seed, void *stream);
/* The 3-D counterpart: `planes` planes of an H x W grid (strides plane_stride,
 * row_stride, x contiguous), local plane 0 = global plane g_z0 of D; cell
 * (gz, y, x) is uniform [0,1) from the hash of (seed, gz * H + y, x), global
 * boundary cells and planes outside [0, D) are 0. */
int spmdb200_fill_jacobi3d_input(float *p, int64_t plane_stride, int64_t row_stride, int64_t planes, int64_t H,
                                 int64_t W, int64_t g_z0, int64_t D, uint64_t seed, void *stream);

/* ---- Jacobi-3D 7-point --------------------------------------------------- */
/* One sweep over the D x H x W grid (index order [z][y][x]):
 *   boundary (any index at 0 or size-1): V = U
 *   interior: V = fmul((((((c + U[z][y][x-1]) + U[z][y][x+1]) + U[z][y-1][x])
 *                      + U[z][y+1][x]) + U[z-1][y][x]) + U[z+1][y][x]), 1.0f/7.0f)
 * with 1.0f/7.0f rounded to f32 once.  Ping-pong and residual contract as
 * spmdb200_jacobi2d. */
int spmdb200_jacobi3d(float *U_base, float *U_aligned, int64_t U_offset,
                      int64_t U_size0, int64_t U_size1, int64_t U_size2,
                      int64_t U_stride0, int64_t U_stride1, int64_t U_stride2,
                      float *V_base, float *V_aligned, int64_t V_offset,
                      int64_t V_size0, int64_t V_size1, int64_t V_size2,
                      int64_t V_stride0, int64_t V_stride1, int64_t V_stride2,
                      int64_t sweeps, int64_t res_every, double *res_out,
                      void *ws, size_t ws_bytes, void *stream);

/* =========================================================================
 * C. End-to-end host entries for configurations without a reference entry.
 * ========================================================================= */

/* Y = a*X + Y on host buffers (copy in, kernel, copy out). */
int spmdb200_axpy_host(float a,
                       float *X_base, float *X_aligned, int64_t X_offset, int64_t X_size, int64_t X_stride,
                       float *Y_base, float *Y_aligned, int64_t Y_offset, int64_t Y_size, int64_t Y_stride,
                       int64_t N);

/* out[] = (float)((double)out[] + sum(A)) on host buffers (deterministic). */
int spmdb200_sum_f32_host(float *A_base, float *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                          float *out_base, float *out_aligned, int64_t out_offset,
                          int64_t N);

/* out[] += sum(A) (int32, wrapping) on host buffers. */
int spmdb200_sum_i32_host(int32_t *A_base, int32_t *A_aligned, int64_t A_offset, int64_t A_size, int64_t A_stride,
                          int32_t *out_base, int32_t *out_aligned, int64_t out_offset,
                          int64_t N);

#ifdef __cplusplus
}
#endif
#endif /* SPMD_B200_H */
