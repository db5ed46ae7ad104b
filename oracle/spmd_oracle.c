/*
 * spmd_oracle.c -- CPU ORACLE for the spmd-dialect hot path.  TEST
 * INFRASTRUCTURE ONLY: the parity tests, the smoke check and the CPU-baseline
 * leg of the benchmark load it as the checker.  The product library
 * (libspmdb200.so) never links, loads or calls anything in this directory.
 *
 * It restates, in plain C with OpenMP, what the reference's CPU lowerings
 * produce for each kernel:
 *   - lib/Conversion/SPMDToSCF/SPMDToSCF.cpp:38-78   forall -> nested scf.for
 *   - lib/Conversion/SPMDToSCF/SPMDToSCF.cpp:147-214 reduce -> scf.for with an
 *     iter_arg, combine acc = acc (+) partial in increasing index order
 *   - lib/Conversion/SPMDToOpenMP/SPMDToOpenMP.cpp:48-118 group forall ->
 *     omp.parallel { omp.wsloop { loop_nest collapse(rank) } }, no clauses, so
 *     the default static schedule over group tiles
 *   - lib/Transforms/MaterializeTilingAndMapping.cpp:136-173 tile split
 *     iv = outer + inner*step with the iv < ub guard on every lane
 *   - lib/Transforms/PlanSPMDSchedule.cpp:74-82 default tile [32, 8, 8 ...]
 *   - lib/Transforms/PromoteGroupMemory.cpp:62-97,256-298: promotion changes
 *     only where a value is read from (tile vs. global), never the arithmetic,
 *     so the oracle reads the global arrays directly.
 * Per-cell arithmetic follows MLIR source order with no contraction; this
 * file must be compiled with -ffp-contract=off and without fast-math.
 *
 * Exported names `ewise`, `stencil_cpu`, `atomic_sum`, `hierarchical_sum`
 * carry the exact unpacked-memref signatures harness/run_host.py:84-203 binds,
 * so the reference's own host harness can drive this library.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define EXPORT __attribute__((visibility("default")))

/* Reads an element of a 2-D descriptor; positions outside (size0, size1)
 * contribute 0.  (The reference CPU twin reads A[i+1][j] and A[i][j+1] with A
 * sized (N+1)x(M+1), harness/run_host.py:121-137, so in-range callers never
 * reach the zero branch.) */
static inline float ld2(const float *a, int64_t off, int64_t s0, int64_t s1,
                        int64_t st0, int64_t st1, int64_t i, int64_t j) {
  if (i < 0 || j < 0 || i >= s0 || j >= s1) return 0.0f;
  return a[off + i * st0 + j * st1];
}

EXPORT int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Sets the OpenMP team size of later parallel regions on the calling thread
 * (launchers such as torchrun export OMP_NUM_THREADS=1; the timed CPU
 * baseline sets the host's core count explicitly).  Returns the new count. */
EXPORT int oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n >= 1) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

/* ---------------------------------------------------------------------------
 * ewise: C[i] = A[i] + B[i]   (test/SPMD/lower-to-gpu-nvptx.mlir:54-71)
 * Group forall over tiles of 32 (spmd.tile_sizes = [32]); OpenMP static over
 * tiles; lane loop guarded by i < N.
 * ------------------------------------------------------------------------- */
EXPORT void ewise(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                  float *B_base, float *B, int64_t B_off, int64_t B_size, int64_t B_st,
                  float *C_base, float *C, int64_t C_off, int64_t C_size, int64_t C_st,
                  int64_t N) {
  (void)A_base; (void)B_base; (void)C_base; (void)A_size; (void)B_size; (void)C_size;
  const int64_t T = 32;
  const int64_t ntiles = (N + T - 1) / T;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < ntiles; ++t) {
    for (int64_t l = 0; l < T; ++l) {
      int64_t i = t * T + l;
      if (i < N) C[C_off + i * C_st] = A[A_off + i * A_st] + B[B_off + i * B_st];
    }
  }
}

/* axpy: Y[i] = fadd(fmul(a, X[i]), Y[i]) -- the elementwise forall
 * y = a*x + y written in MLIR source order (arith.mulf then arith.addf). */
EXPORT void oracle_axpy(float a,
                        float *X_base, float *X, int64_t X_off, int64_t X_size, int64_t X_st,
                        float *Y_base, float *Y, int64_t Y_off, int64_t Y_size, int64_t Y_st,
                        int64_t N) {
  (void)X_base; (void)Y_base; (void)X_size; (void)Y_size;
  if (X_st == 1 && Y_st == 1) {
    const float *x = X + X_off;
    float *y = Y + Y_off;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < N; ++i) {
      float p = a * x[i];
      y[i] = p + y[i];
    }
    return;
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < N; ++i) {
    float p = a * X[X_off + i * X_st];
    Y[Y_off + i * Y_st] = p + Y[Y_off + i * Y_st];
  }
}

/* ---------------------------------------------------------------------------
 * stencil_cpu: B[i,j] = (A[i,j] + A[i,j+1]) + A[i+1,j]
 * (test/SPMD/differential-stencil.mlir:19-37; the promoted GPU instance
 * test/SPMD/lower-to-gpu-nvptx-promoted.mlir:32-67 has the same body).
 * Default plan tile [32, 8], OpenMP static over the collapsed tile loops.
 * ------------------------------------------------------------------------- */
EXPORT void stencil_cpu(float *A_base, float *A, int64_t A_off, int64_t A_s0, int64_t A_s1,
                        int64_t A_st0, int64_t A_st1,
                        float *B_base, float *B, int64_t B_off, int64_t B_s0, int64_t B_s1,
                        int64_t B_st0, int64_t B_st1,
                        int64_t N, int64_t M) {
  (void)A_base; (void)B_base; (void)B_s0; (void)B_s1;
  const int64_t T0 = 32, T1 = 8;
  const int64_t nt0 = (N + T0 - 1) / T0, nt1 = (M + T1 - 1) / T1;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t ti = 0; ti < nt0; ++ti) {
    for (int64_t tj = 0; tj < nt1; ++tj) {
      for (int64_t a = 0; a < T0; ++a) {
        int64_t i = ti * T0 + a;
        if (i >= N) continue;
        for (int64_t b = 0; b < T1; ++b) {
          int64_t j = tj * T1 + b;
          if (j >= M) continue;
          float center = ld2(A, A_off, A_s0, A_s1, A_st0, A_st1, i, j);
          float right = ld2(A, A_off, A_s0, A_s1, A_st0, A_st1, i, j + 1);
          float down = ld2(A, A_off, A_s0, A_s1, A_st0, A_st1, i + 1, j);
          float t0 = center + right;
          float t1 = t0 + down;
          B[B_off + i * B_st0 + j * B_st1] = t1;
        }
      }
    }
  }
}

/* ---------------------------------------------------------------------------
 * atomic_sum: out += A[i] for every i, the SCF lowering's serial order
 * (test/SPMD/lower-to-gpu-nvptx-reduction.mlir:30-44).
 * ------------------------------------------------------------------------- */
EXPORT void atomic_sum(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                       float *o_base, float *o, int64_t o_off, int64_t N) {
  (void)A_base; (void)A_size; (void)o_base;
  float acc = o[o_off];
  for (int64_t i = 0; i < N; ++i) acc = acc + A[A_off + i * A_st];
  o[o_off] = acc;
}

/* hierarchical_sum: for each 256-element tile (group forall step 256), an
 * spmd.reduce over [0,256) starting from 0.0f with out-of-range lanes yielding
 * 0.0f, then one atomic_rmw addf of the tile sum into out; SCF order = tiles in
 * increasing order (test/SPMD/lower-to-gpu-nvptx-hierarchical-reduction.mlir:
 * 58-88, SPMDToSCF.cpp:147-214). */
EXPORT void hierarchical_sum(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                             float *o_base, float *o, int64_t o_off, int64_t N) {
  (void)A_base; (void)A_size; (void)o_base;
  const int64_t T = 256;
  float acc = o[o_off];
  for (int64_t t = 0; t < N; t += T) {
    float s = 0.0f;
    for (int64_t l = 0; l < T; ++l) {
      int64_t g = t + l;
      float v = (g < N) ? A[A_off + g * A_st] : 0.0f;
      s = s + v;
    }
    acc = acc + s;
  }
  o[o_off] = acc;
}

/* The SPMDToOpenMP form of hierarchical_sum (SPMDToOpenMP.cpp:48-118): the
 * group forall over 256-element tiles becomes an OpenMP static worksharing
 * loop, each tile reduces serially from 0.0f, and the tile sums meet in one
 * atomic add -- so the f32 result depends on thread timing.  Used as the
 * timed CPU baseline; parity checks use the serial hierarchical_sum above. */
EXPORT void hierarchical_sum_omp(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                                 float *o_base, float *o, int64_t o_off, int64_t N) {
  (void)A_base; (void)A_size; (void)o_base;
  const int64_t T = 256;
  const int64_t ntiles = (N + T - 1) / T;
  float *out = o + o_off;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < ntiles; ++t) {
    float s = 0.0f;
    for (int64_t l = 0; l < T; ++l) {
      int64_t g = t * T + l;
      float v = (g < N) ? A[A_off + g * A_st] : 0.0f;
      s = s + v;
    }
#pragma omp atomic
    *out += s;
  }
}

/* f64 reference sum (the yardstick the f32 reductions are held to). */
EXPORT double oracle_sum_f64(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                             int64_t N) {
  (void)A_base; (void)A_size;
  double acc = 0.0;
  for (int64_t i = 0; i < N; ++i) acc += (double)A[A_off + i * A_st];
  return acc;
}

/* i32 add reduce: arith.addi wraps modulo 2^32, so any order gives the same
 * bits; ReduceToSCFForGPU / ReduceToSCFFor combine (SPMDToSCF.cpp:153-155). */
EXPORT int32_t oracle_sum_i32(int32_t *A_base, int32_t *A, int64_t A_off, int64_t A_size,
                              int64_t A_st, int64_t N) {
  (void)A_base; (void)A_size;
  uint32_t acc = 0;
#pragma omp parallel for reduction(+ : acc) schedule(static)
  for (int64_t i = 0; i < N; ++i) acc += (uint32_t)A[A_off + i * A_st];
  return (int32_t)acc;
}

/* ---------------------------------------------------------------------------
 * Reduce-kind table (spmd.reduction_kind add/mul/max/min/and/or/xor,
 * include/spmd/IR/SPMDAttrs.td:74-89; combine ops SPMDToGPU.cpp:425-449).
 * Serial in increasing index order from `init`, exactly the SCF fallback.
 * kind: 0 add, 1 mul, 2 max, 3 min, 4 and, 5 or, 6 xor.
 * f32 max/min are arith.maximumf/minimumf: NaN-propagating, -0 < +0.
 * ------------------------------------------------------------------------- */
static inline float f_maximum(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  if (a == b) return signbit(a) ? b : a; /* +0 wins over -0 */
  return a > b ? a : b;
}
static inline float f_minimum(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  if (a == b) return signbit(a) ? a : b; /* -0 wins over +0 */
  return a < b ? a : b;
}
EXPORT float oracle_reduce_f32(int kind, const float *A, int64_t N, float init) {
  float acc = init;
  for (int64_t i = 0; i < N; ++i) {
    float v = A[i];
    switch (kind) {
      case 0: acc = acc + v; break;
      case 1: acc = acc * v; break;
      case 2: acc = f_maximum(acc, v); break;
      case 3: acc = f_minimum(acc, v); break;
      default: return NAN;
    }
  }
  return acc;
}
EXPORT int32_t oracle_reduce_i32(int kind, const int32_t *A, int64_t N, int32_t init) {
  uint32_t acc = (uint32_t)init;
  for (int64_t i = 0; i < N; ++i) {
    uint32_t v = (uint32_t)A[i];
    switch (kind) {
      case 0: acc = acc + v; break;
      case 1: acc = acc * v; break;
      case 2: acc = ((int32_t)acc >= (int32_t)v) ? acc : v; break;
      case 3: acc = ((int32_t)acc <= (int32_t)v) ? acc : v; break;
      case 4: acc = acc & v; break;
      case 5: acc = acc | v; break;
      case 6: acc = acc ^ v; break;
      default: return 0;
    }
  }
  return (int32_t)acc;
}

/* ---------------------------------------------------------------------------
 * Elementwise forall with a general f32 body.  SPMDToSCF.cpp:38-78 turns the
 * forall into nested scf.for loops (row-major order) and the body's arith ops
 * run once per point in SSA order, each rounded on its own.  The body arrives
 * as the straight-line program spmdb200_forall_map takes: two int32 words per
 * instruction, w0 = op | dst << 8 | a << 16 | b << 24, w1 = aux; opcodes
 * 0 LOAD, 1 CONST, 2 ADD, 3 SUB, 4 MUL, 5 DIV, 6 MAXIMUM (arith.maximumf),
 * 7 MINIMUM, 8 NEG, 9 ABS (math.absf), 10 SQRT (math.sqrt), 11 CMP
 * (arith.cmpf, aux = predicate number), 12 SELECT (aux = condition register),
 * 13 AND, 14 OR, 15 XOR (i1 values as 0 / 1), 16 STORE.  Strides in elements,
 * `rank` per input, row after row.
 * ------------------------------------------------------------------------- */
static int cmpf_pred(int pred, float x, float y) {
  const int u = isnan(x) || isnan(y);
  switch (pred) {
    case 1: return x == y;
    case 2: return x > y;
    case 3: return x >= y;
    case 4: return x < y;
    case 5: return x <= y;
    case 6: return !u && x != y;
    case 7: return !u;
    case 8: return u || x == y;
    case 9: return u || x > y;
    case 10: return u || x >= y;
    case 11: return u || x < y;
    case 12: return u || x <= y;
    case 13: return x != y;
    case 14: return u;
    case 15: return 1;
    default: return 0;
  }
}
EXPORT void oracle_forall_map(int rank, const int64_t *sizes, int n_in, const float *const *in,
                              const int64_t *in_st, float *out, const int64_t *out_st, const int32_t *code,
                              int n_insns, const float *consts) {
  int64_t sz[3] = {1, 1, 1}, ost[3] = {0, 0, 0}, ist[8][3];
  memset(ist, 0, sizeof(ist));
  for (int d = 0; d < rank; ++d) {
    sz[3 - rank + d] = sizes[d];
    ost[3 - rank + d] = out_st[d];
    for (int k = 0; k < n_in && k < 8; ++k) ist[k][3 - rank + d] = in_st[k * rank + d];
  }
  for (int64_t i0 = 0; i0 < sz[0]; ++i0)
    for (int64_t i1 = 0; i1 < sz[1]; ++i1)
      for (int64_t i2 = 0; i2 < sz[2]; ++i2) {
        float r[16] = {0};
        for (int pc = 0; pc < n_insns; ++pc) {
          const int32_t w0 = code[2 * pc], aux = code[2 * pc + 1];
          const int op = w0 & 255, d = (w0 >> 8) & 255, a = (w0 >> 16) & 255, b = (int)((uint32_t)w0 >> 24);
          const float x = r[a & 15], y = r[b & 15];
          float v = 0.0f;
          switch (op) {
            case 0: v = in[aux][i0 * ist[aux][0] + i1 * ist[aux][1] + i2 * ist[aux][2]]; break;
            case 1: v = consts[aux]; break;
            case 2: v = x + y; break;
            case 3: v = x - y; break;
            case 4: v = x * y; break;
            case 5: v = x / y; break;
            case 6: v = f_maximum(x, y); break;
            case 7: v = f_minimum(x, y); break;
            case 8: v = -x; break;
            case 9: v = fabsf(x); break;
            case 10: v = sqrtf(x); break;
            case 11: v = cmpf_pred(aux, x, y) ? 1.0f : 0.0f; break;
            case 12: v = r[aux & 15] != 0.0f ? x : y; break;
            case 13: v = (x != 0.0f && y != 0.0f) ? 1.0f : 0.0f; break;
            case 14: v = (x != 0.0f || y != 0.0f) ? 1.0f : 0.0f; break;
            case 15: v = ((x != 0.0f) != (y != 0.0f)) ? 1.0f : 0.0f; break;
            default: out[i0 * ost[0] + i1 * ost[1] + i2 * ost[2]] = x; continue;
          }
          r[d & 15] = v;
        }
      }
}

/* ---------------------------------------------------------------------------
 * Jacobi-2D 5-point sweep over local rows [row_lo, row_hi) of a row-major grid
 * with `pitch` elements per row and W columns.  Global row index of local row r
 * is g_row0 + r; global rows 0 and G-1 and columns 0 and W-1 are the fixed
 * (Dirichlet) boundary and are copied.  Interior order: MLIR source order
 *   ((((c + n) + s) + e) + w) * 0.2f
 * with n = u[i-1][j], s = u[i+1][j], e = u[i][j+1], w = u[i][j-1].
 * When row_res != NULL, row_res[r - row_lo] = sum_j ((double)v - (double)u)^2
 * accumulated left to right.  A single-domain sweep is (row_lo=0, row_hi=H,
 * g_row0=0, G=H); a row slab with halo rows 0 and R+1 is (1, R+1, p*R-1, G).
 * ------------------------------------------------------------------------- */
EXPORT void oracle_jacobi2d_rows(const float *u, float *v, int64_t pitch, int64_t W,
                                 int64_t row_lo, int64_t row_hi, int64_t g_row0, int64_t G,
                                 double *row_res) {
  const float k = 0.2f;
#pragma omp parallel for schedule(static)
  for (int64_t r = row_lo; r < row_hi; ++r) {
    const int64_t g = g_row0 + r;
    const float *uc = u + r * pitch;
    float *vr = v + r * pitch;
    double acc = 0.0;
    if (g == 0 || g == G - 1) {
      for (int64_t j = 0; j < W; ++j) vr[j] = uc[j];
    } else {
      const float *un = uc - pitch;
      const float *us = uc + pitch;
      vr[0] = uc[0];
      if (row_res) {
        for (int64_t j = 1; j < W - 1; ++j) {
          float t = uc[j] + un[j];
          t = t + us[j];
          t = t + uc[j + 1];
          t = t + uc[j - 1];
          float o = t * k;
          vr[j] = o;
          double d = (double)o - (double)uc[j];
          double d2 = d * d;
          acc = acc + d2;
        }
      } else {
        for (int64_t j = 1; j < W - 1; ++j) {
          float t = uc[j] + un[j];
          t = t + us[j];
          t = t + uc[j + 1];
          t = t + uc[j - 1];
          vr[j] = t * k;
        }
      }
      if (W > 1) vr[W - 1] = uc[W - 1];
    }
    if (row_res) row_res[r - row_lo] = acc;
  }
}

/* Full Jacobi-2D run on an H x W grid (same ping-pong and residual contract as
 * spmdb200_jacobi2d).  Residual = f64 sum of per-row partials in row order. */
EXPORT void oracle_jacobi2d(float *U_base, float *U, int64_t U_off, int64_t H, int64_t W,
                            int64_t U_st0, int64_t U_st1,
                            float *V_base, float *V, int64_t V_off, int64_t V_s0, int64_t V_s1,
                            int64_t V_st0, int64_t V_st1,
                            int64_t sweeps, int64_t res_every, double *res_out) {
  (void)U_base; (void)V_base; (void)V_s0; (void)V_s1; (void)V_st0; (void)V_st1; (void)U_st1;
  float *a = U + U_off, *b = V + V_off;
  double *row_res = (res_every > 0) ? (double *)malloc(sizeof(double) * (size_t)(H > 0 ? H : 1)) : NULL;
  for (int64_t k = 1; k <= sweeps; ++k) {
    const int want = (res_every > 0) && (k % res_every == 0);
    oracle_jacobi2d_rows(a, b, U_st0, W, 0, H, 0, H, want ? row_res : NULL);
    if (want) {
      double tot = 0.0;
      for (int64_t r = 0; r < H; ++r) tot = tot + row_res[r];
      res_out[k / res_every - 1] = tot;
    }
    float *t = a; a = b; b = t;
  }
  free(row_res);
}

/* ---------------------------------------------------------------------------
 * Jacobi-3D 7-point sweep over planes [z_lo, z_hi) of a D x H x W grid with
 * strides (sz, sy, 1).  Boundary cells copied; interior in MLIR source order
 *   ((((((c + xm) + xp) + ym) + yp) + zm) + zp) * (1.0f/7.0f)
 * with the constant rounded to f32 once.  plane_res[z - z_lo] (when non-NULL)
 * = per-plane sum of squared updates, rows left to right, planes in order.
 * The arrays may hold a z-slab of a larger grid: local plane z is global plane
 * g_z0 + z of D (the boundary test is on the global index).
 * ------------------------------------------------------------------------- */
EXPORT void oracle_jacobi3d_slab_planes(const float *u, float *v, int64_t g_z0, int64_t D, int64_t H,
                                        int64_t W, int64_t sz, int64_t sy, int64_t z_lo, int64_t z_hi,
                                        double *plane_res) {
  const float k = 1.0f / 7.0f;
#pragma omp parallel for schedule(static)
  for (int64_t z = z_lo; z < z_hi; ++z) {
    double pacc = 0.0;
    const int64_t gz = g_z0 + z;
    for (int64_t y = 0; y < H; ++y) {
      const float *uc = u + z * sz + y * sy;
      float *vr = v + z * sz + y * sy;
      if (gz == 0 || gz == D - 1 || y == 0 || y == H - 1) {
        for (int64_t x = 0; x < W; ++x) vr[x] = uc[x];
        continue;
      }
      const float *uym = uc - sy, *uyp = uc + sy, *uzm = uc - sz, *uzp = uc + sz;
      vr[0] = uc[0];
      double racc = 0.0;
      for (int64_t x = 1; x < W - 1; ++x) {
        float t = uc[x] + uc[x - 1];
        t = t + uc[x + 1];
        t = t + uym[x];
        t = t + uyp[x];
        t = t + uzm[x];
        t = t + uzp[x];
        float o = t * k;
        vr[x] = o;
        if (plane_res) {
          double d = (double)o - (double)uc[x];
          double d2 = d * d;
          racc = racc + d2;
        }
      }
      if (W > 1) vr[W - 1] = uc[W - 1];
      pacc = pacc + racc;
    }
    if (plane_res) plane_res[z - z_lo] = pacc;
  }
}

EXPORT void oracle_jacobi3d_planes(const float *u, float *v, int64_t D, int64_t H, int64_t W,
                                   int64_t sz, int64_t sy, int64_t z_lo, int64_t z_hi,
                                   double *plane_res) {
  oracle_jacobi3d_slab_planes(u, v, 0, D, H, W, sz, sy, z_lo, z_hi, plane_res);
}

EXPORT void oracle_jacobi3d(float *U_base, float *U, int64_t U_off, int64_t D, int64_t H, int64_t W,
                            int64_t U_st0, int64_t U_st1, int64_t U_st2,
                            float *V_base, float *V, int64_t V_off, int64_t V_s0, int64_t V_s1,
                            int64_t V_s2, int64_t V_st0, int64_t V_st1, int64_t V_st2,
                            int64_t sweeps, int64_t res_every, double *res_out) {
  (void)U_base; (void)V_base; (void)V_s0; (void)V_s1; (void)V_s2;
  (void)V_st0; (void)V_st1; (void)V_st2; (void)U_st2;
  float *a = U + U_off, *b = V + V_off;
  double *pres = (res_every > 0) ? (double *)malloc(sizeof(double) * (size_t)(D > 0 ? D : 1)) : NULL;
  for (int64_t k = 1; k <= sweeps; ++k) {
    const int want = (res_every > 0) && (k % res_every == 0);
    oracle_jacobi3d_planes(a, b, D, H, W, U_st0, U_st1, 0, D, want ? pres : NULL);
    if (want) {
      double tot = 0.0;
      for (int64_t z = 0; z < D; ++z) tot = tot + pres[z];
      res_out[k / res_every - 1] = tot;
    }
    float *t = a; a = b; b = t;
  }
  free(pres);
}

/* ---------------------------------------------------------------------------
 * General linear stencil, rank 1-3 (the body behind PromoteGroupMemory's
 * promoted tiles, lib/Transforms/PromoteGroupMemory.cpp:113-314, evaluated on
 * the original arrays since promotion only changes where values are read,
 * rewriteLoadsToTile :62-97):  for every output point p = (k0*step0, ...)
 * inside B's sizes, in row-major order,
 *   t = w0*A[p+off0]; t = t + wk*A[p+offk] (k = 1..); B[p] = t*scale
 * with no multiply when weights == NULL (all 1) or scale == 1.  Reads outside
 * A's sizes are 0.  Strides in elements.
 * ------------------------------------------------------------------------- */
EXPORT void oracle_stencil_nd(int rank, const float *A, const int64_t *a_size, const int64_t *a_stride,
                              float *B, const int64_t *b_size, const int64_t *b_stride, int ntaps,
                              const int64_t *off, const float *w, float scale, const int64_t *step) {
  int64_t npts[3] = {1, 1, 1}, st[3] = {1, 1, 1};
  for (int d = 0; d < rank; ++d) {
    st[d] = step ? step[d] : 1;
    npts[d] = (b_size[d] + st[d] - 1) / st[d];
  }
  const int64_t total = npts[0] * npts[1] * npts[2];
  for (int64_t q = 0; q < total; ++q) {
    int64_t r = q, o[3] = {0, 0, 0}, boff = 0;
    for (int d = rank - 1; d >= 0; --d) {
      o[d] = (r % npts[d]) * st[d];
      r /= npts[d];
      boff += o[d] * b_stride[d];
    }
    float t = 0.0f;
    for (int j = 0; j < ntaps; ++j) {
      int64_t aoff = 0;
      int in = 1;
      for (int d = 0; d < rank; ++d) {
        const int64_t g = o[d] + off[j * rank + d];
        in = in && g >= 0 && g < a_size[d];
        aoff += g * a_stride[d];
      }
      float v = in ? A[aoff] : 0.0f;
      if (w) v = w[j] * v;
      t = j == 0 ? v : t + v;
    }
    B[boff] = scale != 1.0f ? t * scale : t;
  }
}
