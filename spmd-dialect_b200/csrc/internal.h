// internal.h -- launchers shared between the translation units of libspmdb200.
// Every launcher is asynchronous on `stream`, assumes validated arguments and
// returns the cudaError_t of its launch.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace spmdb200 {

// ---- elementwise (ewise.cu) -------------------------------------------------
cudaError_t launch_ewise_add(View1 a, View1 b, View1 c, int64_t n, cudaStream_t s);
cudaError_t launch_axpy(float alpha, View1 x, View1 y, int64_t n, cudaStream_t s);

// ---- reductions (reduce.cu) ---------------------------------------------------
// Workspace of the deterministic f32 sum: [ticket u32 | pad to 256 B | 8-byte
// partials].  All-zero between calls: every kernel that uses it clears the
// ticket and the partial words it wrote (the staged sum reads a non-zero word
// as a written partial).
size_t sum_f32_workspace_bytes(int64_t n);
int sum_f32_grid(int64_t n);
// f64_out set: the unrounded f64 total goes there and `out` is not touched.
cudaError_t launch_sum_f32(View1 a, float *out, int64_t n, void *ws, cudaStream_t s, double *f64_out = nullptr);
cudaError_t launch_sum_i32(const int32_t *a, int64_t stride, int32_t *out, int64_t n, cudaStream_t s);
cudaError_t launch_hier_sum_f32(View1 a, float *out, int64_t n, cudaStream_t s);
// Every spmd.reduce kind (0 add, 1 mul, 2 max, 3 min, 4 and, 5 or, 6 xor):
// out = init (+) reduce(a); ws = [ticket | pad to 256 B | 8-byte partials].
cudaError_t launch_reduce_f32(int kind, const float *a, int64_t sa, int64_t n, float *out, float init, void *ws,
                              cudaStream_t s);
cudaError_t launch_reduce_i32(int kind, const int32_t *a, int64_t sa, int64_t n, int32_t *out, int32_t init,
                              void *ws, cudaStream_t s);
// Device flags set when a bounded wait of a staged sum / staged kind reduction
// expired (-1 on error).
int reduction_timeout_flag(bool clear);
int kind_timeout_flag(bool clear);

// ---- 3-point promoted stencil (stencil3.cu) -----------------------------------------
cudaError_t launch_stencil3(View2 a, View2 b, int64_t n, int64_t m, cudaStream_t s);

// ---- Jacobi (jacobi2d.cu / jacobi3d.cu) ---------------------------------------------
constexpr int kMaxCtas = 2048;
constexpr int kMaxRanks = 8;
constexpr int kMaxResSlots = 1024;
// Residual partial slots: at least twice the residuals one pass can produce
// (a pass fuses up to 8 sweeps).
constexpr int kJacobiPartialSlots = 16;

// Device workspace of every Jacobi run.  The 256-byte header is cleared by the
// host before each run.
struct JacobiWs {
  unsigned barrier;    // grid-barrier arrivals (one per CTA per sweep)
  int status;          // DevStatus of the run
  unsigned from_above; // halo-tile deliveries received from the rank above
  unsigned from_below; // halo-tile deliveries received from the rank below
  unsigned ticket;     // last-block ticket of the per-sweep (generic) path
  unsigned pad[59];
  double partial[kJacobiPartialSlots][kMaxCtas];  // per-CTA residual partials, slot = residual index % 16
  double res_slots[kMaxResSlots][kMaxRanks];  // residual all-gather target (multi-GPU)
};
static_assert(offsetof(JacobiWs, partial) == 256, "JacobiWs header must be 256 bytes");

// Multi-GPU slab parameters (all null / zero for one GPU).
struct SlabPeers {
  float *up_u = nullptr, *up_v = nullptr;  // neighbour above: our first owned row lands in its row up_row
  float *dn_u = nullptr, *dn_v = nullptr;  // neighbour below: our last owned row lands in its row dn_row
  long long up_row = 0, dn_row = 0;
  unsigned *up_flag = nullptr;  // &ws_above->from_below
  unsigned *dn_flag = nullptr;  // &ws_below->from_above
  int rank = 0, nranks = 1;
  JacobiWs *peer_ws[kMaxRanks] = {};  // every rank's workspace (residual all-gather)
};

struct Jacobi2dProblem {
  float *u, *v;       // local arrays, offset applied
  int64_t pitch;      // elements per row
  int64_t h_local;    // rows of the local array (incl. halo rows)
  int64_t w;          // columns
  int64_t row_lo, row_hi;  // local rows updated by a sweep
  int64_t g_row0, g_rows;  // global index of local row 0, global row count
  int64_t sweeps, res_every;
  double *res_out;    // device, [sweeps / res_every]
  JacobiWs *ws;
  int halo = 0;       // slab mode: halo rows on each side (rows exchanged per neighbour per pass)
};

// Halo depth of the multi-GPU Jacobi-2D slab layout: eight rows on each side,
// so a pass may fuse eight sweeps.
constexpr int kSlabHalo = 8;
// Halo depth of the multi-GPU Jacobi-3D z-slab layout (one sweep per pass).
constexpr int kSlabHalo3 = 2;  // the longest 3-D pass (jacobi3d_tb.cu)

// The persistent (register-wavefront) path needs 16-byte aligned rows.
bool jacobi2d_persistent_ok(const Jacobi2dProblem &p);
// Passes the persistent path runs for `sweeps` sweeps: plan[0..3] passes of
// 8, 4, 2 and 1 sweeps (the first three even; no pass longer than res_every
// when res_every > 0, so a pass holds at most one residual sweep).
void jacobi2d_pass_plan(int64_t sweeps, int64_t res_every, int64_t plan[4]);
// Halo deliveries a slab run of `sweeps` sweeps makes to each neighbour (and
// receives from it): one per halo row, tile column and pass, plus one pass's
// worth for the input rows delivered before the first pass.
int64_t jacobi2d_slab_deliveries(int64_t sweeps, int64_t res_every, int64_t w, int halo);
// Runs p.sweeps sweeps on the persistent path (requires
// jacobi2d_persistent_ok) as jacobi2d_pass_plan lays them out (temporal
// blocking), so the result lands in u after an even and in v after an odd
// number of sweeps.  Slab mode: flag_base = deliveries already received from
// each neighbour.  The workspace status word must be clear; the grid barrier
// is reset here on the stream.  Asynchronous.
cudaError_t run_jacobi2d_persistent(const Jacobi2dProblem &p, const SlabPeers &peers, unsigned flag_base,
                                    cudaStream_t s);
// Seeded synthetic Jacobi input (counter-based hash of (seed, global row, column)).
cudaError_t launch_fill_jacobi_input(float *p, int64_t pitch, int64_t rows, int64_t w, int64_t g_row0,
                                     int64_t g_rows, uint64_t seed, cudaStream_t s);
// One launch per sweep, any strides (single GPU only).
cudaError_t launch_jacobi2d_generic(const Jacobi2dProblem &p, int64_t stride1, cudaStream_t s);

struct Jacobi3dProblem {
  float *u, *v;
  int64_t d, h, w;     // sizes [z][y][x] of the (local) arrays
  int64_t sz, sy, sx;  // strides
  int64_t sweeps, res_every;
  double *res_out;
  JacobiWs *ws;
  // z-slab mode (multi-GPU): local planes [z_lo, z_hi) are updated, local
  // plane 0 is global plane g_z0, the global grid has g_d planes, and `halo`
  // planes on each side mirror the neighbours.  One GPU: [0, d), 0, d, 0.
  int64_t z_lo = 0, z_hi = -1, g_z0 = 0, g_d = -1;
  int halo = 0;
};
bool jacobi3d_tma_ok(const Jacobi3dProblem &p);
cudaError_t launch_jacobi3d_generic(const Jacobi3dProblem &p, cudaStream_t s);
// Temporal blocking (jacobi3d_tb.cu): passes of 4, 2 and 1 sweeps (plan[0..2]
// = pass counts; even counts of the multi-sweep passes, at most one residual
// sweep per pass).  Needs jacobi3d_tma_ok(p).  z-slab mode (a neighbour in
// `peers`, p.halo = kSlabHalo3): flag_base = halo deliveries already received
// from each neighbour; a run adds jacobi3d_slab_deliveries(...) to them.
void jacobi3d_pass_plan(int64_t sweeps, int64_t res_every, int64_t plan[3]);
cudaError_t run_jacobi3d_tb(const Jacobi3dProblem &p, const SlabPeers &peers, unsigned flag_base, cudaStream_t s);
int64_t jacobi3d_slab_deliveries(int64_t sweeps, int64_t res_every, int64_t h, int64_t w);
// Seeded synthetic 3-D Jacobi input (counter hash of (seed, gz * h + y, x)).
cudaError_t launch_fill_jacobi3d_input(float *p, int64_t sz, int64_t sy, int64_t planes, int64_t h, int64_t w,
                                       int64_t g_z0, int64_t g_d, uint64_t seed, cudaStream_t s);

// ---- general N-D promoted-tile stencil (stencil_nd.cu) ------------------------------
constexpr int kNdMaxTaps = 64;
enum PlanCode : int {  // promotion decision (PromotionPlanAnalysis.cpp:53-164)
  kPlanPromote = 0,
  kPlanSkipUnbounded = 1,
  kPlanSkipReadWrite = 2,
  kPlanSkipFootprint = 3,
  kPlanSkipNoReuse = 4,
};
// Returns a PlanCode (or -1 for bad arguments); tile_dims_out / footprint
// bytes are filled whenever the offsets are bounded.
int promotion_plan(int rank, const int64_t *tile_sizes, const int64_t *steps, const int64_t *min_off,
                   const int64_t *max_off, int64_t elem_bytes, int64_t max_group_bytes, int read_only,
                   int64_t *tile_dims_out, int64_t *footprint_bytes_out);
struct StencilNdProblem {
  int rank, ntaps;
  const float *a;
  float *b;
  int64_t a_size[3], a_stride[3], b_size[3], b_stride[3];
  int64_t step[3], tile[3];
  const int64_t *offsets;  // ntaps x rank
  const float *weights;    // ntaps, or null (all 1)
  float scale;             // 1: no final multiply
};
cudaError_t launch_stencil_nd(const StencilNdProblem &p, int promote, cudaStream_t s);

// ---- driver entry points resolved at run time (no link-time libcuda) ----------------
// Encodes a row-major f32 tensor map (innermost dimension first).  Returns 0 on success.
int encode_tensor_map_f32(void *tmap /*CUtensorMap*/, void *gaddr, int rank, const uint64_t *dims,
                          const uint64_t *strides_bytes /*rank-1 entries*/, const uint32_t *box);

int num_sms(int device);

// The first out-of-range access a checked build recorded in each file's device
// word (0: none), read and cleared.  Return 1 in a checked build of that file,
// 0 in a release build (nothing read), -1 when the device word could not be
// read; with first == nullptr they only answer whether the build is checked,
// without a CUDA call.
int check_read_forall_map(unsigned long long *first);
int check_read_stencil_nd(unsigned long long *first);

// Bounded-wait limits of the persistent kernels (process-wide, nanoseconds).
unsigned long long wait_budget_ns(bool peer);

// Records a status + message for spmdb200_last_error(); returns `status`.
int record_api_status(int status, const char *fmt, ...);

}  // namespace spmdb200
