// jacobi2d.cu -- Jacobi-2D 5-point sweeps: the PromoteGroupMemory-tiled
// stencil (lib/Transforms/PromoteGroupMemory.cpp:113-314: tile + halo copied
// to group memory, barrier, compute from the tile) rebuilt for B200.
//
// Persistent path (pitch-aligned grids)
// -------------------------------------
// One cooperative launch runs many sweeps.  Each CTA = 1 producer warp + 8
// consumer warps, two CTAs per SM.  The producer stages each tile's
// footprint -- a box starting F rows above and four columns left of the tile,
// so the TMA x coordinate stays 16-byte aligned -- into a 3-deep shared-memory
// ring with cp.async.bulk.tensor.2d, completion tracked by mbarrier expect_tx.
// Out-of-grid box cells are zero-filled by the TMA unit (the guard of
// PromoteGroupMemory.cpp:268-292, done in hardware).  Consumer lanes own 4
// contiguous columns, read north/centre/south as float4 from shared memory,
// get west/east from neighbouring lanes by shuffle, and store float4.
//
// Temporal blocking: a pass advances F sweeps.  F = 1 stages a (BH+2) x 136
// box per 64-row tile and computes one sweep.  F = 2 stages a (BH+4) x 136
// box per 32-row tile, computes the intermediate sweep on the tile plus a
// 1-cell ring into a shared-memory buffer, then the second sweep from that
// buffer: each cell update costs 4 bytes of HBM traffic instead of 8, with
// bit-identical results (the same operations in the same order, only the
// intermediate grid never leaves the SM).  The host runs an even number of
// F = 2 passes and then 0-3 F = 1 sweeps, so the result lands in U after an
// even and in V after an odd number of sweeps.
//
// Passes are separated by a split grid barrier: consumers of a CTA arrive
// (one red.release.gpu per CTA) after their last store of a pass; only the
// producer waits for all arrivals before issuing the next pass's loads, so
// compute never stalls on the barrier itself.  Every wait is bounded
// (%globaltimer budget); on expiry the CTA records a status word, drains its
// in-flight TMA loads and exits.
//
// Row slabs across GPUs (SlabPeers, halo = 2 rows): the consumers that write
// the first (last) two owned rows also store them into the halo rows of the
// neighbour above (below) over NVLink, then bump that neighbour's delivery
// counter (one per row and tile) with a release at system scope.  The
// neighbour's producer acquires the counter before it stages any tile whose
// footprint reaches into that halo.  The last tile row is kept at least two
// rows tall, so only the first and last tile rows touch a halo -- the same
// tiles that deliver -- which also orders every halo overwrite after the
// neighbour's reads of the previous pass.  TMA only ever reads this GPU's own
// memory.
#include <cuda.h>

#include "internal.h"

namespace spmdb200 {
namespace {

constexpr int BW = 128;              // tile columns
constexpr int XPAD = 4;              // left pad of the footprint box (16 bytes)
constexpr int BOXW = BW + 2 * XPAD;  // 136 floats = 544 bytes per box row
constexpr int CWARPS = 8;
constexpr int THREADS = 32 * (CWARPS + 1);
constexpr int CONSUMERS = 32 * CWARPS;

// Tile height and ring depth per fusion depth, chosen by measurement on B200
// (F = 1: 64 x 3 beat 16/32/40/48/96/128-row tiles and 2- or 4-deep rings).
template <int F>
struct Cfg;
template <>
struct Cfg<1> {
  static constexpr int BH = 64, STAGES = 3;
};
template <>
struct Cfg<2> {
  static constexpr int BH = 32, STAGES = 3;
};
template <int F>
struct Geo {
  static constexpr int BH = Cfg<F>::BH;
  static constexpr int STAGES = Cfg<F>::STAGES;
  static constexpr int BOXH = BH + 2 * F;
  static constexpr int RPW = BH / CWARPS;  // output rows per consumer warp
  static constexpr int STAGE_BYTES = BOXW * BOXH * 4;
  static constexpr int STAGE_STRIDE = (STAGE_BYTES + 127) / 128 * 128;
  static constexpr int IROWS = F == 2 ? BH + 2 : 0;  // intermediate buffer rows
  static constexpr int IBYTES = IROWS * BOXW * 4;
  static_assert(BH % CWARPS == 0, "tile rows must split evenly over the consumer warps");
};

struct SmemTail {
  uint64_t full[4];
  uint64_t empty[4];
  double wsum[2][CWARPS];
  int abort;
};
template <int F>
constexpr size_t smem_bytes() {
  return (size_t)Geo<F>::STAGES * Geo<F>::STAGE_STRIDE + Geo<F>::IBYTES + sizeof(SmemTail) + 128;
}

struct J2Kernel {
  float *u, *v;
  long long pitch;
  int w, row_lo, row_hi, tiles_x, tiles_y, last_start;
  long long g_row0, g_rows;
  int passes;      // passes in this launch, each advancing F sweeps
  int sweep_base;  // global index of this launch's first sweep (residual numbering)
  int res_every;
  double *res_out;
  JacobiWs *ws;
  SlabPeers peers;
  unsigned long long grid_budget_ns, peer_budget_ns;  // bounded-wait limits
  int halo;            // rows delivered to / expected from each neighbour per pass (0: no peers)
  unsigned flag_base;  // deliveries already received from each neighbour before this launch
};

__device__ __forceinline__ void record_status(JacobiWs *ws, volatile int *abort, int code) {
  atomicCAS(&ws->status, 0, code);
  *abort = 1;
}

// Waits until *p >= target (wrap-safe); acquire at gpu or sys scope.  Gives
// up when the budget runs out, when this CTA aborts, or when any CTA of the
// grid has recorded an error in the workspace status word.
__device__ __forceinline__ bool wait_counter(const unsigned *p, unsigned target, bool sys,
                                             volatile int *abort, unsigned long long budget,
                                             const JacobiWs *ws) {
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    const unsigned v = sys ? ld_acquire_sys(p) : ld_acquire_gpu(p);
    if ((int)(v - target) >= 0) return true;
    if (*abort) return false;
    if ((i & 7u) == 7u && *reinterpret_cast<const volatile int *>(&ws->status) != 0) return false;
    if (globaltimer_ns() - t0 > budget) return false;
    __nanosleep(64);
  }
}

__device__ __forceinline__ void consumers_sync() { named_bar_sync(1, CONSUMERS); }

// Uniform-across-consumers OR of `pred` at named barrier 1.
__device__ __forceinline__ bool consumers_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(CONSUMERS)
      : "memory");
  return r != 0;
}

// Tile index -> (ty, tx).  In slab mode the first and last tile rows (the
// ones a neighbouring GPU waits for) come first in every pass, so halo rows
// are delivered early and a neighbour's edge tiles never wait for the end of
// this GPU's pass; the interior rows follow in order.  One GPU: row order.
__device__ __forceinline__ void tile_coords(int t, int tiles_x, int tiles_y, bool edges_first, int &ty, int &tx) {
  int row = t / tiles_x;
  tx = t - row * tiles_x;
  if (edges_first && tiles_y > 2) row = row == 0 ? 0 : row == 1 ? tiles_y - 1 : row - 1;
  ty = row;
}

// Local rows [r0, r1) of tile row ty.  All tile rows are BH tall except that
// the last one starts at last_start (so it is at least `halo` rows tall) and
// the one before it ends there.
template <int F>
__device__ __forceinline__ void tile_rows(const J2Kernel &k, int ty, int &r0, int &r1) {
  if (ty == k.tiles_y - 1) {
    r0 = k.last_start;
    r1 = k.row_hi;
  } else {
    r0 = k.row_lo + ty * Geo<F>::BH;
    r1 = min(r0 + Geo<F>::BH, k.last_start);
  }
}

__device__ __forceinline__ void store4_masked(float *p, int gx0, int w, float4 o) {
  if (gx0 + 3 < w) {
    st_f4(p, o);
  } else {
    if (gx0 < w) p[0] = o.x;
    if (gx0 + 1 < w) p[1] = o.y;
    if (gx0 + 2 < w) p[2] = o.z;
  }
}

__device__ __forceinline__ double sq_diff(float a, float b) {
  const double d = __dsub_rn((double)a, (double)b);
  return __dmul_rn(d, d);
}
__device__ __forceinline__ double sq_diff4(float4 a, float4 b, int gx0, int w) {
  double acc = 0.0;
  if (gx0 < w) acc = __dadd_rn(acc, sq_diff(a.x, b.x));
  if (gx0 + 1 < w) acc = __dadd_rn(acc, sq_diff(a.y, b.y));
  if (gx0 + 2 < w) acc = __dadd_rn(acc, sq_diff(a.z, b.z));
  if (gx0 + 3 < w) acc = __dadd_rn(acc, sq_diff(a.w, b.w));
  return acc;
}

// One 5-point update of the 4 cells centred at c (columns gx0..gx0+3 of
// global row g), MLIR source order ((((c + n) + s) + e) + w) * 0.2f; fixed
// boundary cells keep their value.
__device__ __forceinline__ float4 update4(float4 c, float4 n, float4 s, float west, float east, long long g,
                                          long long g_rows, int gx0, int w) {
  float4 o;
  o.x = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.x, n.x), s.x), c.y), west), 0.2f);
  o.y = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.y, n.y), s.y), c.z), c.x), 0.2f);
  o.z = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.z, n.z), s.z), c.w), c.y), 0.2f);
  o.w = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.w, n.w), s.w), east), c.z), 0.2f);
  if (g <= 0 || g >= g_rows - 1) return c;
  const int wl = w - 1;
  if (gx0 == 0) o.x = c.x;
  if (gx0 == wl) o.x = c.x;
  if (gx0 + 1 == wl) o.y = c.y;
  if (gx0 + 2 == wl) o.z = c.z;
  if (gx0 + 3 == wl) o.w = c.w;
  return o;
}

// Scalar 5-point update of one cell (global row g, column gx).
__device__ __forceinline__ float update1(float c, float n, float s, float e, float wv, long long g,
                                         long long g_rows, int gx, int w) {
  if (g <= 0 || g >= g_rows - 1 || gx <= 0 || gx >= w - 1) return c;
  return __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c, n), s), e), wv), 0.2f);
}

// Producer-warp residual combine for residual index r: the CTA partials of
// that sweep in CTA order, lane-strided then a shuffle tree (deterministic).
// CTA 0 combines the residuals of pass p-1 early in pass p, while other CTAs
// may already be writing the partials of pass p; with up to two residuals per
// pass, four slots (index % 4) keep those apart.
__device__ __forceinline__ void combine_residual(const J2Kernel &k, int r, int lane) {
  double p = 0.0;
  for (int i = lane; i < (int)gridDim.x; i += 32) p = __dadd_rn(p, __ldcg(&k.ws->partial[r & 3][i]));
  p = warp_sum_f64(p);
  if (lane == 0) {
    if (k.res_out) k.res_out[r] = p;
    if (k.peers.peer_ws[0] && r < kMaxResSlots) {  // slab mode: all-gather into every rank's slots
      for (int q = 0; q < k.peers.nranks; ++q)
        if (k.peers.peer_ws[q]) k.peers.peer_ws[q]->res_slots[r][k.peers.rank] = p;
      __threadfence_system();
    }
  }
}

// Residual indices produced by pass p (global sweep numbering): -1 if none.
template <int F>
__device__ __forceinline__ void pass_residuals(const J2Kernel &k, int p, int &r_a, int &r_b) {
  r_a = r_b = -1;
  if (k.res_every <= 0) return;
  const int s0 = k.sweep_base + F * p;  // first sweep of the pass (0-based, global)
  if ((s0 + 1) % k.res_every == 0) r_a = (s0 + 1) / k.res_every - 1;
  if (F == 2 && (s0 + 2) % k.res_every == 0) r_b = (s0 + 2) / k.res_every - 1;
}

// Halo deliveries of the owned rows a warp just wrote: stores into the
// neighbours' halo rows happen with the rows; this bumps the counters.
__device__ __forceinline__ void signal_deliveries(const J2Kernel &k, int n_up, int n_dn) {
  if (n_up | n_dn) __threadfence_system();
  if (n_up) red_release_sys_add(k.peers.up_flag, (unsigned)n_up);
  if (n_dn) red_release_sys_add(k.peers.dn_flag, (unsigned)n_dn);
}

// ---------------------------------------------------------------------------
// Interior fast path.  A tile whose computed region (the output rows and
// columns, widened by F-1 for the intermediate ring) holds no fixed boundary
// cell and no row delivered to a neighbour runs straight-line code: no
// boundary tests, no masks, no peer stores.  The arithmetic is the same
// expression as update4, so results are bit-identical to the general path.
// Lanes 0 and 31 take their west/east value from the box pad column (exo);
// all other lanes load the same address as lane 31, a broadcast.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float4 lds4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

__device__ __forceinline__ float4 stencil4(float4 c, float4 n, float4 s, float west, float east) {
  float4 o;
  o.x = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.x, n.x), s.x), c.y), west), 0.2f);
  o.y = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.y, n.y), s.y), c.z), c.x), 0.2f);
  o.z = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.z, n.z), s.z), c.w), c.y), 0.2f);
  o.w = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.w, n.w), s.w), east), c.z), 0.2f);
  return o;
}

__device__ __forceinline__ double acc_sq4(double acc, float4 a, float4 b) {
  double d = __dsub_rn((double)a.x, (double)b.x);
  acc = __fma_rn(d, d, acc);
  d = __dsub_rn((double)a.y, (double)b.y);
  acc = __fma_rn(d, d, acc);
  d = __dsub_rn((double)a.z, (double)b.z);
  acc = __fma_rn(d, d, acc);
  d = __dsub_rn((double)a.w, (double)b.w);
  return __fma_rn(d, d, acc);
}

struct LaneCols {
  int sc;      // first of this lane's 4 columns in a box/buffer row
  int exo;     // pad column: x0-1 for lane 0, x0+BW for the others
  int faro;    // one further out: x0-2 for lane 0, x0+BW+1 for the others
  bool l0, l31;
};

// ROWS output rows from a row-major buffer `in` (row stride BOXW) whose row
// `first` holds the north neighbours of the first output row.  Writes to dp
// (advancing by pitch); RES adds the squared updates to acc.
template <int ROWS, bool RES>
__device__ __forceinline__ void sweep_rows_fast(const float *in, int first, float *dp, long long pitch,
                                                const LaneCols &lc, double &acc) {
  const float *row = in + first * BOXW;
  float4 n = lds4(row + lc.sc);
  float4 c = lds4(row + BOXW + lc.sc);
  float exc = row[BOXW + lc.exo];
#pragma unroll
  for (int q = 0; q < ROWS; ++q) {
    const float *srow = row + (q + 2) * BOXW;
    const float4 s = lds4(srow + lc.sc);
    const float exs = srow[lc.exo];
    const float wu = __shfl_up_sync(0xffffffffu, c.w, 1);
    const float ed = __shfl_down_sync(0xffffffffu, c.x, 1);
    const float4 o = stencil4(c, n, s, lc.l0 ? exc : wu, lc.l31 ? exc : ed);
    *reinterpret_cast<float4 *>(dp) = o;
    dp += pitch;
    if (RES) acc = acc_sq4(acc, o, c);
    n = c;
    c = s;
    exc = exs;
  }
}

// Phase 1 of a two-sweep tile: intermediate rows [a, a + ROWS) (row i from
// box rows i .. i+2) into ibuf, plus the ring cells x0-1 (lane 0) and x0+BW
// (lane 31), each from the same operands in the same order as update1.
template <int ROWS>
__device__ __forceinline__ void intermediate_rows_fast(const float *S, float *ibuf, int a, const LaneCols &lc) {
  const float *row = S + a * BOXW;
  float4 n = lds4(row + lc.sc);
  float4 c = lds4(row + BOXW + lc.sc);
  float exn = row[lc.exo];
  float exc = row[BOXW + lc.exo];
#pragma unroll
  for (int q = 0; q < ROWS; ++q) {
    const float *crow = row + (q + 1) * BOXW;
    const float4 s = lds4(crow + BOXW + lc.sc);
    const float exs = crow[BOXW + lc.exo];
    const float far = crow[lc.faro];
    const float wu = __shfl_up_sync(0xffffffffu, c.w, 1);
    const float ed = __shfl_down_sync(0xffffffffu, c.x, 1);
    float *irow = ibuf + (a + q) * BOXW;
    *reinterpret_cast<float4 *>(irow + lc.sc) = stencil4(c, n, s, lc.l0 ? exc : wu, lc.l31 ? exc : ed);
    const float re = lc.l0 ? c.x : far, rw = lc.l0 ? far : c.w;
    const float ring = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(exc, exn), exs), re), rw), 0.2f);
    if (lc.l0 | lc.l31) irow[lc.exo] = ring;
    n = c;
    c = s;
    exn = exc;
    exc = exs;
  }
}

// Phase 2 of a two-sweep tile: RPW output rows of this warp from ibuf.  RA:
// residual of the first sweep (intermediate minus input, input from the
// staged box), RB: of the second (output minus intermediate).
template <int RPW, bool RA, bool RB>
__device__ __forceinline__ void second_rows_fast(const float *S, const float *ibuf, int j0, float *dp,
                                                 long long pitch, const LaneCols &lc, double &acc_a,
                                                 double &acc_b) {
  const float *row = ibuf + j0 * BOXW;
  float4 n = lds4(row + lc.sc);
  float4 c = lds4(row + BOXW + lc.sc);
  float exc = row[BOXW + lc.exo];
#pragma unroll
  for (int q = 0; q < RPW; ++q) {
    const float *srow = row + (q + 2) * BOXW;
    const float4 s = lds4(srow + lc.sc);
    const float exs = srow[lc.exo];
    const float wu = __shfl_up_sync(0xffffffffu, c.w, 1);
    const float ed = __shfl_down_sync(0xffffffffu, c.x, 1);
    const float4 o = stencil4(c, n, s, lc.l0 ? exc : wu, lc.l31 ? exc : ed);
    *reinterpret_cast<float4 *>(dp) = o;
    dp += pitch;
    if (RA) acc_a = acc_sq4(acc_a, c, lds4(S + (j0 + q + 2) * BOXW + lc.sc));
    if (RB) acc_b = acc_sq4(acc_b, o, c);
    n = c;
    c = s;
    exc = exs;
  }
}

// True when the tile's computed region -- local rows [r0-(F-1), r1+(F-1)),
// columns [x0-(F-1), x0+BW+(F-1)) -- is all interior cells, the tile is full
// height, and none of its output rows is delivered to a neighbour.
template <int F>
__device__ __forceinline__ bool tile_is_interior(const J2Kernel &k, int r0, int r1, int tx) {
  const long long g0 = k.g_row0 + r0 - (F - 1), g1 = k.g_row0 + r1 - 1 + (F - 1);
  const int c0 = tx * BW - (F - 1), c1 = tx * BW + BW - 1 + (F - 1);
  return r1 - r0 == Geo<F>::BH && g0 >= 1 && g1 <= k.g_rows - 2 && c0 >= 1 && c1 <= k.w - 2 &&
         r0 >= k.row_lo + k.halo && r1 <= k.row_hi - k.halo;
}

template <int F>
__global__ void __launch_bounds__(THREADS) jacobi2d_persistent_kernel(
    const __grid_constant__ CUtensorMap map_u, const __grid_constant__ CUtensorMap map_v,
    const __grid_constant__ J2Kernel k) {
  using Gm = Geo<F>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  float *ibuf = reinterpret_cast<float *>(smem + (size_t)Gm::STAGES * Gm::STAGE_STRIDE);  // F == 2 only
  SmemTail *tail = reinterpret_cast<SmemTail *>(smem + (size_t)Gm::STAGES * Gm::STAGE_STRIDE + Gm::IBYTES);
  volatile int *abort = &tail->abort;
  static_assert(Gm::STAGES <= 4, "SmemTail holds four stages");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int T = k.tiles_x * k.tiles_y;
  const bool slab = k.halo > 0;
  const unsigned per_pass = (unsigned)k.tiles_x * (unsigned)k.halo;  // deliveries per neighbour per pass

  if (threadIdx.x == 0) {
    for (int i = 0; i < Gm::STAGES; ++i) {
      mbar_init(&tail->full[i], 1);
      mbar_init(&tail->empty[i], CWARPS);
    }
    tail->abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == CWARPS) {
    // ------------------------------ producer warp ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&map_u);
      tma_prefetch_desc(&map_v);
    }
    uint32_t it = 0;
    bool ok = true;
    for (int p = 0; p < k.passes && ok; ++p) {
      const void *src = (p & 1) ? (const void *)&map_v : (const void *)&map_u;
      if (p > 0) {
        if (lane == 0 &&
            !wait_counter(&k.ws->barrier, (unsigned)p * (unsigned)G, false, abort, k.grid_budget_ns, k.ws)) {
          record_status(k.ws, abort, kDevTimeoutGridBarrier);
          ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (blockIdx.x == 0) {
          int ra, rb;
          pass_residuals<F>(k, p - 1, ra, rb);
          if (ra >= 0) combine_residual(k, ra, lane);
          if (rb >= 0) combine_residual(k, rb, lane);
        }
      }
      if (lane == 0) {
        // Deliveries each neighbour has made once it finished pass p-1 (this
        // launch) -- also the first pass of a later launch waits for all of
        // the previous launch's deliveries.
        const unsigned need = k.flag_base + (unsigned)p * per_pass;
        for (int t = blockIdx.x; t < T; t += G) {
          int ty, tx, r0, r1;
          tile_coords(t, k.tiles_x, k.tiles_y, slab, ty, tx);
          tile_rows<F>(k, ty, r0, r1);
          if (slab) {
            if (k.peers.up_flag && r0 - F < k.row_lo &&
                !wait_counter(&k.ws->from_above, need, true, abort, k.peer_budget_ns, k.ws)) {
              record_status(k.ws, abort, kDevTimeoutPeer);
              ok = false;
              break;
            }
            if (k.peers.dn_flag && r1 + F > k.row_hi &&
                !wait_counter(&k.ws->from_below, need, true, abort, k.peer_budget_ns, k.ws)) {
              record_status(k.ws, abort, kDevTimeoutPeer);
              ok = false;
              break;
            }
          }
          fence_proxy_async_global();
          const uint32_t st = it % Gm::STAGES, ph = (it / Gm::STAGES) & 1u;
          if (!mbar_wait_bounded(&tail->empty[st], ph ^ 1u, abort)) {
            record_status(k.ws, abort, kDevTimeoutEmpty);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&tail->full[st], Gm::STAGE_BYTES);
          tma_load_2d(smem + (size_t)st * Gm::STAGE_STRIDE, src, &tail->full[st], tx * BW - XPAD, r0 - F);
          ++it;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      it = __shfl_sync(0xffffffffu, it, 0);
    }
    if (ok && blockIdx.x == 0 && k.passes > 0) {
      int ra, rb;
      pass_residuals<F>(k, k.passes - 1, ra, rb);
      if (ra >= 0 || rb >= 0) {
        if (lane == 0 && !wait_counter(&k.ws->barrier, (unsigned)k.passes * (unsigned)G, false, abort,
                                       k.grid_budget_ns, k.ws)) {
          record_status(k.ws, abort, kDevTimeoutGridBarrier);
          ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok) {
          if (ra >= 0) combine_residual(k, ra, lane);
          if (rb >= 0) combine_residual(k, rb, lane);
        }
      }
    }
    if (!ok && lane == 0) {
      // Drain: the most recent load issued into each stage must land before
      // this CTA's shared memory can be released.
      const uint32_t n = it < (uint32_t)Gm::STAGES ? it : (uint32_t)Gm::STAGES;
      for (uint32_t j = 0; j < n; ++j) {
        const uint32_t i = it - 1 - j;
        int no_abort = 0;
        mbar_wait_bounded(&tail->full[i % Gm::STAGES], (i / Gm::STAGES) & 1u, &no_abort);
      }
    }
    return;
  }

  // ------------------------------ consumer warps ------------------------------
  const int cw = warp;
  const int j0 = cw * Gm::RPW;  // this warp's first output row within a tile
  const int sc = XPAD + 4 * lane;
  LaneCols lc;
  lc.sc = sc;
  lc.l0 = lane == 0;
  lc.l31 = lane == 31;
  lc.exo = lc.l0 ? XPAD - 1 : XPAD + BW;
  lc.faro = lc.l0 ? XPAD - 2 : XPAD + BW + 1;
  // Intermediate rows of a two-sweep tile, contiguous per warp: IROWS split
  // as evenly as possible (the first IX warps take one more).
  constexpr int IB = F == 2 ? Gm::IROWS / CWARPS : 0, IX = F == 2 ? Gm::IROWS % CWARPS : 0;
  const int ia = cw * IB + (cw < IX ? cw : IX);
  uint32_t it = 0;
  double acc_a = 0.0, acc_b = 0.0;
  for (int p = 0; p < k.passes; ++p) {
    float *dst = (p & 1) ? k.u : k.v;
    float *up_dst = (p & 1) ? k.peers.up_u : k.peers.up_v;
    float *dn_dst = (p & 1) ? k.peers.dn_u : k.peers.dn_v;
    int ra, rb;
    pass_residuals<F>(k, p, ra, rb);
    bool ok = true;
    for (int t = blockIdx.x; t < T; t += G) {
      int ty, tx, r0, r1;
      tile_coords(t, k.tiles_x, k.tiles_y, slab, ty, tx);
      tile_rows<F>(k, ty, r0, r1);
      const uint32_t st = it % Gm::STAGES, ph = (it / Gm::STAGES) & 1u;
      const bool landed = mbar_wait_warp(&tail->full[st], ph, abort);  // warp-uniform outcome
      if (!landed && lane == 0) record_status(k.ws, abort, kDevTimeoutFull);
      if constexpr (F == 1) {
        if (!landed) {
          ok = false;
          break;
        }
      }
      const float *S = reinterpret_cast<const float *>(smem + (size_t)st * Gm::STAGE_STRIDE);
      const int gx0 = tx * BW + 4 * lane;
      int n_up = 0, n_dn = 0;

      // Reads a row of 4 cells plus the west/east neighbours of the row `rowp`.
      auto edges = [&](const float *rowp, float4 c, float &west, float &east) {
        west = __shfl_up_sync(0xffffffffu, c.w, 1);
        east = __shfl_down_sync(0xffffffffu, c.x, 1);
        if (lane == 0) west = rowp[XPAD - 1];
        if (lane == 31) east = rowp[XPAD + BW];
      };
      // Stores an output row (and its halo copies in slab mode).
      auto emit = [&](int L, float4 o) {
        store4_masked(dst + (long long)L * k.pitch + gx0, gx0, k.w, o);
        if (up_dst && L < k.row_lo + k.halo) {
          store4_masked(up_dst + (k.peers.up_row + (L - k.row_lo)) * k.pitch + gx0, gx0, k.w, o);
          ++n_up;
        }
        if (dn_dst && L >= k.row_hi - k.halo) {
          store4_masked(dn_dst + (k.peers.dn_row + (L - (k.row_hi - k.halo))) * k.pitch + gx0, gx0, k.w, o);
          ++n_dn;
        }
      };

      const bool fast = tile_is_interior<F>(k, r0, r1, tx);
      float *dp = dst + (long long)(r0 + j0) * k.pitch + gx0;
      if constexpr (F == 1) {
        if (fast) {
          if (ra >= 0)
            sweep_rows_fast<Gm::RPW, true>(S, j0, dp, k.pitch, lc, acc_a);
          else
            sweep_rows_fast<Gm::RPW, false>(S, j0, dp, k.pitch, lc, acc_a);
        } else {
        // box row of local row L is L - r0 + 1
        float4 n = *reinterpret_cast<const float4 *>(S + j0 * BOXW + sc);
        float4 c = *reinterpret_cast<const float4 *>(S + (j0 + 1) * BOXW + sc);
#pragma unroll
        for (int q = 0; q < Gm::RPW; ++q) {
          const float *crow = S + (j0 + q + 1) * BOXW;
          const float4 so = *reinterpret_cast<const float4 *>(crow + BOXW + sc);
          float west, east;
          edges(crow, c, west, east);
          const int L = r0 + j0 + q;
          if (L < r1) {
            const float4 o = update4(c, n, so, west, east, k.g_row0 + L, k.g_rows, gx0, k.w);
            emit(L, o);
            if (ra >= 0) acc_a = __dadd_rn(acc_a, sq_diff4(o, c, gx0, k.w));
          }
          n = c;
          c = so;
        }
        }
      } else {
        // Phase 1: the intermediate sweep on the tile rows plus a one-cell ring,
        // rows i = 0 .. BH+1 <-> local rows r0-1+i (box row i+1).
        if (landed && fast) {
          if (cw < IX)
            intermediate_rows_fast<IB + 1>(S, ibuf, ia, lc);
          else
            intermediate_rows_fast<IB>(S, ibuf, ia, lc);
        }
        for (int i = cw; landed && !fast && i < Gm::IROWS; i += CWARPS) {
          const float *brow = S + (i + 1) * BOXW;
          const float4 n4 = *reinterpret_cast<const float4 *>(S + i * BOXW + sc);
          const float4 c4 = *reinterpret_cast<const float4 *>(brow + sc);
          const float4 s4 = *reinterpret_cast<const float4 *>(S + (i + 2) * BOXW + sc);
          float west, east;
          edges(brow, c4, west, east);
          const long long g = k.g_row0 + (r0 - 1 + i);
          *reinterpret_cast<float4 *>(ibuf + i * BOXW + sc) =
              update4(c4, n4, s4, west, east, g, k.g_rows, gx0, k.w);
          if (lane == 0) {  // ring column x0 - 1
            const int cc = XPAD - 1;
            ibuf[i * BOXW + cc] = update1(brow[cc], S[i * BOXW + cc], S[(i + 2) * BOXW + cc], brow[cc + 1],
                                          brow[cc - 1], g, k.g_rows, tx * BW - 1, k.w);
          }
          if (lane == 31) {  // ring column x0 + BW
            const int cc = XPAD + BW;
            ibuf[i * BOXW + cc] = update1(brow[cc], S[i * BOXW + cc], S[(i + 2) * BOXW + cc], brow[cc + 1],
                                          brow[cc - 1], g, k.g_rows, tx * BW + BW, k.w);
          }
        }
        // One warp's bounded wait can give up while another's succeeds: the
        // barrier after phase 1 also ORs the failures, so every consumer warp
        // leaves the tile loop together (no warp is left at a named barrier).
        if (consumers_any(!landed)) {
          ok = false;
          break;
        }
        // Phase 2: the second sweep from the intermediate buffer (ibuf row of
        // local row L is L - r0 + 1; box row is L - r0 + 2).
        if (fast) {
          if (ra >= 0 && rb >= 0)
            second_rows_fast<Gm::RPW, true, true>(S, ibuf, j0, dp, k.pitch, lc, acc_a, acc_b);
          else if (ra >= 0)
            second_rows_fast<Gm::RPW, true, false>(S, ibuf, j0, dp, k.pitch, lc, acc_a, acc_b);
          else if (rb >= 0)
            second_rows_fast<Gm::RPW, false, true>(S, ibuf, j0, dp, k.pitch, lc, acc_a, acc_b);
          else
            second_rows_fast<Gm::RPW, false, false>(S, ibuf, j0, dp, k.pitch, lc, acc_a, acc_b);
        } else {
        float4 n = *reinterpret_cast<const float4 *>(ibuf + j0 * BOXW + sc);
        float4 c = *reinterpret_cast<const float4 *>(ibuf + (j0 + 1) * BOXW + sc);
#pragma unroll
        for (int q = 0; q < Gm::RPW; ++q) {
          const float *irow = ibuf + (j0 + q + 1) * BOXW;
          const float4 so = *reinterpret_cast<const float4 *>(irow + BOXW + sc);
          float west, east;
          edges(irow, c, west, east);
          const int L = r0 + j0 + q;
          if (L < r1) {
            const float4 o = update4(c, n, so, west, east, k.g_row0 + L, k.g_rows, gx0, k.w);
            emit(L, o);
            if (ra >= 0) {  // first sweep of the pair: intermediate minus input
              const float4 in = *reinterpret_cast<const float4 *>(S + (j0 + q + 2) * BOXW + sc);
              acc_a = __dadd_rn(acc_a, sq_diff4(c, in, gx0, k.w));
            }
            if (rb >= 0) acc_b = __dadd_rn(acc_b, sq_diff4(o, c, gx0, k.w));
          }
          n = c;
          c = so;
        }
        }
        consumers_sync();  // the buffer is rewritten by the next tile
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tail->empty[st]);
        if (slab) signal_deliveries(k, n_up, n_dn);
      }
      ++it;
    }
    // ---- end of pass p: CTA partials, then one grid-barrier arrival ----
    if (ra >= 0) {
      const double wv = warp_sum_f64(acc_a);
      if (lane == 0) tail->wsum[ra & 1][cw] = wv;
      acc_a = 0.0;
    }
    if (rb >= 0) {
      const double wv = warp_sum_f64(acc_b);
      if (lane == 0) tail->wsum[rb & 1][cw] = wv;
      acc_b = 0.0;
    }
    fence_proxy_async_global();
    __syncwarp();
    const bool fail = consumers_any(!ok || *abort);
    if (fail) break;
    if (threadIdx.x == 0) {
      const int rs[2] = {ra, rb};
      for (int j = 0; j < 2; ++j) {
        const int r = rs[j];
        if (r < 0) continue;
        double tot = 0.0;
        for (int i = 0; i < CWARPS; ++i) tot = __dadd_rn(tot, tail->wsum[r & 1][i]);
        k.ws->partial[r & 3][blockIdx.x] = tot;
      }
      __threadfence();
      red_release_gpu_add(&k.ws->barrier, 1u);
    }
  }
}

// One sweep, any strides: one thread per cell, residual partials combined by
// the last block (ticket) in block order.
__global__ void __launch_bounds__(256) jacobi2d_sweep_generic_kernel(
    const float *__restrict__ u, float *__restrict__ v, long long s0, long long s1, long long h,
    long long w, int want, double *partials, unsigned *ticket, double *res_slot) {
  __shared__ double sh[32];
  __shared__ int last;
  const long long nth = (long long)gridDim.x * blockDim.x;
  double acc = 0.0;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < h * w; idx += nth) {
    const long long i = idx / w, j = idx - i * w;
    const float c = u[i * s0 + j * s1];
    float o = c;
    if (i > 0 && i < h - 1 && j > 0 && j < w - 1) {
      const float nn = u[(i - 1) * s0 + j * s1], ss = u[(i + 1) * s0 + j * s1];
      const float ee = u[i * s0 + (j + 1) * s1], ww = u[i * s0 + (j - 1) * s1];
      o = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c, nn), ss), ee), ww), 0.2f);
      if (want) acc = __dadd_rn(acc, sq_diff(o, c));
    }
    v[i * s0 + j * s1] = o;
  }
  if (!want) return;
  // Block partial (warp shuffles + one slot per warp), then the ticket.
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

// splitmix64 finaliser over (seed, row, column): a counter-based generator, so
// any rank can produce any global cell without coordination.
__device__ __forceinline__ float hash_uniform(uint64_t seed, uint64_t g, uint64_t c) {
  uint64_t x = seed * 0x9E3779B97F4A7C15ull + g * 0xD1B54A32D192ED03ull + c * 0x8CB92BA72F3D8DD7ull;
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return (float)(x >> 40) * (1.0f / 16777216.0f);  // 24 random bits -> [0, 1)
}

__global__ void __launch_bounds__(256) fill_jacobi_input_kernel(float *p, long long pitch, long long rows,
                                                                long long w, long long g_row0, long long g_rows,
                                                                uint64_t seed) {
  const long long nth = (long long)gridDim.x * blockDim.x;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < rows * w; idx += nth) {
    const long long r = idx / w, c = idx - r * w;
    const long long g = g_row0 + r;
    const bool interior = g > 0 && g < g_rows - 1 && c > 0 && c < w - 1;
    p[r * pitch + c] = interior ? hash_uniform(seed, (uint64_t)g, (uint64_t)c) : 0.0f;
  }
}

}  // namespace

cudaError_t launch_fill_jacobi_input(float *p, int64_t pitch, int64_t rows, int64_t w, int64_t g_row0,
                                     int64_t g_rows, uint64_t seed, cudaStream_t s) {
  if (rows <= 0 || w <= 0) return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  long long g = (rows * w + 255) / 256;
  const long long cap = (long long)num_sms(dev) * 8;
  if (g > cap) g = cap;
  fill_jacobi_input_kernel<<<(unsigned)g, 256, 0, s>>>(p, pitch, rows, w, g_row0, g_rows, seed);
  return cudaGetLastError();
}

bool jacobi2d_tma_ok(const Jacobi2dProblem &p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p.u), b = reinterpret_cast<uintptr_t>(p.v);
  return ((a | b) & 15u) == 0 && (p.pitch * 4) % 16 == 0 && p.w >= 1 && p.h_local >= 1 &&
         p.w <= (1ll << 31) - 1 - BW && p.h_local <= (1ll << 31) - 1 - 128 && p.pitch < (1ll << 37) &&
         p.row_lo >= 0 && p.row_hi <= p.h_local && p.row_hi > p.row_lo && p.sweeps <= (1ll << 30);
}

namespace {

template <int F>
cudaError_t launch_passes(const Jacobi2dProblem &p, const SlabPeers &peers, int64_t passes, int64_t sweep_base,
                          unsigned flag_base, cudaStream_t s) {
  using Gm = Geo<F>;
  CUtensorMap mu, mv;
  const uint64_t dims[2] = {(uint64_t)p.w, (uint64_t)p.h_local};
  const uint64_t strides[1] = {(uint64_t)p.pitch * 4u};
  const uint32_t box[2] = {(uint32_t)BOXW, (uint32_t)Gm::BOXH};
  if (encode_tensor_map_f32(&mu, p.u, 2, dims, strides, box) != 0) return cudaErrorInvalidValue;
  if (encode_tensor_map_f32(&mv, p.v, 2, dims, strides, box) != 0) return cudaErrorInvalidValue;

  J2Kernel k{};
  k.u = p.u;
  k.v = p.v;
  k.pitch = p.pitch;
  k.w = (int)p.w;
  k.row_lo = (int)p.row_lo;
  k.row_hi = (int)p.row_hi;
  const int rows = (int)(p.row_hi - p.row_lo);
  k.tiles_x = (int)((p.w + BW - 1) / BW);
  k.tiles_y = (rows + Gm::BH - 1) / Gm::BH;
  const int rem = rows - (k.tiles_y - 1) * Gm::BH;
  k.last_start = (p.halo > 0 && k.tiles_y >= 2 && rem < p.halo) ? (int)p.row_hi - p.halo
                                                                  : (int)p.row_lo + (k.tiles_y - 1) * Gm::BH;
  k.g_row0 = p.g_row0;
  k.g_rows = p.g_rows;
  k.passes = (int)passes;
  k.sweep_base = (int)sweep_base;
  k.res_every = (int)p.res_every;
  k.res_out = p.res_out;
  k.ws = p.ws;
  k.peers = peers;
  k.grid_budget_ns = wait_budget_ns(false);
  k.peer_budget_ns = wait_budget_ns(true);
  k.halo = p.halo;
  k.flag_base = flag_base;

  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e;
  if (configured_dev != dev) {
    e = cudaFuncSetAttribute(jacobi2d_persistent_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes<F>());
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, jacobi2d_persistent_kernel<F>, THREADS,
                                                    smem_bytes<F>());
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  long long g = (long long)per_sm * num_sms(dev);
  const long long tiles = (long long)k.tiles_x * k.tiles_y;
  if (g > tiles) g = tiles;
  if (g > kMaxCtas) g = kMaxCtas;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)g);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem_bytes<F>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, jacobi2d_persistent_kernel<F>, mu, mv, k);
}

}  // namespace

cudaError_t run_jacobi2d_persistent(const Jacobi2dProblem &p, const SlabPeers &peers, cudaStream_t s) {
  // An even number of two-sweep passes keeps the ping-pong parity of single
  // sweeps; the 0-3 sweeps left over run as single-sweep passes.
  const int64_t fused = (p.sweeps / 4) * 2;
  const int64_t single = p.sweeps - 2 * fused;
  const unsigned per_pass = (unsigned)((p.w + BW - 1) / BW) * (unsigned)p.halo;
  cudaError_t e = cudaSuccess;
  if (fused > 0) {
    e = launch_passes<2>(p, peers, fused, 0, 0u, s);
    if (e != cudaSuccess) return e;
  }
  if (single > 0) {
    if (fused > 0) {
      e = cudaMemsetAsync(&p.ws->barrier, 0, sizeof(unsigned), s);  // fresh grid barrier, same status word
      if (e != cudaSuccess) return e;
    }
    e = launch_passes<1>(p, peers, single, 2 * fused, (unsigned)fused * per_pass, s);
  }
  return e;
}

cudaError_t launch_jacobi2d_generic(const Jacobi2dProblem &p, int64_t stride1, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  long long cells = p.h_local * p.w;
  long long g = (cells + 255) / 256;
  const long long cap = (long long)num_sms(dev) * 8;
  if (g > cap) g = cap;
  if (g > kMaxCtas) g = kMaxCtas;
  if (g < 1) g = 1;
  float *a = p.u, *b = p.v;
  for (long long sw = 1; sw <= p.sweeps; ++sw) {
    const int want = p.res_every > 0 && sw % p.res_every == 0;
    double *slot = want ? p.res_out + (sw / p.res_every - 1) : nullptr;
    jacobi2d_sweep_generic_kernel<<<(unsigned)g, 256, 0, s>>>(a, b, p.pitch, stride1, p.h_local, p.w, want,
                                                               p.ws->partial[0], &p.ws->ticket, slot);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    float *t = a;
    a = b;
    b = t;
  }
  return cudaSuccess;
}

}  // namespace spmdb200
