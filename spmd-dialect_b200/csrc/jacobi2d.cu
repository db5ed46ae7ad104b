// jacobi2d.cu -- Jacobi-2D 5-point sweeps: the PromoteGroupMemory-tiled
// stencil (lib/Transforms/PromoteGroupMemory.cpp:113-314: tile + halo copied
// to group memory, barrier, compute from the tile) rebuilt for B200.
//
// Persistent path (pitch-aligned grids)
// -------------------------------------
// One cooperative launch runs many passes; a pass advances F sweeps
// (temporal blocking, F = 1, 2 or 4).  Each CTA = 1 producer warp + 8
// consumer warps, two CTAs per SM.  A tile is BH rows x 120 columns.  The
// producer stages its footprint -- a (BH + 2F) x 128 box starting F rows above
// and 4 columns left of the tile, so the TMA x coordinate stays 16-byte
// aligned -- into a shared-memory ring with cp.async.bulk.tensor.2d,
// completion tracked by mbarrier expect_tx.  Out-of-grid box cells are
// zero-filled by the TMA unit (the guard of PromoteGroupMemory.cpp:268-292,
// done in hardware).
//
// Consumer lanes own 4 contiguous box columns each (the warp covers all 128),
// read north/centre/south as float4 from shared memory, get west/east from the
// neighbouring lanes by shuffle, and write float4.  Sweep k of a pass computes
// box rows [k, BOXH - k): every sweep the valid region shrinks by one row and
// one column on each side (lane 0's west and lane 31's east neighbours are
// simply not valid), and after F sweeps box rows [F, F + BH) x columns
// [4, 124) -- the tile -- are exact.  Intermediate sweeps ping-pong between an
// intermediate buffer and the stage itself (S -> I -> S -> I -> global for
// F = 4); only the last sweep writes HBM.  A pass costs one read and one write
// of the grid however many sweeps it advances, and every cell value is the
// same operations in the same order as a sweep-by-sweep run (bit-identical).
//
// The host runs an even number of 4-sweep passes, an even number of 2-sweep
// passes and 0-3 single sweeps, so the result lands in U after an even and in
// V after an odd number of sweeps.
//
// Interior tiles (no fixed boundary cell in the valid region, full height, no
// row delivered to a neighbour) run straight-line code; other tiles apply the
// boundary rule and column masks per cell.
//
// Passes are separated by a split grid barrier: consumers of a CTA arrive
// (one red.release.gpu per CTA) after their last store of a pass; only the
// producer waits for all arrivals before issuing the next pass's loads.  Every
// wait is bounded (%globaltimer budget); on expiry the CTA records a status
// word, drains its in-flight TMA loads and exits.
//
// Row slabs across GPUs (SlabPeers, halo = 4 rows): the consumers that write
// the first (last) four owned rows also store them into the halo rows of the
// neighbour above (below) over NVLink, then bump that neighbour's delivery
// counter (one per row and tile) with a release at system scope.  The
// neighbour's producer acquires the counter before it stages any tile whose
// footprint reaches into that halo.  The last tile row is kept at least four
// rows tall, so only the first and last tile rows touch a halo -- the same
// tiles that deliver -- which also orders every halo overwrite after the
// neighbour's reads of the previous pass.  TMA only ever reads this GPU's own
// memory.
#include <cuda.h>

#include "internal.h"

namespace spmdb200 {
namespace {

constexpr int LW = 128;            // box columns: 32 lanes x 4
constexpr int XOFF = 4;            // the box starts 4 columns (16 bytes) left of its tile
constexpr int TW = LW - 2 * XOFF;  // 120 output columns per tile
constexpr int CWARPS = 8;
constexpr int THREADS = 32 * (CWARPS + 1);
constexpr int CONSUMERS = 32 * CWARPS;
constexpr int kMaxF = 4;
constexpr int kPartialSlots = 8;  // >= 2 x the residuals one pass can produce
static_assert(kSlabHalo == kMaxF, "slab halos must cover the deepest pass");

// Tile height, ring depth and intermediate buffers per pass depth, chosen by
// measurement on B200 (32768^2 x 200 sweeps, four-sweep passes: 40 rows, a
// 2-deep ring and one intermediate buffer -- 73.7 KB, three CTAs per SM --
// at 1876 Gcell/s beat 32/48/56 rows (1774-1815), two intermediate buffers
// (1744, two CTAs per SM) and a 3-deep ring (1726); interleaving two row
// chains per warp was slower (1856)).
template <int F>
struct Cfg;
template <>
struct Cfg<1> {
  static constexpr int BH = 64, STAGES = 3, IBUFS = 0;
};
template <>
struct Cfg<2> {
  static constexpr int BH = 48, STAGES = 2, IBUFS = 2;
};
template <>
struct Cfg<4> {
  static constexpr int BH = 40, STAGES = 2, IBUFS = 1;
};
template <int F>
struct Geo {
  static constexpr int BH = Cfg<F>::BH;
  static constexpr int STAGES = Cfg<F>::STAGES;
  static constexpr int IBUFS = Cfg<F>::IBUFS;
  static constexpr int BOXH = BH + 2 * F;
  static constexpr int RPW = BH / CWARPS;  // final-sweep rows per consumer warp
  static constexpr int STAGE_BYTES = LW * BOXH * 4;
  static constexpr int STAGE_STRIDE = (STAGE_BYTES + 127) / 128 * 128;
  static constexpr int IBYTES = STAGE_STRIDE;
  static_assert(BH % CWARPS == 0, "tile rows must split evenly over the consumer warps");
  static_assert(BH >= kSlabHalo, "a tile row must hold a whole halo");
  static_assert(F == 1 || IBUFS >= 1, "multi-sweep passes need an intermediate buffer");
  static_assert(STAGES <= 4, "SmemTail holds four stages");
};

struct SmemTail {
  uint64_t full[4];
  uint64_t empty[4];
  double wsum[kMaxF][CWARPS];
  int abort;
};
template <int F>
constexpr size_t smem_bytes() {
  return (size_t)Geo<F>::STAGES * Geo<F>::STAGE_STRIDE + (size_t)Geo<F>::IBUFS * Geo<F>::IBYTES +
         sizeof(SmemTail) + 128;
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

__device__ __forceinline__ float4 lds4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void sts4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }

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

// The 5-point update of 4 cells centred at c, MLIR source order
// ((((c + n) + s) + e) + w) * 0.2f.
__device__ __forceinline__ float4 stencil4(float4 c, float4 n, float4 s, float west, float east) {
  float4 o;
  o.x = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.x, n.x), s.x), c.y), west), 0.2f);
  o.y = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.y, n.y), s.y), c.z), c.x), 0.2f);
  o.z = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.z, n.z), s.z), c.w), c.y), 0.2f);
  o.w = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.w, n.w), s.w), east), c.z), 0.2f);
  return o;
}

// The same update for cells of global row g, columns gx0..gx0+3: fixed
// boundary cells (and cells outside the grid) keep their value.
__device__ __forceinline__ float4 update4(float4 c, float4 n, float4 s, float west, float east, long long g,
                                          long long g_rows, int gx0, int w) {
  float4 o = stencil4(c, n, s, west, east);
  if (g <= 0 || g >= g_rows - 1) return c;
  const int wl = w - 1;
  if (gx0 <= 0 || gx0 >= wl) o.x = c.x;
  if (gx0 + 1 <= 0 || gx0 + 1 >= wl) o.y = c.y;
  if (gx0 + 2 <= 0 || gx0 + 2 >= wl) o.z = c.z;
  if (gx0 + 3 <= 0 || gx0 + 3 >= wl) o.w = c.w;
  return o;
}

// ---------------------------------------------------------------------------
// Straight-line rows of one sweep (interior tiles).  Rows [b0, b0 + ROWS) of
// the box from `in` into `out` (same box layout) or, for the last sweep, into
// global memory at dp (lanes 1..30 hold the tile's 120 columns).  RES adds the
// squared updates of owned cells (box rows [own_lo, own_hi), lanes 1..30).
// ---------------------------------------------------------------------------
// One output row of a straight-line sweep: box row b (its south neighbour at
// p + (q + 2) * LW), sliding the north/centre window down by one row.
template <bool TO_GLOBAL, bool RES>
__device__ __forceinline__ void row_step(const float *p, int q, int b, float4 &n, float4 &c, float *out, int c4,
                                         float *&dp, long long pitch, bool out_lane, int own_lo, int own_hi,
                                         double &acc) {
  const float4 s = lds4(p + (q + 2) * LW);
  const float wv = __shfl_up_sync(0xffffffffu, c.w, 1);
  const float ev = __shfl_down_sync(0xffffffffu, c.x, 1);
  const float4 o = stencil4(c, n, s, wv, ev);
  if (TO_GLOBAL) {
    if (out_lane) *reinterpret_cast<float4 *>(dp) = o;
    dp += pitch;
    if (RES && out_lane) acc = acc_sq4(acc, o, c);
  } else {
    sts4(out + b * LW + c4, o);
    if (RES && out_lane && b >= own_lo && b < own_hi) acc = acc_sq4(acc, o, c);
  }
  n = c;
  c = s;
}

template <int ROWS, bool TO_GLOBAL, bool RES>
__device__ __forceinline__ void rows_fast(const float *in, float *out, int b0, int c4, float *dp, long long pitch,
                                          bool out_lane, int own_lo, int own_hi, double &acc) {
  const float *p = in + (b0 - 1) * LW + c4;
  float4 n = lds4(p);
  float4 c = lds4(p + LW);
#pragma unroll
  for (int q = 0; q < ROWS; ++q)
    row_step<TO_GLOBAL, RES>(p, q, b0 + q, n, c, out, c4, dp, pitch, out_lane, own_lo, own_hi, acc);
}

// Per-tile context of the general (boundary) rows.
struct TileCtx {
  long long g_box0;  // global row of box row 0
  int l_box0;        // local row of box row 0
  int r1;            // end of the tile's owned local rows
  int gx0;           // global column of this lane's first cell
  bool out_lane;     // lanes 1..30
};

// General rows [b_lo, b_hi) of one sweep: the boundary rule per cell, column
// masks, owned-row limits; the last sweep also stores the rows a neighbour
// needs into its halo (peer memory) and counts them.
template <bool TO_GLOBAL>
__device__ __noinline__ void rows_general(const J2Kernel &k, const float *in, float *out, int b_lo, int b_hi,
                                          int c4, const TileCtx &t, int own_lo, int own_hi, bool res,
                                          double &acc, float *dst, float *up_dst, float *dn_dst, int &n_up,
                                          int &n_dn) {
  for (int b = b_lo; b < b_hi; ++b) {
    const float4 n = lds4(in + (b - 1) * LW + c4);
    const float4 c = lds4(in + b * LW + c4);
    const float4 s = lds4(in + (b + 1) * LW + c4);
    const float wv = __shfl_up_sync(0xffffffffu, c.w, 1);
    const float ev = __shfl_down_sync(0xffffffffu, c.x, 1);
    const float4 o = update4(c, n, s, wv, ev, t.g_box0 + b, k.g_rows, t.gx0, k.w);
    const int L = t.l_box0 + b;
    const bool owned = b >= own_lo && b < own_hi && L < t.r1;
    if (!TO_GLOBAL) {
      sts4(out + b * LW + c4, o);
    } else if (owned) {
      if (t.out_lane && t.gx0 < k.w) store4_masked(dst + (long long)L * k.pitch + t.gx0, t.gx0, k.w, o);
      if (up_dst && L < k.row_lo + k.halo) {
        if (t.out_lane && t.gx0 < k.w)
          store4_masked(up_dst + (k.peers.up_row + (L - k.row_lo)) * k.pitch + t.gx0, t.gx0, k.w, o);
        ++n_up;
      }
      if (dn_dst && L >= k.row_hi - k.halo) {
        if (t.out_lane && t.gx0 < k.w)
          store4_masked(dn_dst + (k.peers.dn_row + (L - (k.row_hi - k.halo))) * k.pitch + t.gx0, t.gx0, k.w, o);
        ++n_dn;
      }
    }
    if (res && owned && t.out_lane) acc = __dadd_rn(acc, sq_diff4(o, c, t.gx0, k.w));
  }
}

// Sweep K (1..F) of a pass for consumer warp cw: the warp's share of box rows
// [K, BOXH - K) -- contiguous, split as evenly as possible (the final sweep:
// RPW rows each) -- from `in` into `out` or, for K == F, global memory.
template <int F, int K>
__device__ __forceinline__ void sweep_rows(const J2Kernel &k, bool fast, const float *in, float *out, int cw,
                                           int c4, const TileCtx &t, float *dst, long long out_row0, bool res,
                                           double &acc, float *up_dst, float *dn_dst, int &n_up, int &n_dn) {
  using Gm = Geo<F>;
  constexpr int own_lo = F, own_hi = F + Gm::BH;
  if constexpr (K == F) {
    const int b0 = F + cw * Gm::RPW;
    if (fast) {
      float *dp = dst + (out_row0 + cw * Gm::RPW) * k.pitch + t.gx0;
      if (res)
        rows_fast<Gm::RPW, true, true>(in, nullptr, b0, c4, dp, k.pitch, t.out_lane, own_lo, own_hi, acc);
      else
        rows_fast<Gm::RPW, true, false>(in, nullptr, b0, c4, dp, k.pitch, t.out_lane, own_lo, own_hi, acc);
    } else {
      rows_general<true>(k, in, nullptr, b0, b0 + Gm::RPW, c4, t, own_lo, own_hi, res, acc, dst, up_dst, dn_dst,
                         n_up, n_dn);
    }
  } else {
    constexpr int N = Gm::BOXH - 2 * K;
    constexpr int B = N / CWARPS, X = N % CWARPS;
    const int b0 = K + cw * B + (cw < X ? cw : X);
    if (fast) {
      if (cw < X) {
        if (res)
          rows_fast<B + 1, false, true>(in, out, b0, c4, nullptr, 0, t.out_lane, own_lo, own_hi, acc);
        else
          rows_fast<B + 1, false, false>(in, out, b0, c4, nullptr, 0, t.out_lane, own_lo, own_hi, acc);
      } else {
        if (res)
          rows_fast<B, false, true>(in, out, b0, c4, nullptr, 0, t.out_lane, own_lo, own_hi, acc);
        else
          rows_fast<B, false, false>(in, out, b0, c4, nullptr, 0, t.out_lane, own_lo, own_hi, acc);
      }
    } else {
      int dummy_up = 0, dummy_dn = 0;
      rows_general<false>(k, in, out, b0, b0 + B + (cw < X ? 1 : 0), c4, t, own_lo, own_hi, res, acc, nullptr,
                          nullptr, nullptr, dummy_up, dummy_dn);
    }
  }
}

// True when the union of the pass's valid regions -- local rows
// [r0-F+1, r1+F-1), columns [x0-3, x0+123) -- is all interior cells, the tile
// is full height, and none of its rows is delivered to a neighbour.
template <int F>
__device__ __forceinline__ bool tile_is_interior(const J2Kernel &k, int r0, int r1, int x0) {
  return r1 - r0 == Geo<F>::BH && k.g_row0 + r0 - F + 1 >= 1 && k.g_row0 + r1 + F - 2 <= k.g_rows - 2 &&
         x0 >= XOFF && x0 + TW + XOFF <= k.w && r0 >= k.row_lo + k.halo && r1 <= k.row_hi - k.halo;
}

// Producer-warp residual combine for residual index r: the CTA partials of
// that sweep in CTA order, lane-strided then a shuffle tree (deterministic).
// CTA 0 combines the residuals of pass p-1 early in pass p, while other CTAs
// may already be writing the partials of pass p; with up to four residuals
// per pass, eight slots (index % 8) keep those apart.
__device__ __forceinline__ void combine_residual(const J2Kernel &k, int r, int lane) {
  double p = 0.0;
  for (int i = lane; i < (int)gridDim.x; i += 32)
    p = __dadd_rn(p, __ldcg(&k.ws->partial[r % kPartialSlots][i]));
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

// Residual index of sweep K (1-based within the pass) of pass p, or -1.
template <int F>
__device__ __forceinline__ int sweep_residual(const J2Kernel &k, int p, int K) {
  if (k.res_every <= 0) return -1;
  const int s = k.sweep_base + F * p + K;  // global 1-based sweep number
  return s % k.res_every == 0 ? s / k.res_every - 1 : -1;
}

template <int F>
__device__ __forceinline__ void combine_pass(const J2Kernel &k, int p, int lane) {
#pragma unroll
  for (int K = 1; K <= F; ++K) {
    const int r = sweep_residual<F>(k, p, K);
    if (r >= 0) combine_residual(k, r, lane);
  }
}

// Halo deliveries of the owned rows a warp just wrote: stores into the
// neighbours' halo rows happen with the rows; this bumps the counters.
__device__ __forceinline__ void signal_deliveries(const J2Kernel &k, int n_up, int n_dn) {
  if (n_up | n_dn) __threadfence_system();
  if (n_up) red_release_sys_add(k.peers.up_flag, (unsigned)n_up);
  if (n_dn) red_release_sys_add(k.peers.dn_flag, (unsigned)n_dn);
}

template <int F>
__global__ void __launch_bounds__(THREADS) jacobi2d_persistent_kernel(
    const __grid_constant__ CUtensorMap map_u, const __grid_constant__ CUtensorMap map_v,
    const __grid_constant__ J2Kernel k) {
  using Gm = Geo<F>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  // Aligned by pointer arithmetic on the shared array itself, so the compiler
  // keeps shared-space addressing (LDS/STS) for everything derived from it.
  unsigned char *smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  float *ibase = reinterpret_cast<float *>(smem + (size_t)Gm::STAGES * Gm::STAGE_STRIDE);
  SmemTail *tail = reinterpret_cast<SmemTail *>(smem + (size_t)Gm::STAGES * Gm::STAGE_STRIDE +
                                                (size_t)Gm::IBUFS * Gm::IBYTES);
  volatile int *abort = &tail->abort;

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
        if (blockIdx.x == 0) combine_pass<F>(k, p - 1, lane);
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
          tma_load_2d(smem + (size_t)st * Gm::STAGE_STRIDE, src, &tail->full[st], tx * TW - XOFF, r0 - F);
          ++it;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      it = __shfl_sync(0xffffffffu, it, 0);
    }
    if (ok && blockIdx.x == 0 && k.passes > 0) {
      bool any = false;
      for (int K = 1; K <= F; ++K) any |= sweep_residual<F>(k, k.passes - 1, K) >= 0;
      if (any) {
        if (lane == 0 && !wait_counter(&k.ws->barrier, (unsigned)k.passes * (unsigned)G, false, abort,
                                       k.grid_budget_ns, k.ws)) {
          record_status(k.ws, abort, kDevTimeoutGridBarrier);
          ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok) combine_pass<F>(k, k.passes - 1, lane);
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
  const int c4 = 4 * lane;  // this lane's first box column
  uint32_t it = 0;
  double acc[F];
#pragma unroll
  for (int K = 0; K < F; ++K) acc[K] = 0.0;
  for (int p = 0; p < k.passes; ++p) {
    float *dst = (p & 1) ? k.u : k.v;
    float *up_dst = (p & 1) ? k.peers.up_u : k.peers.up_v;
    float *dn_dst = (p & 1) ? k.peers.dn_u : k.peers.dn_v;
    int rk[F];
#pragma unroll
    for (int K = 0; K < F; ++K) rk[K] = sweep_residual<F>(k, p, K + 1);
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
      float *S = reinterpret_cast<float *>(smem + (size_t)st * Gm::STAGE_STRIDE);
      float *I = ibase + (Gm::IBUFS == 2 ? (it & 1u) : 0u) * (Gm::IBYTES / 4);
      const int x0 = tx * TW;
      const bool fast = tile_is_interior<F>(k, r0, r1, x0);
      TileCtx tc;
      tc.g_box0 = k.g_row0 + r0 - F;
      tc.l_box0 = r0 - F;
      tc.r1 = r1;
      tc.gx0 = x0 - XOFF + c4;
      tc.out_lane = lane >= 1 && lane <= 30;
      int n_up = 0, n_dn = 0;

      // Sweep 1 (S -> I, or S -> global when F == 1).  A warp whose wait gave
      // up skips it; the barrier after it ORs the failures so every consumer
      // warp leaves the tile loop together.
      if (landed)
        sweep_rows<F, 1>(k, fast, S, I, cw, c4, tc, dst, r0, rk[0] >= 0, acc[0], up_dst, dn_dst, n_up, n_dn);
      if constexpr (F >= 2) {
        if (consumers_any(!landed)) {
          ok = false;
          break;
        }
        // Sweep 2: I -> global (F == 2) or I -> S (F == 4).
        sweep_rows<F, 2>(k, fast, I, S, cw, c4, tc, dst, r0, rk[1] >= 0, acc[1], up_dst, dn_dst, n_up, n_dn);
      }
      if constexpr (F == 4) {
        consumers_sync();
        sweep_rows<F, 3>(k, fast, S, I, cw, c4, tc, dst, r0, rk[2] >= 0, acc[2], up_dst, dn_dst, n_up, n_dn);
        consumers_sync();
        sweep_rows<F, 4>(k, fast, I, nullptr, cw, c4, tc, dst, r0, rk[3] >= 0, acc[3], up_dst, dn_dst, n_up,
                         n_dn);
        fence_proxy_async_shared();  // the stage was written by sweep 2; TMA refills it next
      }
      if constexpr (Gm::IBUFS == 1) consumers_sync();  // one intermediate buffer: the next tile rewrites it
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tail->empty[st]);
        if (slab) signal_deliveries(k, n_up, n_dn);
      }
      ++it;
    }
    // ---- end of pass p: CTA partials, then one grid-barrier arrival ----
#pragma unroll
    for (int K = 0; K < F; ++K) {
      if (rk[K] >= 0) {
        const double wv = warp_sum_f64(acc[K]);
        if (lane == 0) tail->wsum[K][cw] = wv;
        acc[K] = 0.0;
      }
    }
    fence_proxy_async_global();
    __syncwarp();
    const bool fail = consumers_any(!ok || *abort);
    if (fail) break;
    if (threadIdx.x == 0) {
      for (int K = 0; K < F; ++K) {
        if (rk[K] < 0) continue;
        double tot = 0.0;
        for (int i = 0; i < CWARPS; ++i) tot = __dadd_rn(tot, tail->wsum[K][i]);
        k.ws->partial[rk[K] % kPartialSlots][blockIdx.x] = tot;
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
         p.w <= (1ll << 31) - 1 - LW && p.h_local <= (1ll << 31) - 1 - 256 && p.pitch < (1ll << 37) &&
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
  const uint32_t box[2] = {(uint32_t)LW, (uint32_t)Gm::BOXH};
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
  k.tiles_x = (int)((p.w + TW - 1) / TW);
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

void jacobi2d_pass_plan(int64_t sweeps, int64_t plan[3]) {
  // Even pass counts keep the ping-pong parity of single sweeps.
  plan[0] = (sweeps / 8) * 2;                             // four-sweep passes
  plan[1] = ((sweeps - 4 * plan[0]) / 4) * 2;             // two-sweep passes (0 or 2)
  plan[2] = sweeps - 4 * plan[0] - 2 * plan[1];           // single sweeps (0-3)
}

cudaError_t run_jacobi2d_persistent(const Jacobi2dProblem &p, const SlabPeers &peers, cudaStream_t s) {
  int64_t plan[3];
  jacobi2d_pass_plan(p.sweeps, plan);
  const unsigned per_pass = (unsigned)((p.w + TW - 1) / TW) * (unsigned)p.halo;
  int64_t sweeps_done = 0, passes_done = 0;
  cudaError_t e = cudaSuccess;
  for (int d = 0; d < 3; ++d) {
    if (plan[d] == 0) continue;
    if (passes_done > 0) {
      e = cudaMemsetAsync(&p.ws->barrier, 0, sizeof(unsigned), s);  // fresh grid barrier, same status word
      if (e != cudaSuccess) return e;
    }
    const unsigned fb = (unsigned)passes_done * per_pass;
    if (d == 0)
      e = launch_passes<4>(p, peers, plan[0], sweeps_done, fb, s);
    else if (d == 1)
      e = launch_passes<2>(p, peers, plan[1], sweeps_done, fb, s);
    else
      e = launch_passes<1>(p, peers, plan[2], sweeps_done, fb, s);
    if (e != cudaSuccess) return e;
    sweeps_done += plan[d] * (d == 0 ? 4 : d == 1 ? 2 : 1);
    passes_done += plan[d];
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
