// jacobi2d.cu -- Jacobi-2D 5-point sweeps: the PromoteGroupMemory-tiled
// stencil (lib/Transforms/PromoteGroupMemory.cpp:113-314: tile + halo copied
// to group memory, barrier, compute from the tile) rebuilt for B200.
//
// Persistent path (16-byte aligned rows): the register wavefront
// -------------------------------------------------------------
// One cooperative launch runs many passes; a pass advances F sweeps
// (temporal blocking, F = 8, 4, 2 or 1), reading every cell of the grid once
// and writing it once.
//
// Every warp works alone on its own tiles.  A tile is BH rows x TW columns;
// its warp streams the tile's footprint -- BH + 2F rows of a 128-column strip
// starting XO columns left of the tile (XO = F rounded up to a multiple of 4,
// so each lane's 16-byte chunk stays aligned; TW = 128 - 2 XO) -- one row at
// a time through a 12-row cp.async ring in shared memory.  Each lane copies,
// and later reads, only its own 16 bytes of a row, so the ring needs no
// barrier; row i + 1 is read while row i is computed, and rows up to i + 10
// are in flight.  The F sweeps of the pass run as a pipeline in registers:
// when box row i arrives, sweep 1 computes row i-1, sweep 2 row i-2, ...,
// sweep F row i-F, each from a three-row window of the sweep below it (north
// and centre kept in registers, south just computed); west/east come from
// the neighbouring lanes by shuffle.  The valid region shrinks by one row per
// sweep at the strip's top and bottom and by one column per sweep at its
// sides, so after F sweeps box rows [F, F + BH) x columns [XO, XO + TW) are
// exact and are stored.  Nothing but the input row and the output row touches
// memory, and every cell value is the same operations in the same order as a
// sweep-by-sweep run (bit-identical).
//
// A CTA (8 warps) takes 8 neighbouring tiles of a tile row at a time, so its
// warps stream adjacent 512-byte segments of the same rows.  Tiles without a
// fixed boundary cell, halo row or grid edge in reach run an unmasked loop
// with the pass's residual sweep fixed at compile time; the others (a few
// percent) zero-fill loads outside the array, keep fixed
// boundary cells, mask stores past the last column and deliver slab halo
// rows to the neighbours.
//
// The host runs even numbers of 8-, 4- and 2-sweep passes and 0-1 single
// sweeps (no pass longer than the residual interval), so the result lands in
// U after an even and in V after an odd number of sweeps.  Passes are
// separated by a grid barrier (one release per CTA, every wait bounded by
// %globaltimer; on expiry the CTA records a status word and exits).
//
// Row slabs across GPUs (SlabPeers, halo = 8 rows): the warps that write the
// first (last) `halo` owned rows of a pass also store them into the halo rows
// of the neighbour above (below) over NVLink, then bump that neighbour's
// delivery counter (one per row and tile) with a release at system scope.
// Before the first pass every slab launch also delivers the edge rows of its
// input the same way, so a launch's halo rows never depend on what an earlier
// launch left behind.  A tile whose footprint reaches into a halo first
// acquires the counter.  Counters only grow: the host passes the deliveries
// already received (flag_base), so back-to-back launches need no host
// synchronisation between them.  The last tile row is kept at least `halo`
// rows tall, so only the first and last tile rows touch a halo -- the same
// tiles that deliver -- which also orders every halo overwrite after the
// neighbour's reads of the previous pass.  Only plain loads and stores cross
// NVLink; there is no TMA and no multicast here.
#include "internal.h"

namespace spmdb200 {
namespace {

constexpr int kPartialSlots = kJacobiPartialSlots;  // >= 2 x the residuals one pass can produce
// Warps per CTA and resident CTAs per SM, per pass depth: the register
// windows of an eight-sweep pass need more registers than 2 x 8 warps leave
// (65,536 / 512 = 128 per thread).  Measured at 32768^2 x 200 (residual every
// 10): 3 CTAs of 4 warps (168 registers) 3019-3027 Gcell/s, 2 of 6 (168)
// 2979-2992, 2 of 8 (128, spills) 2873-2889, 1 of 8 (216, no spills)
// 2734-2739.
#ifndef WV_WARPS_DEEP
#define WV_WARPS_DEEP 4
#endif
#ifndef WV_MINB_DEEP
#define WV_MINB_DEEP 3
#endif
template <int F>
struct WvLaunch {
  static constexpr int WARPS = F > 4 ? WV_WARPS_DEEP : 8;
  static constexpr int MINB = F > 4 ? WV_MINB_DEEP : 2;
  static constexpr int THREADS = 32 * WARPS;
};
constexpr int WV_U = 6;         // unroll of the row loop (the register windows rotate with period 3)
constexpr int WV_D = 2 * WV_U;  // ring rows per warp
constexpr int WV_ROW = 512;     // bytes of one ring row (128 floats)
// Tile rows: chosen per launch (wave_tile_rows) between WV_BH_MIN and the
// grid height.
constexpr int WV_BH = 128;
#ifndef WV_BH_MIN
#define WV_BH_MIN 32
#endif
constexpr int kMaxWaveF = 8;
static_assert(kSlabHalo >= kMaxWaveF, "slab halos must cover the deepest pass");
static_assert(WV_BH_MIN >= kSlabHalo, "a tile row must hold a whole halo");

template <int F>
struct Wv {
  static constexpr int XO = (F + 3) / 4 * 4;                     // box starts XO columns left of its tile
  static constexpr int TW = 128 - 2 * XO;                        // output columns per tile
  static constexpr int LANE_LO = XO / 4, LANE_HI = 32 - XO / 4;  // lanes holding output columns
  static_assert(F >= 1 && F <= kMaxWaveF, "1..8 sweeps per pass");
};

template <int NW>
struct WvSmem {
  alignas(128) unsigned char ring[NW][WV_D][WV_ROW];
  double racc[NW][32];  // per-lane residual sums of the current pass
  double wsum[NW];
  int abort;
};

struct J2Kernel {
  float *u, *v;
  long long pitch;
  int w, h_local, row_lo, row_hi, tiles_x, tiles_y, last_start;
  int bh;  // tile rows
  long long g_row0, g_rows;
  int passes;      // passes in this launch, each advancing F sweeps
  int sweep_base;  // global index of this launch's first sweep (residual numbering)
  int res_every;
  double *res_out;
  JacobiWs *ws;
  SlabPeers peers;
  unsigned long long grid_budget_ns, peer_budget_ns;  // bounded-wait limits
  int halo;            // rows delivered to / expected from each neighbour per pass (0: no peers)
  int init_halo;       // deliver the input's edge rows before the first pass
  unsigned flag_base;  // deliveries already received from each neighbour before this launch
};

__device__ __forceinline__ void record_status(JacobiWs *ws, volatile int *abort, int code) {
  atomicCAS(&ws->status, 0, code);
  *abort = 1;
}

// Waits until *p >= target (wrap-safe); acquire at gpu or sys scope.  Gives
// up when the budget runs out, when this CTA aborts, or when any CTA of the
// grid has recorded an error in the workspace status word.
__device__ __forceinline__ bool wait_counter(const unsigned *p, unsigned target, bool sys, volatile int *abort,
                                             unsigned long long budget, const JacobiWs *ws) {
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
__device__ __forceinline__ void tile_rows(const J2Kernel &k, int ty, int &r0, int &r1) {
  if (ty == k.tiles_y - 1) {
    r0 = k.last_start;
    r1 = k.row_hi;
  } else {
    r0 = k.row_lo + ty * k.bh;
    r1 = min(r0 + k.bh, k.last_start);
  }
}

// Stores the cells of o whose columns gx0 + j are < w (plain stores).
__device__ __forceinline__ void store4_masked(float *p, int gx0, int w, float4 o) {
  if (gx0 + 3 < w) {
    *reinterpret_cast<float4 *>(p) = o;
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
// ((((c + n) + s) + e) + w) * 0.2f.  Packed pairs (add.rn.f32x2 /
// mul.rn.f32x2, which round every lane exactly like add.rn.f32 /
// mul.rn.f32) where the operands are already aligned register pairs -- the
// (c + n) + s of cells (0, 1) and (2, 3) and the final * 0.2 -- and scalar
// adds for the east / west terms, whose operands straddle the pairs, so no
// register moves are needed to build pairs.
__device__ __forceinline__ float4 stencil4(float4 c, float4 n, float4 s, float west, float east) {
  float2 a = __fadd2_rn(make_float2(c.x, c.y), make_float2(n.x, n.y));
  float2 b = __fadd2_rn(make_float2(c.z, c.w), make_float2(n.z, n.w));
  a = __fadd2_rn(a, make_float2(s.x, s.y));
  b = __fadd2_rn(b, make_float2(s.z, s.w));
  const float v0 = __fadd_rn(__fadd_rn(a.x, c.y), west);
  const float v1 = __fadd_rn(__fadd_rn(a.y, c.z), c.x);
  const float v2 = __fadd_rn(__fadd_rn(b.x, c.w), c.y);
  const float v3 = __fadd_rn(__fadd_rn(b.y, east), c.z);
  a = __fmul2_rn(make_float2(v0, v1), make_float2(0.2f, 0.2f));
  b = __fmul2_rn(make_float2(v2, v3), make_float2(0.2f, 0.2f));
  return make_float4(a.x, a.y, b.x, b.y);
}

// CTA 0's combine of residual r: the CTA partials of that sweep in CTA order,
// lane-strided then a shuffle tree (deterministic).  CTA 0 combines the
// residual of pass p early in pass p + 1, while other CTAs may already be
// writing the partials of pass p + 1; kPartialSlots >= 2 x the residuals of
// one pass keep those apart.
__device__ __forceinline__ void combine_residual(const J2Kernel &k, int r, int lane) {
  double p = 0.0;
  for (int i = lane; i < (int)gridDim.x; i += 32) p = __dadd_rn(p, __ldcg(&k.ws->partial[r % kPartialSlots][i]));
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

// Halo deliveries of the rows a warp just stored into its neighbours: the
// stores happened with the rows; this bumps the counters (lane 0, after a
// __syncwarp has ordered the warp's stores before it).
__device__ __forceinline__ void signal_deliveries(const J2Kernel &k, int n_up, int n_dn) {
  if (n_up | n_dn) __threadfence_system();
  if (n_up) red_release_sys_add(k.peers.up_flag, (unsigned)n_up);
  if (n_dn) red_release_sys_add(k.peers.dn_flag, (unsigned)n_dn);
}

// ---- per-warp cp.async ring ------------------------------------------------
// These asm statements carry no "memory" clobber: they touch only the warp's
// own ring (volatile asm keeps their relative order: wait, then read, then
// refill), so the compiler stays free to interleave the arithmetic and the
// global stores of neighbouring rows around them.
// 16-byte cp.async of `bytes` (0..16) valid source bytes; the rest is zero-filled.
__device__ __forceinline__ void wv_cp16(uint32_t dst, const float *src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes));
}
__device__ __forceinline__ void wv_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void wv_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}
__device__ __forceinline__ float4 wv_lds4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
// Predicated 16-byte global store (no branch around it).
__device__ __forceinline__ void wv_st4_if(bool pred, float *p, float4 v) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %0, 0;\n\t"
      "@q st.global.v4.f32 [%1], {%2, %3, %4, %5};\n\t}" ::"r"((uint32_t)pred),
      "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w));
}

// No masks needed: every row and column the tile reads is inside the array,
// no fixed boundary cell lies inside a sweep's valid region, and the tile
// neither reads a halo row nor delivers one.
template <int F>
__device__ __forceinline__ bool tile_interior(const J2Kernel &k, int r0, int r1, int x0) {
  using W = Wv<F>;
  return k.g_row0 + r0 - F >= 0 && k.g_row0 + r1 + F <= k.g_rows && r0 - F >= 0 && r1 + F <= k.h_local &&
         x0 - W::XO >= 0 && x0 - W::XO + 128 <= k.w && r0 >= k.row_lo + k.halo && r1 <= k.row_hi - k.halo;
}

// One tile of one pass.  With RES, the squared updates of sweep RL + 1 (or,
// for RL < 0, of the run-time sweep rl + 1) over the tile's cells are added
// to the lane's slot *racc (a pass holds at most one residual sweep: the
// host keeps passes no longer than the residual interval).  Returns the halo
// rows delivered to the neighbour above (low 16 bits) and below (high 16).
template <int F, bool EDGE, bool RES, int RL = -1>
__device__ __forceinline__ unsigned wave_tile(const J2Kernel &k, const float *src, float *dst, float *up_dst,
                                              float *dn_dst, int r0, int r1, int x0, uint32_t ring, int lane,
                                              int rl, double *racc) {
  using W = Wv<F>;
  constexpr int U = WV_U, D = WV_D;
  double acc = 0.0;
  int n_up = 0, n_dn = 0;
  // Kernel fields in registers (read once, not through `k` in the loop).
  const long long pitch = k.pitch;
  const int w = k.w, h_local = k.h_local;
  const int h = r1 - r0;
  const int nb = h + 2 * F;  // box rows
  const int lr0 = r0 - F;    // local row of box row 0
  const int gx0 = x0 - W::XO + 4 * lane;
  const bool out_lane = lane >= W::LANE_LO && lane < W::LANE_HI;
  uint32_t cbytes = 16u;
  if (EDGE) cbytes = (gx0 < 0 || gx0 >= w) ? 0u : (gx0 + 4 <= w ? 16u : 4u * (uint32_t)(w - gx0));
  const uint32_t slot = ring + 16u * (uint32_t)lane;

  // Box row b into ring slot b % D, one commit group per row (rows are issued
  // in order).  Rows past the box (and, on edge tiles, outside the array)
  // copy zero bytes from a valid address, so the loop body has no branch.
  const float *lq = src + (long long)lr0 * pitch + gx0;
  int b_next = 0;
  auto issue = [&](uint32_t slot_off) {
    uint32_t nbytes = b_next < nb ? cbytes : 0u;
    if (EDGE) {
      const int lr = lr0 + b_next;
      if (lr < 0 || lr >= h_local) nbytes = 0u;
    }
    wv_cp16(slot + slot_off, nbytes ? lq : src, nbytes);
    wv_commit();
    lq += pitch;
    ++b_next;
  };

  int bl = 0, bspan = 0;  // non-fixed box rows [bl, bl + bspan)
  bool cm0 = false, cm1 = false, cm2 = false, cm3 = false;
  if (EDGE) {
    const long long gb0 = k.g_row0 + lr0;
    const long long lo = 1 - gb0, hi = k.g_rows - 1 - gb0;
    bl = (int)max(lo, -(1ll << 30));
    bspan = (int)max(min(hi, 1ll << 30) - (long long)bl, 0ll);
    cm0 = gx0 <= 0 || gx0 >= w - 1;
    cm1 = gx0 + 1 <= 0 || gx0 + 1 >= w - 1;
    cm2 = gx0 + 2 <= 0 || gx0 + 2 >= w - 1;
    cm3 = gx0 + 3 <= 0 || gx0 + 3 >= w - 1;
  }

  float4 wn[F], wc[F];  // input window (north, centre) of each sweep
#pragma unroll
  for (int L = 0; L < F; ++L) {
    wn[L] = make_float4(0.f, 0.f, 0.f, 0.f);
    wc[L] = wn[L];
  }
#pragma unroll
  for (int b = 0; b < D - 1; ++b) issue((uint32_t)b * WV_ROW);

  float *dp = dst + (long long)(lr0 - F) * pitch + gx0;  // output row of step i: local row lr0 + i - F
  const int iters = (nb + U - 1) / U;
  wv_wait<D - 2>();  // box row 0 has landed
  float4 s_next = wv_lds4(slot);
  for (int it = 0; it < iters; ++it) {
    // Ring slot of row i = it * U + j is j in this iteration's half of the
    // ring (it even: slots 0..U-1, odd: U..2U-1).
    const uint32_t cur = (uint32_t)((it & 1) * U * WV_ROW), oth = (uint32_t)((~it & 1) * U * WV_ROW);
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int i = it * U + j;
      // Row i was read one step ago; read row i + 1 now (rows up to
      // i + D - 2 were issued, so at most D - 3 groups may still be in
      // flight), then refill the slot of row i - 1 with row i + D - 1.
      float4 s = s_next;
      wv_wait<D - 3>();
      s_next = wv_lds4(slot + (j + 1 < U ? cur + (uint32_t)(j + 1) * WV_ROW : oth));
      issue(j >= 1 ? cur + (uint32_t)(j - 1) * WV_ROW : oth + (uint32_t)(U - 1) * WV_ROW);
#pragma unroll
      for (int L = 1; L <= F; ++L) {
        const float4 n = wn[L - 1], c = wc[L - 1];
        const float we = __shfl_up_sync(0xffffffffu, c.w, 1);
        const float ea = __shfl_down_sync(0xffffffffu, c.x, 1);
        float4 o = stencil4(c, n, s, we, ea);
        const int b = i - L;  // box row of this sweep's output
        if (EDGE) {
          if ((unsigned)(b - bl) >= (unsigned)bspan) {
            o = c;
          } else {
            if (cm0) o.x = c.x;
            if (cm1) o.y = c.y;
            if (cm2) o.z = c.z;
            if (cm3) o.w = c.w;
          }
        }
        if (RES && (RL >= 0 ? RL == L - 1 : rl == L - 1) && out_lane && (unsigned)(b - F) < (unsigned)h) {
          if (EDGE) {
            acc = __dadd_rn(acc, sq_diff4(o, c, gx0, w));
          } else {
            // Through the lane's shared-memory slot, so the f64 sum holds no
            // register across rows (two register chains measured the same).
            volatile double *ra = racc;
            *ra = acc_sq4(*ra, o, c);
          }
        }
        wn[L - 1] = c;
        wc[L - 1] = s;
        s = o;
      }
      // s: sweep F at box row i - F, i.e. tile row f.
      const int f = i - 2 * F;
      if (!EDGE) {
        wv_st4_if(out_lane && (unsigned)f < (unsigned)h, dp, s);
      } else if ((unsigned)f < (unsigned)h) {
        if (out_lane && gx0 < w) store4_masked(dp, gx0, w, s);
        const int L = r0 + f;
        if (up_dst && L < k.row_lo + k.halo) {
          if (out_lane && gx0 < w)
            store4_masked(up_dst + (k.peers.up_row + (L - k.row_lo)) * pitch + gx0, gx0, w, s);
          ++n_up;
        }
        if (dn_dst && L >= k.row_hi - k.halo) {
          if (out_lane && gx0 < w)
            store4_masked(dn_dst + (k.peers.dn_row + (L - (k.row_hi - k.halo))) * pitch + gx0, gx0, w, s);
          ++n_dn;
        }
      }
      dp += pitch;
    }
  }
  if (RES && EDGE) *racc = __dadd_rn(*racc, acc);
  return (unsigned)n_up | ((unsigned)n_dn << 16);
}

// Edge tile with the residual sweep RL fixed at compile time, inlined like
// the interior tiles.  A pass waits for its slowest warp, and edge tiles set
// the pace wherever a warp holds few tiles: out of line with the residual
// sweep a run-time value they ran 2.55x slower than interior tiles (every
// tile forced onto the edge path at 32768^2: 1172 Gcell/s), inlined 1.76x
// (1693); with normal dispatch 4096^2 x 100 went 1038 -> 1321 Gcell/s and
// 32768^2 x 200 2991 -> 3250.
template <int F, int RL>
__device__ __forceinline__ unsigned wave_tile_edge(const J2Kernel &k, const float *src, float *dst, float *up_dst,
                                                   float *dn_dst, int r0, int r1, int x0, uint32_t ring, int lane,
                                                   int rl, double *racc) {
  if constexpr (RL >= F) {
    return 0u;
  } else {
    if (rl == RL)
      return wave_tile<F, true, true, RL>(k, src, dst, up_dst, dn_dst, r0, r1, x0, ring, lane, rl, racc);
    return wave_tile_edge<F, RL + 1>(k, src, dst, up_dst, dn_dst, r0, r1, x0, ring, lane, rl, racc);
  }
}

// Interior tile with the residual sweep RL (0-based within the pass) fixed at
// compile time: the residual costs its own sweep's f64 sums and nothing else.
template <int F, int RL>
__device__ __forceinline__ unsigned wave_tile_interior(const J2Kernel &k, const float *src, float *dst, int r0,
                                                       int r1, int x0, uint32_t ring, int lane, int rl,
                                                       double *racc) {
  if constexpr (RL >= F) {
    return 0u;
  } else {
    if (rl == RL)
      return wave_tile<F, false, true, RL>(k, src, dst, nullptr, nullptr, r0, r1, x0, ring, lane, rl, racc);
    return wave_tile_interior<F, RL + 1>(k, src, dst, r0, r1, x0, ring, lane, rl, racc);
  }
}

// Before pass 0 of a slab launch: the first (last) `halo` owned rows of the
// input go into the halo rows of the neighbour above (below), one tile column
// per warp, counted like a pass of deliveries.
template <int F>
__device__ __forceinline__ void deliver_input_halo(const J2Kernel &k, int gw, int GW, int lane) {
  using W = Wv<F>;
  for (int tx = gw; tx < k.tiles_x; tx += GW) {
    const int gx0 = tx * W::TW - W::XO + 4 * lane;
    const bool mine = lane >= W::LANE_LO && lane < W::LANE_HI && gx0 < k.w;
    for (int j = 0; j < k.halo; ++j) {
      if (k.peers.up_u && mine) {
        const float *q = k.u + (long long)(k.row_lo + j) * k.pitch + gx0;
        const float4 v = make_float4(q[0], gx0 + 1 < k.w ? q[1] : 0.f, gx0 + 2 < k.w ? q[2] : 0.f,
                                     gx0 + 3 < k.w ? q[3] : 0.f);
        store4_masked(k.peers.up_u + (k.peers.up_row + j) * k.pitch + gx0, gx0, k.w, v);
      }
      if (k.peers.dn_u && mine) {
        const float *q = k.u + (long long)(k.row_hi - k.halo + j) * k.pitch + gx0;
        const float4 v = make_float4(q[0], gx0 + 1 < k.w ? q[1] : 0.f, gx0 + 2 < k.w ? q[2] : 0.f,
                                     gx0 + 3 < k.w ? q[3] : 0.f);
        store4_masked(k.peers.dn_u + (k.peers.dn_row + j) * k.pitch + gx0, gx0, k.w, v);
      }
    }
    __syncwarp();
    if (lane == 0) signal_deliveries(k, k.peers.up_u ? k.halo : 0, k.peers.dn_u ? k.halo : 0);
  }
}

// Two CTAs of 8 warps per SM (128 registers, no spills in the interior loop)
// beat three (80 registers, spills) by 11 % at 32768^2 with four-sweep passes.
template <int F>
__global__ void __launch_bounds__(WvLaunch<F>::THREADS, WvLaunch<F>::MINB)
    jacobi2d_wave_kernel(const __grid_constant__ J2Kernel k) {
  constexpr int NW = WvLaunch<F>::WARPS;
  extern __shared__ __align__(128) unsigned char wv_smem_raw[];
  WvSmem<NW> &sm = *reinterpret_cast<WvSmem<NW> *>(wv_smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) sm.abort = 0;
  __syncthreads();
  volatile int *abort = &sm.abort;
  const int G = gridDim.x;
  const int GW = G * NW;
  const int gw = blockIdx.x * NW + warp;  // a CTA takes neighbouring tiles: adjacent row segments
  const int T = k.tiles_x * k.tiles_y;
  const bool slab = k.halo > 0;
  const unsigned per_pass = (unsigned)k.tiles_x * (unsigned)k.halo;
  const uint32_t ring = smem_u32(&sm.ring[warp][0][0]);
  double *racc = &sm.racc[warp][lane];
  *racc = 0.0;

  if (slab && k.init_halo) deliver_input_halo<F>(k, gw, GW, lane);

  for (int p = 0; p < k.passes; ++p) {
    const float *src = (p & 1) ? k.v : k.u;
    float *dst = (p & 1) ? k.u : k.v;
    float *up_dst = (p & 1) ? k.peers.up_u : k.peers.up_v;
    float *dn_dst = (p & 1) ? k.peers.dn_u : k.peers.dn_v;
    int rl = -1;  // the pass's residual sweep (0-based within the pass), if any
#pragma unroll
    for (int K = F - 1; K >= 0; --K)
      if (sweep_residual<F>(k, p, K + 1) >= 0) rl = K;
    const bool any = rl >= 0;
    bool ok = true;
    // Deliveries each neighbour has made once it finished pass p-1 of this
    // launch (and, with init_halo, its input rows), on top of earlier launches.
    const unsigned need = k.flag_base + (unsigned)(p + k.init_halo) * per_pass;
    for (int t = gw; t < T; t += GW) {
      int ty, tx, r0, r1;
      tile_coords(t, k.tiles_x, k.tiles_y, slab, ty, tx);
      tile_rows(k, ty, r0, r1);
      if (slab) {
        // The neighbours' halo rows must have arrived before this tile reads them.
        if (lane == 0) {
          if (k.peers.up_flag && r0 - F < k.row_lo &&
              !wait_counter(&k.ws->from_above, need, true, abort, k.peer_budget_ns, k.ws)) {
            record_status(k.ws, abort, kDevTimeoutPeer);
            ok = false;
          }
          if (ok && k.peers.dn_flag && r1 + F > k.row_hi &&
              !wait_counter(&k.ws->from_below, need, true, abort, k.peer_budget_ns, k.ws)) {
            record_status(k.ws, abort, kDevTimeoutPeer);
            ok = false;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
      const int x0 = tx * Wv<F>::TW;
      unsigned nd;
      if (tile_interior<F>(k, r0, r1, x0)) {
        if (any)
          nd = wave_tile_interior<F, 0>(k, src, dst, r0, r1, x0, ring, lane, rl, racc);
        else
          nd = wave_tile<F, false, false>(k, src, dst, up_dst, dn_dst, r0, r1, x0, ring, lane, rl, racc);
      } else {
        if (any)
          nd = wave_tile_edge<F, 0>(k, src, dst, up_dst, dn_dst, r0, r1, x0, ring, lane, rl, racc);
        else
          nd = wave_tile<F, true, false>(k, src, dst, up_dst, dn_dst, r0, r1, x0, ring, lane, rl, racc);
      }
      if (slab && nd) {
        __syncwarp();
        if (lane == 0) signal_deliveries(k, (int)(nd & 0xffffu), (int)(nd >> 16));
      }
    }
    // ---- end of pass p: CTA partial of the residual, grid barrier ----
    if (any) {
      const double wv = warp_sum_f64(*racc);
      if (lane == 0) sm.wsum[warp] = wv;
      *racc = 0.0;
    }
    if (__syncthreads_or(!ok || *abort)) break;
    const bool last = p + 1 == k.passes;
    if (threadIdx.x == 0) {
      if (any) {
        double tot = 0.0;
        for (int i = 0; i < NW; ++i) tot = __dadd_rn(tot, sm.wsum[i]);
        k.ws->partial[sweep_residual<F>(k, p, rl + 1) % kPartialSlots][blockIdx.x] = tot;
      }
      __threadfence();
      red_release_gpu_add(&k.ws->barrier, 1u);
      // Every CTA waits before the next pass; after the last pass only CTA 0
      // waits, and only when it has a residual to combine.
      if ((!last || (blockIdx.x == 0 && any)) &&
          !wait_counter(&k.ws->barrier, (unsigned)(p + 1) * (unsigned)G, false, abort, k.grid_budget_ns, k.ws))
        record_status(k.ws, abort, kDevTimeoutGridBarrier);
    }
    __syncthreads();
    if (*abort) break;
    if (blockIdx.x == 0 && warp == 0 && any) combine_residual(k, sweep_residual<F>(k, p, rl + 1), lane);
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

// Tile rows of a pass: warp w takes tiles w, w + warps, ...; every tile
// streams its rows plus 2F halo rows, so a pass lasts about
// ceil(tiles / warps) * (bh + 2F) row steps.  The height up to 128 with the
// least of that wins: small grids get one wave of shorter tiles (4096^2:
// 86-row tiles on all 1776 warps instead of 128-row tiles on 1120 of them,
// 803 -> 1039 Gcell/s).  Taller tiles re-sweep fewer halo rows but lose
// more: one wave of 5461-row tiles at 32768^2 measured 1323 against 3019
// Gcell/s (a pass waits for its slowest tile, and the edge tiles' masked
// path is the slow one).
static int wave_tile_rows(int rows, int tiles_x, long long warps, int F) {
#ifdef WV_BH_FIXED
  return WV_BH_FIXED;
#endif
  const long long t128 = (long long)tiles_x * ((rows + WV_BH - 1) / WV_BH);
  const long long n128 = (t128 + warps - 1) / warps;
  long long best_cost = -1, best = WV_BH;
  for (long long n = 1; n <= n128 + 1; ++n) {
    const long long per_col = n * warps / tiles_x;
    if (per_col < 1) continue;
    long long bh = (rows + per_col - 1) / per_col;
    if (bh > WV_BH) continue;
    if (bh < WV_BH_MIN) bh = WV_BH_MIN;
    const long long tiles = (long long)tiles_x * ((rows + bh - 1) / bh);
    const long long cost = (tiles + warps - 1) / warps * (bh + 2 * F);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bh;
    }
  }
  return (int)best;
}

template <int F>
cudaError_t launch_wave(const Jacobi2dProblem &p, const SlabPeers &peers, int64_t passes, int64_t sweep_base,
                        unsigned flag_base, int init_halo, cudaStream_t s) {
  using W = Wv<F>;
  J2Kernel k{};
  k.u = p.u;
  k.v = p.v;
  k.pitch = p.pitch;
  k.w = (int)p.w;
  k.h_local = (int)p.h_local;
  k.row_lo = (int)p.row_lo;
  k.row_hi = (int)p.row_hi;
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
  k.init_halo = init_halo;
  k.flag_base = flag_base;

  using L = WvLaunch<F>;
  constexpr size_t smem = sizeof(WvSmem<L::WARPS>);
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int configured_dev = -1;
  cudaError_t e;
  if (configured_dev != dev) {
    e = cudaFuncSetAttribute(jacobi2d_wave_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, jacobi2d_wave_kernel<F>, L::THREADS, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  long long g = (long long)per_sm * num_sms(dev);
  const int rows = (int)(p.row_hi - p.row_lo);
  k.tiles_x = (int)((p.w + W::TW - 1) / W::TW);
  k.bh = wave_tile_rows(rows, k.tiles_x, g * L::WARPS, F);
  k.tiles_y = (rows + k.bh - 1) / k.bh;
  const int rem = rows - (k.tiles_y - 1) * k.bh;
  k.last_start = (p.halo > 0 && k.tiles_y >= 2 && rem < p.halo) ? (int)p.row_hi - p.halo
                                                                  : (int)p.row_lo + (k.tiles_y - 1) * k.bh;
  const long long tiles = (long long)k.tiles_x * k.tiles_y;
  const long long want = (tiles + L::WARPS - 1) / L::WARPS;
  if (g > want) g = want;
  if (g > kMaxCtas) g = kMaxCtas;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)g);
  cfg.blockDim = dim3(L::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, jacobi2d_wave_kernel<F>, k);
}

// Tile columns of a pass fusing f sweeps over w columns.
int64_t tile_cols(int f, int64_t w) {
  const int64_t tw = f > 4 ? Wv<8>::TW : Wv<4>::TW;
  return (w + tw - 1) / tw;
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

bool jacobi2d_persistent_ok(const Jacobi2dProblem &p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p.u), b = reinterpret_cast<uintptr_t>(p.v);
  return ((a | b) & 15u) == 0 && (p.pitch * 4) % 16 == 0 && p.w >= 1 && p.h_local >= 1 &&
         p.w <= (1ll << 31) - 1 - 256 && p.h_local <= (1ll << 31) - 1 - 256 && p.pitch < (1ll << 37) &&
         p.row_lo >= 0 && p.row_hi <= p.h_local && p.row_hi > p.row_lo && p.sweeps <= (1ll << 30);
}

void jacobi2d_pass_plan(int64_t sweeps, int64_t res_every, int64_t plan[4]) {
  int fmax = kMaxWaveF;
  while (res_every > 0 && fmax > res_every) fmax >>= 1;  // at most one residual sweep per pass
  int64_t left = sweeps;
  for (int d = 0, f = kMaxWaveF; d < 4; ++d, f >>= 1) {
    // Even counts of the multi-sweep passes keep the ping-pong parity of the
    // single sweeps left over.
    plan[d] = f > fmax ? 0 : f == 1 ? left : (left / (2 * f)) * 2;
    left -= plan[d] * f;
  }
}

int64_t jacobi2d_slab_deliveries(int64_t sweeps, int64_t res_every, int64_t w, int halo) {
  int64_t plan[4];
  jacobi2d_pass_plan(sweeps, res_every, plan);
  int64_t total = 0;
  bool first = true;
  for (int d = 0, f = kMaxWaveF; d < 4; ++d, f >>= 1) {
    if (plan[d] == 0) continue;
    total += (plan[d] + (first ? 1 : 0)) * tile_cols(f, w) * halo;
    first = false;
  }
  return total;
}

cudaError_t run_jacobi2d_persistent(const Jacobi2dProblem &p, const SlabPeers &peers, unsigned flag_base,
                                    cudaStream_t s) {
  int64_t plan[4];
  jacobi2d_pass_plan(p.sweeps, p.res_every, plan);
  int64_t sweeps_done = 0;
  unsigned flags = flag_base;
  bool first = true;
  cudaError_t e = cudaSuccess;
  for (int d = 0, f = kMaxWaveF; d < 4; ++d, f >>= 1) {
    const int64_t n = plan[d];
    if (n == 0) continue;
    e = cudaMemsetAsync(&p.ws->barrier, 0, sizeof(unsigned), s);  // fresh grid barrier, same status word
    if (e != cudaSuccess) return e;
    // A slab run delivers its input's edge rows before its first pass.
    const int init = (p.halo > 0 && first) ? 1 : 0;
    switch (f) {
      case 8: e = launch_wave<8>(p, peers, n, sweeps_done, flags, init, s); break;
      case 4: e = launch_wave<4>(p, peers, n, sweeps_done, flags, init, s); break;
      case 2: e = launch_wave<2>(p, peers, n, sweeps_done, flags, init, s); break;
      default: e = launch_wave<1>(p, peers, n, sweeps_done, flags, init, s); break;
    }
    if (e != cudaSuccess) return e;
    flags += (unsigned)((n + init) * tile_cols(f, p.w) * p.halo);
    sweeps_done += n * f;
    first = false;
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
