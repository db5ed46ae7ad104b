// jacobi3d_tb.cu -- Jacobi-3D 7-point sweeps, F sweeps per pass over HBM.
//
// Temporal blocking along z (3.5-D blocking).  A work item is a tile of 128
// columns x TH rows over a chunk of consecutive planes [z0, z1).  Its CTA
// streams the planes of the item's box -- 136 columns (4 more on each side,
// so TMA x offsets stay 16-byte aligned) x BHB = TH + 2F rows, from plane
// z0 - F to z1 + F - 1 -- through a ring of RING plane buffers
// (cp.async.bulk.tensor.3d, mbarrier completion, issued by thread 0 three
// planes ahead, across item boundaries).  Every input plane advances a
// wavefront of F sweeps: when input plane q lands, sweep 1 computes plane
// q - 1, sweep 2 plane q - 2, ..., sweep F plane q - F, which is stored.
//
// Thread layout: 34 float4 column groups x 15 bands in 16 warps (the last two
// threads only take part in barriers and shuffles; 16 warps, 4 per SM
// sub-partition, leave 128 registers a thread); a thread owns one group of RPW
// consecutive box rows.  For every sweep level it keeps its cells'
// values in the two planes below the newest one in registers, so the z
// neighbours and the rows inside its band never leave registers and the x
// neighbours come by shuffles.  Only band-edge rows, and the groups of the
// lanes at warp edges, pass through shared memory: one double-buffered plane
// per intermediate level, written at one plane step and read at the next, so
// a single __syncthreads per plane step orders every hand-off.  The box loses
// one cell per sweep on every side, and exactly the owned tile is valid after
// F sweeps; that redundant halo work is the price of keeping F sweeps on chip.
//
// Passes are separated by a grid barrier (cooperative launch; the per-pass
// CTA residual partials are combined in CTA order by CTA 0).  Every wait is
// bounded and records a DevStatus on expiry.
//
// z-slabs across GPUs (SlabPeers, kSlabHalo3 = 2 halo planes on each side): a
// rank updates its owned planes [z_lo, z_hi).  The work items of the first
// (last) z-chunk come first in every pass; when one has finished, its threads
// copy their cells of the first (last) F owned planes into the neighbour's
// halo planes over NVLink and thread 0 bumps the neighbour's delivery counter
// (release, system scope; one delivery per tile per pass, counters only grow
// across launches).  Before thread 0 stages a halo plane it
// acquires the counter it needs.  A run's first launch first copies the
// input's edge planes into the neighbours' halos (counted as one pass).  TMA
// only ever reads this GPU's own memory.  Arithmetic per cell is the
// reference order ((((((c + xm) + xp) + ym) + yp) + zm) + zp) * (1/7) with
// IEEE round-to-nearest adds, so results are bit-identical to one sweep at a
// time.
#include <cuda.h>

#include "internal.h"

namespace spmdb200 {
namespace {

// The longest pass the plan uses.  Measured at 512^3 x 50 (residual every
// 10) on B200: two-sweep passes 704 Gcell/s, four-sweep passes (with 2
// single sweeps) 547, single sweeps 644 -- per sweep level the kernel is
// issue- and latency-bound, and the four-sweep tile re-sweeps 45 % more
// cells than it owns (two sweeps: 17 %).
#ifndef SPMDB200_J3TB_FMAX
#define SPMDB200_J3TB_FMAX 2
#endif
constexpr int kTbMaxF = SPMDB200_J3TB_FMAX;
static_assert(kSlabHalo3 >= kTbMaxF, "z-slab halos hold the planes of the longest pass");
constexpr int kTbGroups = 34;                  // float4 column groups per box row
constexpr int kTbBoxW = 4 * kTbGroups;         // 136 columns: 128 owned + 4 each side
constexpr int kTbOwnW = 128;
constexpr int kTbBands = 15;
constexpr int kTbThreads = 512;                 // 510 cell threads + 2 idle
constexpr int kTbWarps = kTbThreads / 32;
static_assert(kTbGroups * kTbBands <= kTbThreads && kTbThreads % 32 == 0, "whole warps");

template <int F>
struct Tb {
#ifndef SPMDB200_J3TB_RPW2
#define SPMDB200_J3TB_RPW2 3
#endif
  static constexpr int RPW = F >= 4 ? 2 : F == 2 ? SPMDB200_J3TB_RPW2 : 3;  // rows per thread (12 * RPW registers per level)
  // Sweep level 0 (the input) read from the ring instead of registers (four
  // sweeps: 3 x 4 x 24 registers would not fit); the ring then keeps one
  // more plane (the centre's z - 1).
#ifndef SPMDB200_J3TB_L0F
#define SPMDB200_J3TB_L0F 4
#endif
  static constexpr int L0 = F >= SPMDB200_J3TB_L0F ? 1 : 0;
  static constexpr int RING = 4 + L0;              // input plane buffers; RING - 1 - L0 planes in flight
  static constexpr int BHB = kTbBands * RPW;       // box rows
  static constexpr int TH = BHB - 2 * F;           // owned rows per tile
  static constexpr int PLANE = BHB * kTbBoxW;      // floats of one box plane
  static constexpr int PSTR = (PLANE + 31) / 32 * 32;  // plane buffer stride (128-byte aligned)
  static constexpr int PUB = F - 1;                // intermediate levels handed over in shared memory
  static constexpr size_t SMEM = ((size_t)RING + 2 * PUB) * PSTR * 4 + 128;
  static_assert(TH >= 1, "tile too short for F sweeps");
};

struct J3Tb {
  float *u, *v;             // pass p reads (p even ? u : v) and writes the other
  long long sy, sz;         // strides in elements (x contiguous)
  int d, h, w;              // local planes, rows, columns
  int z_lo, z_hi;           // owned local planes
  long long g_z0, g_d;      // global plane of local plane 0, global plane count
  int tiles_x, tiles_y, zchunks, bz;
  int passes, sweep_base, res_every;
  double *res_out;
  JacobiWs *ws;
  unsigned long long budget_ns, peer_budget_ns;
  SlabPeers peers;          // z-slab mode
  int halo;                 // halo planes on each side (z-slab mode)
  int init_halo;            // 1: deliver the input's edge planes before pass 0
  unsigned flag_base;       // deliveries received from each neighbour before this launch
};

__device__ __forceinline__ float4 lds4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void sts4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }

// Four cells of one row: scalar adds for the x terms (their operands straddle
// the float4's pairs), then packed pair adds for y and z and the scale.
__device__ __forceinline__ float4 j7x4(float4 c, float west, float east, float4 n, float4 s, float4 zm,
                                       float4 zp) {
  const float v0 = __fadd_rn(__fadd_rn(c.x, west), c.y);
  const float v1 = __fadd_rn(__fadd_rn(c.y, c.x), c.z);
  const float v2 = __fadd_rn(__fadd_rn(c.z, c.y), c.w);
  const float v3 = __fadd_rn(__fadd_rn(c.w, c.z), east);
  float2 a = __fadd2_rn(make_float2(v0, v1), make_float2(n.x, n.y));
  float2 b = __fadd2_rn(make_float2(v2, v3), make_float2(n.z, n.w));
  a = __fadd2_rn(a, make_float2(s.x, s.y));
  b = __fadd2_rn(b, make_float2(s.z, s.w));
  a = __fadd2_rn(a, make_float2(zm.x, zm.y));
  b = __fadd2_rn(b, make_float2(zm.z, zm.w));
  a = __fadd2_rn(a, make_float2(zp.x, zp.y));
  b = __fadd2_rn(b, make_float2(zp.z, zp.w));
  const float k7 = 1.0f / 7.0f;
  a = __fmul2_rn(a, make_float2(k7, k7));
  b = __fmul2_rn(b, make_float2(k7, k7));
  return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ double sq4(float4 o, float4 c, bool m0, bool m1, bool m2, bool m3) {
  double acc = 0.0;
  const float oo[4] = {o.x, o.y, o.z, o.w}, cc[4] = {c.x, c.y, c.z, c.w};
  const bool mm[4] = {m0, m1, m2, m3};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (mm[i]) {
      const double e = __dsub_rn((double)oo[i], (double)cc[i]);
      acc = __dadd_rn(acc, __dmul_rn(e, e));
    }
  }
  return acc;
}

// Item t -> box origin and plane range.  Tiles of one z-chunk are
// consecutive, so the CTAs of one wave share their halo rows in L2; the
// first and the last z-chunk (the items a neighbour waits for) come first.
struct TbItem {
  int bx, by;        // box origin (column, row); bx is a multiple of 4
  int z0, z1;        // owned planes
  int n;             // input planes streamed: z1 - z0 + 2F
  bool edge;         // the box holds boundary or outside cells in x or y (z: checked per plane)
  bool first, last;  // first / last z-chunk of the owned planes
};

template <int F>
__device__ __forceinline__ TbItem tb_item(const J3Tb &k, int t) {
  TbItem it;
  const int txy = k.tiles_x * k.tiles_y;
  const int zi = t / txy, rest = t - zi * txy;
  const int zc = k.zchunks < 3 ? zi : zi == 0 ? 0 : zi == 1 ? k.zchunks - 1 : zi - 1;
  const int tx = rest % k.tiles_x, ty = rest / k.tiles_x;
  it.bx = tx * kTbOwnW - 4;
  it.by = ty * Tb<F>::TH - F;
  it.z0 = k.z_lo + zc * k.bz;
  it.z1 = min(k.z_hi, it.z0 + k.bz);
  it.n = it.z1 - it.z0 + 2 * F;
  it.edge = !(it.bx >= 1 && it.bx + kTbBoxW <= k.w - 1 && it.by >= 1 && it.by + Tb<F>::BHB <= k.h - 1);
  it.first = zc == 0;
  it.last = zc == k.zchunks - 1;
  return it;
}

__device__ __forceinline__ void tb_record(JacobiWs *ws, volatile int *abort, int code) {
  atomicCAS(&ws->status, 0, code);
  *abort = 1;
}

// Bounded wait until *p (a counter that only grows) reaches target.
__device__ __forceinline__ bool tb_wait_counter(const J3Tb &k, const unsigned *p, unsigned target, bool sys,
                                                unsigned long long budget) {
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if ((int)((sys ? ld_acquire_sys(p) : ld_acquire_gpu(p)) - target) >= 0) return true;
    if ((i & 7u) == 7u && *reinterpret_cast<const volatile int *>(&k.ws->status) != 0) return false;
    if (globaltimer_ns() - t0 > budget) return false;
    __nanosleep(64);
  }
}
__device__ __forceinline__ bool tb_wait_barrier(const J3Tb &k, unsigned target) {
  return tb_wait_counter(k, &k.ws->barrier, target, false, k.budget_ns);
}

// z-slab mode, thread 0, before staging a halo plane: wait until the
// neighbour delivered it (out of line: it runs a few times per pass).
__device__ __noinline__ bool tb_halo_wait(const J3Tb &k, bool wait_up, bool wait_dn, unsigned need) {
  if (wait_up && !tb_wait_counter(k, &k.ws->from_above, need, true, k.peer_budget_ns)) return false;
  if (wait_dn && !tb_wait_counter(k, &k.ws->from_below, need, true, k.peer_budget_ns)) return false;
  // the acquire above, then the async-proxy read of the peer-written plane
  fence_proxy_async_global();
  return true;
}

// Thread 0: stage the next plane of this CTA's stream for pass p into the
// ring.  z-slab mode: a halo plane only once the neighbour delivered it.
// Thread 0's issue cursor, kept in shared memory (in registers it would
// occupy every thread's: the plane loop runs at the 128-register limit).
struct TbCursor {
  uint32_t ic;  // input planes issued
  int t, j;     // item and plane of the item the next load belongs to
  TbItem it;
};

template <int F, bool SLAB>
__device__ __forceinline__ bool tb_issue(const J3Tb &k, const void *src, float *ring, uint64_t *full, TbCursor &cur,
                                         int items, unsigned need) {
  uint32_t &ic = cur.ic;
  int &t_i = cur.t, &j_i = cur.j;
  TbItem &it_i = cur.it;
  constexpr int PL = Tb<F>::PSTR;
  const int q = it_i.z0 - F + j_i;
  if constexpr (SLAB) {
    const bool wait_up = it_i.first && k.peers.up_u && q < k.z_lo;
    const bool wait_dn = it_i.last && k.peers.dn_u && q >= k.z_hi;
    if ((wait_up || wait_dn) && !tb_halo_wait(k, wait_up, wait_dn, need)) return false;
  }
  const uint32_t slot = ic % Tb<F>::RING;
  mbar_arrive_expect_tx(&full[slot], (uint32_t)Tb<F>::PLANE * 4u);
  tma_load_3d(ring + slot * PL, src, &full[slot], it_i.bx, it_i.by, q);
  ++ic;
  if (++j_i == it_i.n) {
    j_i = 0;
    t_i += gridDim.x;
    if (t_i < items) it_i = tb_item<F>(k, t_i);
  }
  return true;
}

// Residual index of sweep level l (1-based) of pass p, or -1.
template <int F>
__device__ __forceinline__ int tb_residual(const J3Tb &k, int p, int l) {
  if (k.res_every <= 0) return -1;
  const int s = k.sweep_base + F * p + l;
  return s % k.res_every == 0 ? s / k.res_every - 1 : -1;
}

// CTA 0: residual r = the CTA partials in CTA order (warp 0); in z-slab mode
// also all-gathered into every rank's slot array.
__device__ __forceinline__ void tb_combine(const J3Tb &k, int r, int lane) {
  double p = 0.0;
  for (int i = lane; i < (int)gridDim.x; i += 32)
    p = __dadd_rn(p, __ldcg(&k.ws->partial[r % kJacobiPartialSlots][i]));
  p = warp_sum_f64(p);
  if (lane == 0) {
    if (k.res_out) k.res_out[r] = p;
    if (k.peers.peer_ws[0] && r < kMaxResSlots) {
      for (int q = 0; q < k.peers.nranks; ++q)
        if (k.peers.peer_ws[q]) k.peers.peer_ws[q]->res_slots[r][k.peers.rank] = p;
      __threadfence_system();
    }
  }
}

__device__ __forceinline__ void tb_store4(float *p, int gx0, int w, float4 o) {
  if (gx0 + 3 < w) {
    st_f4(p, o);
  } else {
    p[0] = o.x;
    if (gx0 + 1 < w) p[1] = o.y;
    if (gx0 + 2 < w) p[2] = o.z;
  }
}

// z-slab mode, before pass 0 of a run: the first (last) F owned planes of the
// input go into the halo planes of the neighbour above (below), counted as
// one pass of deliveries (split over the CTAs).
template <int F>
__device__ __forceinline__ void tb_deliver_input_halo(const J3Tb &k, unsigned per_pass) {
  const int gpr = (k.w + 3) / 4;
  const long long per_plane = (long long)k.h * gpr;
  const long long total = 2ll * F * per_plane;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int side = (int)(i / (F * per_plane));
    const long long rem = i - side * F * per_plane;
    const int f = (int)(rem / per_plane);
    const long long rg = rem - f * per_plane;
    const int y = (int)(rg / gpr), gx0 = 4 * (int)(rg - (long long)y * gpr);
    const long long yo = (long long)y * k.sy + gx0;
    if (side == 0 && k.peers.up_u) {
      const float4 v = ld_f4(k.u + (long long)(k.z_lo + f) * k.sz + yo);
      tb_store4(k.peers.up_u + (k.peers.up_row + f) * k.sz + yo, gx0, k.w, v);
    } else if (side == 1 && k.peers.dn_u) {
      const float4 v = ld_f4(k.u + (long long)(k.z_hi - F + f) * k.sz + yo);
      tb_store4(k.peers.dn_u + (k.peers.dn_row + k.halo - F + f) * k.sz + yo, gx0, k.w, v);
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned share = per_pass / gridDim.x + (blockIdx.x < per_pass % gridDim.x ? 1u : 0u);
    if (share) {
      if (k.peers.up_flag) red_release_sys_add(k.peers.up_flag, share);
      if (k.peers.dn_flag) red_release_sys_add(k.peers.dn_flag, share);
    }
  }
}

// Per-item constants of one thread.
template <int F>
struct TbLanes {
  bool rfix[Tb<F>::RPW];   // row on the y boundary or outside the grid: keeps its value
  bool rown[Tb<F>::RPW];   // row owned by the tile
  bool cm0, cm1, cm2, cm3; // column on the x boundary or outside the grid: keeps its value
  bool ow0, ow1, ow2, ow3; // column owned (residual)
  int gx0;                 // global column of the thread's first cell
};

// Mutable state of one thread; registers once everything is inlined.
template <int F>
struct TbCtx {
  uint32_t pc;      // input planes consumed
  double acc;       // residual partial
  // A[l - L0][s][r]: the thread's cells of box row r0 + r at sweep level l
  // (0: the input) in the plane of the last plane step congruent to s mod 3,
  // so the z windows rotate with the unrolled step loop and never move.
  float4 A[F - Tb<F>::L0][3][Tb<F>::RPW];
};

__device__ __forceinline__ void tb_st4_if(bool pred, float *p, float4 v) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %0, 0;\n\t"
      "@q st.global.v4.f32 [%1], {%2, %3, %4, %5};\n\t}" ::"r"((uint32_t)pred),
      "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w));
}

// z-slab mode, after an item of the first / last z-chunk has stored its
// planes: the first / last F owned planes (each thread re-reads the cells it
// stored, L2-resident) go to the neighbour's halo planes over NVLink, then
// thread 0 counts the delivery.  Outside the plane loop, so that loop is the
// one-GPU loop (inside it, the slab path spilled and ran ~1.5x slower).
template <int F>
__device__ __forceinline__ void tb_deliver_item(const J3Tb &k, const TbLanes<F> &L, const TbItem &it, int p, int r0,
                                                const float *dst) {
  const bool up = it.first && k.peers.up_u != nullptr, dn = it.last && k.peers.dn_u != nullptr;
  if (!up && !dn) return;
#pragma unroll 1
  for (int e = 0; e < 2; ++e) {
    if (e == 0 ? !up : !dn) continue;
    float *to = e == 0 ? ((p & 1) ? k.peers.up_u : k.peers.up_v) : ((p & 1) ? k.peers.dn_u : k.peers.dn_v);
#pragma unroll 1
    for (int f = 0; f < F; ++f) {
      const long long gz = e == 0 ? k.z_lo + f : k.z_hi - F + f;
      const long long tz = e == 0 ? k.peers.up_row + f : k.peers.dn_row + k.halo - F + f;
#pragma unroll
      for (int r = 0; r < Tb<F>::RPW; ++r) {
        if (!L.rown[r] || !L.ow0) continue;
        const long long yo = (long long)(it.by + r0 + r) * k.sy + L.gx0;
        // a full float4 stays inside the row pitch (a multiple of 4 floats)
        tb_store4(to + tz * k.sz + yo, L.gx0, k.w, ld_f4(dst + gz * k.sz + yo));
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (up) red_release_sys_add(k.peers.up_flag, 1u);
    if (dn) red_release_sys_add(k.peers.dn_flag, 1u);
  }
}

// One plane step of item `it` (PH = j mod 3): input plane q = z0 - F + j has
// landed in the ring; sweep l computes plane q - l from the registers of
// level l - 1 (z neighbours and the rows inside the band), shuffles (x), and
// the band-edge rows and warp-edge groups of level l - 1's previous plane
// from shared memory.  EDGE: the tile touches the grid's x or y boundary.
// Returns false if the wait for the plane timed out (warp-uniform).
template <int F, bool EDGE, int PH>
__device__ __forceinline__ bool tb_step(const J3Tb &k, TbCtx<F> &C, const TbLanes<F> &L, const TbItem &it, int j,
                                        int p, int rl, float *dst, const float *ring, float *pub, uint64_t *full,
                                        volatile int *abort, int lane, int g, int r0, bool active, int top_off,
                                        int bot_off, bool w_edge, bool e_edge) {
  constexpr int RPW = Tb<F>::RPW, PL = Tb<F>::PSTR, RING = Tb<F>::RING, L0 = Tb<F>::L0;
  constexpr int P1 = (PH + 2) % 3, P2 = (PH + 1) % 3;  // the previous step, two steps back
  const uint32_t slot = C.pc % RING;
  if (!mbar_wait_warp(&full[slot], (C.pc / RING) & 1u, abort)) return false;
  const int q = it.z0 - F + j;
  const int off = r0 * kTbBoxW + 4 * g;  // the thread's first cell in a plane buffer
  const float *P = ring + slot * PL;
  const float *nb = ring + ((C.pc + RING - 1) % RING) * PL;  // level 0, plane q - 1
  float4 in_m[L0 ? RPW : 1], in_c[L0 ? RPW : 1], in_p[L0 ? RPW : 1];  // level 0 from the ring (L0)
  if constexpr (L0) {
    const float *Pm = ring + ((C.pc + RING - 2) % RING) * PL;  // plane q - 2
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      in_m[r] = lds4(Pm + off + r * kTbBoxW);
      in_c[r] = lds4(nb + off + r * kTbBoxW);
      in_p[r] = lds4(P + off + r * kTbBoxW);
    }
  } else {
#pragma unroll
    for (int r = 0; r < RPW; ++r) C.A[0][PH][r] = lds4(P + off + r * kTbBoxW);
  }
  const int par = j & 1;  // hand-off buffer written at this step
#pragma unroll
  for (int l = 1; l <= F; ++l) {
    const int gz = q - l;  // plane computed by sweep l
    const float4 *zm, *c, *zp;
    if (L0 && l == 1) {
      zm = in_m;
      c = in_c;
      zp = in_p;
    } else {
      zm = C.A[l - 1 - L0][P2];
      c = C.A[l - 1 - L0][P1];
      zp = C.A[l - 1 - L0][PH];
    }
    // the rows above / below the band (band 0 and the last band read their own
    // edge row instead: their outer rows are halo rows, never kept)
    const float4 top = lds4(nb + off + top_off);
    const float4 bot = lds4(nb + off + bot_off);
    float4 o[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const float4 cc = c[r];
      float west = __shfl_up_sync(0xffffffffu, cc.w, 1);
      float east = __shfl_down_sync(0xffffffffu, cc.x, 1);
      if (w_edge) west = nb[off + r * kTbBoxW - 1];
      if (e_edge) east = nb[off + r * kTbBoxW + 4];
      float4 v = j7x4(cc, west, east, r == 0 ? top : c[r - 1], r == RPW - 1 ? bot : c[r + 1], zm[r], zp[r]);
      if (EDGE) {
        if (L.rfix[r]) v = cc;
        if (L.cm0) v.x = cc.x;
        if (L.cm1) v.y = cc.y;
        if (L.cm2) v.z = cc.z;
        if (L.cm3) v.w = cc.w;
      }
      o[r] = v;
    }
    const long long gzg = k.g_z0 + gz;
    if (gzg <= 0 || gzg >= k.g_d - 1) {  // a fixed plane (or outside the grid)
#pragma unroll
      for (int r = 0; r < RPW; ++r) o[r] = c[r];
    }
    if (l == rl && gz >= it.z0 && gz < it.z1) {
#pragma unroll
      for (int r = 0; r < RPW; ++r)
        if (L.rown[r]) C.acc = __dadd_rn(C.acc, sq4(o[r], c[r], L.ow0, L.ow1, L.ow2, L.ow3));
    }
    if (l < F) {
      // keep the plane, and hand it to the next plane step: band-edge rows for
      // the bands above / below, every row of the warp-edge groups
      float *Q = pub + ((l - 1) * 2 + par) * PL + off;
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        C.A[l - L0][PH][r] = o[r];
        if (active && (r == 0 || r == RPW - 1 || lane == 0 || lane == 31)) sts4(Q + r * kTbBoxW, o[r]);
      }
      nb = pub + ((l - 1) * 2 + (par ^ 1)) * PL;  // level l, plane q - l - 1 (the previous step's)
    } else if (j >= 2 * F) {
      // sweep F: plane q - F of the owned tile
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const long long yo = (long long)(it.by + r0 + r) * k.sy + L.gx0;
        float *op = dst + (long long)gz * k.sz + yo;
        if (EDGE) {
          if (L.rown[r] && L.ow0) tb_store4(op, L.gx0, k.w, o[r]);
        } else {
          tb_st4_if(L.rown[r] && L.ow0, op, o[r]);
        }
      }
    }
  }
  return true;
}

// After a plane step: the CTA barrier, and thread 0 refilling the ring slot
// the step freed.  Returns false if any warp's wait timed out.
template <int F, bool SLAB>
__device__ __forceinline__ bool tb_after_step(const J3Tb &k, TbCtx<F> &C, TbCursor &cur, bool got, const void *src,
                                              float *ring, uint64_t *full, volatile int *abort, int items,
                                              unsigned need) {
  ++C.pc;
  if (__syncthreads_or(!got)) {
    if (threadIdx.x == 0 && *abort == 0) tb_record(k.ws, abort, kDevTimeoutFull);
    --C.pc;  // this step's plane did not land (or was never issued)
    return false;
  }
  if (threadIdx.x == 0) {
    // the slot of the step's centre plane is free: refill it
    if (cur.t < items && !tb_issue<F, SLAB>(k, src, ring, full, cur, items, need)) {
      tb_record(k.ws, abort, kDevTimeoutPeer);
      cur.t = items;
    }
  }
  return true;
}

// All plane steps of one item, unrolled by three (the register rotation).
template <int F, bool SLAB, bool EDGE>
__device__ __forceinline__ bool tb_run_item(const J3Tb &k, TbCtx<F> &C, TbCursor &cur, const TbLanes<F> &L,
                                            const TbItem &it,
                                            int p, int rl, const void *src, float *dst, float *ring, float *pub,
                                            uint64_t *full, volatile int *abort, int items, unsigned need, int lane,
                                            int g, int r0, bool active, int top_off, int bot_off, bool w_edge,
                                            bool e_edge) {
#define TB_STEP(PH)                                                                                              \
  {                                                                                                              \
    const bool got = tb_step<F, EDGE, PH>(k, C, L, it, j + PH, p, rl, dst, ring, pub, full, abort, lane, g,       \
                                                r0, active, top_off, bot_off, w_edge, e_edge);                  \
    if (!tb_after_step<F, SLAB>(k, C, cur, got, src, ring, full, abort, items, need)) return false;           \
  }
  int j = 0;
  for (; j + 3 <= it.n; j += 3) {
    TB_STEP(0)
    TB_STEP(1)
    TB_STEP(2)
  }
  if (j < it.n) TB_STEP(0)
  if (j + 1 < it.n) TB_STEP(1)
#undef TB_STEP
  return true;
}

// SLAB: z-slab mode (peer deliveries and waits); the one-GPU instantiation
// carries none of that code.
template <int F, bool SLAB>
__global__ void __launch_bounds__(kTbThreads, 1) jacobi3d_tb_kernel(const __grid_constant__ CUtensorMap map_u,
                                                                    const __grid_constant__ CUtensorMap map_v,
                                                                    const __grid_constant__ J3Tb k) {
  using T = Tb<F>;
  constexpr int RPW = T::RPW;
  extern __shared__ __align__(128) unsigned char tb_raw[];
  __shared__ uint64_t full[T::RING];
  __shared__ double wsum[kTbWarps];
  __shared__ int abort_s;
  __shared__ TbCursor cur;
  float *ring = reinterpret_cast<float *>(tb_raw + ((128u - (smem_u32(tb_raw) & 127u)) & 127u));
  float *pub = ring + T::RING * T::PSTR;  // [level 1..F-1][2] planes
  volatile int *abort = &abort_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool active = tid < kTbGroups * kTbBands;  // idle threads read band 14, store nothing
  const int g = tid % kTbGroups, band = active ? tid / kTbGroups : kTbBands - 1, r0 = band * RPW;
  const int G = gridDim.x;
  const int items = k.tiles_x * k.tiles_y * k.zchunks;
  const bool own_g = active && g >= 1 && g <= kTbGroups - 2;
  const int top_off = band > 0 ? -kTbBoxW : 0;                               // row above the band
  const int bot_off = (band < kTbBands - 1 ? RPW : RPW - 1) * kTbBoxW;        // row below the band
  const bool w_edge = lane == 0 && g > 0, e_edge = lane == 31 && g < kTbGroups - 1;
  const unsigned per_pass = (unsigned)(k.tiles_x * k.tiles_y);  // deliveries to each neighbour per pass

  if (tid == 0) {
    for (int i = 0; i < T::RING; ++i) mbar_init(&full[i], 1);
    abort_s = 0;
    cur.ic = 0;
    mbar_fence_init();
    tma_prefetch_desc(&map_u);
    tma_prefetch_desc(&map_v);
  }
  __syncthreads();
  if constexpr (SLAB) {
    if (k.init_halo) tb_deliver_input_halo<F>(k, per_pass);
  }

  TbCtx<F> C;
  C.pc = 0;

  C.acc = 0.0;
#pragma unroll
  for (int l = 0; l < F - T::L0; ++l)
#pragma unroll
    for (int s = 0; s < 3; ++s)
#pragma unroll
      for (int r = 0; r < RPW; ++r) C.A[l][s][r] = make_float4(0.f, 0.f, 0.f, 0.f);
  bool failed = false;
  int prev_r = -1;  // residual of the previous pass

  for (int p = 0; p < k.passes; ++p) {
    const void *src = (p & 1) ? (const void *)&map_v : (const void *)&map_u;
    float *dst = (p & 1) ? k.u : k.v;
    int rl = -1, ridx = -1;  // residual sweep level of this pass (at most one)
#pragma unroll
    for (int l = 1; l <= F; ++l) {
      const int r = tb_residual<F>(k, p, l);
      if (r >= 0) {
        rl = l;
        ridx = r;
      }
    }
    if (p > 0) {
      if (tid == 0 && !tb_wait_barrier(k, (unsigned)p * (unsigned)G)) tb_record(k.ws, abort, kDevTimeoutGridBarrier);
      if (__syncthreads_or(*abort != 0)) {
        failed = true;
        break;
      }
      if (blockIdx.x == 0 && warp == 0 && prev_r >= 0) tb_combine(k, prev_r, lane);
    }

    const unsigned need = k.flag_base + (unsigned)(k.init_halo + p) * per_pass;  // halo deliveries for pass p
    if (tid == 0) {
      cur.t = blockIdx.x;
      cur.j = 0;
      if (cur.t < items) cur.it = tb_item<F>(k, cur.t);
      for (int s = 0; s < T::RING - 1 - T::L0 && cur.t < items; ++s)
        if (!tb_issue<F, SLAB>(k, src, ring, full, cur, items, need)) {
          tb_record(k.ws, abort, kDevTimeoutPeer);
          cur.t = items;  // issue nothing more; the consumers see the abort flag
        }
    }

    for (int t = blockIdx.x; t < items; t += G) {
      const TbItem it = tb_item<F>(k, t);
      TbLanes<F> L;
      L.gx0 = it.bx + 4 * g;
      L.cm0 = L.gx0 <= 0 || L.gx0 >= k.w - 1;
      L.cm1 = L.gx0 + 1 <= 0 || L.gx0 + 1 >= k.w - 1;
      L.cm2 = L.gx0 + 2 <= 0 || L.gx0 + 2 >= k.w - 1;
      L.cm3 = L.gx0 + 3 <= 0 || L.gx0 + 3 >= k.w - 1;
      L.ow0 = own_g && L.gx0 < k.w;
      L.ow1 = own_g && L.gx0 + 1 < k.w;
      L.ow2 = own_g && L.gx0 + 2 < k.w;
      L.ow3 = own_g && L.gx0 + 3 < k.w;
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int gy = it.by + r0 + r;
        L.rfix[r] = gy <= 0 || gy >= k.h - 1;
        L.rown[r] = r0 + r >= F && r0 + r < F + T::TH && gy < k.h;
      }
      const bool ok = it.edge ? tb_run_item<F, SLAB, true>(k, C, cur, L, it, p, rl, src, dst, ring, pub, full, abort, items,
                                                            need, lane, g, r0, active, top_off, bot_off, w_edge,
                                                            e_edge)
                              : tb_run_item<F, SLAB, false>(k, C, cur, L, it, p, rl, src, dst, ring, pub, full, abort,
                                                             items, need, lane, g, r0, active, top_off, bot_off,
                                                             w_edge, e_edge);
      if constexpr (SLAB) {
        if (ok) tb_deliver_item<F>(k, L, it, p, r0, dst);
      }
      if (!ok) {
        failed = true;
        break;
      }
    }
    if (failed) break;

    // end of pass: residual partial, then arrive on the grid barrier
    if (rl >= 0) {
      const double wv = warp_sum_f64(C.acc);
      if (lane == 0) wsum[warp] = wv;
      C.acc = 0.0;
    }
    fence_proxy_async_global();  // this pass's stores before the next pass's TMA reads
    __syncthreads();
    if (tid == 0) {
      if (rl >= 0) {
        double tot = 0.0;
        for (int i = 0; i < kTbWarps; ++i) tot = __dadd_rn(tot, wsum[i]);
        k.ws->partial[ridx % kJacobiPartialSlots][blockIdx.x] = tot;
      }
      __threadfence();
      red_release_gpu_add(&k.ws->barrier, 1u);
    }
    prev_r = ridx;
  }

  if (!failed && blockIdx.x == 0 && prev_r >= 0) {
    if (tid == 0 && !tb_wait_barrier(k, (unsigned)k.passes * (unsigned)G))
      tb_record(k.ws, abort, kDevTimeoutGridBarrier);
    if (!__syncthreads_or(*abort != 0) && warp == 0) tb_combine(k, prev_r, lane);
  }
  if (failed && tid == 0) {
    // planes issued but not consumed must land before shared memory is released
    for (uint32_t i = C.pc; (int)(cur.ic - i) > 0; ++i) {
      int no_abort = 0;
      mbar_wait_bounded(&full[i % T::RING], (i / T::RING) & 1u, &no_abort);
    }
  }
}

// z-chunks of the owned planes: about three items per CTA, chunks of at least
// 4F planes, and first / last chunks of at least F planes (the planes a
// neighbour waits for come from one item).
inline void tb_chunks(int64_t planes, int64_t txy, int64_t ctas, int F, int &bz, int &zchunks) {
  int64_t zc = (3 * ctas) / (txy > 0 ? txy : 1);
  const int64_t zc_max = (planes + 4 * F - 1) / (4 * F);
  if (zc > zc_max) zc = zc_max;
  if (zc < 1) zc = 1;
  for (;; --zc) {
    const int64_t b = (planes + zc - 1) / zc;
    const int64_t n = (planes + b - 1) / b;
    if (zc == 1 || planes - (n - 1) * b >= F) {
      bz = (int)b;
      zchunks = (int)n;
      return;
    }
  }
}

template <int F>
int64_t tb_tiles(int64_t h, int64_t w) {
  return ((w + kTbOwnW - 1) / kTbOwnW) * ((h + Tb<F>::TH - 1) / Tb<F>::TH);
}

template <int F, bool SLAB>
cudaError_t launch_tb(const Jacobi3dProblem &p, const SlabPeers &peers, int64_t passes, int64_t sweep_base,
                      unsigned flag_base, int init_halo, cudaStream_t s) {
  using T = Tb<F>;
  CUtensorMap mu, mv;
  const uint64_t dims[3] = {(uint64_t)p.w, (uint64_t)p.h, (uint64_t)p.d};
  const uint64_t strides[2] = {(uint64_t)p.sy * 4u, (uint64_t)p.sz * 4u};
  const uint32_t box[3] = {(uint32_t)kTbBoxW, (uint32_t)T::BHB, 1u};
  if (encode_tensor_map_f32(&mu, p.u, 3, dims, strides, box) != 0) return cudaErrorInvalidValue;
  if (encode_tensor_map_f32(&mv, p.v, 3, dims, strides, box) != 0) return cudaErrorInvalidValue;
  auto kernel = jacobi3d_tb_kernel<F, SLAB>;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e;
  if (configured_dev != dev) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)T::SMEM);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kTbThreads, T::SMEM);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  long long g = (long long)per_sm * num_sms(dev);
  if (g > kMaxCtas) g = kMaxCtas;

  J3Tb k{};
  k.u = p.u;
  k.v = p.v;
  k.sy = p.sy;
  k.sz = p.sz;
  k.d = (int)p.d;
  k.h = (int)p.h;
  k.w = (int)p.w;
  k.z_lo = (int)p.z_lo;
  k.z_hi = (int)(p.z_hi < 0 ? p.d : p.z_hi);
  k.g_z0 = p.g_z0;
  k.g_d = p.g_d < 0 ? p.d : p.g_d;
  k.tiles_x = (int)((p.w + kTbOwnW - 1) / kTbOwnW);
  k.tiles_y = (int)((p.h + T::TH - 1) / T::TH);
  const long long txy = (long long)k.tiles_x * k.tiles_y;
  tb_chunks(k.z_hi - k.z_lo, txy, g, F, k.bz, k.zchunks);
  k.passes = (int)passes;
  k.sweep_base = (int)sweep_base;
  k.res_every = (int)p.res_every;
  k.res_out = p.res_out;
  k.ws = p.ws;
  k.budget_ns = wait_budget_ns(false);
  k.peer_budget_ns = wait_budget_ns(true);
  k.peers = peers;
  k.halo = p.halo;
  k.init_halo = init_halo;
  k.flag_base = flag_base;
  const long long items = txy * k.zchunks;
  if (g > items) g = items;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)g);
  cfg.blockDim = dim3(kTbThreads);
  cfg.dynamicSmemBytes = T::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, mu, mv, k);
}

template <int F>
cudaError_t launch_tb_any(const Jacobi3dProblem &p, const SlabPeers &peers, int64_t passes, int64_t sweep_base,
                          unsigned flag_base, int init_halo, cudaStream_t s) {
  const bool slab = peers.up_u != nullptr || peers.dn_u != nullptr;  // a neighbour exists
  return slab ? launch_tb<F, true>(p, peers, passes, sweep_base, flag_base, init_halo, s)
              : launch_tb<F, false>(p, peers, passes, sweep_base, flag_base, init_halo, s);
}

}  // namespace

void jacobi3d_pass_plan(int64_t sweeps, int64_t res_every, int64_t plan[3]) {
  int fmax = kTbMaxF;
  while (res_every > 0 && fmax > res_every) fmax >>= 1;  // at most one residual sweep per pass
  int64_t left = sweeps;
  for (int d = 0, f = 4; d < 3; ++d, f >>= 1) {
    // even counts of the multi-sweep passes keep the ping-pong parity of the
    // single sweeps left over
    plan[d] = f > fmax ? 0 : f == 1 ? left : (left / (2 * f)) * 2;
    left -= plan[d] * f;
  }
}

int64_t jacobi3d_slab_deliveries(int64_t sweeps, int64_t res_every, int64_t h, int64_t w) {
  int64_t plan[3];
  jacobi3d_pass_plan(sweeps, res_every, plan);
  int64_t total = 0;
  bool first = true;
  for (int d = 0, f = 4; d < 3; ++d, f >>= 1) {
    if (plan[d] == 0) continue;
    const int64_t tiles = f == 4 ? tb_tiles<4>(h, w) : f == 2 ? tb_tiles<2>(h, w) : tb_tiles<1>(h, w);
    total += (plan[d] + (first ? 1 : 0)) * tiles;
    first = false;
  }
  return total;
}

cudaError_t run_jacobi3d_tb(const Jacobi3dProblem &p, const SlabPeers &peers, unsigned flag_base, cudaStream_t s) {
  int64_t plan[3];
  jacobi3d_pass_plan(p.sweeps, p.res_every, plan);
  int64_t done = 0;
  unsigned flags = flag_base;
  bool first = true;
  cudaError_t e = cudaSuccess;
  for (int d = 0, f = 4; d < 3; ++d, f >>= 1) {
    const int64_t n = plan[d];
    if (n == 0) continue;
    e = cudaMemsetAsync(&p.ws->barrier, 0, sizeof(unsigned), s);  // fresh grid barrier, same status word
    if (e != cudaSuccess) return e;
    // a slab run delivers its input's edge planes before its first pass
    const int init = (p.halo > 0 && first) ? 1 : 0;
    int64_t tiles = 0;
    switch (f) {
      case 4: e = launch_tb_any<4>(p, peers, n, done, flags, init, s); tiles = tb_tiles<4>(p.h, p.w); break;
      case 2: e = launch_tb_any<2>(p, peers, n, done, flags, init, s); tiles = tb_tiles<2>(p.h, p.w); break;
      default: e = launch_tb_any<1>(p, peers, n, done, flags, init, s); tiles = tb_tiles<1>(p.h, p.w); break;
    }
    if (e != cudaSuccess) return e;
    flags += (unsigned)((n + init) * tiles);
    done += n * f;
    first = false;
  }
  return e;
}

}  // namespace spmdb200
