// jacobi2d.cu -- Jacobi-2D 5-point sweeps: the PromoteGroupMemory-tiled
// stencil (lib/Transforms/PromoteGroupMemory.cpp:113-314: tile + halo copied
// to group memory, barrier, compute from the tile) rebuilt for B200.
//
// Persistent path (pitch-aligned grids)
// -------------------------------------
// One cooperative launch runs every sweep.  Each CTA = 1 producer warp + 8
// consumer warps, two CTAs per SM.  Tiles are 64 rows x 128 columns of
// output; the producer stages each tile's footprint -- a 66 x 136 box starting
// one row above and four columns left of the tile, so the TMA x coordinate
// stays 16-byte aligned -- into a 3-deep shared-memory ring (3 x 36 KB) with
// cp.async.bulk.tensor.2d, completion tracked by mbarrier expect_tx.  (Tile
// height and ring depth were chosen by measurement on B200: 1 CTA per SM or a
// 2-deep ring leaves HBM idle; 64 x 3 beat 16/32/40/48/96/128-row tiles.)  Out-of-grid box cells are zero-filled by the
// TMA unit (the guard of PromoteGroupMemory.cpp:268-292, done in hardware).
// Consumer warp w computes tile rows 8w..8w+7; lane l owns 4 contiguous
// columns, reads north/centre/south as float4 from the ring (sliding down the
// rows), gets west/east from neighbouring lanes by shuffle and stores float4.
//
// Sweeps are separated by a split grid barrier: consumers of a CTA arrive
// (one red.release.gpu per CTA) after their last store of sweep s; only the
// producer waits for all arrivals before issuing sweep s+1's loads, so
// compute never stalls on the barrier itself.  Every wait is bounded
// (%globaltimer budget); on expiry the CTA records a status word, drains its
// in-flight TMA loads and exits.
//
// Row slabs across GPUs (SlabPeers): the consumer that writes the first
// (last) owned row also stores it into the halo row of the neighbour above
// (below) over NVLink, then bumps that neighbour's delivery counter with a
// release at system scope.  The neighbour's producer acquires the counter
// before it stages any tile whose footprint includes that halo row.  TMA only
// ever reads this GPU's own memory.
#include <cuda.h>

#include "internal.h"

namespace spmdb200 {
namespace {

#ifndef SPMDB200_J2_BH
#define SPMDB200_J2_BH 64
#endif
#ifndef SPMDB200_J2_STAGES
#define SPMDB200_J2_STAGES 3
#endif
constexpr int BW = 128;                   // tile columns
constexpr int BH = SPMDB200_J2_BH;        // tile rows (multiple of 8)
constexpr int XPAD = 4;                   // left pad of the footprint box (16 bytes)
constexpr int BOXW = BW + 2 * XPAD;       // 136 floats = 544 bytes per box row
constexpr int BOXH = BH + 2;              // footprint rows
constexpr int STAGES = SPMDB200_J2_STAGES;
constexpr int STAGE_BYTES = BOXW * BOXH * 4;
constexpr int STAGE_STRIDE = (STAGE_BYTES + 127) / 128 * 128;
constexpr int CWARPS = 8;
constexpr int RPW = BH / CWARPS;          // rows per consumer warp
constexpr int THREADS = 32 * (CWARPS + 1);
constexpr int CONSUMERS = 32 * CWARPS;

struct SmemTail {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  double wsum[2][CWARPS];
  int abort;
};
constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_STRIDE + sizeof(SmemTail) + 128;

struct J2Kernel {
  float *u, *v;
  long long pitch;
  int w, row_lo, row_hi, tiles_x, tiles_y;
  long long g_row0, g_rows;
  int sweeps, res_every;
  double *res_out;
  JacobiWs *ws;
  SlabPeers peers;
  unsigned long long grid_budget_ns, peer_budget_ns;  // bounded-wait limits
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
// ones a neighbouring GPU waits for) come first in every sweep, so halo rows
// are delivered early and a neighbour's edge tiles never wait for the end of
// this GPU's sweep; the interior rows follow in order.  One GPU: row order.
__device__ __forceinline__ void tile_coords(int t, int tiles_x, int tiles_y, bool edges_first, int &ty, int &tx) {
  int row = t / tiles_x;
  tx = t - row * tiles_x;
  if (edges_first && tiles_y > 2) row = row == 0 ? 0 : row == 1 ? tiles_y - 1 : row - 1;
  ty = row;
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

// Producer-warp residual combine for residual index r: the CTA partials of
// that sweep in CTA order, lane-strided then a shuffle tree (deterministic).
__device__ __forceinline__ void combine_residual(const J2Kernel &k, int r, int lane) {
  double p = 0.0;
  for (int i = lane; i < (int)gridDim.x; i += 32) p = __dadd_rn(p, __ldcg(&k.ws->partial[r & 1][i]));
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

__global__ void __launch_bounds__(THREADS) jacobi2d_persistent_kernel(
    const __grid_constant__ CUtensorMap map_u, const __grid_constant__ CUtensorMap map_v,
    const __grid_constant__ J2Kernel k) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  SmemTail *tail = reinterpret_cast<SmemTail *>(smem + (size_t)STAGES * STAGE_STRIDE);
  volatile int *abort = &tail->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int T = k.tiles_x * k.tiles_y;
  const bool edges_first = k.peers.up_flag != nullptr || k.peers.dn_flag != nullptr;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
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
    for (int s = 0; s < k.sweeps && ok; ++s) {
      const void *src = (s & 1) ? (const void *)&map_v : (const void *)&map_u;
      if (s > 0) {
        if (lane == 0 && !wait_counter(&k.ws->barrier, (unsigned)s * (unsigned)G, false, abort, k.grid_budget_ns, k.ws)) {
          record_status(k.ws, abort, kDevTimeoutGridBarrier);
          ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (blockIdx.x == 0 && k.res_every > 0 && s % k.res_every == 0)
          combine_residual(k, s / k.res_every - 1, lane);
      }
      if (lane == 0) {
        for (int t = blockIdx.x; t < T; t += G) {
          int ty, tx;
          tile_coords(t, k.tiles_x, k.tiles_y, edges_first, ty, tx);
          if (s > 0) {
            const unsigned need = (unsigned)s * (unsigned)k.tiles_x;
            if (ty == 0 && k.peers.up_flag &&
                !wait_counter(&k.ws->from_above, need, true, abort, k.peer_budget_ns, k.ws)) {
              record_status(k.ws, abort, kDevTimeoutPeer);
              ok = false;
              break;
            }
            if (ty == k.tiles_y - 1 && k.peers.dn_flag &&
                !wait_counter(&k.ws->from_below, need, true, abort, k.peer_budget_ns, k.ws)) {
              record_status(k.ws, abort, kDevTimeoutPeer);
              ok = false;
              break;
            }
          }
          fence_proxy_async_global();
          const uint32_t st = it % STAGES, ph = (it / STAGES) & 1u;
          if (!mbar_wait_bounded(&tail->empty[st], ph ^ 1u, abort)) {
            record_status(k.ws, abort, kDevTimeoutEmpty);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&tail->full[st], STAGE_BYTES);
          tma_load_2d(smem + (size_t)st * STAGE_STRIDE, src, &tail->full[st], tx * BW - XPAD,
                      k.row_lo + ty * BH - 1);
          ++it;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      it = __shfl_sync(0xffffffffu, it, 0);
    }
    if (ok && blockIdx.x == 0 && k.sweeps > 0 && k.res_every > 0 && k.sweeps % k.res_every == 0) {
      if (lane == 0 &&
          !wait_counter(&k.ws->barrier, (unsigned)k.sweeps * (unsigned)G, false, abort, k.grid_budget_ns, k.ws)) {
        record_status(k.ws, abort, kDevTimeoutGridBarrier);
        ok = false;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok) combine_residual(k, k.sweeps / k.res_every - 1, lane);
    }
    if (!ok && lane == 0) {
      // Drain: the most recent load issued into each stage must land before
      // this CTA's shared memory can be released.
      const uint32_t n = it < (uint32_t)STAGES ? it : (uint32_t)STAGES;
      for (uint32_t j = 0; j < n; ++j) {
        const uint32_t i = it - 1 - j;
        int no_abort = 0;
        mbar_wait_bounded(&tail->full[i % STAGES], (i / STAGES) & 1u, &no_abort);
      }
    }
    return;
  }

  // ------------------------------ consumer warps ------------------------------
  const int cw = warp;
  uint32_t it = 0;
  double acc = 0.0;
  for (int s = 0; s < k.sweeps; ++s) {
    float *dst = (s & 1) ? k.u : k.v;
    float *up_dst = (s & 1) ? k.peers.up_u : k.peers.up_v;
    float *dn_dst = (s & 1) ? k.peers.dn_u : k.peers.dn_v;
    const bool want = k.res_every > 0 && ((s + 1) % k.res_every == 0);
    bool ok = true;
    for (int t = blockIdx.x; t < T; t += G) {
      int ty, tx;
      tile_coords(t, k.tiles_x, k.tiles_y, edges_first, ty, tx);
      const uint32_t st = it % STAGES, ph = (it / STAGES) & 1u;
      if (!mbar_wait_warp(&tail->full[st], ph, abort)) {  // warp-uniform outcome
        if (lane == 0) record_status(k.ws, abort, kDevTimeoutFull);
        ok = false;
        break;
      }
      const float *S = reinterpret_cast<const float *>(smem + (size_t)st * STAGE_STRIDE);
      const int gx0 = tx * BW + 4 * lane;
      const int sc = XPAD + 4 * lane;
      const int r0 = cw * RPW;
      const int lr0 = k.row_lo + ty * BH + r0;  // local row of this warp's first row
      float4 n = *reinterpret_cast<const float4 *>(S + r0 * BOXW + sc);
      float4 c = *reinterpret_cast<const float4 *>(S + (r0 + 1) * BOXW + sc);
#pragma unroll
      for (int q = 0; q < RPW; ++q) {
        const float *crow = S + (r0 + q + 1) * BOXW;
        const float4 so = *reinterpret_cast<const float4 *>(crow + BOXW + sc);
        float west = __shfl_up_sync(0xffffffffu, c.w, 1);
        float east = __shfl_down_sync(0xffffffffu, c.x, 1);
        if (lane == 0) west = crow[XPAD - 1];
        if (lane == 31) east = crow[XPAD + BW];
        const int lr = lr0 + q;
        if (lr < k.row_hi) {
          float4 o;
          o.x = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.x, n.x), so.x), c.y), west), 0.2f);
          o.y = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.y, n.y), so.y), c.z), c.x), 0.2f);
          o.z = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.z, n.z), so.z), c.w), c.y), 0.2f);
          o.w = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(c.w, n.w), so.w), east), c.z), 0.2f);
          const long long g = k.g_row0 + lr;
          if (g == 0 || g == k.g_rows - 1) {
            o = c;
          } else {
            if (gx0 == 0) o.x = c.x;
            const int wl = k.w - 1;
            if (gx0 == wl) o.x = c.x;
            if (gx0 + 1 == wl) o.y = c.y;
            if (gx0 + 2 == wl) o.z = c.z;
            if (gx0 + 3 == wl) o.w = c.w;
          }
          store4_masked(dst + (long long)lr * k.pitch + gx0, gx0, k.w, o);
          if (up_dst && lr == k.row_lo) store4_masked(up_dst + k.peers.up_row * k.pitch + gx0, gx0, k.w, o);
          if (dn_dst && lr == k.row_hi - 1)
            store4_masked(dn_dst + k.peers.dn_row * k.pitch + gx0, gx0, k.w, o);
          if (want) {
            if (gx0 < k.w) acc = __dadd_rn(acc, sq_diff(o.x, c.x));
            if (gx0 + 1 < k.w) acc = __dadd_rn(acc, sq_diff(o.y, c.y));
            if (gx0 + 2 < k.w) acc = __dadd_rn(acc, sq_diff(o.z, c.z));
            if (gx0 + 3 < k.w) acc = __dadd_rn(acc, sq_diff(o.w, c.w));
          }
        }
        n = c;
        c = so;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tail->empty[st]);
        // Halo delivery: the warp that owns the first / last owned row publishes
        // it to the neighbouring GPU once its peer stores are issued.
        if (k.peers.up_flag && ty == 0 && cw == 0) {
          __threadfence_system();
          red_release_sys_add(k.peers.up_flag, 1u);
        }
        if (k.peers.dn_flag && ty == k.tiles_y - 1) {
          const int rr = (k.row_hi - 1) - (k.row_lo + ty * BH);
          if (rr / RPW == cw) {
            __threadfence_system();
            red_release_sys_add(k.peers.dn_flag, 1u);
          }
        }
      }
      ++it;
    }
    // ---- end of sweep s: CTA partial, then one grid-barrier arrival ----
    if (want) {
      const double wv = warp_sum_f64(acc);
      if (lane == 0) tail->wsum[s & 1][cw] = wv;
      acc = 0.0;
    }
    fence_proxy_async_global();
    __syncwarp();
    const bool fail = consumers_any(!ok || *abort);
    if (fail) break;
    if (threadIdx.x == 0) {
      if (want) {
        double tot = 0.0;
        for (int i = 0; i < CWARPS; ++i) tot = __dadd_rn(tot, tail->wsum[s & 1][i]);
        k.ws->partial[((s + 1) / k.res_every - 1) & 1][blockIdx.x] = tot;
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
         p.w <= (1ll << 31) - 1 - BW && p.h_local <= (1ll << 31) - 1 - BH && p.pitch < (1ll << 37) &&
         p.row_lo >= 0 && p.row_hi <= p.h_local && p.row_hi > p.row_lo && p.sweeps <= (1ll << 30);
}

cudaError_t launch_jacobi2d_persistent(const Jacobi2dProblem &p, const SlabPeers &peers,
                                       cudaStream_t s, int *grid_out) {
  CUtensorMap mu, mv;
  const uint64_t dims[2] = {(uint64_t)p.w, (uint64_t)p.h_local};
  const uint64_t strides[1] = {(uint64_t)p.pitch * 4u};
  const uint32_t box[2] = {(uint32_t)BOXW, (uint32_t)BOXH};
  if (encode_tensor_map_f32(&mu, p.u, 2, dims, strides, box) != 0) return cudaErrorInvalidValue;
  if (encode_tensor_map_f32(&mv, p.v, 2, dims, strides, box) != 0) return cudaErrorInvalidValue;

  J2Kernel k{};
  k.u = p.u;
  k.v = p.v;
  k.pitch = p.pitch;
  k.w = (int)p.w;
  k.row_lo = (int)p.row_lo;
  k.row_hi = (int)p.row_hi;
  k.tiles_x = (int)((p.w + BW - 1) / BW);
  k.tiles_y = (int)((p.row_hi - p.row_lo + BH - 1) / BH);
  k.g_row0 = p.g_row0;
  k.g_rows = p.g_rows;
  k.sweeps = (int)p.sweeps;
  k.res_every = (int)p.res_every;
  k.res_out = p.res_out;
  k.ws = p.ws;
  k.peers = peers;
  k.grid_budget_ns = wait_budget_ns(false);
  k.peer_budget_ns = wait_budget_ns(true);

  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e;
  if (configured_dev != dev) {
    e = cudaFuncSetAttribute(jacobi2d_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, jacobi2d_persistent_kernel, THREADS, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  long long g = (long long)per_sm * num_sms(dev);
  const long long tiles = (long long)k.tiles_x * k.tiles_y;
  if (g > tiles) g = tiles;
  if (g > kMaxCtas) g = kMaxCtas;
  if (grid_out) *grid_out = (int)g;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)g);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, jacobi2d_persistent_kernel, mu, mv, k);
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
