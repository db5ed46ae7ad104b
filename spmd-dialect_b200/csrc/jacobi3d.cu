// jacobi3d.cu -- Jacobi-3D 7-point sweeps.
//
// Persistent path (x contiguous, 16-byte aligned rows and planes)
// --------------------------------------------------------------
// 2.5-D blocking.  A work item is a BH x BW tile of (y, x) over a chunk of BZ
// consecutive z-planes.  The producer warp streams the item's BZ + 2 planes
// (z0 - 1 .. z0 + BZ) -- each a (BH + 2) x (BW + 8) footprint box taken from a
// 3-D tensor map with cp.async.bulk.tensor.3d -- through a ring of STAGES
// plane buffers (mbarrier expect_tx).  Consumer warp w owns tile rows
// w*RPW .. w*RPW + RPW-1, lane l four contiguous columns; each thread keeps the
// centre and z-1 values of its cells in registers and slides up the z-chunk,
// so computing a plane needs only its z+1 row and the two y-halo rows from
// shared memory (plus shuffles for x +- 1).  A plane buffer is released as soon
// as the plane above it has been computed.  Sweeps are separated by the same
// split grid barrier as the 2-D kernel (consumers arrive, the producer waits),
// every wait is bounded, and out-of-grid box cells are zero-filled by TMA.
//
// z-slabs across GPUs (SlabPeers, halo = 1 plane): a rank updates local planes
// [z_lo, z_hi) and mirrors one plane of each neighbour.  The work items that
// compute the first (last) owned plane also store it into the neighbour's halo
// plane over NVLink, and each consumer warp then bumps the neighbour's
// delivery counter with a release at system scope; the producer acquires that
// counter before it stages a halo plane.  Those edge items come first in
// every sweep.  TMA only ever reads this GPU's own memory.
//
// Generic path: one launch per sweep, one thread per cell (x fastest), any
// strides; residual partials combined by the last block in block order.
#include <cuda.h>

#include "internal.h"

namespace spmdb200 {
namespace {

__device__ __forceinline__ double sq_diff3(float a, float b) {
  const double d = __dsub_rn((double)a, (double)b);
  return __dmul_rn(d, d);
}

__global__ void __launch_bounds__(256) jacobi3d_sweep_generic_kernel(
    const float *__restrict__ u, float *__restrict__ v, long long sz, long long sy, long long sx,
    long long d, long long h, long long w, int want, double *partials, unsigned *ticket, double *res_slot) {
  __shared__ double sh[32];
  __shared__ int last;
  const float k7 = 1.0f / 7.0f;
  const long long nth = (long long)gridDim.x * blockDim.x;
  const long long total = d * h * w;
  double acc = 0.0;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += nth) {
    const long long z = idx / (h * w), rem = idx - z * h * w;
    const long long y = rem / w, x = rem - y * w;
    const long long o0 = z * sz + y * sy + x * sx;
    const float c = u[o0];
    float o = c;
    if (z > 0 && z < d - 1 && y > 0 && y < h - 1 && x > 0 && x < w - 1) {
      float t = __fadd_rn(c, u[o0 - sx]);
      t = __fadd_rn(t, u[o0 + sx]);
      t = __fadd_rn(t, u[o0 - sy]);
      t = __fadd_rn(t, u[o0 + sy]);
      t = __fadd_rn(t, u[o0 - sz]);
      t = __fadd_rn(t, u[o0 + sz]);
      o = __fmul_rn(t, k7);
      if (want) acc = __dadd_rn(acc, sq_diff3(o, c));
    }
    v[o0] = o;
  }
  if (!want) return;
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

// Seeded synthetic 3-D input: cell (gz, y, x) of the global g_d x h x w grid
// is uniform [0, 1) from the counter hash of (seed, gz * h + y, x); global
// boundary cells and planes outside [0, g_d) are 0.
__global__ void __launch_bounds__(256) fill_jacobi3d_input_kernel(float *p, long long sz, long long sy,
                                                                  long long planes, long long h, long long w,
                                                                  long long g_z0, long long g_d, uint64_t seed) {
  const long long nth = (long long)gridDim.x * blockDim.x;
  const long long total = planes * h * w;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += nth) {
    const long long z = idx / (h * w), rem = idx - z * h * w;
    const long long y = rem / w, x = rem - y * w;
    const long long gz = g_z0 + z;
    const bool interior = gz > 0 && gz < g_d - 1 && y > 0 && y < h - 1 && x > 0 && x < w - 1;
    p[z * sz + y * sy + x] = interior ? hash_uniform(seed, (uint64_t)(gz * h + y), (uint64_t)x) : 0.0f;
  }
}

}  // namespace

cudaError_t launch_fill_jacobi3d_input(float *p, int64_t sz, int64_t sy, int64_t planes, int64_t h, int64_t w,
                                       int64_t g_z0, int64_t g_d, uint64_t seed, cudaStream_t s) {
  if (planes <= 0 || h <= 0 || w <= 0) return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  long long g = (planes * h * w + 255) / 256;
  const long long cap = (long long)num_sms(dev) * 8;
  if (g > cap) g = cap;
  fill_jacobi3d_input_kernel<<<(unsigned)g, 256, 0, s>>>(p, sz, sy, planes, h, w, g_z0, g_d, seed);
  return cudaGetLastError();
}

cudaError_t launch_jacobi3d_generic(const Jacobi3dProblem &p, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  const long long cells = p.d * p.h * p.w;
  long long g = (cells + 255) / 256;
  const long long cap = (long long)num_sms(dev) * 8;
  if (g > cap) g = cap;
  if (g > kMaxCtas) g = kMaxCtas;
  if (g < 1) g = 1;
  float *a = p.u, *b = p.v;
  for (long long sw = 1; sw <= p.sweeps; ++sw) {
    const int want = p.res_every > 0 && sw % p.res_every == 0;
    double *slot = want ? p.res_out + (sw / p.res_every - 1) : nullptr;
    jacobi3d_sweep_generic_kernel<<<(unsigned)g, 256, 0, s>>>(a, b, p.sz, p.sy, p.sx, p.d, p.h, p.w, want,
                                                               p.ws->partial[0], &p.ws->ticket, slot);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    float *t = a;
    a = b;
    b = t;
  }
  return cudaSuccess;
}


namespace {

#ifndef SPMDB200_J3_BH
#define SPMDB200_J3_BH 16
#endif
#ifndef SPMDB200_J3_BZ
#define SPMDB200_J3_BZ 16
#endif
#ifndef SPMDB200_J3_STAGES
#define SPMDB200_J3_STAGES 8
#endif
constexpr int BW3 = 128;
constexpr int BH3 = SPMDB200_J3_BH;          // tile rows (multiple of 8)
constexpr int BZ3 = SPMDB200_J3_BZ;          // planes per work item
constexpr int XP3 = 4;                        // left pad (keeps TMA x 16-byte aligned)
constexpr int BOXW3 = BW3 + 2 * XP3;          // 136
constexpr int BOXH3 = BH3 + 2;
constexpr int ST3 = SPMDB200_J3_STAGES;       // plane buffers (>= 4: three held + one in flight)
constexpr int PLANE_BYTES = BOXW3 * BOXH3 * 4;
constexpr int PLANE_STRIDE = (PLANE_BYTES + 127) / 128 * 128;
constexpr int CW3 = 8;                        // consumer warps
constexpr int RPW3 = BH3 / CW3;
constexpr int THREADS3 = 32 * (CW3 + 1);
constexpr int CONSUMERS3 = 32 * CW3;
static_assert(ST3 >= 4, "the consumer holds three planes at a time");
static_assert(BH3 % CW3 == 0, "tile rows must split evenly over the consumer warps");

struct Smem3Tail {
  uint64_t full[ST3];
  uint64_t empty[ST3];
  double wsum[2][CW3];
  int abort;
};
constexpr size_t SMEM3_BYTES = (size_t)ST3 * PLANE_STRIDE + sizeof(Smem3Tail) + 128;

struct J3Kernel {
  float *u, *v;
  long long sy, sz;  // strides in elements (x contiguous)
  int d, h, w;       // local planes, rows, columns
  int z_lo, z_hi;    // local planes updated by a sweep
  long long g_z0, g_d;  // global plane of local plane 0, global plane count
  int tiles_x, tiles_y, zchunks;
  int sweeps, res_every;
  double *res_out;
  JacobiWs *ws;
  unsigned long long budget_ns, peer_budget_ns;
  SlabPeers peers;
  int halo;            // 1 in z-slab mode, 0 on one GPU
  unsigned flag_base;  // halo-plane deliveries already received from each neighbour
};

// Work item t -> (zc, tx, ty).  One GPU: z-chunk fastest.  z-slab mode: the
// first and last z-chunks (the items a neighbour waits for) come first.
__device__ __forceinline__ void item_coords3(const J3Kernel &k, int t, int &zc, int &tx, int &ty) {
  const int txy = k.tiles_x * k.tiles_y;
  int rest;
  if (k.halo > 0 && k.zchunks > 2) {
    if (t < 2 * txy) {
      zc = t < txy ? 0 : k.zchunks - 1;
      rest = t < txy ? t : t - txy;
    } else {
      const int u = t - 2 * txy;
      zc = 1 + u % (k.zchunks - 2);
      rest = u / (k.zchunks - 2);
    }
  } else {
    zc = t % k.zchunks;
    rest = t / k.zchunks;
  }
  tx = rest % k.tiles_x;
  ty = rest / k.tiles_x;
}

// Residual r: the CTA partials in CTA order (producer warp of CTA 0); in
// z-slab mode also all-gathered into every rank's slot array.
__device__ __forceinline__ void combine3(const J3Kernel &k, int r, int lane) {
  double p = 0.0;
  for (int i = lane; i < (int)gridDim.x; i += 32) p = __dadd_rn(p, __ldcg(&k.ws->partial[r & 1][i]));
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

__device__ __forceinline__ void record3(JacobiWs *ws, volatile int *abort, int code) {
  atomicCAS(&ws->status, 0, code);
  *abort = 1;
}

__device__ __forceinline__ bool wait_counter3(const unsigned *p, unsigned target, volatile int *abort,
                                              unsigned long long budget, const JacobiWs *ws, bool sys = false) {
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if ((int)((sys ? ld_acquire_sys(p) : ld_acquire_gpu(p)) - target) >= 0) return true;
    if (*abort) return false;
    if ((i & 7u) == 7u && *reinterpret_cast<const volatile int *>(&ws->status) != 0) return false;
    if (globaltimer_ns() - t0 > budget) return false;
    __nanosleep(64);
  }
}

__device__ __forceinline__ bool consumers3_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(CONSUMERS3)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float4 ld4s(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// Stores the 4 cells at columns gx0..gx0+3 of a row, masked to the grid width.
__device__ __forceinline__ void store4_w(float *p, int gx0, int w, float4 o) {
  if (gx0 + 3 < w) {
    st_f4(p, o);
  } else {
    if (gx0 < w) p[0] = o.x;
    if (gx0 + 1 < w) p[1] = o.y;
    if (gx0 + 2 < w) p[2] = o.z;
  }
}

__device__ __forceinline__ float j7(float c, float xm, float xp, float ym, float yp, float zm, float zp) {
  float t = __fadd_rn(c, xm);
  t = __fadd_rn(t, xp);
  t = __fadd_rn(t, ym);
  t = __fadd_rn(t, yp);
  t = __fadd_rn(t, zm);
  t = __fadd_rn(t, zp);
  return __fmul_rn(t, 1.0f / 7.0f);
}

// SLAB: z-slab mode (peer waits, halo deliveries); the one-GPU instantiation
// carries none of that code.
template <bool SLAB>
__global__ void __launch_bounds__(THREADS3) jacobi3d_persistent_kernel(
    const __grid_constant__ CUtensorMap map_u, const __grid_constant__ CUtensorMap map_v,
    const __grid_constant__ J3Kernel k) {
  extern __shared__ __align__(128) unsigned char smem3_raw[];
  // Aligned by pointer arithmetic on the shared array, so shared-space
  // addressing (LDS) survives for everything derived from it.
  unsigned char *smem = smem3_raw + ((128u - (smem_u32(smem3_raw) & 127u)) & 127u);
  Smem3Tail *tail = reinterpret_cast<Smem3Tail *>(smem + (size_t)ST3 * PLANE_STRIDE);
  volatile int *abort = &tail->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int T = k.tiles_x * k.tiles_y * k.zchunks;
  const unsigned per_sweep = (unsigned)(k.tiles_x * k.tiles_y * CW3);  // deliveries per neighbour per sweep

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST3; ++i) {
      mbar_init(&tail->full[i], 1);
      mbar_init(&tail->empty[i], CW3);
    }
    tail->abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == CW3) {
    // ------------------------------------------------------------ producer warp
    if (lane == 0) {
      tma_prefetch_desc(&map_u);
      tma_prefetch_desc(&map_v);
    }
    uint32_t pc = 0;  // planes issued
    bool ok = true;
    for (int s = 0; s < k.sweeps && ok; ++s) {
      const void *src = (s & 1) ? (const void *)&map_v : (const void *)&map_u;
      if (s > 0) {
        if (lane == 0 &&
            !wait_counter3(&k.ws->barrier, (unsigned)s * (unsigned)G, abort, k.budget_ns, k.ws)) {
          record3(k.ws, abort, kDevTimeoutGridBarrier);
          ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (blockIdx.x == 0 && k.res_every > 0 && s % k.res_every == 0) combine3(k, s / k.res_every - 1, lane);
      }
      if (lane == 0) {
        for (int t = blockIdx.x; t < T && ok; t += G) {
          int zc, tx, ty;
          item_coords3(k, t, zc, tx, ty);
          const int z0 = k.z_lo + zc * BZ3;
          if constexpr (SLAB) {
            // a halo plane is staged only once the neighbour delivered it for
            // every earlier sweep; the proxy fence orders that acquire before
            // the TMA (async-proxy) read of the peer-written plane
            const unsigned need = k.flag_base + (unsigned)s * per_sweep;
            const bool wait_up = k.peers.up_flag && z0 - 1 < k.z_lo;
            const bool wait_dn = k.peers.dn_flag && z0 + BZ3 >= k.z_hi;
            if (wait_up && !wait_counter3(&k.ws->from_above, need, abort, k.peer_budget_ns, k.ws, true)) {
              record3(k.ws, abort, kDevTimeoutPeer);
              ok = false;
              break;
            }
            if (wait_dn && !wait_counter3(&k.ws->from_below, need, abort, k.peer_budget_ns, k.ws, true)) {
              record3(k.ws, abort, kDevTimeoutPeer);
              ok = false;
              break;
            }
            if (wait_up || wait_dn) fence_proxy_async_global();
          }
          for (int l = 0; l < BZ3 + 2; ++l) {
            const uint32_t st = pc % ST3, ph = (pc / ST3) & 1u;
            if (!mbar_wait_bounded(&tail->empty[st], ph ^ 1u, abort)) {
              record3(k.ws, abort, kDevTimeoutEmpty);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&tail->full[st], PLANE_BYTES);
            tma_load_3d(smem + (size_t)st * PLANE_STRIDE, src, &tail->full[st], tx * BW3 - XP3, ty * BH3 - 1,
                        z0 - 1 + l);
            ++pc;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      pc = __shfl_sync(0xffffffffu, pc, 0);
    }
    if (ok && blockIdx.x == 0 && k.sweeps > 0 && k.res_every > 0 && k.sweeps % k.res_every == 0) {
      if (lane == 0 &&
          !wait_counter3(&k.ws->barrier, (unsigned)k.sweeps * (unsigned)G, abort, k.budget_ns, k.ws)) {
        record3(k.ws, abort, kDevTimeoutGridBarrier);
        ok = false;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok) combine3(k, k.sweeps / k.res_every - 1, lane);
    }
    if (!ok && lane == 0) {
      const uint32_t n = pc < (uint32_t)ST3 ? pc : (uint32_t)ST3;
      for (uint32_t j = 0; j < n; ++j) {
        const uint32_t i = pc - 1 - j;
        int no_abort = 0;
        mbar_wait_bounded(&tail->full[i % ST3], (i / ST3) & 1u, &no_abort);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumer warps
  const int cw = warp;
  const int r0 = cw * RPW3;        // this warp's first tile row
  const int sc = XP3 + 4 * lane;   // this lane's first box column
  uint32_t pc = 0;                 // planes consumed (ring position)
  double acc = 0.0;
  for (int s = 0; s < k.sweeps; ++s) {
    float *dst = (s & 1) ? k.u : k.v;
    const bool has_up = SLAB && k.peers.up_u != nullptr, has_dn = SLAB && k.peers.dn_u != nullptr;
    const bool want = k.res_every > 0 && ((s + 1) % k.res_every == 0);
    bool ok = true;
    for (int t = blockIdx.x; t < T && ok; t += G) {
      int zc, tx, ty;
      item_coords3(k, t, zc, tx, ty);
      const int z0 = k.z_lo + zc * BZ3;
      const int gx0 = tx * BW3 + 4 * lane;
      const int y0 = ty * BH3 + r0;
      // planes 0 (z0-1) and 1 (z0) of this item
      bool got = mbar_wait_warp(&tail->full[pc % ST3], (pc / ST3) & 1u, abort) &&
                 mbar_wait_warp(&tail->full[(pc + 1) % ST3], ((pc + 1) / ST3) & 1u, abort);
      if (!got) {
        if (lane == 0) record3(k.ws, abort, kDevTimeoutFull);
        ok = false;
        break;
      }
      float4 zm[RPW3], c[RPW3];
      {
        const float *P0 = reinterpret_cast<const float *>(smem + (size_t)(pc % ST3) * PLANE_STRIDE);
        const float *P1 = reinterpret_cast<const float *>(smem + (size_t)((pc + 1) % ST3) * PLANE_STRIDE);
#pragma unroll
        for (int q = 0; q < RPW3; ++q) {
          zm[q] = ld4s(P0 + (r0 + q + 1) * BOXW3 + sc);
          c[q] = ld4s(P1 + (r0 + q + 1) * BOXW3 + sc);
        }
      }
      for (int j = 1; j <= BZ3; ++j) {
        const uint32_t pz = pc + j, pp = pc + j + 1;  // ring positions of planes z and z+1
        got = mbar_wait_warp(&tail->full[pp % ST3], (pp / ST3) & 1u, abort);
        if (!got) {
          if (lane == 0) record3(k.ws, abort, kDevTimeoutFull);
          ok = false;
          break;
        }
        const int z = z0 + j - 1;
        const float *Pz = reinterpret_cast<const float *>(smem + (size_t)(pz % ST3) * PLANE_STRIDE);
        const float *Pp = reinterpret_cast<const float *>(smem + (size_t)(pp % ST3) * PLANE_STRIDE);
        const float4 top = ld4s(Pz + r0 * BOXW3 + sc);
        const float4 bot = ld4s(Pz + (r0 + RPW3 + 1) * BOXW3 + sc);
        float4 zp[RPW3];
#pragma unroll
        for (int q = 0; q < RPW3; ++q) zp[q] = ld4s(Pp + (r0 + q + 1) * BOXW3 + sc);
        if (z < k.z_hi) {
          const long long gz = k.g_z0 + z;
          const bool zb = (gz == 0 || gz == k.g_d - 1);
#pragma unroll
          for (int q = 0; q < RPW3; ++q) {
            const int y = y0 + q;
            const float *crow = Pz + (r0 + q + 1) * BOXW3;
            const float4 cc = c[q];
            const float4 n = q == 0 ? top : c[q - 1];
            const float4 so = q == RPW3 - 1 ? bot : c[q + 1];
            float west = __shfl_up_sync(0xffffffffu, cc.w, 1);
            float east = __shfl_down_sync(0xffffffffu, cc.x, 1);
            if (lane == 0) west = crow[XP3 - 1];
            if (lane == 31) east = crow[XP3 + BW3];
            if (y < k.h) {
              float4 o;
              o.x = j7(cc.x, west, cc.y, n.x, so.x, zm[q].x, zp[q].x);
              o.y = j7(cc.y, cc.x, cc.z, n.y, so.y, zm[q].y, zp[q].y);
              o.z = j7(cc.z, cc.y, cc.w, n.z, so.z, zm[q].z, zp[q].z);
              o.w = j7(cc.w, cc.z, east, n.w, so.w, zm[q].w, zp[q].w);
              if (zb || y == 0 || y == k.h - 1) {
                o = cc;
              } else {
                const int wl = k.w - 1;
                if (gx0 == 0) o.x = cc.x;
                if (gx0 == wl) o.x = cc.x;
                if (gx0 + 1 == wl) o.y = cc.y;
                if (gx0 + 2 == wl) o.z = cc.z;
                if (gx0 + 3 == wl) o.w = cc.w;
              }
              store4_w(dst + (long long)z * k.sz + (long long)y * k.sy + gx0, gx0, k.w, o);
              if (want) {
                if (gx0 < k.w) acc = __dadd_rn(acc, __dmul_rn(__dsub_rn((double)o.x, (double)cc.x), __dsub_rn((double)o.x, (double)cc.x)));
                if (gx0 + 1 < k.w) acc = __dadd_rn(acc, __dmul_rn(__dsub_rn((double)o.y, (double)cc.y), __dsub_rn((double)o.y, (double)cc.y)));
                if (gx0 + 2 < k.w) acc = __dadd_rn(acc, __dmul_rn(__dsub_rn((double)o.z, (double)cc.z), __dsub_rn((double)o.z, (double)cc.z)));
                if (gx0 + 3 < k.w) acc = __dadd_rn(acc, __dmul_rn(__dsub_rn((double)o.w, (double)cc.w), __dsub_rn((double)o.w, (double)cc.w)));
              }
            }
          }
        }
#pragma unroll
        for (int q = 0; q < RPW3; ++q) {
          zm[q] = c[q];
          c[q] = zp[q];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tail->empty[(pz - 1) % ST3]);  // plane z-1 is no longer needed
      }
      if (!ok) break;
      if constexpr (SLAB) {
        // An edge item of the slab: copy this warp's rows of the first / last
        // owned plane (its own stores, L2-resident) into the neighbour's halo
        // plane, then count the delivery.  Done once per item, outside the
        // plane loop, which keeps that loop the one-GPU loop.
        const bool up_item = has_up && zc == 0, dn_item = has_dn && zc == k.zchunks - 1;
        if (up_item || dn_item) {
          float *up_dst = (s & 1) ? k.peers.up_u : k.peers.up_v;
          float *dn_dst = (s & 1) ? k.peers.dn_u : k.peers.dn_v;
#pragma unroll 1
          for (int e = 0; e < 2; ++e) {
            if (e == 0 ? !up_item : !dn_item) continue;
            const int z = e == 0 ? k.z_lo : k.z_hi - 1;
            float *to = e == 0 ? up_dst + k.peers.up_row * k.sz : dn_dst + k.peers.dn_row * k.sz;
#pragma unroll 1
            for (int q = 0; q < RPW3; ++q) {
              const int y = y0 + q;
              if (y >= k.h || gx0 >= k.w) continue;
              const long long yo = (long long)y * k.sy + gx0;
              const float *mine = dst + (long long)z * k.sz + yo;
              float4 o;
              o.x = mine[0];
              o.y = gx0 + 1 < k.w ? mine[1] : 0.0f;
              o.z = gx0 + 2 < k.w ? mine[2] : 0.0f;
              o.w = gx0 + 3 < k.w ? mine[3] : 0.0f;
              store4_w(to + yo, gx0, k.w, o);
            }
          }
          __syncwarp();
          if (lane == 0) {
            __threadfence_system();
            if (up_item) red_release_sys_add(k.peers.up_flag, 1u);
            if (dn_item) red_release_sys_add(k.peers.dn_flag, 1u);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {  // the item's last two planes
        mbar_arrive(&tail->empty[(pc + BZ3) % ST3]);
        mbar_arrive(&tail->empty[(pc + BZ3 + 1) % ST3]);
      }
      pc += BZ3 + 2;
    }
    if (want) {
      const double wv = warp_sum_f64(acc);
      if (lane == 0) tail->wsum[s & 1][cw] = wv;
      acc = 0.0;
    }
    fence_proxy_async_global();  // this sweep's stores before the next sweep's TMA reads
    __syncwarp();
    const bool fail = consumers3_any(!ok || *abort);
    if (fail) break;
    if (threadIdx.x == 0) {
      if (want) {
        double tot = 0.0;
        for (int i = 0; i < CW3; ++i) tot = __dadd_rn(tot, tail->wsum[s & 1][i]);
        k.ws->partial[((s + 1) / k.res_every - 1) & 1][blockIdx.x] = tot;
      }
      __threadfence();
      red_release_gpu_add(&k.ws->barrier, 1u);
    }
  }
}

}  // namespace

bool jacobi3d_tma_ok(const Jacobi3dProblem &p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p.u), b = reinterpret_cast<uintptr_t>(p.v);
  return p.sx == 1 && ((a | b) & 15u) == 0 && (p.sy * 4) % 16 == 0 && (p.sz * 4) % 16 == 0 && p.w >= 1 &&
         p.h >= 1 && p.d >= 1 && p.sy >= p.w && p.sz >= p.sy * p.h && p.w < (1ll << 30) && p.h < (1ll << 30) &&
         p.d < (1ll << 30) && p.sz < (1ll << 37) && p.sweeps <= (1ll << 30);
}

int64_t jacobi3d_slab_deliveries(int64_t sweeps, int64_t h, int64_t w) {
  return sweeps * ((w + BW3 - 1) / BW3) * ((h + BH3 - 1) / BH3) * CW3;
}

cudaError_t launch_jacobi3d_persistent(const Jacobi3dProblem &p, const SlabPeers &peers, cudaStream_t s,
                                       int *grid_out, unsigned flag_base) {
  CUtensorMap mu, mv;
  const uint64_t dims[3] = {(uint64_t)p.w, (uint64_t)p.h, (uint64_t)p.d};
  const uint64_t strides[2] = {(uint64_t)p.sy * 4u, (uint64_t)p.sz * 4u};
  const uint32_t box[3] = {(uint32_t)BOXW3, (uint32_t)BOXH3, 1u};
  if (encode_tensor_map_f32(&mu, p.u, 3, dims, strides, box) != 0) return cudaErrorInvalidValue;
  if (encode_tensor_map_f32(&mv, p.v, 3, dims, strides, box) != 0) return cudaErrorInvalidValue;
  J3Kernel k{};
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
  k.halo = p.halo;
  k.peers = peers;
  k.tiles_x = (int)((p.w + BW3 - 1) / BW3);
  k.tiles_y = (int)((p.h + BH3 - 1) / BH3);
  k.zchunks = (k.z_hi - k.z_lo + BZ3 - 1) / BZ3;
  k.sweeps = (int)p.sweeps;
  k.res_every = (int)p.res_every;
  k.res_out = p.res_out;
  k.ws = p.ws;
  k.budget_ns = wait_budget_ns(false);
  k.peer_budget_ns = wait_budget_ns(true);
  k.flag_base = flag_base;

  const bool slab = peers.up_u != nullptr || peers.dn_u != nullptr;  // a neighbour exists
  auto kernel = slab ? jacobi3d_persistent_kernel<true> : jacobi3d_persistent_kernel<false>;
  static thread_local int configured_dev[2] = {-1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e;
  if (configured_dev[slab] != dev) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM3_BYTES);
    if (e != cudaSuccess) return e;
    configured_dev[slab] = dev;
  }
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, THREADS3, SMEM3_BYTES);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  long long g = (long long)per_sm * num_sms(dev);
  const long long items = (long long)k.tiles_x * k.tiles_y * k.zchunks;
  if (g > items) g = items;
  if (g > kMaxCtas) g = kMaxCtas;
  if (grid_out) *grid_out = (int)g;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)g);
  cfg.blockDim = dim3(THREADS3);
  cfg.dynamicSmemBytes = SMEM3_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, mu, mv, k);
}

}  // namespace spmdb200
