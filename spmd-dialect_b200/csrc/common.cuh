// common.cuh -- shared device/host helpers for libspmdb200 (sm_100a only).
//
// Memref views: the unpacked MLIR descriptors of include/spmd_b200.h collapse
// into these small structs once validated (element (i,j) = ptr[i*s0 + j*s1],
// offset already applied).  Inline-PTX wrappers for mbarrier, TMA
// (cp.async.bulk.tensor) and acquire/release flags live here so every kernel
// file spells them the same way.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libspmdb200 is written for sm_100a (B200) only"
#endif

namespace spmdb200 {

struct View1 {
  float *p;
  int64_t n, s;
};
struct View2 {
  float *p;
  int64_t n0, n1, s0, s1;
};
struct View3 {
  float *p;
  int64_t n0, n1, n2, s0, s1, s2;
};

// Device status words shared by kernels with bounded waits.
enum DevStatus : int {
  kDevOk = 0,
  kDevTimeoutGridBarrier = 1,
  kDevTimeoutFull = 2,
  kDevTimeoutEmpty = 3,
  kDevTimeoutPeer = 4,
};

// Bounded-wait budgets (nanoseconds of %globaltimer).
constexpr unsigned long long kWaitBudgetNs = 4000000000ull;      // 4 s inside one GPU
constexpr unsigned long long kPeerWaitBudgetNs = 20000000000ull; // 20 s across GPUs

#ifdef __CUDACC__

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// The suspend-time hint (20 us) lets the hardware park a waiting thread until
// the phase completes instead of spinning: measured +0.8 % on the power-capped
// Jacobi-2D headline run (fewer wasted issue slots), neutral elsewhere.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 20000;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for phase `parity` of `bar` to complete, giving up after the budget or
// as soon as *abort becomes non-zero.  Returns true when the phase completed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15u) == 0) {  // poll the abort flag and the clock every 16 tries
      if (*abort) return false;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
    }
  }
}

// Warp-wide bounded wait for phase `parity` of `bar`: every lane polls (a
// lane-0-only poll with a __syncwarp hand-off measured 5-8 % slower on B200:
// the extra wake-up latency lands on every tile), and the outcome is made
// warp-uniform.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort) {
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort));
}

// ---- TMA (bulk tensor copies), no multicast anywhere -----------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, uint64_t *bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
// Orders this thread's generic-proxy view of global memory before its later
// async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- flags --------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned *p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(unsigned *p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Named barrier among `nthreads` threads (warp multiples), id 1..15.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- streaming vector memory ops ---------------------------------------------
__device__ __forceinline__ float4 ld_stream_f4(const float *p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_f4(const float *p) {
  float4 v;
  asm volatile("ld.global.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_f4(float *p, float4 v) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// ---- programmatic dependent launch -----------------------------------------------
// A kernel launched with launch_pdl() may start while the previous kernel of
// its stream is finishing (its launch and prologue overlap that kernel's
// tail); pdl_wait() then blocks until the previous kernel has completed and
// its memory is visible, so nothing may read or write global memory before
// it (an L2 prefetch, which returns no data, may run earlier).
// pdl_trigger() lets the next such launch start early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned *p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- checked builds -----------------------------------------------------------
// Compiled with -DSPMDB200_CHECKED, the general kernels (forall_map.cu,
// stencil_nd.cu) test their global and shared indices against the extent of
// what they address.  An access that fails is skipped, and the first failure
// of each file is kept in a device word of that file (bit 63 set, the site in
// bits 48-62, the low 48 bits of the index), which spmdb200_check_status()
// reads and clears.  Nothing traps.  Release builds compile the checks to
// nothing.
__device__ __forceinline__ bool record_check(unsigned long long *word, bool ok, unsigned site, long long idx) {
  if (!ok)
    atomicCAS(word, 0ull,
              (1ull << 63) | ((unsigned long long)(site & 0x7fffu) << 48) | ((unsigned long long)idx & 0xffffffffffffull));
  return ok;
}

template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- seeded synthetic input ---------------------------------------------------
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

// ---- reductions -----------------------------------------------------------------
__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

#endif  // __CUDACC__

}  // namespace spmdb200
