// reduce_bulk.cuh -- shared-memory-staged reduction bodies (unit stride,
// 16-byte aligned input).
//
// A register-streaming reduction keeps only a few loads in flight per thread,
// so a 64 MiB input costs ~7 dependent DRAM round trips per thread.  Here each
// CTA owns one contiguous range of the input (equal split, so no tail CTA) and
// pulls it through a ring of kStages x 16 KB shared-memory stages with
// cp.async.bulk (completion on an mbarrier): 128 KB in flight per SM,
// independent of register count.  Threads reduce a
// landed stage from shared memory, __syncthreads, and thread 0 refills the
// stage with the chunk kStages ahead.  Every wait is bounded; on expiry the
// CTA records a flag, drains its in-flight copies and stops.
#pragma once

#include "common.cuh"

namespace spmdb200 {

constexpr int kBulkThreads = 256;
// 4 x 32 KB per CTA (one CTA per SM): measured on B200 against 4-16 KB chunks,
// 2-8 stages and per-warp stage release without CTA barriers, 32 KB x 4 was
// fastest at 2^24 (f32 17.5 us, i32 14.6 us vs 18.7 / 15.5 at 16 KB x 4) and
// at 2^28.
constexpr int kBulkChunk = 32768;  // bytes per stage
constexpr int kBulkStages = 4;
constexpr size_t kBulkSmem = (size_t)kBulkStages * kBulkChunk + 128;

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch of the first kBulkStages chunks of [u_lo, u_hi).  A prefetch
// returns no data, so it may run before griddepcontrol.wait: lines that the
// previous kernel still writes are updated in L2, the point of coherence, and
// the stage loads after the wait read them from there.  (Prefetching a whole
// 64 MiB input into L2 at kernel start measured slower: 2^24 f32 single
// launch 21.5 against 19.5 us.)
__device__ __forceinline__ void bulk_prefetch_head(const uint4 *base, int64_t u_lo, int64_t u_hi) {
  constexpr int kUnits = kBulkChunk / 16;
  for (int s = 0; s < kBulkStages; ++s) {
    const int64_t c0 = u_lo + (int64_t)s * kUnits;
    if (c0 >= u_hi) break;
    const uint32_t bytes = (uint32_t)(min((int64_t)kUnits, u_hi - c0) * 16);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + c0), "r"(bytes) : "memory");
  }
}

// Streams the 16-byte units [u_lo, u_hi) of `base` through shared memory and
// calls f(float4 as the element type's 16 bytes) for every unit, each thread
// seeing a fixed, deterministic subset.  Returns false if a wait timed out.
template <class F>
__device__ __forceinline__ bool bulk_stream(const uint4 *base, int64_t u_lo, int64_t u_hi, unsigned char *smem,
                                            uint64_t *full, volatile int *abort, F f) {
  constexpr int kUnits = kBulkChunk / 16;
  const int64_t units = u_hi - u_lo;
  const int64_t nch = (units + kUnits - 1) / kUnits;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages && s < nch; ++s) {
      const int64_t c0 = u_lo + (int64_t)s * kUnits;
      const uint32_t bytes = (uint32_t)(min((int64_t)kUnits, u_hi - c0) * 16);
      mbar_arrive_expect_tx(&full[s], bytes);
      bulk_load(smem + (size_t)s * kBulkChunk, base + c0, bytes, &full[s]);
    }
  }
  int64_t failed_at = -1;
  for (int64_t k = 0; k < nch; ++k) {
    const int st = (int)(k % kBulkStages);
    const uint32_t ph = (uint32_t)((k / kBulkStages) & 1);
    const bool got = mbar_wait_bounded(&full[st], ph, abort);
    if (!__syncthreads_and(got)) {  // uniform decision for the whole CTA
      failed_at = k;
      break;
    }
    const int64_t c0 = u_lo + k * kUnits;
    const int cnt = (int)min((int64_t)kUnits, u_hi - c0);
    const uint4 *sv = reinterpret_cast<const uint4 *>(smem + (size_t)st * kBulkChunk);
    for (int i = threadIdx.x; i < cnt; i += kBulkThreads) f(sv[i]);
    __syncthreads();  // every thread is done with stage st
    if (threadIdx.x == 0 && k + kBulkStages < nch) {
      const int64_t n0 = c0 + (int64_t)kBulkStages * kUnits;
      const uint32_t bytes = (uint32_t)(min((int64_t)kUnits, u_hi - n0) * 16);
      mbar_arrive_expect_tx(&full[st], bytes);
      bulk_load(smem + (size_t)st * kBulkChunk, base + n0, bytes, &full[st]);
    }
  }
  if (failed_at >= 0 && threadIdx.x == 0) {
    // Drain: chunks [0, horizon) were issued; the latest one in each stage
    // must land before this CTA's shared memory is released.
    int no_abort = 0;
    const int64_t horizon = min(failed_at + kBulkStages, nch);
    for (int s = 0; s < kBulkStages && s < horizon; ++s) {
      const int64_t last = s + ((horizon - 1 - s) / kBulkStages) * kBulkStages;
      mbar_wait_bounded(&full[s], (uint32_t)((last / kBulkStages) & 1), &no_abort);
    }
  }
  return failed_at < 0;
}

// Block partials of the staged reductions travel as one 64-bit word each.
// An f64 partial is stored as its bits XOR a signalling-NaN key.  Every partial is the result of
// __dadd_rn (a number or the canonical quiet NaN), never the key itself, so a
// stored word is never 0 and 0 means "not written yet".  One word carries the
// value and its presence, so the writer needs no fence and the combiner no
// ticket: it polls the words and sees each partial one store latency after
// it is written.
constexpr unsigned long long kPartialKey = 0x7FF0DEADBEEF0001ull;

__device__ __forceinline__ void st_relaxed_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// A 4-byte partial (f32 or i32 bits) is stored with bit 32 set.
__device__ __forceinline__ unsigned long long partial_word(double v) {
  return (unsigned long long)__double_as_longlong(v) ^ kPartialKey;
}
__device__ __forceinline__ unsigned long long partial_word(float v) { return (1ull << 32) | __float_as_uint(v); }
__device__ __forceinline__ unsigned long long partial_word(uint32_t v) { return (1ull << 32) | v; }
__device__ __forceinline__ void partial_value(unsigned long long w, double &v) {
  v = __longlong_as_double((long long)(w ^ kPartialKey));
}
__device__ __forceinline__ void partial_value(unsigned long long w, float &v) { v = __uint_as_float((uint32_t)w); }
__device__ __forceinline__ void partial_value(unsigned long long w, uint32_t &v) { v = (uint32_t)w; }
// Bounded wait for a non-zero word; returns 0 if the wait budget ran out.
__device__ __forceinline__ unsigned long long poll_partial(const unsigned long long *p) {
  unsigned long long v = ld_relaxed_u64(p);
  if (v) return v;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    v = ld_relaxed_u64(p);
    if (v) return v;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) return 0ull;
  }
}

// This CTA's contiguous share [lo, hi) of `total` units (equal split).
__device__ __forceinline__ void cta_range(int64_t total, int64_t &lo, int64_t &hi) {
  lo = total * (int64_t)blockIdx.x / gridDim.x;
  hi = total * (int64_t)(blockIdx.x + 1) / gridDim.x;
}

}  // namespace spmdb200
