// noalloc.cu -- spmdb200_sum_f32_noalloc: the deterministic f32 sum for
// callers that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- inside a
// stream capture that must not allocate, in a plugin whose host application
// owns every device allocation, or in a latency-critical path that has no
// workspace to hand out.  spmdb200_sum_f32 needs a caller-provided workspace
// (a ticket word and one f64 partial per block); this entry keeps that
// scratch in a file-scope __device__ array instead, so the caller passes only
// the input and the output.
//
// The array is fixed at 256 bytes of header (the ticket) plus 2048 f64 block
// partials (16,640 bytes in all).  Every GPU that loads the library holds it
// until the process exits.  The reduction launches at most 2048 blocks, so
// every N fits; the entry still checks the block count against the capacity
// and rejects a launch that would need more.
//
// In host code the array's name is only a host-side stand-in, not a device
// address, so the entry looks the address up with cudaGetSymbolAddress with
// the device current and passes it to the kernel.  A __device__ array has one
// instance per CUDA context, so the address is cached per context (the
// primary context, or one a caller created with cuCtxCreate and made
// current): the first call in each context does the look-up, so that first
// call should come before any stream capture.  A context that is destroyed
// and replaced by a new one with the same handle value would reuse the old
// address, so a caller that destroys contexts must not call this entry again
// in the process afterwards.
//
// All calls share the one array.  Each call clears the header and the
// partial words its launch will use before the launch (a partial that a
// block stored after a bounded wait gave up would otherwise be read by the
// next call as already written), and calls that overlap on the GPU
// (different streams, or different host threads on one device) race on it
// and must be serialised by the caller.  No cudaMalloc, cudaFree or
// allocating library routine is called.
#include <mutex>

#include "../../include/spmd_b200.h"
#include "internal.h"

namespace spmdb200 {
namespace {

constexpr int kNoAllocMaxBlocks = 2048;
constexpr size_t kNoAllocHeader = 256;  // ticket word + padding (the partials start 256 bytes in)
constexpr size_t kNoAllocBytes = kNoAllocHeader + sizeof(double) * kNoAllocMaxBlocks;

static __device__ __align__(256) unsigned char g_sum_scratch[kNoAllocBytes];

// Address cache: (CUcontext, address of g_sum_scratch in it).  The runtime
// resolves the context itself; the driver's cuCtxGetCurrent names it.
constexpr int kMaxContexts = 64;
std::mutex g_mu;
struct CtxAddr {
  void *ctx;
  void *addr;
};
CtxAddr g_scratch_addr[kMaxContexts] = {};
int g_scratch_n = 0;

using CtxGetCurrentFn = int (*)(void **);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
    tried = true;
  }
  return fn;
}

// Device address of g_sum_scratch in the current context (looked up once per
// context).
cudaError_t scratch_address(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return cudaErrorDeviceUninitialized;
  std::lock_guard<std::mutex> lk(g_mu);
  void *ctx = nullptr;
  if (get(&ctx) != 0) return cudaErrorDeviceUninitialized;
  for (int i = 0; ctx && i < g_scratch_n; ++i)
    if (g_scratch_addr[i].ctx == ctx) {
      *out = g_scratch_addr[i].addr;
      return cudaSuccess;
    }
  // First call in this context (or on a thread the runtime has not bound to
  // a context yet: the look-up binds the device's primary context).
  void *p = nullptr;
  e = cudaGetSymbolAddress(&p, g_sum_scratch);
  if (e != cudaSuccess) return e;
  if (!p) return cudaErrorInvalidSymbol;
  if (!ctx && (get(&ctx) != 0 || !ctx)) return cudaErrorDeviceUninitialized;
  bool known = false;
  for (int i = 0; i < g_scratch_n; ++i) known |= g_scratch_addr[i].ctx == ctx;
  if (!known) {
    if (g_scratch_n < kMaxContexts)
      g_scratch_addr[g_scratch_n++] = CtxAddr{ctx, p};
    else
      g_scratch_addr[kMaxContexts - 1] = CtxAddr{ctx, p};  // full: the newest context replaces the last entry
  }
  *out = p;
  return cudaSuccess;
}

}  // namespace
}  // namespace spmdb200

extern "C" int spmdb200_sum_f32_noalloc(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                                        float *o_base, float *o, int64_t o_off, int64_t N, void *stream) {
  using namespace spmdb200;
  (void)A_base;
  (void)o_base;
  if (N < 0) return record_api_status(SPMDB200_ERR_INVALID_ARG, "A: negative loop bound %lld", (long long)N);
  if (N > 0 && (!A || A_off < 0 || A_size < N || A_st < 1))
    return record_api_status(SPMDB200_ERR_INVALID_ARG, "A: null pointer, negative offset, size < N or stride < 1");
  if (!o || o_off < 0) return record_api_status(SPMDB200_ERR_INVALID_ARG, "out: null pointer or negative offset");
  const int blocks = sum_f32_grid(N);
  if (blocks > kNoAllocMaxBlocks)
    return record_api_status(SPMDB200_ERR_WORKSPACE,
                         "N=%lld needs %d block partials; the no-alloc scratch holds %d (%zu bytes)",
                         (long long)N, blocks, kNoAllocMaxBlocks, kNoAllocBytes);
  void *scratch = nullptr;
  cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return record_api_status(SPMDB200_ERR_CUDA, "cudaGetSymbolAddress(g_sum_scratch): %s", cudaGetErrorString(e));
  }
  cudaStream_t s = (cudaStream_t)stream;
  // The header and every partial word this launch can touch start at zero.
  e = cudaMemsetAsync(scratch, 0, kNoAllocHeader + sizeof(double) * (size_t)blocks, s);
  if (e == cudaSuccess) e = launch_sum_f32(View1{A ? A + A_off : nullptr, N, A_st}, o + o_off, N, scratch, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return record_api_status(SPMDB200_ERR_CUDA, "sum_f32_noalloc launch: %s", cudaGetErrorString(e));
  }
  return record_api_status(SPMDB200_OK, "");
}

