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
// address, so the entry looks the address up with cudaGetSymbolAddress once
// per device (with that device current) and passes it to the kernel.  That
// look-up happens on the first call on each device, so the first call on a
// device should come before any stream capture.
//
// All calls share the one array: each call clears the ticket before its
// launch, and calls that overlap on the GPU (different streams, or different
// host threads on one device) race on it and must be serialised by the
// caller.  No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "../../include/spmd_b200.h"
#include "internal.h"

namespace spmdb200 {
namespace {

constexpr int kNoAllocMaxBlocks = 2048;
constexpr size_t kNoAllocHeader = 256;  // ticket word + padding (the partials start 256 bytes in)
constexpr size_t kNoAllocBytes = kNoAllocHeader + sizeof(double) * kNoAllocMaxBlocks;

static __device__ __align__(256) unsigned char g_sum_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of g_sum_scratch on the current device (looked up once).
cudaError_t scratch_address(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sum_scratch);
    if (e != cudaSuccess) return e;
    if (!p) return cudaErrorInvalidSymbol;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
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
  e = cudaMemsetAsync(scratch, 0, sizeof(unsigned), s);  // the ticket starts at zero
  if (e == cudaSuccess) e = launch_sum_f32(View1{A ? A + A_off : nullptr, N, A_st}, o + o_off, N, scratch, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return record_api_status(SPMDB200_ERR_CUDA, "sum_f32_noalloc launch: %s", cudaGetErrorString(e));
  }
  return record_api_status(SPMDB200_OK, "");
}
