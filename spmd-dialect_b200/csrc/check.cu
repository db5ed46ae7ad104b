// check.cu -- spmdb200_check_status: the out-of-range records of a checked
// build (-DSPMDB200_CHECKED on forall_map.cu and stencil_nd.cu).  The
// reference's checks are static (barrier placement, SPMDToGPU.cpp:771-780;
// VerifySPMDInvariants.cpp); a checked build adds run-time index checks that
// record instead of trapping, for shapes the parity tests compare with the
// oracle.
#include "../../include/spmd_b200.h"
#include "internal.h"

using namespace spmdb200;

extern "C" int spmdb200_check_status(unsigned long long *first_out) {
  if (first_out) *first_out = 0;
  if (!check_read_forall_map(nullptr) && !check_read_stencil_nd(nullptr))
    return record_api_status(SPMDB200_ERR_UNSUPPORTED, "not a checked build");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return record_api_status(SPMDB200_ERR_CUDA, "check_status: %s", cudaGetErrorString(e));
  }
  unsigned long long a = 0, b = 0;
  if (check_read_forall_map(&a) < 0 || check_read_stencil_nd(&b) < 0) {
    e = cudaGetLastError();
    return record_api_status(SPMDB200_ERR_CUDA, "check_status: reading the record: %s", cudaGetErrorString(e));
  }
  const unsigned long long first = a ? a : b;
  if (!first) return record_api_status(SPMDB200_OK, "");
  if (first_out) *first_out = first;
  return record_api_status(SPMDB200_ERR_BOUNDS, "%s: site %u, index %lld", a ? "forall_map" : "stencil_nd",
                           (unsigned)((first >> 48) & 0x7fff), (long long)(first & 0xffffffffffffull));
}
