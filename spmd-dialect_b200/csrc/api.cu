// api.cu -- the extern "C" entry points declared in include/spmd_b200.h.
//
// Argument validation happens here, before anything touches the GPU: a bad
// descriptor returns SPMDB200_ERR_INVALID_ARG and launches nothing.  The
// reference-named host entries keep the reference's void signatures and
// report failures on stderr plus spmdb200_last_error().
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <vector>

#include "../../include/spmd_b200.h"
#include "internal.h"

using namespace spmdb200;

namespace {

thread_local int g_last_status = SPMDB200_OK;
thread_local char g_last_msg[512] = "";

int fail(int status, const char *fmt, ...) {
  g_last_status = status;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_msg, sizeof(g_last_msg), fmt, ap);
  va_end(ap);
  return status;
}
int ok() {
  g_last_status = SPMDB200_OK;
  g_last_msg[0] = '\0';
  return SPMDB200_OK;
}
int cuda_fail(cudaError_t e, const char *what) {
  cudaGetLastError();  // clear a sticky launch error so the next call starts clean
  return fail(SPMDB200_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}
#define CUDA_TRY(expr)                                     \
  do {                                                     \
    cudaError_t e_ = (expr);                               \
    if (e_ != cudaSuccess) return cuda_fail(e_, #expr);    \
  } while (0)

void report_void(const char *fn, int st) {
  if (st != SPMDB200_OK) fprintf(stderr, "spmdb200: %s failed: %s\n", fn, g_last_msg);
}

// ---- descriptor validation ----------------------------------------------------
int check1(const char *nm, const void *p, int64_t off, int64_t size, int64_t stride, int64_t n) {
  if (n < 0) return fail(SPMDB200_ERR_INVALID_ARG, "%s: negative loop bound %lld", nm, (long long)n);
  if (n == 0) return SPMDB200_OK;
  if (!p) return fail(SPMDB200_ERR_INVALID_ARG, "%s: null aligned pointer", nm);
  if (off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "%s: negative offset", nm);
  if (size < n) return fail(SPMDB200_ERR_INVALID_ARG, "%s: size %lld < loop bound %lld", nm, (long long)size, (long long)n);
  if (stride < 1) return fail(SPMDB200_ERR_INVALID_ARG, "%s: stride %lld < 1", nm, (long long)stride);
  return SPMDB200_OK;
}
int check2(const char *nm, const void *p, int64_t off, int64_t n0, int64_t n1, int64_t s0, int64_t s1) {
  if (n0 < 0 || n1 < 0) return fail(SPMDB200_ERR_INVALID_ARG, "%s: negative size", nm);
  if (n0 == 0 || n1 == 0) return SPMDB200_OK;
  if (!p) return fail(SPMDB200_ERR_INVALID_ARG, "%s: null aligned pointer", nm);
  if (off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "%s: negative offset", nm);
  if (s0 < 1 || s1 < 1) return fail(SPMDB200_ERR_INVALID_ARG, "%s: strides must be >= 1", nm);
  return SPMDB200_OK;
}
int check3(const char *nm, const void *p, int64_t off, int64_t n0, int64_t n1, int64_t n2, int64_t s0,
           int64_t s1, int64_t s2) {
  if (n0 < 0 || n1 < 0 || n2 < 0) return fail(SPMDB200_ERR_INVALID_ARG, "%s: negative size", nm);
  if (n0 == 0 || n1 == 0 || n2 == 0) return SPMDB200_OK;
  if (!p) return fail(SPMDB200_ERR_INVALID_ARG, "%s: null aligned pointer", nm);
  if (off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "%s: negative offset", nm);
  if (s0 < 1 || s1 < 1 || s2 < 1) return fail(SPMDB200_ERR_INVALID_ARG, "%s: strides must be >= 1", nm);
  return SPMDB200_OK;
}
#define CHECK(expr)                        \
  do {                                     \
    int st_ = (expr);                      \
    if (st_ != SPMDB200_OK) return st_;    \
  } while (0)

int have_device() {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n < 1) {
    cudaGetLastError();
    return fail(SPMDB200_ERR_NO_DEVICE, "no CUDA device visible (%s)", cudaGetErrorString(e));
  }
  return SPMDB200_OK;
}

// ---- staging buffers for the host entries --------------------------------------
struct Staging {
  std::vector<std::pair<void *, size_t>> slots;  // per slot: ptr, capacity
};
std::mutex g_stage_mu;
std::vector<Staging> g_stage;  // indexed by device

int staging(int slot, size_t bytes, void **out) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_stage_mu);
  if ((int)g_stage.size() <= dev) g_stage.resize(dev + 1);
  auto &sl = g_stage[dev].slots;
  if ((int)sl.size() <= slot) sl.resize(slot + 1, {nullptr, 0});
  if (sl[slot].second < bytes) {
    if (sl[slot].first) cudaFree(sl[slot].first);
    sl[slot] = {nullptr, 0};
    void *p = nullptr;
    CUDA_TRY(cudaMalloc(&p, bytes < 256 ? 256 : bytes));
    sl[slot] = {p, bytes < 256 ? 256 : bytes};
  }
  *out = sl[slot].first;
  return SPMDB200_OK;
}

// Strided host <-> dense device copies of rank-1 f32/i32 memrefs.
int h2d_1d(void *dst, const void *src_elem0, int64_t n, int64_t stride, size_t esz) {
  if (n <= 0) return SPMDB200_OK;
  if (stride == 1) {
    CUDA_TRY(cudaMemcpy(dst, src_elem0, (size_t)n * esz, cudaMemcpyHostToDevice));
  } else {
    CUDA_TRY(cudaMemcpy2D(dst, esz, src_elem0, (size_t)stride * esz, esz, (size_t)n, cudaMemcpyHostToDevice));
  }
  return SPMDB200_OK;
}
int d2h_1d(void *dst_elem0, const void *src, int64_t n, int64_t stride, size_t esz) {
  if (n <= 0) return SPMDB200_OK;
  if (stride == 1) {
    CUDA_TRY(cudaMemcpy(dst_elem0, src, (size_t)n * esz, cudaMemcpyDeviceToHost));
  } else {
    CUDA_TRY(cudaMemcpy2D(dst_elem0, (size_t)stride * esz, src, esz, esz, (size_t)n, cudaMemcpyDeviceToHost));
  }
  return SPMDB200_OK;
}
// Rank-2: host (n0 x n1, strides s0, s1) <-> device dense with row pitch dp elements.
int h2d_2d(float *dst, int64_t dp, const float *src, int64_t n0, int64_t n1, int64_t s0, int64_t s1) {
  if (n0 <= 0 || n1 <= 0) return SPMDB200_OK;
  if (s1 == 1) {
    CUDA_TRY(cudaMemcpy2D(dst, (size_t)dp * 4, src, (size_t)s0 * 4, (size_t)n1 * 4, (size_t)n0,
                          cudaMemcpyHostToDevice));
  } else {
    for (int64_t i = 0; i < n0; ++i)
      CUDA_TRY(cudaMemcpy2D(dst + i * dp, 4, src + i * s0, (size_t)s1 * 4, 4, (size_t)n1, cudaMemcpyHostToDevice));
  }
  return SPMDB200_OK;
}
int d2h_2d(float *dst, int64_t n0, int64_t n1, int64_t s0, int64_t s1, const float *src, int64_t sp) {
  if (n0 <= 0 || n1 <= 0) return SPMDB200_OK;
  if (s1 == 1) {
    CUDA_TRY(cudaMemcpy2D(dst, (size_t)s0 * 4, src, (size_t)sp * 4, (size_t)n1 * 4, (size_t)n0,
                          cudaMemcpyDeviceToHost));
  } else {
    for (int64_t i = 0; i < n0; ++i)
      CUDA_TRY(cudaMemcpy2D(dst + i * s0, (size_t)s1 * 4, src + i * sp, 4, 4, (size_t)n1, cudaMemcpyDeviceToHost));
  }
  return SPMDB200_OK;
}

int64_t round_up4(int64_t x) { return (x + 3) & ~int64_t(3); }

int jacobi_status_from_ws(JacobiWs *ws, cudaStream_t s) {
  CUDA_TRY(cudaStreamSynchronize(s));
  int st = 0;
  CUDA_TRY(cudaMemcpy(&st, &ws->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st != kDevOk)
    return fail(SPMDB200_ERR_TIMEOUT, "device-side bounded wait expired (code %d: %s)", st,
                st == kDevTimeoutGridBarrier ? "grid barrier"
                : st == kDevTimeoutFull      ? "TMA stage full"
                : st == kDevTimeoutEmpty     ? "TMA stage empty"
                : st == kDevTimeoutPeer      ? "peer halo delivery"
                                             : "unknown");
  return SPMDB200_OK;
}

}  // namespace

// ---- helpers used by the kernel translation units ------------------------------
namespace spmdb200 {

int num_sms(int device) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= device) cache.resize(device + 1, 0);
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n < 1) n = 148;
    cache[device] = n;
  }
  return cache[device];
}

static std::atomic<unsigned long long> g_grid_budget_ns{kWaitBudgetNs};
static std::atomic<unsigned long long> g_peer_budget_ns{kPeerWaitBudgetNs};

unsigned long long wait_budget_ns(bool peer) { return peer ? g_peer_budget_ns.load() : g_grid_budget_ns.load(); }

int record_api_status(int status, const char *fmt, ...) {
  g_last_status = status;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_msg, sizeof(g_last_msg), fmt, ap);
  va_end(ap);
  return status;
}

int encode_tensor_map_f32(void *tmap, void *gaddr, int rank, const uint64_t *dims,
                          const uint64_t *strides_bytes, const uint32_t *box) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) return -1;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) st[i] = strides_bytes[i];
  CUresult r = fn(reinterpret_cast<CUtensorMap *>(tmap), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, gaddr, d,
                  st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

}  // namespace spmdb200

// =================================================================================
extern "C" {

const char *spmdb200_status_string(int status) {
  switch (status) {
    case SPMDB200_OK: return "ok";
    case SPMDB200_ERR_INVALID_ARG: return "invalid argument";
    case SPMDB200_ERR_CUDA: return "CUDA error";
    case SPMDB200_ERR_TIMEOUT: return "device wait timed out";
    case SPMDB200_ERR_UNSUPPORTED: return "unsupported layout";
    case SPMDB200_ERR_WORKSPACE: return "bad workspace";
    case SPMDB200_ERR_NO_DEVICE: return "no CUDA device";
    case SPMDB200_ERR_BOUNDS: return "out-of-range access recorded (checked build)";
    default: return "unknown status";
  }
}
int spmdb200_last_error(void) { return g_last_status; }
const char *spmdb200_last_error_message(void) { return g_last_msg; }
const char *spmdb200_version(void) { return "spmdb200 0.1.0 (sm_100a)"; }

int spmdb200_release_cache(void) {
  std::lock_guard<std::mutex> lk(g_stage_mu);
  int cur = 0;
  cudaGetDevice(&cur);
  for (size_t d = 0; d < g_stage.size(); ++d) {
    if (g_stage[d].slots.empty()) continue;
    cudaSetDevice((int)d);
    for (auto &s : g_stage[d].slots)
      if (s.first) cudaFree(s.first);
    g_stage[d].slots.clear();
  }
  cudaSetDevice(cur);
  return ok();
}

// ---------------------------------------------------------------- device entries
int spmdb200_ewise(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                   float *B_base, float *B, int64_t B_off, int64_t B_size, int64_t B_st,
                   float *C_base, float *C, int64_t C_off, int64_t C_size, int64_t C_st,
                   int64_t N, void *stream) {
  (void)A_base; (void)B_base; (void)C_base;
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  CHECK(check1("B", B, B_off, B_size, B_st, N));
  CHECK(check1("C", C, C_off, C_size, C_st, N));
  if (N == 0) return ok();
  CUDA_TRY(launch_ewise_add(View1{A + A_off, N, A_st}, View1{B + B_off, N, B_st}, View1{C + C_off, N, C_st}, N,
                            (cudaStream_t)stream));
  return ok();
}

int spmdb200_axpy(float a, float *X_base, float *X, int64_t X_off, int64_t X_size, int64_t X_st,
                  float *Y_base, float *Y, int64_t Y_off, int64_t Y_size, int64_t Y_st, int64_t N, void *stream) {
  (void)X_base; (void)Y_base;
  CHECK(check1("X", X, X_off, X_size, X_st, N));
  CHECK(check1("Y", Y, Y_off, Y_size, Y_st, N));
  if (N == 0) return ok();
  CUDA_TRY(launch_axpy(a, View1{X + X_off, N, X_st}, View1{Y + Y_off, N, Y_st}, N, (cudaStream_t)stream));
  return ok();
}

int spmdb200_stencil3pt(float *A_base, float *A, int64_t A_off, int64_t A_n0, int64_t A_n1, int64_t A_s0,
                        int64_t A_s1, float *B_base, float *B, int64_t B_off, int64_t B_n0, int64_t B_n1,
                        int64_t B_s0, int64_t B_s1, int64_t N, int64_t M, void *stream) {
  (void)A_base; (void)B_base;
  CHECK(check2("A", A, A_off, A_n0, A_n1, A_s0, A_s1));
  CHECK(check2("B", B, B_off, B_n0, B_n1, B_s0, B_s1));
  if (N < 0 || M < 0 || N > B_n0 || M > B_n1)
    return fail(SPMDB200_ERR_INVALID_ARG, "loop bounds (%lld, %lld) exceed B (%lld, %lld)", (long long)N,
                (long long)M, (long long)B_n0, (long long)B_n1);
  if (N == 0 || M == 0) return ok();
  const View2 a{A ? A + A_off : nullptr, A_n0, A_n1, A_s0, A_s1};
  const View2 b{B + B_off, B_n0, B_n1, B_s0, B_s1};
  CUDA_TRY(launch_stencil3(a, b, N, M, (cudaStream_t)stream));
  return ok();
}

int spmdb200_promotion_plan(int rank, const int64_t *tile_sizes, const int64_t *steps,
                            const int64_t *min_offsets, const int64_t *max_offsets, int64_t elem_bytes,
                            int64_t max_group_bytes, int read_only, int64_t *tile_dims_out,
                            int64_t *footprint_bytes_out) {
  const int r = promotion_plan(rank, tile_sizes, steps, min_offsets, max_offsets, elem_bytes, max_group_bytes,
                               read_only, tile_dims_out, footprint_bytes_out);
  if (r < 0) return fail(SPMDB200_ERR_INVALID_ARG, "promotion plan: rank 1-3, non-null sizes, elem_bytes >= 1");
  ok();
  return r;
}

int spmdb200_stencil_nd(int rank, const float *A, const int64_t *A_sizes, const int64_t *A_strides, float *B,
                        const int64_t *B_sizes, const int64_t *B_strides, int ntaps, const int64_t *offsets,
                        const float *weights, float scale, const int64_t *tile_sizes, const int64_t *steps,
                        int64_t max_group_bytes, int policy, int *promoted_out, void *stream) {
  if (promoted_out) *promoted_out = 0;
  if (rank < 1 || rank > 3) return fail(SPMDB200_ERR_INVALID_ARG, "rank %d: must be 1, 2 or 3", rank);
  if (ntaps < 1 || ntaps > kNdMaxTaps) return fail(SPMDB200_ERR_INVALID_ARG, "ntaps %d: 1..%d", ntaps, kNdMaxTaps);
  if (!A_sizes || !A_strides || !B_sizes || !B_strides || !offsets || !tile_sizes)
    return fail(SPMDB200_ERR_INVALID_ARG, "null size / stride / offset / tile array");
  if (policy != 0 && policy != 1) return fail(SPMDB200_ERR_INVALID_ARG, "policy must be 0 or 1");
  if (max_group_bytes <= 0) max_group_bytes = SPMDB200_DEFAULT_GROUP_MEM_BYTES;
  if (max_group_bytes > 227 * 1024) return fail(SPMDB200_ERR_UNSUPPORTED, "max_group_bytes above 227 KB");
  StencilNdProblem p{};
  p.rank = rank;
  p.ntaps = ntaps;
  p.a = A;
  p.b = B;
  p.offsets = offsets;
  p.weights = weights;
  p.scale = scale;
  int64_t a_cells = 1, b_cells = 1, a_span = 1, b_span = 1, mn[3], mx[3];
  for (int d = 0; d < rank; ++d) {
    if (A_sizes[d] < 0 || B_sizes[d] < 0 || A_strides[d] < 0 || B_strides[d] < 0)
      return fail(SPMDB200_ERR_INVALID_ARG, "negative size or stride in dimension %d", d);
    if (tile_sizes[d] < 1 || tile_sizes[d] > 1024 || (steps && (steps[d] < 1 || steps[d] > (1 << 20))))
      return fail(SPMDB200_ERR_INVALID_ARG, "tile size 1..1024 and step 1..2^20 in dimension %d", d);
    p.a_size[d] = A_sizes[d];
    p.a_stride[d] = A_strides[d];
    p.b_size[d] = B_sizes[d];
    p.b_stride[d] = B_strides[d];
    p.tile[d] = tile_sizes[d];
    p.step[d] = steps ? steps[d] : 1;
    a_cells *= A_sizes[d];
    b_cells *= B_sizes[d];
    a_span += (A_sizes[d] > 0 ? A_sizes[d] - 1 : 0) * A_strides[d];
    b_span += (B_sizes[d] > 0 ? B_sizes[d] - 1 : 0) * B_strides[d];
    mn[d] = mx[d] = offsets[d];
  }
  for (int j = 0; j < ntaps; ++j)
    for (int d = 0; d < rank; ++d) {
      const int64_t o = offsets[j * rank + d];
      if (o < -(1 << 20) || o > (1 << 20)) return fail(SPMDB200_ERR_INVALID_ARG, "offset %lld out of range", (long long)o);
      mn[d] = o < mn[d] ? o : mn[d];
      mx[d] = o > mx[d] ? o : mx[d];
    }
  if (b_cells == 0) return ok();
  if (!B || (a_cells > 0 && !A)) return fail(SPMDB200_ERR_INVALID_ARG, "null A or B");
  const bool overlap = a_cells > 0 && (const void *)A < (const void *)(B + b_span) && (const void *)B < (const void *)(A + a_span);
  if (overlap) return fail(SPMDB200_ERR_INVALID_ARG, "A and B overlap (the stencil's input must be read-only)");
  if (a_cells == 0) {
    p.a = B;  // every read is outside A: reads return 0 without touching memory
    for (int d = 0; d < rank; ++d) p.a_size[d] = 0;
  }
  int64_t dims[3], bytes = 0;
  const int plan = policy == 0 ? promotion_plan(rank, tile_sizes, steps, mn, mx, 4, max_group_bytes, 1, dims, &bytes)
                               : kPlanSkipNoReuse;
  const int promote = plan == kPlanPromote ? 1 : 0;
  CUDA_TRY(launch_stencil_nd(p, promote, (cudaStream_t)stream));
  if (promoted_out) *promoted_out = promote;
  return ok();
}

size_t spmdb200_sum_workspace_bytes(int64_t N) { return sum_f32_workspace_bytes(N); }

int spmdb200_sum_f32(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                     float *o_base, float *o, int64_t o_off, int64_t N, void *ws, size_t ws_bytes, void *stream) {
  (void)A_base; (void)o_base;
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  if (!o || o_off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "out: null pointer or negative offset");
  if (!ws || ((uintptr_t)ws & 255u) != 0 || ws_bytes < sum_f32_workspace_bytes(N))
    return fail(SPMDB200_ERR_WORKSPACE, "workspace must be >= %zu bytes and 256-byte aligned",
                sum_f32_workspace_bytes(N));
  CUDA_TRY(launch_sum_f32(View1{A ? A + A_off : nullptr, N, A_st}, o + o_off, N, ws, (cudaStream_t)stream));
  return ok();
}

int spmdb200_sum_f32_partial(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st, int64_t N,
                             double *partial, void *ws, size_t ws_bytes, void *stream) {
  (void)A_base;
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  if (!partial) return fail(SPMDB200_ERR_INVALID_ARG, "partial: null pointer");
  if (!ws || ((uintptr_t)ws & 255u) != 0 || ws_bytes < sum_f32_workspace_bytes(N))
    return fail(SPMDB200_ERR_WORKSPACE, "workspace must be >= %zu bytes and 256-byte aligned",
                sum_f32_workspace_bytes(N));
  CUDA_TRY(launch_sum_f32(View1{A ? A + A_off : nullptr, N, A_st}, nullptr, N, ws, (cudaStream_t)stream, partial));
  return ok();
}

int spmdb200_sum_i32(int32_t *A_base, int32_t *A, int64_t A_off, int64_t A_size, int64_t A_st,
                     int32_t *o_base, int32_t *o, int64_t o_off, int64_t N, void *stream) {
  (void)A_base; (void)o_base;
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  if (!o || o_off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "out: null pointer or negative offset");
  if (N == 0) return ok();
  CUDA_TRY(launch_sum_i32(A + A_off, A_st, o + o_off, N, (cudaStream_t)stream));
  return ok();
}

int spmdb200_hierarchical_sum(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                              float *o_base, float *o, int64_t o_off, int64_t N, void *stream) {
  (void)A_base; (void)o_base;
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  if (!o || o_off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "out: null pointer or negative offset");
  if (N == 0) return ok();
  CUDA_TRY(launch_hier_sum_f32(View1{A + A_off, N, A_st}, o + o_off, N, (cudaStream_t)stream));
  return ok();
}

static int check_reduce_args(int kind, int max_kind, const void *A, int64_t A_off, int64_t A_size, int64_t A_st,
                             const void *o, int64_t o_off, int64_t N, void *ws, size_t ws_bytes) {
  if (kind < 0 || kind > max_kind)
    return fail(SPMDB200_ERR_INVALID_ARG, "reduction kind %d not in [0, %d]", kind, max_kind);
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  if (!o || o_off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "out: null pointer or negative offset");
  if (!ws || ((uintptr_t)ws & 255u) != 0 || ws_bytes < sum_f32_workspace_bytes(N))
    return fail(SPMDB200_ERR_WORKSPACE, "workspace must be >= %zu bytes and 256-byte aligned",
                sum_f32_workspace_bytes(N));
  return SPMDB200_OK;
}

int spmdb200_reduce_f32(int kind, float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                        float *o_base, float *o, int64_t o_off, int64_t N, float init, void *ws, size_t ws_bytes,
                        void *stream) {
  (void)A_base; (void)o_base;
  CHECK(check_reduce_args(kind, 3, A, A_off, A_size, A_st, o, o_off, N, ws, ws_bytes));
  CUDA_TRY(launch_reduce_f32(kind, A ? A + A_off : nullptr, A_st, N, o + o_off, init, ws, (cudaStream_t)stream));
  return ok();
}

int spmdb200_reduce_i32(int kind, int32_t *A_base, int32_t *A, int64_t A_off, int64_t A_size, int64_t A_st,
                        int32_t *o_base, int32_t *o, int64_t o_off, int64_t N, int32_t init, void *ws,
                        size_t ws_bytes, void *stream) {
  (void)A_base; (void)o_base;
  CHECK(check_reduce_args(kind, 6, A, A_off, A_size, A_st, o, o_off, N, ws, ws_bytes));
  CUDA_TRY(launch_reduce_i32(kind, A ? A + A_off : nullptr, A_st, N, o + o_off, init, ws, (cudaStream_t)stream));
  return ok();
}

int spmdb200_reduction_status(void) {
  CUDA_TRY(cudaDeviceSynchronize());
  const int f0 = reduction_timeout_flag(true), f1 = kind_timeout_flag(true);
  if (f0 < 0 || f1 < 0) return fail(SPMDB200_ERR_CUDA, "reading the reduction status flag failed");
  if (f0 || f1) return fail(SPMDB200_ERR_TIMEOUT, "a staged reduction's bounded wait expired; its result is invalid");
  return ok();
}

size_t spmdb200_jacobi_workspace_bytes(void) { return sizeof(JacobiWs); }

int spmdb200_set_wait_budget_ms(int64_t grid_ms, int64_t peer_ms) {
  if (grid_ms < 1 || peer_ms < 1 || grid_ms > 600000 || peer_ms > 600000)
    return fail(SPMDB200_ERR_INVALID_ARG, "wait budgets must be in [1, 600000] ms");
  g_grid_budget_ns.store((unsigned long long)grid_ms * 1000000ull);
  g_peer_budget_ns.store((unsigned long long)peer_ms * 1000000ull);
  return ok();
}

int spmdb200_workspace_status(void *ws, void *stream) {
  if (!ws) return fail(SPMDB200_ERR_WORKSPACE, "null workspace");
  CHECK(jacobi_status_from_ws(static_cast<JacobiWs *>(ws), (cudaStream_t)stream));
  return ok();
}

static int check_jacobi_ws(void *ws, size_t ws_bytes) {
  if (!ws || ((uintptr_t)ws & 255u) != 0 || ws_bytes < sizeof(JacobiWs))
    return fail(SPMDB200_ERR_WORKSPACE, "workspace must be >= %zu bytes and 256-byte aligned", sizeof(JacobiWs));
  return SPMDB200_OK;
}
static int check_res(int64_t sweeps, int64_t res_every, const double *res_out) {
  if (sweeps < 0 || res_every < 0) return fail(SPMDB200_ERR_INVALID_ARG, "negative sweeps / res_every");
  if (res_every > 0 && sweeps >= res_every && !res_out)
    return fail(SPMDB200_ERR_INVALID_ARG, "res_out is null but %lld residuals are due",
                (long long)(sweeps / res_every));
  return SPMDB200_OK;
}

int spmdb200_jacobi2d(float *U_base, float *U, int64_t U_off, int64_t U_n0, int64_t U_n1, int64_t U_s0, int64_t U_s1,
                      float *V_base, float *V, int64_t V_off, int64_t V_n0, int64_t V_n1, int64_t V_s0, int64_t V_s1,
                      int64_t sweeps, int64_t res_every, double *res_out, void *ws, size_t ws_bytes, void *stream) {
  (void)U_base; (void)V_base;
  CHECK(check2("U", U, U_off, U_n0, U_n1, U_s0, U_s1));
  CHECK(check2("V", V, V_off, V_n0, V_n1, V_s0, V_s1));
  if (U_n0 != V_n0 || U_n1 != V_n1 || U_s0 != V_s0 || U_s1 != V_s1)
    return fail(SPMDB200_ERR_INVALID_ARG, "U and V must have identical sizes and strides");
  CHECK(check_res(sweeps, res_every, res_out));
  CHECK(check_jacobi_ws(ws, ws_bytes));
  if (sweeps == 0 || U_n0 == 0 || U_n1 == 0) return ok();
  cudaStream_t s = (cudaStream_t)stream;
  JacobiWs *w = static_cast<JacobiWs *>(ws);
  CUDA_TRY(cudaMemsetAsync(w, 0, 256, s));
  Jacobi2dProblem p{};
  p.u = U + U_off;
  p.v = V + V_off;
  p.pitch = U_s0;
  p.h_local = U_n0;
  p.w = U_n1;
  p.row_lo = 0;
  p.row_hi = U_n0;
  p.g_row0 = 0;
  p.g_rows = U_n0;
  p.sweeps = sweeps;
  p.res_every = res_every;
  p.res_out = res_out;
  p.ws = w;
  if (U_s1 == 1 && jacobi2d_persistent_ok(p)) {
    CUDA_TRY(run_jacobi2d_persistent(p, SlabPeers{}, 0u, s));
  } else {
    CUDA_TRY(launch_jacobi2d_generic(p, U_s1, s));
  }
  return ok();
}

int spmdb200_jacobi3d(float *U_base, float *U, int64_t U_off, int64_t U_n0, int64_t U_n1, int64_t U_n2,
                      int64_t U_s0, int64_t U_s1, int64_t U_s2,
                      float *V_base, float *V, int64_t V_off, int64_t V_n0, int64_t V_n1, int64_t V_n2,
                      int64_t V_s0, int64_t V_s1, int64_t V_s2,
                      int64_t sweeps, int64_t res_every, double *res_out, void *ws, size_t ws_bytes, void *stream) {
  (void)U_base; (void)V_base;
  CHECK(check3("U", U, U_off, U_n0, U_n1, U_n2, U_s0, U_s1, U_s2));
  CHECK(check3("V", V, V_off, V_n0, V_n1, V_n2, V_s0, V_s1, V_s2));
  if (U_n0 != V_n0 || U_n1 != V_n1 || U_n2 != V_n2 || U_s0 != V_s0 || U_s1 != V_s1 || U_s2 != V_s2)
    return fail(SPMDB200_ERR_INVALID_ARG, "U and V must have identical sizes and strides");
  CHECK(check_res(sweeps, res_every, res_out));
  CHECK(check_jacobi_ws(ws, ws_bytes));
  if (sweeps == 0 || U_n0 == 0 || U_n1 == 0 || U_n2 == 0) return ok();
  cudaStream_t s = (cudaStream_t)stream;
  JacobiWs *w = static_cast<JacobiWs *>(ws);
  CUDA_TRY(cudaMemsetAsync(w, 0, 256, s));
  Jacobi3dProblem p{};
  p.u = U + U_off;
  p.v = V + V_off;
  p.d = U_n0;
  p.h = U_n1;
  p.w = U_n2;
  p.sz = U_s0;
  p.sy = U_s1;
  p.sx = U_s2;
  p.sweeps = sweeps;
  p.res_every = res_every;
  p.res_out = res_out;
  p.ws = w;
  if (jacobi3d_tma_ok(p)) {
    CUDA_TRY(run_jacobi3d_tb(p, SlabPeers{}, 0u, s));
  } else {
    CUDA_TRY(launch_jacobi3d_generic(p, s));
  }
  return ok();
}

// ---------------------------------------------------------------- multi-GPU slabs
int spmdb200_jacobi_slab_halo(int dims) { return dims == 2 ? kSlabHalo : dims == 3 ? kSlabHalo3 : -1; }

int spmdb200_jacobi_ws_reset(void *ws, void *stream) {
  if (!ws) return fail(SPMDB200_ERR_WORKSPACE, "null workspace");
  CUDA_TRY(cudaMemsetAsync(ws, 0, 256, (cudaStream_t)stream));
  return ok();
}

int spmdb200_jacobi2d_slab(float *U_base, float *U, int64_t U_off, int64_t U_n0, int64_t U_n1, int64_t U_s0,
                           int64_t U_s1, float *V_base, float *V, int64_t V_off, int64_t V_n0, int64_t V_n1,
                           int64_t V_s0, int64_t V_s1, int64_t g_first, int64_t G, int64_t sweeps,
                           int64_t res_every, double *res_out, void *ws, float *up_u, float *up_v, void *up_ws,
                           int64_t up_rows, float *dn_u, float *dn_v, void *dn_ws, int rank, int nranks,
                           void *const *all_ws, int64_t *deliveries, void *stream) {
  (void)U_base; (void)V_base;
  CHECK(check2("U", U, U_off, U_n0, U_n1, U_s0, U_s1));
  CHECK(check2("V", V, V_off, V_n0, V_n1, V_s0, V_s1));
  if (U_n0 != V_n0 || U_n1 != V_n1 || U_s0 != V_s0 || U_s1 != V_s1)
    return fail(SPMDB200_ERR_INVALID_ARG, "U and V must have identical sizes and strides");
  const int64_t H = kSlabHalo;
  if (U_n0 < 3 * H || U_n1 < 1)
    return fail(SPMDB200_ERR_INVALID_ARG, "a slab needs >= %lld owned rows plus %lld halo rows on each side",
                (long long)H, (long long)H);
  const int64_t R = U_n0 - 2 * H;
  if (U_s1 != 1) return fail(SPMDB200_ERR_UNSUPPORTED, "slab rows must be contiguous (stride1 == 1)");
  if (g_first < 0 || G < 1 || g_first + R > G)
    return fail(SPMDB200_ERR_INVALID_ARG, "owned rows [%lld, %lld) outside the %lld global rows",
                (long long)g_first, (long long)(g_first + R), (long long)G);
  if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
    return fail(SPMDB200_ERR_INVALID_ARG, "rank %d of %d (at most %d ranks)", rank, nranks, kMaxRanks);
  if ((g_first > 0) != (up_u != nullptr) || (g_first + R < G) != (dn_u != nullptr))
    return fail(SPMDB200_ERR_INVALID_ARG, "neighbour pointers must be given exactly where a neighbour exists");
  if ((up_u && (!up_v || !up_ws)) || (dn_u && (!dn_v || !dn_ws)))
    return fail(SPMDB200_ERR_INVALID_ARG, "incomplete neighbour (U, V, workspace)");
  if (up_u && (up_rows < H || up_rows > g_first))
    return fail(SPMDB200_ERR_INVALID_ARG, "neighbour above owns %lld rows: must be in [%lld, %lld]",
                (long long)up_rows, (long long)H, (long long)g_first);
  if (nranks > 1 && !all_ws) return fail(SPMDB200_ERR_INVALID_ARG, "all_ws is required for nranks > 1");
  if (sweeps < 0 || res_every < 0) return fail(SPMDB200_ERR_INVALID_ARG, "negative sweeps / res_every");
  if (res_every > 0 && sweeps / res_every > kMaxResSlots)
    return fail(SPMDB200_ERR_UNSUPPORTED, "at most %d residuals per slab run", kMaxResSlots);
  CHECK(check_jacobi_ws(ws, sizeof(JacobiWs)));
  if (sweeps == 0) return ok();
  Jacobi2dProblem p{};
  p.u = U + U_off;
  p.v = V + V_off;
  p.pitch = U_s0;
  p.h_local = U_n0;
  p.w = U_n1;
  p.row_lo = H;
  p.row_hi = R + H;
  p.g_row0 = g_first - H;
  p.g_rows = G;
  p.halo = (int)H;
  p.sweeps = sweeps;
  p.res_every = res_every;
  p.res_out = res_out;
  p.ws = static_cast<JacobiWs *>(ws);
  if (!jacobi2d_persistent_ok(p))
    return fail(SPMDB200_ERR_UNSUPPORTED, "slab arrays need 16-byte aligned rows (pitch multiple of 4 floats)");
  if (!deliveries) return fail(SPMDB200_ERR_INVALID_ARG, "deliveries (the halo-delivery count) is required");
  SlabPeers peers;
  peers.up_u = up_u;
  peers.up_v = up_v;
  peers.dn_u = dn_u;
  peers.dn_v = dn_v;
  peers.up_row = up_rows + H;  // our first owned rows are the bottom halo rows of the rank above
  peers.dn_row = 0;            // our last owned rows are the top halo rows of the rank below
  peers.up_flag = up_ws ? &static_cast<JacobiWs *>(up_ws)->from_below : nullptr;
  peers.dn_flag = dn_ws ? &static_cast<JacobiWs *>(dn_ws)->from_above : nullptr;
  peers.rank = rank;
  peers.nranks = nranks;
  for (int q = 0; q < nranks; ++q)
    peers.peer_ws[q] = static_cast<JacobiWs *>(all_ws ? all_ws[q] : (q == rank ? ws : nullptr));
  if (!peers.peer_ws[rank]) peers.peer_ws[rank] = static_cast<JacobiWs *>(ws);
  CUDA_TRY(run_jacobi2d_persistent(p, peers, (unsigned)*deliveries, (cudaStream_t)stream));
  *deliveries += jacobi2d_slab_deliveries(sweeps, res_every, U_n1, (int)H);
  return ok();
}

int spmdb200_jacobi3d_slab(float *U_base, float *U, int64_t U_off, int64_t U_n0, int64_t U_n1, int64_t U_n2,
                           int64_t U_s0, int64_t U_s1, int64_t U_s2, float *V_base, float *V, int64_t V_off,
                           int64_t V_n0, int64_t V_n1, int64_t V_n2, int64_t V_s0, int64_t V_s1, int64_t V_s2,
                           int64_t z_first, int64_t D, int64_t sweeps, int64_t res_every, double *res_out,
                           void *ws, float *up_u, float *up_v, void *up_ws, int64_t up_planes, float *dn_u,
                           float *dn_v, void *dn_ws, int rank, int nranks, void *const *all_ws,
                           int64_t *deliveries, void *stream) {
  (void)U_base; (void)V_base;
  CHECK(check3("U", U, U_off, U_n0, U_n1, U_n2, U_s0, U_s1, U_s2));
  CHECK(check3("V", V, V_off, V_n0, V_n1, V_n2, V_s0, V_s1, V_s2));
  if (U_n0 != V_n0 || U_n1 != V_n1 || U_n2 != V_n2 || U_s0 != V_s0 || U_s1 != V_s1 || U_s2 != V_s2)
    return fail(SPMDB200_ERR_INVALID_ARG, "U and V must have identical sizes and strides");
  const int64_t H = kSlabHalo3;
  if (U_n0 < 3 * H || U_n1 < 1 || U_n2 < 1)
    return fail(SPMDB200_ERR_INVALID_ARG, "a z-slab needs >= %lld owned planes plus %lld halo planes on each side",
                (long long)H, (long long)H);
  const int64_t Z = U_n0 - 2 * H;
  if (z_first < 0 || D < 1 || z_first + Z > D)
    return fail(SPMDB200_ERR_INVALID_ARG, "owned planes [%lld, %lld) outside the %lld global planes",
                (long long)z_first, (long long)(z_first + Z), (long long)D);
  if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
    return fail(SPMDB200_ERR_INVALID_ARG, "rank %d of %d (at most %d ranks)", rank, nranks, kMaxRanks);
  if ((z_first > 0) != (up_u != nullptr) || (z_first + Z < D) != (dn_u != nullptr))
    return fail(SPMDB200_ERR_INVALID_ARG, "neighbour pointers must be given exactly where a neighbour exists");
  if ((up_u && (!up_v || !up_ws)) || (dn_u && (!dn_v || !dn_ws)))
    return fail(SPMDB200_ERR_INVALID_ARG, "incomplete neighbour (U, V, workspace)");
  if (up_u && (up_planes < H || up_planes > z_first))
    return fail(SPMDB200_ERR_INVALID_ARG, "neighbour above owns %lld planes: must be in [%lld, %lld]",
                (long long)up_planes, (long long)H, (long long)z_first);
  if (nranks > 1 && !all_ws) return fail(SPMDB200_ERR_INVALID_ARG, "all_ws is required for nranks > 1");
  if (sweeps < 0 || res_every < 0) return fail(SPMDB200_ERR_INVALID_ARG, "negative sweeps / res_every");
  if (res_every > 0 && sweeps / res_every > kMaxResSlots)
    return fail(SPMDB200_ERR_UNSUPPORTED, "at most %d residuals per slab run", kMaxResSlots);
  CHECK(check_jacobi_ws(ws, sizeof(JacobiWs)));
  if (sweeps == 0) return ok();
  Jacobi3dProblem p{};
  p.u = U + U_off;
  p.v = V + V_off;
  p.d = U_n0;
  p.h = U_n1;
  p.w = U_n2;
  p.sz = U_s0;
  p.sy = U_s1;
  p.sx = U_s2;
  p.sweeps = sweeps;
  p.res_every = res_every;
  p.res_out = res_out;
  p.ws = static_cast<JacobiWs *>(ws);
  p.z_lo = H;
  p.z_hi = Z + H;
  p.g_z0 = z_first - H;
  p.g_d = D;
  p.halo = (int)H;
  if (!jacobi3d_tma_ok(p))
    return fail(SPMDB200_ERR_UNSUPPORTED,
                "z-slab arrays need contiguous x and 16-byte aligned rows and planes (pitch multiple of 4 floats)");
  SlabPeers peers;
  peers.up_u = up_u;
  peers.up_v = up_v;
  peers.dn_u = dn_u;
  peers.dn_v = dn_v;
  // plane indices: our first owned plane lands in the first bottom halo plane
  // of the rank above; our last H owned planes land in the top halo planes
  // [0, H) of the rank below
  peers.up_row = up_planes + H;
  peers.dn_row = 0;
  peers.up_flag = up_ws ? &static_cast<JacobiWs *>(up_ws)->from_below : nullptr;
  peers.dn_flag = dn_ws ? &static_cast<JacobiWs *>(dn_ws)->from_above : nullptr;
  peers.rank = rank;
  peers.nranks = nranks;
  for (int q = 0; q < nranks; ++q)
    peers.peer_ws[q] = static_cast<JacobiWs *>(all_ws ? all_ws[q] : (q == rank ? ws : nullptr));
  if (!peers.peer_ws[rank]) peers.peer_ws[rank] = static_cast<JacobiWs *>(ws);
  if (!deliveries) return fail(SPMDB200_ERR_INVALID_ARG, "deliveries (the halo-delivery count) is required");
  // Each launch of the run starts from a fresh grid barrier (stream-ordered
  // memsets); the status word and the delivery counters carry over.
  CUDA_TRY(run_jacobi3d_tb(p, peers, (unsigned)*deliveries, (cudaStream_t)stream));
  *deliveries += jacobi3d_slab_deliveries(sweeps, res_every, U_n1, U_n2);
  return ok();
}

int spmdb200_jacobi2d_slab_residuals(void *ws, int nranks, int64_t nres, double *res_host) {
  if (!ws) return fail(SPMDB200_ERR_WORKSPACE, "null workspace");
  if (nranks < 1 || nranks > kMaxRanks || nres < 0 || nres > kMaxResSlots || (nres > 0 && !res_host))
    return fail(SPMDB200_ERR_INVALID_ARG, "bad nranks / nres / output");
  if (nres == 0) return ok();
  std::vector<double> slots((size_t)nres * kMaxRanks);
  CUDA_TRY(cudaMemcpy(slots.data(), static_cast<JacobiWs *>(ws)->res_slots, slots.size() * sizeof(double),
                      cudaMemcpyDeviceToHost));
  for (int64_t r = 0; r < nres; ++r) {
    double t = 0.0;
    for (int q = 0; q < nranks; ++q) t += slots[(size_t)r * kMaxRanks + q];
    res_host[r] = t;
  }
  return ok();
}

int spmdb200_dev_alloc(size_t bytes, void **out) {
  if (!out) return fail(SPMDB200_ERR_INVALID_ARG, "null output pointer");
  *out = nullptr;
  CHECK(have_device());
  CUDA_TRY(cudaMalloc(out, bytes ? bytes : 256));
  return ok();
}
int spmdb200_dev_free(void *p) {
  if (p) CUDA_TRY(cudaFree(p));
  return ok();
}
int spmdb200_memcpy(void *dst, const void *src, size_t bytes, void *stream) {
  if (bytes == 0) return ok();
  if (!dst || !src) return fail(SPMDB200_ERR_INVALID_ARG, "null pointer");
  CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, (cudaStream_t)stream));
  CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
  return ok();
}
int spmdb200_memcpy_async(void *dst, const void *src, size_t bytes, void *stream) {
  if (bytes == 0) return ok();
  if (!dst || !src) return fail(SPMDB200_ERR_INVALID_ARG, "null pointer");
  CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, (cudaStream_t)stream));
  return ok();
}
int spmdb200_ipc_handle(void *dev_ptr, void *handle64_out) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  if (!dev_ptr || !handle64_out) return fail(SPMDB200_ERR_INVALID_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  CUDA_TRY(cudaIpcGetMemHandle(&h, dev_ptr));
  memcpy(handle64_out, &h, sizeof(h));
  return ok();
}
int spmdb200_ipc_open(const void *handle64, void **dev_ptr_out) {
  if (!handle64 || !dev_ptr_out) return fail(SPMDB200_ERR_INVALID_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  CUDA_TRY(cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
  return ok();
}
int spmdb200_ipc_close(void *dev_ptr) {
  if (dev_ptr) CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr));
  return ok();
}
int spmdb200_fill_jacobi3d_input(float *p, int64_t plane_stride, int64_t row_stride, int64_t planes, int64_t H,
                                 int64_t W, int64_t g_z0, int64_t D, uint64_t seed, void *stream) {
  if (planes < 0 || H < 0 || W < 0 || row_stride < W || plane_stride < row_stride * H ||
      (planes > 0 && H > 0 && W > 0 && !p))
    return fail(SPMDB200_ERR_INVALID_ARG, "bad fill arguments");
  CUDA_TRY(launch_fill_jacobi3d_input(p, plane_stride, row_stride, planes, H, W, g_z0, D, seed,
                                      (cudaStream_t)stream));
  return ok();
}
int spmdb200_fill_jacobi_input(float *p, int64_t pitch, int64_t rows, int64_t W, int64_t g_row0, int64_t G,
                               uint64_t seed, void *stream) {
  if (rows < 0 || W < 0 || pitch < W || (rows > 0 && W > 0 && !p))
    return fail(SPMDB200_ERR_INVALID_ARG, "bad fill arguments");
  CUDA_TRY(launch_fill_jacobi_input(p, pitch, rows, W, g_row0, G, seed, (cudaStream_t)stream));
  return ok();
}

// ---------------------------------------------------------------- host entries (A)
static int ewise_host_impl(float *A, int64_t A_off, int64_t A_size, int64_t A_st, float *B, int64_t B_off,
                           int64_t B_size, int64_t B_st, float *C, int64_t C_off, int64_t C_size, int64_t C_st,
                           int64_t N) {
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  CHECK(check1("B", B, B_off, B_size, B_st, N));
  CHECK(check1("C", C, C_off, C_size, C_st, N));
  if (N == 0) return ok();
  CHECK(have_device());
  void *da, *db, *dc;
  CHECK(staging(0, (size_t)N * 4, &da));
  CHECK(staging(1, (size_t)N * 4, &db));
  CHECK(staging(2, (size_t)N * 4, &dc));
  CHECK(h2d_1d(da, A + A_off, N, A_st, 4));
  CHECK(h2d_1d(db, B + B_off, N, B_st, 4));
  CUDA_TRY(launch_ewise_add(View1{(float *)da, N, 1}, View1{(float *)db, N, 1}, View1{(float *)dc, N, 1}, N, 0));
  CHECK(d2h_1d(C + C_off, dc, N, C_st, 4));
  return ok();
}

void ewise(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
           float *B_base, float *B, int64_t B_off, int64_t B_size, int64_t B_st,
           float *C_base, float *C, int64_t C_off, int64_t C_size, int64_t C_st, int64_t N) {
  (void)A_base; (void)B_base; (void)C_base;
  report_void("ewise", ewise_host_impl(A, A_off, A_size, A_st, B, B_off, B_size, B_st, C, C_off, C_size, C_st, N));
}

static int stencil_host_impl(float *A, int64_t A_off, int64_t A_n0, int64_t A_n1, int64_t A_s0, int64_t A_s1,
                             float *B, int64_t B_off, int64_t B_n0, int64_t B_n1, int64_t B_s0, int64_t B_s1,
                             int64_t N, int64_t M) {
  CHECK(check2("A", A, A_off, A_n0, A_n1, A_s0, A_s1));
  CHECK(check2("B", B, B_off, B_n0, B_n1, B_s0, B_s1));
  if (N < 0 || M < 0 || N > B_n0 || M > B_n1)
    return fail(SPMDB200_ERR_INVALID_ARG, "loop bounds exceed B's sizes");
  if (N == 0 || M == 0) return ok();
  CHECK(have_device());
  const int64_t ap = round_up4(A_n1 > 0 ? A_n1 : 1), bp = round_up4(M);
  void *da, *db;
  CHECK(staging(0, (size_t)(A_n0 > 0 ? A_n0 : 1) * ap * 4, &da));
  CHECK(staging(1, (size_t)N * bp * 4, &db));
  CHECK(h2d_2d((float *)da, ap, A ? A + A_off : nullptr, A_n0, A_n1, A_s0, A_s1));
  CUDA_TRY(launch_stencil3(View2{(float *)da, A_n0, A_n1, ap, 1}, View2{(float *)db, N, M, bp, 1}, N, M, 0));
  CHECK(d2h_2d(B + B_off, N, M, B_s0, B_s1, (float *)db, bp));
  return ok();
}

void stencil_cpu(float *A_base, float *A, int64_t A_off, int64_t A_n0, int64_t A_n1, int64_t A_s0, int64_t A_s1,
                 float *B_base, float *B, int64_t B_off, int64_t B_n0, int64_t B_n1, int64_t B_s0, int64_t B_s1,
                 int64_t N, int64_t M) {
  (void)A_base; (void)B_base;
  report_void("stencil_cpu",
              stencil_host_impl(A, A_off, A_n0, A_n1, A_s0, A_s1, B, B_off, B_n0, B_n1, B_s0, B_s1, N, M));
}

static int sum_host_impl(float *A, int64_t A_off, int64_t A_size, int64_t A_st, float *o, int64_t o_off, int64_t N) {
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  if (!o || o_off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "out: null pointer or negative offset");
  CHECK(have_device());
  void *da, *dout, *dws;
  CHECK(staging(0, (size_t)(N > 0 ? N : 1) * 4, &da));
  CHECK(staging(1, 256, &dout));
  const size_t wsb = sum_f32_workspace_bytes(N);
  CHECK(staging(2, wsb, &dws));
  CHECK(h2d_1d(da, A ? A + A_off : nullptr, N, A_st, 4));
  CUDA_TRY(cudaMemcpy(dout, o + o_off, 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemset(dws, 0, wsb));  // the whole workspace: ticket and partial words start at zero
  CUDA_TRY(launch_sum_f32(View1{(float *)da, N, 1}, (float *)dout, N, dws, 0));
  CUDA_TRY(cudaMemcpy(o + o_off, dout, 4, cudaMemcpyDeviceToHost));
  return ok();
}

void atomic_sum(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                float *o_base, float *o, int64_t o_off, int64_t N) {
  (void)A_base; (void)o_base;
  report_void("atomic_sum", sum_host_impl(A, A_off, A_size, A_st, o, o_off, N));
}

void hierarchical_sum(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                      float *o_base, float *o, int64_t o_off, int64_t N) {
  (void)A_base; (void)o_base;
  report_void("hierarchical_sum", sum_host_impl(A, A_off, A_size, A_st, o, o_off, N));
}

// ---------------------------------------------------------------- host entries (C)
int spmdb200_axpy_host(float a, float *X_base, float *X, int64_t X_off, int64_t X_size, int64_t X_st,
                       float *Y_base, float *Y, int64_t Y_off, int64_t Y_size, int64_t Y_st, int64_t N) {
  (void)X_base; (void)Y_base;
  CHECK(check1("X", X, X_off, X_size, X_st, N));
  CHECK(check1("Y", Y, Y_off, Y_size, Y_st, N));
  if (N == 0) return ok();
  CHECK(have_device());
  void *dx, *dy;
  CHECK(staging(0, (size_t)N * 4, &dx));
  CHECK(staging(1, (size_t)N * 4, &dy));
  CHECK(h2d_1d(dx, X + X_off, N, X_st, 4));
  CHECK(h2d_1d(dy, Y + Y_off, N, Y_st, 4));
  CUDA_TRY(launch_axpy(a, View1{(float *)dx, N, 1}, View1{(float *)dy, N, 1}, N, 0));
  CHECK(d2h_1d(Y + Y_off, dy, N, Y_st, 4));
  return ok();
}

int spmdb200_sum_f32_host(float *A_base, float *A, int64_t A_off, int64_t A_size, int64_t A_st,
                          float *o_base, float *o, int64_t o_off, int64_t N) {
  (void)A_base; (void)o_base;
  return sum_host_impl(A, A_off, A_size, A_st, o, o_off, N);
}

int spmdb200_sum_i32_host(int32_t *A_base, int32_t *A, int64_t A_off, int64_t A_size, int64_t A_st,
                          int32_t *o_base, int32_t *o, int64_t o_off, int64_t N) {
  (void)A_base; (void)o_base;
  CHECK(check1("A", A, A_off, A_size, A_st, N));
  if (!o || o_off < 0) return fail(SPMDB200_ERR_INVALID_ARG, "out: null pointer or negative offset");
  if (N == 0) return ok();
  CHECK(have_device());
  void *da, *dout;
  CHECK(staging(0, (size_t)N * 4, &da));
  CHECK(staging(1, 256, &dout));
  CHECK(h2d_1d(da, A + A_off, N, A_st, 4));
  CUDA_TRY(cudaMemcpy(dout, o + o_off, 4, cudaMemcpyHostToDevice));
  CUDA_TRY(launch_sum_i32((int32_t *)da, 1, (int32_t *)dout, N, 0));
  CUDA_TRY(cudaMemcpy(o + o_off, dout, 4, cudaMemcpyDeviceToHost));
  return ok();
}

int spmdb200_jacobi2d_host(float *U_base, float *U, int64_t U_off, int64_t U_n0, int64_t U_n1, int64_t U_s0,
                           int64_t U_s1, int64_t sweeps, int64_t res_every, double *res_out) {
  (void)U_base;
  CHECK(check2("U", U, U_off, U_n0, U_n1, U_s0, U_s1));
  CHECK(check_res(sweeps, res_every, res_out));
  if (U_n0 == 0 || U_n1 == 0) return ok();
  CHECK(have_device());
  const int64_t dp = round_up4(U_n1);  // 16-byte row pitch on the device: always the TMA path
  const size_t grid_bytes = (size_t)U_n0 * dp * 4;
  const int64_t nres = res_every > 0 ? sweeps / res_every : 0;
  void *du, *dv, *dws, *dres;
  CHECK(staging(0, grid_bytes, &du));
  CHECK(staging(1, grid_bytes, &dv));
  CHECK(staging(2, sizeof(JacobiWs), &dws));
  CHECK(staging(3, (size_t)(nres > 0 ? nres : 1) * 8, &dres));
  CHECK(h2d_2d((float *)du, dp, U + U_off, U_n0, U_n1, U_s0, U_s1));
  const int st = spmdb200_jacobi2d(nullptr, (float *)du, 0, U_n0, U_n1, dp, 1, nullptr, (float *)dv, 0, U_n0, U_n1,
                                    dp, 1, sweeps, res_every, (double *)dres, dws, sizeof(JacobiWs), nullptr);
  if (st != SPMDB200_OK) return st;
  CHECK(jacobi_status_from_ws((JacobiWs *)dws, 0));
  const float *fin = (sweeps % 2 == 0) ? (float *)du : (float *)dv;
  CHECK(d2h_2d(U + U_off, U_n0, U_n1, U_s0, U_s1, fin, dp));
  if (nres > 0) CUDA_TRY(cudaMemcpy(res_out, dres, (size_t)nres * 8, cudaMemcpyDeviceToHost));
  return ok();
}

// A batch of independent host grids through two device slots.  Grid k uses
// slot k % 2.  Uploads run on `in`, sweeps on `comp`, downloads on `out`.
// Grid k's upload waits for grid k-2's download, which was the last reader of
// that slot.  So grid k+1's upload and grid k-1's download overlap grid k's
// sweeps: PCIe copies both ways while HBM serves the sweep kernel.  Residuals
// and status words come back through a pinned host buffer: a download into
// pageable memory would block this thread and serialise the pipeline.
int spmdb200_jacobi2d_host_batch(int64_t count, float *const *U, int64_t U_off, int64_t U_n0, int64_t U_n1,
                                 int64_t U_s0, int64_t U_s1, int64_t sweeps, int64_t res_every,
                                 double *const *res_out) {
  if (count < 0 || (count > 0 && !U)) return fail(SPMDB200_ERR_INVALID_ARG, "negative count or null grid list");
  if (U_s1 != 1) return fail(SPMDB200_ERR_UNSUPPORTED, "batch grids need contiguous rows (stride1 == 1)");
  const int64_t nres = res_every > 0 ? sweeps / res_every : 0;
  for (int64_t k = 0; k < count; ++k) {
    CHECK(check2("U", U[k], U_off, U_n0, U_n1, U_s0, U_s1));
    CHECK(check_res(sweeps, res_every, res_out ? res_out[k] : nullptr));
    if (U_n0 > 0 && U_n1 > 0 && U_s0 < U_n1) return fail(SPMDB200_ERR_INVALID_ARG, "U: row pitch below the row length");
  }
  if (count == 0 || U_n0 == 0 || U_n1 == 0) return ok();
  CHECK(have_device());
  const int64_t dp = round_up4(U_n1);
  const size_t grid_bytes = (size_t)U_n0 * dp * 4, rows_bytes = (size_t)U_n1 * 4;
  void *du[2], *dv[2], *dws[2], *dres[2];
  for (int j = 0; j < 2; ++j) {  // staging slots 8..15: apart from the single-grid entries' slots
    CHECK(staging(8 + 4 * j, grid_bytes, &du[j]));
    CHECK(staging(9 + 4 * j, grid_bytes, &dv[j]));
    CHECK(staging(10 + 4 * j, sizeof(JacobiWs), &dws[j]));
    CHECK(staging(11 + 4 * j, (size_t)(nres > 0 ? nres : 1) * 8, &dres[j]));
  }
  cudaStream_t in = nullptr, comp = nullptr, out = nullptr;
  cudaEvent_t ev[6] = {};  // in_done[2], comp_done[2], out_done[2]
  char *pin = nullptr;     // per grid: status word (8 B) + residuals
  const size_t per_grid = 8 + (size_t)nres * 8;
  int st = SPMDB200_OK;
  auto body = [&]() -> int {
    CUDA_TRY(cudaStreamCreateWithFlags(&in, cudaStreamNonBlocking));
    CUDA_TRY(cudaStreamCreateWithFlags(&comp, cudaStreamNonBlocking));
    CUDA_TRY(cudaStreamCreateWithFlags(&out, cudaStreamNonBlocking));
    for (auto &e : ev) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    CUDA_TRY(cudaHostAlloc((void **)&pin, per_grid * (size_t)count, cudaHostAllocDefault));
    // Status words read as OK when a grid runs no sweep (zero sweeps launch nothing).
    for (int j = 0; j < 2; ++j) CUDA_TRY(cudaMemsetAsync(dws[j], 0, 256, comp));
    for (int64_t k = 0; k < count; ++k) {
      const int j = (int)(k & 1);
      float *hu = U[k] + U_off;
      if (k >= 2) CUDA_TRY(cudaStreamWaitEvent(in, ev[4 + j], 0));
      CUDA_TRY(cudaMemcpy2DAsync(du[j], (size_t)dp * 4, hu, (size_t)U_s0 * 4, rows_bytes, (size_t)U_n0,
                                 cudaMemcpyHostToDevice, in));
      CUDA_TRY(cudaEventRecord(ev[j], in));
      CUDA_TRY(cudaStreamWaitEvent(comp, ev[j], 0));
      CHECK(spmdb200_jacobi2d(nullptr, (float *)du[j], 0, U_n0, U_n1, dp, 1, nullptr, (float *)dv[j], 0, U_n0, U_n1,
                              dp, 1, sweeps, res_every, (double *)dres[j], dws[j], sizeof(JacobiWs), comp));
      CUDA_TRY(cudaEventRecord(ev[2 + j], comp));
      CUDA_TRY(cudaStreamWaitEvent(out, ev[2 + j], 0));
      const void *fin = (sweeps % 2 == 0) ? du[j] : dv[j];
      CUDA_TRY(cudaMemcpy2DAsync(hu, (size_t)U_s0 * 4, fin, (size_t)dp * 4, rows_bytes, (size_t)U_n0,
                                 cudaMemcpyDeviceToHost, out));
      char *slot = pin + per_grid * (size_t)k;
      CUDA_TRY(cudaMemcpyAsync(slot, &static_cast<JacobiWs *>(dws[j])->status, sizeof(int), cudaMemcpyDeviceToHost,
                               out));
      if (nres > 0) CUDA_TRY(cudaMemcpyAsync(slot + 8, dres[j], (size_t)nres * 8, cudaMemcpyDeviceToHost, out));
      CUDA_TRY(cudaEventRecord(ev[4 + j], out));
    }
    CUDA_TRY(cudaStreamSynchronize(out));
    for (int64_t k = 0; k < count; ++k) {
      const char *slot = pin + per_grid * (size_t)k;
      int dev_status = 0;
      std::memcpy(&dev_status, slot, sizeof(int));
      if (dev_status != kDevOk)
        return fail(SPMDB200_ERR_TIMEOUT, "grid %lld: a bounded device wait expired (status %d)", (long long)k,
                    dev_status);
      if (nres > 0 && res_out && res_out[k]) std::memcpy(res_out[k], slot + 8, (size_t)nres * 8);
    }
    return SPMDB200_OK;
  };
  st = body();
  // Every stream drains before its resources go, on success and on error.
  for (cudaStream_t s : {in, comp, out})
    if (s) cudaStreamSynchronize(s);
  for (cudaStream_t s : {in, comp, out})
    if (s) cudaStreamDestroy(s);
  for (auto e : ev)
    if (e) cudaEventDestroy(e);
  if (pin) cudaFreeHost(pin);
  if (st != SPMDB200_OK) return st;
  return ok();
}

}  // extern "C"
