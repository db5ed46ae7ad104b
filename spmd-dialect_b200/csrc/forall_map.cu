// forall_map.cu -- elementwise spmd.forall with a general f32 body.
//
// The reference lowers every spmd.forall body to one GPU thread per point:
// the lane lowering of lib/Conversion/SPMDToGPU/SPMDToGPU.cpp:491-580 with the
// bounds guard of lib/Transforms/MaterializeTilingAndMapping.cpp:153-173; its
// elementwise instance is C = A + B (test/SPMD/lower-to-gpu-nvptx.mlir:54-71),
// and the dialect's tests carry others (C = A * B over a 2-D domain,
// test/SPMD/ewise.mlir:50-64; B = A + 1, test/SPMD/cross-pipeline-regression.mlir:
// 132-146).  The library's fixed kernels cover C = A + B and y = a*x + y; this
// file runs any body of f32 arith ops, given as a straight-line program (the
// body's SSA ops in order, registers allocated by the caller; opcodes and
// encoding in include/spmd_b200.h, SPMDB200_MAP_*).
//
// Execution: one pass over the domain, grid-stride over chunks of
// 256 threads x 2 slots x 4 points.  A thread owns two float4 groups of
// points per chunk (four consecutive points each for aligned contiguous
// views; otherwise points 256 apart, see MapMode) and keeps the program's
// registers for them in its own rows of shared memory (row r, slot s at
// [(r*2 + s)*256 + thread]:
// 16-byte accesses by consecutive threads, no bank conflicts, no barriers,
// since no thread reads another's rows).  Every instruction is decoded once
// per 8 points, uniformly across the warp.  The loads of all inputs are
// issued before the first operation (the LOADs are a prefix of the program),
// so a chunk's input traffic is in flight at once.  Contiguous, 16-byte
// aligned views take 128-bit loads and stores; other views 4-byte accesses,
// 32 consecutive points per warp access (MapMode below).
//
// Arithmetic is spelled with the _rn intrinsics (round to nearest even, never
// contracted to an FMA), so the result equals a CPU evaluation of the same
// program op by op; maximumf / minimumf follow arith's NaN and signed-zero
// rules.
#include <cmath>
#include <cstdint>

#include "../../include/spmd_b200.h"
#include "common.cuh"
#include "internal.h"

namespace spmdb200 {
namespace {

constexpr int kMapThreads = 256;
constexpr int kMaxLoads = SPMDB200_MAP_MAX_INPUTS;

// float4 groups a thread owns per chunk, for a body with nl inputs.
constexpr int map_slots(int /*nl*/) { return 2; }
constexpr int64_t map_chunk(int nl) { return (int64_t)kMapThreads * map_slots(nl) * 4; }

struct MapParams {
  const float *ld_src[kMaxLoads];  // source of the i-th leading LOAD
  int64_t ld_st[kMaxLoads][3];     // its strides (elements), dimension 0 outermost
  int ld_dst[kMaxLoads];           // its destination register
  float *out;
  int64_t out_st[3];
  int64_t size[3];  // domain, padded to rank 3 with leading 1s
  int64_t n;        // points
  int32_t code[2 * SPMDB200_MAP_MAX_INSNS];
  float consts[SPMDB200_MAP_MAX_CONSTS];
  int n_insns;  // all instructions, the LOAD prefix and the final STORE included
  int out_reg;
  int n_regs;
  int64_t ld_span[kMaxLoads];  // elements each view covers (1 + max offset), for checked builds
  int64_t out_span;
};

#ifdef SPMDB200_CHECKED
__device__ unsigned long long g_check_first;  // first out-of-range access (see common.cuh)
#define IN_RANGE(cond, site, idx) record_check(&g_check_first, (cond), (site), (long long)(idx))
#else
#define IN_RANGE(cond, site, idx) true
#endif

__device__ __forceinline__ float f_maximum(float a, float b) {
  if (isnan(a) || isnan(b)) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
__device__ __forceinline__ float f_minimum(float a, float b) {
  if (isnan(a) || isnan(b)) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

// arith.cmpf with the predicate numbering of include/spmd_b200.h.
__device__ __forceinline__ bool cmpf(int pred, float x, float y) {
  const bool u = isnan(x) || isnan(y);
  switch (pred) {
    case 1: return x == y;
    case 2: return x > y;
    case 3: return x >= y;
    case 4: return x < y;
    case 5: return x <= y;
    case 6: return !u && x != y;
    case 7: return !u;
    case 8: return u || x == y;
    case 9: return u || x > y;
    case 10: return u || x >= y;
    case 11: return u || x < y;
    case 12: return u || x <= y;
    case 13: return x != y;
    case 14: return u;
    case 15: return true;
    default: return false;
  }
}

__device__ __forceinline__ float bool_f(bool b) { return b ? 1.0f : 0.0f; }

// rd = f(ra, rb) for each of the thread's S slots (float4s kMapThreads
// apart).  Operands are read before the result is written, so rd may be ra or
// rb.
template <int S, class F>
__device__ __forceinline__ void apply(float4 *rd, const float4 *ra, const float4 *rb, F f) {
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int o = s * kMapThreads;
    const float4 x = ra[o], y = rb[o];
    rd[o] = make_float4(f(x.x, y.x), f(x.y, y.y), f(x.z, y.z), f(x.w, y.w));
  }
}

// How a launch addresses its views.  VEC: every view contiguous in the
// domain's row-major order and 16-byte aligned: a thread's float4 holds four
// consecutive points, moved with 128-bit accesses at the flat index.
// CONTIG (every view contiguous, some not 16-byte aligned) and GENERAL (any
// strides): component k of slot s is point (4s + k) * threads + thread of the
// chunk, so a warp access covers 32 consecutive points; CONTIG addresses them
// at the flat index, GENERAL from the (i0, i1, i2) index of the thread's
// first point, decomposed once per chunk, with each view's offset advanced
// along the row and plane wraps of the following steps.
// ROWS (strided views whose rows hold at least kRowsMin points): a chunk is
// a segment of one row, component k of slot s its column (4s + k) *
// threads + thread, each view's offset the row's plus the column times the
// column stride, advanced by one add per point.
enum MapMode { kVec = 0, kContig = 1, kGeneral = 2, kRows = 3 };
constexpr int64_t kRowsMin = 1024;

// Offset of flat point e in a view with strides st over the rank-3 domain sz.
__device__ __forceinline__ int64_t point_offset(int64_t e, const int64_t *sz, const int64_t *st) {
  const int64_t i2 = e % sz[2], q = e / sz[2];
  const int64_t i1 = q % sz[1], i0 = q / sz[1];
  return i0 * st[0] + i1 * st[1] + i2 * st[2];
}

// GENERAL: the (i0, i1, i2) index of flat point e.
struct Idx3 {
  int64_t i0, i1, i2;
};
__device__ __forceinline__ Idx3 point_index(const MapParams &p, int64_t e) {
  Idx3 x;
  x.i2 = e % p.size[2];
  const int64_t q = e / p.size[2];
  x.i1 = q % p.size[1];
  x.i0 = q / p.size[1];
  return x;
}

// GENERAL, per chunk: the index of the thread's first point and, for each of
// the 4 * S - 1 steps of `threads` points that follow, whether it wraps a row
// (bit 2j) and a plane (bit 2j + 1).  Rows shorter than `threads` can wrap
// more than once per step: those are decomposed point by point (`multi`).
struct ChunkIdx {
  Idx3 x;
  uint32_t wraps;
  bool multi;
};
template <int S>
__device__ __forceinline__ ChunkIdx chunk_index(const MapParams &p, int64_t first) {
  ChunkIdx g;
  g.x = point_index(p, first);
  g.wraps = 0;
  g.multi = p.size[2] < kMapThreads;
  if (!g.multi) {
    Idx3 y = g.x;
#pragma unroll
    for (int j = 0; j < 4 * S - 1; ++j) {
      y.i2 += kMapThreads;
      if (y.i2 >= p.size[2]) {
        y.i2 -= p.size[2];
        g.wraps |= 1u << (2 * j);
        if (++y.i1 >= p.size[1]) {
          y.i1 = 0;
          ++y.i0;
          g.wraps |= 2u << (2 * j);
        }
      }
    }
  }
  return g;
}

// GENERAL: the 4 * S points of a chunk for one view (component k of slot s =
// point first + (4s + k) * threads), the offset advanced by adds along the
// chunk's recorded wraps.
template <int S>
__device__ __forceinline__ void load_general(const float *src, const int64_t *st, int64_t span, const MapParams &p,
                                             int64_t first, const ChunkIdx &g, float4 *out) {
  int64_t o = g.x.i0 * st[0] + g.x.i1 * st[1] + g.x.i2 * st[2];
  const int64_t d_step = (int64_t)kMapThreads * st[2];
  const int64_t d_row = st[1] - p.size[2] * st[2], d_plane = st[0] - p.size[1] * st[1];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * s + k;
      const int64_t q = first + (int64_t)j * kMapThreads;
      const int64_t oq = g.multi ? point_offset(q, p.size, st) : o;
      v[k] = 0.0f;
      if (q < p.n && IN_RANGE(oq >= 0 && oq < span, 1, oq)) v[k] = src[oq];
      if (j < 4 * S - 1) {
        o += d_step;
        if (g.wraps & (1u << (2 * j))) o += d_row;
        if (g.wraps & (2u << (2 * j))) o += d_plane;
      }
    }
    out[s] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

template <int S>
__device__ __forceinline__ void store_general(const MapParams &p, int64_t first, const ChunkIdx &g,
                                              const float4 *vals, int row) {
  const int64_t *st = p.out_st;
  int64_t o = g.x.i0 * st[0] + g.x.i1 * st[1] + g.x.i2 * st[2];
  const int64_t d_step = (int64_t)kMapThreads * st[2];
  const int64_t d_row = st[1] - p.size[2] * st[2], d_plane = st[0] - p.size[1] * st[1];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const float4 v4 = vals[s * row];
    const float w[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * s + k;
      const int64_t q = first + (int64_t)j * kMapThreads;
      const int64_t oq = g.multi ? point_offset(q, p.size, st) : o;
      if (q < p.n && IN_RANGE(oq >= 0 && oq < p.out_span, 2, oq)) p.out[oq] = w[k];
      if (j < 4 * S - 1) {
        o += d_step;
        if (g.wraps & (1u << (2 * j))) o += d_row;
        if (g.wraps & (2u << (2 * j))) o += d_plane;
      }
    }
  }
}

// ROWS: the chunk's row (i0, i1) and the thread's first column.
struct RowChunk {
  int64_t i0, i1, col0;
};

template <int S>
__device__ __forceinline__ void load_rows(const float *src, const int64_t *st, int64_t span, const MapParams &p,
                                          const RowChunk &rc, float4 *out) {
  int64_t o = rc.i0 * st[0] + rc.i1 * st[1] + rc.col0 * st[2];
  const int64_t d_step = (int64_t)kMapThreads * st[2];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t col = rc.col0 + (int64_t)(4 * s + k) * kMapThreads;
      v[k] = 0.0f;
      if (col < p.size[2] && IN_RANGE(o >= 0 && o < span, 1, o)) v[k] = src[o];
      o += d_step;
    }
    out[s] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

template <int S>
__device__ __forceinline__ void store_rows(const MapParams &p, const RowChunk &rc, const float4 *vals, int row) {
  const int64_t *st = p.out_st;
  int64_t o = rc.i0 * st[0] + rc.i1 * st[1] + rc.col0 * st[2];
  const int64_t d_step = (int64_t)kMapThreads * st[2];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const float4 v4 = vals[s * row];
    const float w[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t col = rc.col0 + (int64_t)(4 * s + k) * kMapThreads;
      if (col < p.size[2] && IN_RANGE(o >= 0 && o < p.out_span, 2, o)) p.out[o] = w[k];
      o += d_step;
    }
  }
}

// VEC / CONTIG: the four points of a slot whose first point is e (VEC:
// e..e+3; CONTIG: threads apart); points at or past n read as 0.
template <int MODE>
__device__ __forceinline__ float4 load4(const float *src, int64_t span, const MapParams &p, int64_t e) {
  if (MODE == kVec && e + 3 < p.n) {
    if (!IN_RANGE(e + 3 < span, 1, e)) return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    return ld_f4(src + e);
  }
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = 0.0f;
    const int64_t q = MODE == kVec ? e + k : e + (int64_t)k * kMapThreads;
    if (q < p.n && IN_RANGE(q < span, 1, q)) v[k] = src[q];
  }
  return make_float4(v[0], v[1], v[2], v[3]);
}

template <int MODE>
__device__ __forceinline__ void store4(const MapParams &p, int64_t e, float4 v) {
  if (MODE == kVec && e + 3 < p.n) {
    if (IN_RANGE(e + 3 < p.out_span, 2, e)) st_f4(p.out + e, v);
    return;
  }
  const float w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t q = MODE == kVec ? e + k : e + (int64_t)k * kMapThreads;
    if (q < p.n && IN_RANGE(q < p.out_span, 2, q)) p.out[q] = w[k];
  }
}

// NL: the number of leading LOAD instructions (1..8); MODE: a MapMode.
template <int NL, int MODE>
__global__ void __launch_bounds__(kMapThreads) forall_map_kernel(const __grid_constant__ MapParams p) {
  constexpr int S = map_slots(NL);
  constexpr int64_t kChunk = map_chunk(NL);
  extern __shared__ float4 regs[];  // n_regs x S x kMapThreads
  __shared__ int32_t s_code[2 * SPMDB200_MAP_MAX_INSNS];
  __shared__ float s_consts[SPMDB200_MAP_MAX_CONSTS];
  const int t = threadIdx.x;
  for (int i = t; i < 2 * p.n_insns; i += kMapThreads) s_code[i] = p.code[i];
  for (int i = t; i < SPMDB200_MAP_MAX_CONSTS; i += kMapThreads) s_consts[i] = p.consts[i];
  __syncthreads();
  constexpr int kRow = S * kMapThreads;  // float4s per register
  float4 *mine = regs + t;
  const int64_t row_chunks = MODE == kRows ? (p.size[2] + kChunk - 1) / kChunk : 1;  // chunks per row
  const int64_t nchunks = MODE == kRows ? p.size[0] * p.size[1] * row_chunks : (p.n + kChunk - 1) / kChunk;
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    // slot s starts at base + s * 4 * threads (VEC: its components are
    // consecutive; otherwise threads apart)
    const int64_t base = c * kChunk + (MODE == kVec ? 4 * (int64_t)t : (int64_t)t);
    ChunkIdx g{};
    if constexpr (MODE == kGeneral) g = chunk_index<S>(p, base);
    RowChunk rc{};
    if constexpr (MODE == kRows) {
      const int64_t r = c / row_chunks;
      rc.i0 = r / p.size[1];
      rc.i1 = r - rc.i0 * p.size[1];
      rc.col0 = (c - r * row_chunks) * kChunk + t;
    }
    float4 v[NL][S];
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      if constexpr (MODE == kGeneral) {
        load_general<S>(p.ld_src[i], p.ld_st[i], p.ld_span[i], p, base, g, v[i]);
      } else if constexpr (MODE == kRows) {
        load_rows<S>(p.ld_src[i], p.ld_st[i], p.ld_span[i], p, rc, v[i]);
      } else {
#pragma unroll
        for (int s = 0; s < S; ++s)
          v[i][s] = load4<MODE>(p.ld_src[i], p.ld_span[i], p, base + (int64_t)s * 4 * kMapThreads);
      }
    }
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      if (!IN_RANGE(p.ld_dst[i] < p.n_regs, 3, p.ld_dst[i])) continue;
#pragma unroll
      for (int s = 0; s < S; ++s) mine[p.ld_dst[i] * kRow + s * kMapThreads] = v[i][s];
    }
    for (int pc = NL; pc < p.n_insns - 1; ++pc) {
      const int w0 = s_code[2 * pc], aux = s_code[2 * pc + 1];
      if (!IN_RANGE(((w0 >> 8) & 255) < p.n_regs && ((w0 >> 16) & 255) < p.n_regs &&
                        (int)((unsigned)w0 >> 24) < p.n_regs,
                    3, pc))
        continue;
      float4 *rd = mine + ((w0 >> 8) & 255) * kRow;
      const float4 *ra = mine + ((w0 >> 16) & 255) * kRow;
      const float4 *rb = mine + ((unsigned)w0 >> 24) * kRow;
      switch (w0 & 255) {
        case SPMDB200_MAP_CONST: {
          const float cv = s_consts[aux];
#pragma unroll
          for (int s = 0; s < S; ++s) rd[s * kMapThreads] = make_float4(cv, cv, cv, cv);
          break;
        }
        case SPMDB200_MAP_ADD: apply<S>(rd, ra, rb, [](float a, float b) { return __fadd_rn(a, b); }); break;
        case SPMDB200_MAP_SUB: apply<S>(rd, ra, rb, [](float a, float b) { return __fsub_rn(a, b); }); break;
        case SPMDB200_MAP_MUL: apply<S>(rd, ra, rb, [](float a, float b) { return __fmul_rn(a, b); }); break;
        case SPMDB200_MAP_DIV: apply<S>(rd, ra, rb, [](float a, float b) { return __fdiv_rn(a, b); }); break;
        case SPMDB200_MAP_MAXIMUM: apply<S>(rd, ra, rb, [](float a, float b) { return f_maximum(a, b); }); break;
        case SPMDB200_MAP_MINIMUM: apply<S>(rd, ra, rb, [](float a, float b) { return f_minimum(a, b); }); break;
        case SPMDB200_MAP_NEG:
          apply<S>(rd, ra, ra, [](float a, float) { return __int_as_float(__float_as_int(a) ^ (int)0x80000000u); });
          break;
        case SPMDB200_MAP_ABS:
          apply<S>(rd, ra, ra, [](float a, float) { return __int_as_float(__float_as_int(a) & 0x7fffffff); });
          break;
        case SPMDB200_MAP_SQRT: apply<S>(rd, ra, ra, [](float a, float) { return __fsqrt_rn(a); }); break;
        case SPMDB200_MAP_CMP: apply<S>(rd, ra, rb, [aux](float a, float b) { return bool_f(cmpf(aux, a, b)); }); break;
        case SPMDB200_MAP_SELECT: {
          if (!IN_RANGE(aux < p.n_regs, 3, aux)) break;
          const float4 *rk = mine + aux * kRow;
#pragma unroll
          for (int s = 0; s < S; ++s) {
            const int o = s * kMapThreads;
            const float4 k = rk[o], x = ra[o], y = rb[o];
            rd[o] = make_float4(k.x != 0.0f ? x.x : y.x, k.y != 0.0f ? x.y : y.y, k.z != 0.0f ? x.z : y.z,
                                k.w != 0.0f ? x.w : y.w);
          }
          break;
        }
        case SPMDB200_MAP_AND:
          apply<S>(rd, ra, rb, [](float a, float b) { return bool_f(a != 0.0f && b != 0.0f); });
          break;
        case SPMDB200_MAP_OR:
          apply<S>(rd, ra, rb, [](float a, float b) { return bool_f(a != 0.0f || b != 0.0f); });
          break;
        default:  // XOR: the host accepts no other opcode before the STORE
          apply<S>(rd, ra, rb, [](float a, float b) { return bool_f((a != 0.0f) != (b != 0.0f)); });
          break;
      }
    }
    if (IN_RANGE(p.out_reg < p.n_regs, 3, p.out_reg)) {
      if constexpr (MODE == kGeneral) {
        store_general<S>(p, base, g, mine + p.out_reg * kRow, kMapThreads);
      } else if constexpr (MODE == kRows) {
        store_rows<S>(p, rc, mine + p.out_reg * kRow, kMapThreads);
      } else {
#pragma unroll
        for (int s = 0; s < S; ++s)
          store4<MODE>(p, base + (int64_t)s * 4 * kMapThreads, mine[p.out_reg * kRow + s * kMapThreads]);
      }
    }
  }
}

template <int NL>
cudaError_t launch_nl(const MapParams &p, int mode, int n_regs, cudaStream_t stream) {
  const size_t smem = (size_t)n_regs * map_slots(NL) * kMapThreads * sizeof(float4);
  auto kern = mode == kVec      ? forall_map_kernel<NL, kVec>
              : mode == kContig ? forall_map_kernel<NL, kContig>
              : mode == kRows   ? forall_map_kernel<NL, kRows>
                                : forall_map_kernel<NL, kGeneral>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int dev = 0, per_sm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kMapThreads, smem)) != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  const int64_t nchunks = mode == kRows ? p.size[0] * p.size[1] * ((p.size[2] + map_chunk(NL) - 1) / map_chunk(NL))
                                        : (p.n + map_chunk(NL) - 1) / map_chunk(NL);
  const int64_t cap = (int64_t)num_sms(dev) * per_sm;
  const int grid = (int)(nchunks < cap ? nchunks : cap);
  kern<<<grid, kMapThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

bool contiguous(const int64_t *sz, const int64_t *st) {
  int64_t want = 1;
  for (int d = 2; d >= 0; --d) {
    if (sz[d] > 1 && st[d] != want) return false;
    want *= sz[d];
  }
  return true;
}

// Elements a view covers: 1 + its largest offset over the domain.
int64_t view_span(const int64_t *sz, const int64_t *st) {
  int64_t sp = 1;
  for (int d = 0; d < 3; ++d) sp += (sz[d] - 1) * st[d];
  return sp;
}

}  // namespace

int check_read_forall_map(unsigned long long *first) {
#ifdef SPMDB200_CHECKED
  if (!first) return 1;  // only asks whether this is a checked build
  unsigned long long v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_check_first, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_check_first, &z, sizeof(z)) != cudaSuccess)
    return -1;
  *first = v;
  return 1;
#else
  if (first) *first = 0;
  return 0;
#endif
}

}  // namespace spmdb200

using namespace spmdb200;

extern "C" int spmdb200_forall_map(int rank, const int64_t *sizes, int n_inputs, const float *const *inputs,
                                   const int64_t *input_strides, float *out, const int64_t *out_strides,
                                   const int32_t *code, int n_insns, const float *consts, int n_consts,
                                   int n_regs, void *stream) {
  auto bad = [](const char *fmt, auto... a) { return record_api_status(SPMDB200_ERR_INVALID_ARG, fmt, a...); };
  if (rank < 1 || rank > 3) return bad("rank %d: must be 1, 2 or 3", rank);
  if (!sizes || !out_strides || !code) return bad("null sizes, out_strides or code");
  if (n_inputs < 0 || n_inputs > SPMDB200_MAP_MAX_INPUTS) return bad("n_inputs %d: 0..%d", n_inputs, kMaxLoads);
  if (n_inputs > 0 && (!inputs || !input_strides)) return bad("null inputs or input_strides");
  if (n_insns < 2 || n_insns > SPMDB200_MAP_MAX_INSNS) return bad("n_insns %d: 2..%d", n_insns, SPMDB200_MAP_MAX_INSNS);
  if (n_consts < 0 || n_consts > SPMDB200_MAP_MAX_CONSTS || (n_consts > 0 && !consts))
    return bad("n_consts %d: 0..%d with a non-null table", n_consts, SPMDB200_MAP_MAX_CONSTS);
  if (n_regs < 1 || n_regs > SPMDB200_MAP_MAX_REGS) return bad("n_regs %d: 1..%d", n_regs, SPMDB200_MAP_MAX_REGS);

  MapParams p{};
  p.size[0] = p.size[1] = p.size[2] = 1;
  p.n = 1;
  for (int d = 0; d < rank; ++d) {
    if (sizes[d] < 0) return bad("negative size in dimension %d", d);
    p.size[3 - rank + d] = sizes[d];
    p.out_st[3 - rank + d] = out_strides[d];
    p.n *= sizes[d];
  }
  // The program: a LOAD prefix, then operations, then exactly one STORE.
  bool written[SPMDB200_MAP_MAX_REGS] = {};
  int nl = 0;
  for (int i = 0; i < n_insns; ++i) {
    const int w0 = code[2 * i], aux = code[2 * i + 1];
    const int op = w0 & 255, d = (w0 >> 8) & 255, a = (w0 >> 16) & 255, b = (int)((unsigned)w0 >> 24);
    const bool last = i == n_insns - 1;
    if (op > SPMDB200_MAP_STORE) return bad("instruction %d: unknown opcode %d", i, op);
    // The kernel may read the a / b fields of any instruction: all in range.
    if (d >= n_regs || a >= n_regs || b >= n_regs)
      return bad("instruction %d: register field beyond n_regs %d", i, n_regs);
    if ((op == SPMDB200_MAP_STORE) != last) return bad("instruction %d: exactly one STORE, the last", i);
    if (op == SPMDB200_MAP_LOAD) {
      if (i != nl) return bad("instruction %d: LOADs must come before every other instruction", i);
      if (aux < 0 || aux >= n_inputs) return bad("instruction %d: input %d of %d", i, aux, n_inputs);
      if (nl == kMaxLoads) return bad("more than %d LOADs", kMaxLoads);
      ++nl;
    }
    const bool unary = op == SPMDB200_MAP_NEG || op == SPMDB200_MAP_ABS || op == SPMDB200_MAP_SQRT;
    const bool reads_a = op >= SPMDB200_MAP_ADD || op == SPMDB200_MAP_STORE;
    const bool reads_b = op >= SPMDB200_MAP_ADD && op != SPMDB200_MAP_STORE && !unary;
    if (reads_a && (a >= n_regs || !written[a])) return bad("instruction %d: register %d read before written", i, a);
    if (reads_b && (b >= n_regs || !written[b])) return bad("instruction %d: register %d read before written", i, b);
    if (op == SPMDB200_MAP_CONST && (aux < 0 || aux >= n_consts)) return bad("instruction %d: constant %d", i, aux);
    if (op == SPMDB200_MAP_CMP && (aux < 0 || aux > 15)) return bad("instruction %d: predicate %d", i, aux);
    if (op == SPMDB200_MAP_SELECT && (aux < 0 || aux >= n_regs || !written[aux]))
      return bad("instruction %d: condition register %d read before written", i, aux);
    if (op != SPMDB200_MAP_STORE) {
      written[d] = true;
    } else {
      p.out_reg = a;
    }
    p.code[2 * i] = w0;
    p.code[2 * i + 1] = aux;
  }
  if (nl == 0) return record_api_status(SPMDB200_ERR_UNSUPPORTED, "a body with no LOAD (a fill) is not mapped");
  p.n_insns = n_insns;
  p.n_regs = n_regs;
  for (int j = 0; j < n_consts; ++j) p.consts[j] = consts[j];
  if (p.n == 0) return record_api_status(SPMDB200_OK, "");
  if (!out) return bad("null out");
  p.out = out;
  bool contig = contiguous(p.size, p.out_st), aligned = ((uintptr_t)out & 15u) == 0;
  for (int i = 0; i < nl; ++i) {
    const int in = code[2 * i + 1];
    const float *src = inputs[in];
    if (!src) return bad("null input %d", in);
    p.ld_src[i] = src;
    p.ld_dst[i] = (code[2 * i] >> 8) & 255;
    for (int d = 0; d < 3; ++d) p.ld_st[i][d] = 0;
    for (int d = 0; d < rank; ++d) p.ld_st[i][3 - rank + d] = input_strides[in * rank + d];
    contig = contig && contiguous(p.size, p.ld_st[i]);
    aligned = aligned && ((uintptr_t)src & 15u) == 0;
    p.ld_span[i] = view_span(p.size, p.ld_st[i]);
  }
  p.out_span = view_span(p.size, p.out_st);
  for (int d = 0; d < 3; ++d)
    for (int i = 0; i < nl; ++i)
      if (p.ld_st[i][d] < 0 || p.out_st[d] < 0) return bad("negative stride");
  const int mode = contig ? (aligned ? kVec : kContig) : p.size[2] >= kRowsMin ? kRows : kGeneral;
  cudaError_t e;
  cudaStream_t s = (cudaStream_t)stream;
  switch (nl) {
    case 1: e = launch_nl<1>(p, mode, n_regs, s); break;
    case 2: e = launch_nl<2>(p, mode, n_regs, s); break;
    case 3: e = launch_nl<3>(p, mode, n_regs, s); break;
    case 4: e = launch_nl<4>(p, mode, n_regs, s); break;
    case 5: e = launch_nl<5>(p, mode, n_regs, s); break;
    case 6: e = launch_nl<6>(p, mode, n_regs, s); break;
    case 7: e = launch_nl<7>(p, mode, n_regs, s); break;
    default: e = launch_nl<8>(p, mode, n_regs, s); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return record_api_status(SPMDB200_ERR_CUDA, "forall_map launch: %s", cudaGetErrorString(e));
  }
  return record_api_status(SPMDB200_OK, "");
}
