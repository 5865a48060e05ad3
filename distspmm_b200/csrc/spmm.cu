// spmm.cu — sm_100a CSR x dense fp32 SpMM kernels and the single-GPU plan API.
//
// C[rows x N] (+)= A[rows x cols] * B[cols x N]; A in CSR with int32 column ids, B and C
// row-major fp32. This is a gather-and-accumulate bound by L2 / HBM bandwidth and by the
// number of B-row loads in flight, not a dense contraction, so it runs on the CUDA cores.
//
// Two work decompositions, picked per operand from its row-length statistics:
//   row-split  one item per row; rows longer than `piece_cap` nonzeros are cut into
//              balanced pieces. Good for regular rows (stencils, fixed-degree rows).
//   nnz-split  equal chunks of `chunk_nnz` consecutive nonzeros per lane group regardless
//              of row boundaries (merge-path style): every group keeps the same number of
//              B-row loads in flight even when rows hold 1-3 nonzeros (R-MAT). Rows are
//              flushed as the chunk crosses them; rows cut by a chunk boundary write
//              partial rows to slots.
// In both, partial rows are summed in a fixed order by a fixup kernel (deterministic, no
// atomics), so repeated runs are bit-identical.
//
// Per group of LPR lanes (a warp for N >= 128) each lane holds VPL vectors of W floats of
// the output row, so one B row is read as LPR*W*4 contiguous bytes (512 B at N = 128:
// 32 lanes x float4). (column, value[, row]) triples are loaded once per lane per 32
// nonzeros with streaming loads and broadcast by warp shuffles; B rows go through the
// read-only path with an L2 evict_last policy (A and C stream past them); final C rows
// are written once with streaming stores.
// Replaces cusparseSpMM(COO, ALG_DEFAULT, beta = 1) of src/dist_spmm_node.cu:354-385.
#include <cuda.h>  // CUtensorMap and its enums (the encoder is fetched through the runtime)
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "device.cuh"
#include "internal.h"
#include "mbar.cuh"

namespace dsp {

// ------------------------------------------------------------------ vector helpers
template <int W>
struct Vec;
template <>
struct Vec<4> {
  using T = float4;
  static __device__ __forceinline__ T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  // B rows: read-only path, kept in L2 ahead of the streamed A and C (evict_last policy)
  static __device__ __forceinline__ T ldg(const float *p, uint64_t pol) {
    T v;
    asm("ld.global.nc.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p), "l"(pol));
    return v;
  }
  static __device__ __forceinline__ T ld(const float *p) { return *reinterpret_cast<const float4 *>(p); }
  static __device__ __forceinline__ void st(float *p, T v) { *reinterpret_cast<float4 *>(p) = v; }
  // final C rows are not re-read by this kernel: streaming store, no L2 residency
  static __device__ __forceinline__ void st_stream(float *p, T v) { __stcs(reinterpret_cast<float4 *>(p), v); }
  static __device__ __forceinline__ void fma(T &acc, float s, T b) {
    acc.x = fmaf(s, b.x, acc.x);
    acc.y = fmaf(s, b.y, acc.y);
    acc.z = fmaf(s, b.z, acc.z);
    acc.w = fmaf(s, b.w, acc.w);
  }
  static __device__ __forceinline__ void add(T &acc, T b) {
    acc.x += b.x;
    acc.y += b.y;
    acc.z += b.z;
    acc.w += b.w;
  }
};
// 256-bit vectors (sm_100 ld/st .v8.f32): with 4 lanes per row one warp instruction reads
// eight whole 128-byte lines of B, twice the bytes per L1 wavefront of the float4 path.
struct Float8 {
  float4 lo, hi;
};
template <>
struct Vec<8> {
  using T = Float8;
  static __device__ __forceinline__ T zero() {
    return {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  }
  static __device__ __forceinline__ T ldg(const float *p, uint64_t pol) {
    T v;
    asm("ld.global.nc.L2::cache_hint.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], %9;"
        : "=f"(v.lo.x), "=f"(v.lo.y), "=f"(v.lo.z), "=f"(v.lo.w), "=f"(v.hi.x), "=f"(v.hi.y), "=f"(v.hi.z),
          "=f"(v.hi.w)
        : "l"(p), "l"(pol));
    return v;
  }
  static __device__ __forceinline__ T ld(const float *p) {
    T v;
    asm volatile("ld.global.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(v.lo.x), "=f"(v.lo.y), "=f"(v.lo.z), "=f"(v.lo.w), "=f"(v.hi.x), "=f"(v.hi.y),
                   "=f"(v.hi.z), "=f"(v.hi.w)
                 : "l"(p)
                 : "memory");
    return v;
  }
  static __device__ __forceinline__ void st(float *p, T v) {
    asm volatile("st.global.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v.lo.x), "f"(v.lo.y),
                 "f"(v.lo.z), "f"(v.lo.w), "f"(v.hi.x), "f"(v.hi.y), "f"(v.hi.z), "f"(v.hi.w)
                 : "memory");
  }
  static __device__ __forceinline__ void st_stream(float *p, T v) {
    asm volatile("st.global.cs.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v.lo.x), "f"(v.lo.y),
                 "f"(v.lo.z), "f"(v.lo.w), "f"(v.hi.x), "f"(v.hi.y), "f"(v.hi.z), "f"(v.hi.w)
                 : "memory");
  }
  static __device__ __forceinline__ void fma(T &acc, float s, T b) {
    Vec<4>::fma(acc.lo, s, b.lo);
    Vec<4>::fma(acc.hi, s, b.hi);
  }
  static __device__ __forceinline__ void add(T &acc, T b) {
    Vec<4>::add(acc.lo, b.lo);
    Vec<4>::add(acc.hi, b.hi);
  }
};
template <>
struct Vec<1> {
  using T = float;
  static __device__ __forceinline__ T zero() { return 0.f; }
  static __device__ __forceinline__ T ldg(const float *p, uint64_t) { return __ldg(p); }
  static __device__ __forceinline__ T ld(const float *p) { return *p; }
  static __device__ __forceinline__ void st(float *p, T v) { *p = v; }
  static __device__ __forceinline__ void st_stream(float *p, T v) { __stcs(p, v); }
  static __device__ __forceinline__ void fma(T &acc, float s, T b) { acc = fmaf(s, b, acc); }
  static __device__ __forceinline__ void add(T &acc, T b) { acc += b; }
};

__device__ __forceinline__ uint64_t evict_last_policy() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Stored column ids of CSR operands carry the L2 policy of their B row in bit 31: set for
// the operand's most-referenced ("hot") columns, whose rows are read with evict_last so that
// they stay in L2; clear for the others, read with evict_first so that rows used once or
// twice do not push the hot rows out (mark_hot_columns decides on the host).
__device__ __forceinline__ int32_t col_id(int32_t stored) { return stored & 0x7fffffff; }
__device__ __forceinline__ uint64_t col_policy(int32_t stored, uint64_t hot, uint64_t cold) {
  return stored < 0 ? hot : cold;
}

template <int LPR>
__device__ __forceinline__ unsigned group_mask() {
  return LPR == 32 ? 0xffffffffu : (((1u << LPR) - 1u) << ((threadIdx.x & 31) & ~(LPR - 1)));
}

// nonzeros whose B vectors are loaded before their FMAs: about 8 vectors (4 of 256 bits)
// in flight per lane, never more nonzeros than one shuffle round holds
template <int LPR, int VPL, int W>
__host__ __device__ constexpr int loads_in_flight() {
  const int per_nonzero = (W == 8 ? 4 : 8) / VPL;
  const int u = per_nonzero < 1 ? 1 : per_nonzero;
  return u < LPR ? u : LPR;
}

// (column, value[, row]) entries each lane loads per round: one round covers up to 32
// nonzeros of the group, so the streamed A loads are issued together
template <int LPR>
__host__ __device__ constexpr int entries_per_lane() {
  return 32 / LPR < 8 ? 32 / LPR : 8;
}

// Whether output row `row` adds to C: the launch accumulates, or (split pipeline) an
// earlier phase already wrote the row.
template <bool kAccum>
__device__ __forceinline__ bool accumulates(const SpmmArgs &a, int32_t row) {
  return kAccum || (a.first_phase != nullptr && (int)a.first_phase[row] < a.phase);
}

// Write one output row held in acc: to its partial slot, or to C (adding C when
// accumulating). col0 is this lane's first column.
template <int LPR, int VPL, int W, bool kAccum>
__device__ __forceinline__ void flush_row(const SpmmArgs &a, int32_t row, int32_t slot, int col0,
                                          const typename Vec<W>::T (&acc)[VPL]) {
  using V = Vec<W>;
  using T = typename V::T;
  if (slot >= 0) {
    float *dst = a.partial + (int64_t)slot * a.N;
#pragma unroll
    for (int w = 0; w < VPL; ++w) {
      const int col = col0 + w * LPR * W;
      if (col < a.N) V::st(dst + col, acc[w]);
    }
  } else {
    float *dst = a.C + (int64_t)row * a.ldc;
    const bool add = accumulates<kAccum>(a, row);
#pragma unroll
    for (int w = 0; w < VPL; ++w) {
      const int col = col0 + w * LPR * W;
      if (col < a.N) {
        T r = acc[w];
        if (add) V::add(r, V::ld(dst + col));
        V::st_stream(dst + col, r);
      }
    }
  }
}

// Rows [r0, r1) hold no nonzeros: write their zeros (non-accumulating launches only).
template <int LPR, int VPL, int W>
__device__ __forceinline__ void zero_rows(const SpmmArgs &a, int64_t r0, int64_t r1, int col0) {
  using V = Vec<W>;
  for (int64_t r = r0; r < r1; ++r) {
    float *dst = a.C + r * a.ldc;
#pragma unroll
    for (int w = 0; w < VPL; ++w) {
      const int col = col0 + w * LPR * W;
      if (col < a.N) V::st_stream(dst + col, V::zero());
    }
  }
}

// ------------------------------------------------------------------ row-split kernel

// One item per group of LPR lanes; blockIdx.y selects a chunk of LPR*VPL*W columns.
template <int LPR, int VPL, int W, bool kAccum>
__global__ void __launch_bounds__(kSpmmThreads) spmm_rows_kernel(const SpmmArgs a) {
  using V = Vec<W>;
  using T = typename V::T;
  constexpr int U = loads_in_flight<LPR, VPL, W>();
  const int lane = threadIdx.x & (LPR - 1);
  const int64_t item = ((int64_t)blockIdx.x * kSpmmThreads + threadIdx.x) / LPR;
  if (item >= a.n_items) return;
  const unsigned gmask = group_mask<LPR>();
  const int col0 = blockIdx.y * (LPR * VPL * W) + lane * W;
  const int64_t beg = a.item_ptr[item], end = a.item_ptr[item + 1];
  const uint64_t pol_hot = evict_last_policy(), pol_cold = evict_first_policy();

  constexpr int K = entries_per_lane<LPR>();
  T acc[VPL];
#pragma unroll
  for (int w = 0; w < VPL; ++w) acc[w] = V::zero();

  for (int64_t base = beg; base < end; base += LPR * K) {
    int c[K];
    float v[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t p = base + k * LPR + lane;
      c[k] = p < end ? __ldcs(a.cols + p) : 0;
      v[k] = p < end ? __ldcs(a.vals + p) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t kb = base + k * LPR;
      if (kb >= end) break;
      const int n = (int)min((int64_t)LPR, end - kb);
      for (int j = 0; j < n; j += U) {
        T b[U][VPL];
        float s[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int cs = __shfl_sync(gmask, c[k], j + u, LPR);
          s[u] = __shfl_sync(gmask, v[k], j + u, LPR);
          const uint64_t pol = col_policy(cs, pol_hot, pol_cold);
          const float *brow = a.B + (int64_t)col_id(cs) * a.ldb;
#pragma unroll
          for (int w = 0; w < VPL; ++w) {
            const int col = col0 + w * LPR * W;
            b[u][w] = (j + u < n && col < a.N) ? V::ldg(brow + col, pol) : V::zero();
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int w = 0; w < VPL; ++w)
            if (j + u < n) V::fma(acc[w], s[u], b[u][w]);
      }
    }
  }
  const int32_t o = a.item_out[item];
  flush_row<LPR, VPL, W, kAccum>(a, o, o >= 0 ? -1 : -(o + 1), col0, acc);
}

// ------------------------------------------------------------------ nnz-split kernel

// One chunk of chunk_nnz consecutive nonzeros per group of LPR lanes.
template <int LPR, int VPL, int W, bool kAccum>
__global__ void __launch_bounds__(kSpmmThreads) spmm_nnz_kernel(const SpmmArgs a) {
  using V = Vec<W>;
  using T = typename V::T;
  constexpr int U = loads_in_flight<LPR, VPL, W>();
  const int lane = threadIdx.x & (LPR - 1);
  const int64_t chunk = ((int64_t)blockIdx.x * kSpmmThreads + threadIdx.x) / LPR;
  if (chunk >= a.n_chunks) return;
  const unsigned gmask = group_mask<LPR>();
  const int col0 = blockIdx.y * (LPR * VPL * W) + lane * W;
  const int64_t s = chunk * a.chunk_nnz, e = min(s + a.chunk_nnz, a.nnz);
  const int32_t head_slot = a.chunk_slot[2 * chunk], tail_slot = a.chunk_slot[2 * chunk + 1];
  const uint64_t pol_hot = evict_last_policy(), pol_cold = evict_first_policy();

  int32_t row = a.coo_row[s];
  const int32_t head_row = row;
  // empty rows between the previous chunk's last row and this chunk's first row
  // (only operands that list every output row, zero_rows > 0, own the rows in between)
  if (!kAccum && a.zero_rows > 0) zero_rows<LPR, VPL, W>(a, s > 0 ? (int64_t)a.coo_row[s - 1] + 1 : 0, row, col0);

  constexpr int K = entries_per_lane<LPR>();
  T acc[VPL];
#pragma unroll
  for (int w = 0; w < VPL; ++w) acc[w] = V::zero();

  for (int64_t base = s; base < e; base += LPR * K) {
    int c[K], rr[K];
    float v[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t p = base + k * LPR + lane;
      c[k] = p < e ? __ldcs(a.cols + p) : 0;
      v[k] = p < e ? __ldcs(a.vals + p) : 0.f;
      rr[k] = p < e ? __ldcs(a.coo_row + p) : 0;
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t kb = base + k * LPR;
      if (kb >= e) break;
      const int n = (int)min((int64_t)LPR, e - kb);
      for (int j = 0; j < n; j += U) {
        T b[U][VPL];
        float sv[U];
        int ru[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int cs = __shfl_sync(gmask, c[k], j + u, LPR);
          sv[u] = __shfl_sync(gmask, v[k], j + u, LPR);
          ru[u] = __shfl_sync(gmask, rr[k], j + u, LPR);
          const uint64_t pol = col_policy(cs, pol_hot, pol_cold);
          const float *brow = a.B + (int64_t)col_id(cs) * a.ldb;
#pragma unroll
          for (int w = 0; w < VPL; ++w) {
            const int col = col0 + w * LPR * W;
            b[u][w] = (j + u < n && col < a.N) ? V::ldg(brow + col, pol) : V::zero();
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (j + u < n) {
            if (ru[u] != row) {  // group-uniform: the chunk crosses into the next row
              flush_row<LPR, VPL, W, kAccum>(a, row, row == head_row ? head_slot : -1, col0, acc);
              if (!kAccum && a.zero_rows > 0) zero_rows<LPR, VPL, W>(a, (int64_t)row + 1, ru[u], col0);
              row = ru[u];
#pragma unroll
              for (int w = 0; w < VPL; ++w) acc[w] = V::zero();
            }
#pragma unroll
            for (int w = 0; w < VPL; ++w) V::fma(acc[w], sv[u], b[u][w]);
          }
        }
      }
    }
  }
  flush_row<LPR, VPL, W, kAccum>(a, row, tail_slot >= 0 ? tail_slot : (row == head_row ? head_slot : -1), col0,
                                 acc);
  if (!kAccum && chunk == a.n_chunks - 1) zero_rows<LPR, VPL, W>(a, (int64_t)row + 1, a.zero_rows, col0);
}

// ------------------------------------------------------------------ nnz-split, warp per chunk

// 4 consecutive 32-bit words read by every lane of the warp from the same 16-byte address
// (one request, served to the whole warp).
__device__ __forceinline__ int4 ldg_uniform_i4(const int32_t *p) {
  int4 v;
  asm("ld.global.nc.v4.s32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ldg_uniform_f4(const float *p) {
  float4 v;
  asm("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// One chunk of chunk_nnz consecutive nonzeros per warp; lane l holds output columns
// col0 + 128 v .. +3 (v < VPL) of the current row, blockIdx.y selecting a block of
// 128 * VPL columns. Each step reads the column, value and output row of U nonzeros (every
// lane reads the same words: one request each, served to the whole warp), then requests
// their U B rows (one 512-byte row per warp instruction at VPL = 1) and does the FMAs. A
// row change is met when the next nonzero's row id differs, which is the same for every
// lane, so no lane diverges; the finished row is written (to its partial slot when it is
// cut by a chunk boundary, as in spmm_nnz_kernel). No loads are carried across steps: with
// few registers per lane, many warps per SM keep the B rows in flight instead (measured on
// B200 against software-pipelined and lane-group forms of the same loop: 1.06 / 1.68 /
// 1.43 ms on the R-MAT scale-20 stream).
template <int VPL, int U, bool kAccum, int kMinBlocks>
__global__ void __launch_bounds__(kSpmmThreads, kMinBlocks) spmm_warp_kernel(const SpmmArgs a) {
  static_assert(U % 4 == 0, "steps read groups of 4 nonzeros");
  using V = Vec<4>;
  const int lane = threadIdx.x & 31;
  const int64_t chunk = ((int64_t)blockIdx.x * kSpmmThreads + threadIdx.x) >> 5;
  if (chunk >= a.n_chunks) return;
  const int col0 = blockIdx.y * (128 * VPL) + lane * 4;
  const int64_t s = chunk * a.chunk_nnz, e = min(s + a.chunk_nnz, a.nnz);
  const int32_t head_slot = a.chunk_slot[2 * chunk], tail_slot = a.chunk_slot[2 * chunk + 1];
  const uint64_t pol_hot = evict_last_policy(), pol_cold = evict_first_policy();

  int32_t row = __ldg(a.coo_row + s);
  const int32_t head_row = row;
  float4 acc[VPL];
  // rows [r0, r1) hold no nonzeros: zeros (only operands that list every output row,
  // zero_rows > 0, own the rows in between)
  auto zeros = [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r)
#pragma unroll
      for (int w = 0; w < VPL; ++w) V::st_stream(a.C + r * a.ldc + col0 + 128 * w, V::zero());
  };
  auto flush = [&](int32_t slot) {
    if (slot >= 0) {
      float *dst = a.partial + (int64_t)slot * a.N + col0;
#pragma unroll
      for (int w = 0; w < VPL; ++w) V::st(dst + 128 * w, acc[w]);
    } else {
      float *dst = a.C + (int64_t)row * a.ldc + col0;
      const bool add = accumulates<kAccum>(a, row);
#pragma unroll
      for (int w = 0; w < VPL; ++w) {
        float4 r = acc[w];
        if (add) V::add(r, V::ld(dst + 128 * w));
        V::st_stream(dst + 128 * w, r);
      }
    }
  };
  if (!kAccum && a.zero_rows > 0) zeros(s > 0 ? (int64_t)__ldg(a.coo_row + s - 1) + 1 : 0, row);
#pragma unroll
  for (int w = 0; w < VPL; ++w) acc[w] = V::zero();
  // nonzero with column cs, value v, row r (warp-uniform row change)
  auto add = [&](int32_t r, float v, const float4 (&b)[VPL]) {
    if (r != row) {
      flush(row == head_row ? head_slot : -1);
      if (!kAccum && a.zero_rows > 0) zeros((int64_t)row + 1, r);
      row = r;
#pragma unroll
      for (int w = 0; w < VPL; ++w) acc[w] = V::zero();
    }
#pragma unroll
    for (int w = 0; w < VPL; ++w) V::fma(acc[w], v, b[w]);
  };

  // B rows as float4 from this lane's first column: one 32 x 32 -> 64-bit multiply-add per
  // nonzero (the host keeps ldb / 4 within int32 for this kernel)
  const float4 *B4 = reinterpret_cast<const float4 *>(a.B + col0);
  const int32_t ld4 = (int32_t)(a.ldb >> 2);

  // full steps of U nonzeros: p stays a multiple of 4 (chunk_nnz is a multiple of 16), so
  // the column ids, values and row ids of 4 nonzeros come in one 16-byte load each, and no
  // entry needs a bounds test
  int64_t p = s;
  for (; p + U <= e; p += U) {
    int32_t cs[U], r[U];
    float v[U];
#pragma unroll
    for (int q = 0; q < U / 4; ++q) {
      const int4 c4 = ldg_uniform_i4(a.cols + p + 4 * q);
      const float4 v4 = ldg_uniform_f4(a.vals + p + 4 * q);
      const int4 r4 = ldg_uniform_i4(a.coo_row + p + 4 * q);
      cs[4 * q] = c4.x, cs[4 * q + 1] = c4.y, cs[4 * q + 2] = c4.z, cs[4 * q + 3] = c4.w;
      v[4 * q] = v4.x, v[4 * q + 1] = v4.y, v[4 * q + 2] = v4.z, v[4 * q + 3] = v4.w;
      r[4 * q] = r4.x, r[4 * q + 1] = r4.y, r[4 * q + 2] = r4.z, r[4 * q + 3] = r4.w;
    }
    float4 b[U][VPL];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float4 *brow = B4 + (int64_t)col_id(cs[u]) * ld4;
      const uint64_t pol = col_policy(cs[u], pol_hot, pol_cold);
#pragma unroll
      for (int w = 0; w < VPL; ++w) b[u][w] = V::ldg(reinterpret_cast<const float *>(brow + 32 * w), pol);
    }
    // the step stays in the current row (the common case on rows longer than a step): the
    // multiply-adds without per-nonzero row tests
    bool same = true;
#pragma unroll
    for (int u = 0; u < U; ++u) same &= r[u] == row;
    if (same) {
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int w = 0; w < VPL; ++w) V::fma(acc[w], v[u], b[u][w]);
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) add(r[u], v[u], b[u]);
    }
  }
  // the chunk's last nonzeros (the matrix's end)
  for (; p < e; ++p) {
    const int32_t cs = __ldg(a.cols + p);
    float4 b[VPL];
    const float *brow = reinterpret_cast<const float *>(B4 + (int64_t)col_id(cs) * ld4);
#pragma unroll
    for (int w = 0; w < VPL; ++w) b[w] = V::ldg(brow + 128 * w, col_policy(cs, pol_hot, pol_cold));
    add(__ldg(a.coo_row + p), __ldg(a.vals + p), b);
  }
  flush(tail_slot >= 0 ? tail_slot : (row == head_row ? head_slot : -1));
  if (!kAccum && a.zero_rows > 0 && chunk == a.n_chunks - 1) zeros((int64_t)row + 1, a.zero_rows);
}

// ------------------------------------------------------------------ banded operands (diagonals)

// One block of kDiaRows (8) consecutive rows per warp, on the diagonal form: row i holds
// the entries (i, i + diag_off[d]). Offsets that follow one another (o, o+1, ..., a run of
// up to 4, e.g. the x-neighbours of a stencil) share B rows: the 8 rows of a block need
// B rows jb + k, k < 8 + L - 1, of a run of length L, and each such row is read once and
// applied to every row r = k - l of the block it touches, so a 27-point stencil reads about
// 11 B rows per output row instead of 27, and no column ids. The block's values are staged
// once in shared memory (one load latency per block, then broadcast reads); each run is
// done by code specialised for its length (run_len, set on the host). Presence bits (one
// byte per block and diagonal) mark the entries that exist: a B row no entry of the block
// uses is not read and an absent entry adds nothing, so the result is the CSR product
// exactly (an explicit zero in A counts as present). Lane l holds output columns
// col0 .. col0 + 3, blockIdx.y selecting a block of 128 columns. Needs N % 128 == 0 and
// 16-byte aligned B / C rows.
template <int RB, int L>
__device__ __forceinline__ void dia_run(const SpmmArgs &a, const float *sv, int d0, const uint32_t (&pb)[4],
                                        int64_t jb, int col0, uint64_t pol, float4 (&acc)[RB]) {
  using V = Vec<4>;
  constexpr uint32_t kFull = (1u << RB) - 1u;
  bool all = true;  // every entry of the run is present: no per-entry tests
#pragma unroll
  for (int l = 0; l < L; ++l) all = all && pb[l] == kFull;
  float4 b[RB + L - 1];
  if (all) {
#pragma unroll
    for (int k = 0; k < RB + L - 1; ++k) b[k] = V::ldg(a.B + (jb + k) * a.ldb + col0, pol);
#pragma unroll
    for (int k = 0; k < RB + L - 1; ++k)
#pragma unroll
      for (int l = 0; l < L; ++l)
        if (k - l >= 0 && k - l < RB) V::fma(acc[k - l], sv[(d0 + l) * RB + k - l], b[k]);
    return;
  }
#pragma unroll
  for (int k = 0; k < RB + L - 1; ++k) {
    uint32_t need = 0;  // some present entry of the block uses B row jb + k
#pragma unroll
    for (int l = 0; l < L; ++l)
      if (k - l >= 0 && k - l < RB) need |= (pb[l] >> (k - l)) & 1u;
    b[k] = need ? V::ldg(a.B + (jb + k) * a.ldb + col0, pol) : V::zero();
  }
#pragma unroll
  for (int k = 0; k < RB + L - 1; ++k)
#pragma unroll
    for (int l = 0; l < L; ++l)
      if (k - l >= 0 && k - l < RB && ((pb[l] >> (k - l)) & 1u))
        V::fma(acc[k - l], sv[(d0 + l) * RB + k - l], b[k]);
}

// RB (4 or 8) consecutive rows per warp; the presence bytes cover 8-row blocks, so a 4-row
// warp uses half of each byte.
template <int RB, bool kAccum>
__global__ void __launch_bounds__(kSpmmThreads) spmm_dia_kernel(const SpmmArgs a) {
  static_assert(RB == 4 || RB == 8, "rows per warp");
  using V = Vec<4>;
  __shared__ float s_val[kSpmmThreads / 32][kMaxDiag * RB];
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t wid = ((int64_t)blockIdx.x * kSpmmThreads + threadIdx.x) >> 5;
  const int64_t i0 = wid * RB;
  if (i0 >= a.dia_m) return;
  const int col0 = blockIdx.y * 128 + lane * 4;
  const int64_t orow0 = a.dia_row0 + i0;
  const uint64_t pol = evict_last_policy();
  // this warp's values, diagonal-major (RB rows each), into its shared slice
  float *sv = s_val[wib];
  for (int idx = lane; idx < a.n_diag * RB; idx += 32) {
    const int d = idx / RB, r = idx % RB;
    sv[idx] = i0 + r < a.dia_m ? __ldg(a.dia_vals + (int64_t)d * a.dia_m + i0 + r) : 0.f;
  }
  // lane d holds the presence bits of diagonal d for the RB rows of this warp
  const int64_t blk = i0 / kDiaRows;
  const int shift = (int)(i0 % kDiaRows);
  const uint32_t pbyte =
      lane < a.n_diag ? ((uint32_t)__ldg(a.dia_pres + blk * a.n_diag + lane) >> shift) & ((1u << RB) - 1u) : 0u;
  __syncwarp();
  float4 acc[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) acc[r] = V::zero();

  int d0 = 0;
  for (int q = 0; q < a.n_runs; ++q) {
    const int L = a.run_len[q];
    uint32_t pb[4];
#pragma unroll
    for (int l = 0; l < 4; ++l) pb[l] = __shfl_sync(full, pbyte, min(d0 + l, 31));
    const int64_t jb = orow0 + a.diag_off[d0];  // B row of k = 0
    switch (L) {
      case 1: dia_run<RB, 1>(a, sv, d0, pb, jb, col0, pol, acc); break;
      case 2: dia_run<RB, 2>(a, sv, d0, pb, jb, col0, pol, acc); break;
      case 3: dia_run<RB, 3>(a, sv, d0, pb, jb, col0, pol, acc); break;
      default: dia_run<RB, 4>(a, sv, d0, pb, jb, col0, pol, acc); break;
    }
    d0 += L;
  }
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    if (i0 + r >= a.dia_m) break;
    const int32_t row = (int32_t)(orow0 + r);
    float *dst = a.C + (int64_t)row * a.ldc + col0;
    float4 out = acc[r];
    if (accumulates<kAccum>(a, row)) V::add(out, V::ld(dst));
    V::st_stream(dst, out);
  }
}

// ------------------------------------------------------------------ diagonal kernel, TMA-staged B
//
// The banded kernel with its B rows staged in shared memory by the tensor-memory
// accelerator. Persistent CTAs (MB per SM) of W consumer warps and one producer warp (W + 1
// a multiple of 4: whole warps per scheduler). A work item is R = 8W consecutive listed
// rows x 128 columns. For each run of consecutive offsets
// [o, o + L) the item's rows need B rows [row0 + o, row0 + o + R + L - 1); the producer
// loads that window (a box of R + 3 rows x 128 columns; rows outside B are zero-filled, and
// no present entry uses them) with one cp.async.bulk.tensor.2d into an S-stage ring, its
// completion counted in bytes on the stage's mbarrier. A consumer warp reads its 8 + L - 1
// rows of the window from shared memory once each and applies each to the up to L of its 8
// rows that use it, so a B element crosses L2 -> SM once per run (9 times per output row of
// a 27-point stencil) and no warp waits on a global load in the inner loop. Values and
// presence bits of the next item are loaded into registers during the current one.
// Every mbarrier wait is bounded: on timeout the kernel records a code in *a.err, the
// producer waits (bounded) for the windows it issued, and the CTA returns.
template <int W>
struct DiaTmaShape {
  static constexpr int kRows = 8 * W;              // rows per item
  static constexpr int kBoxRows = kRows + 3;       // window rows (runs are at most 4 long)
  static constexpr int kStageBytes = kBoxRows * 128 * 4;
  static constexpr int kThreads = 32 * (W + 1);
  static constexpr int kValBytes = W * kMaxDiag * 8 * 4;  // per warp: [diag][8 rows]
};

// One run of L consecutive diagonals for a warp's 8 rows: each window row the warp needs is
// read from shared memory once and applied to the up to L rows that use it.
template <int L, bool kAll>
__device__ __forceinline__ void dia_tma_run(const float *wrow, const float *sv, int d0, const uint32_t (&pb)[4],
                                            float4 (&acc)[8]) {
  using V = Vec<4>;
  float v[L][8];
#pragma unroll
  for (int l = 0; l < L; ++l) {
    const float4 lo = *reinterpret_cast<const float4 *>(sv + (d0 + l) * 8);
    const float4 hi = *reinterpret_cast<const float4 *>(sv + (d0 + l) * 8 + 4);
    v[l][0] = lo.x, v[l][1] = lo.y, v[l][2] = lo.z, v[l][3] = lo.w;
    v[l][4] = hi.x, v[l][5] = hi.y, v[l][6] = hi.z, v[l][7] = hi.w;
  }
#pragma unroll
  for (int k = 0; k < 8 + L - 1; ++k) {
    const float4 b = *reinterpret_cast<const float4 *>(wrow + k * 128);
#pragma unroll
    for (int l = 0; l < L; ++l) {
      const int r = k - l;
      if (r >= 0 && r < 8 && (kAll || ((pb[l] >> r) & 1u))) V::fma(acc[r], v[l][r], b);
    }
  }
}

template <int W, int S, int MB, bool kAccum>
__global__ void __launch_bounds__(32 * (W + 1), MB)
    spmm_dia_tma_kernel(const SpmmArgs a, const __grid_constant__ CUtensorMap tmap) {
  using V = Vec<4>;
  using D = DiaTmaShape<W>;
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S];
  float *win = reinterpret_cast<float *>(dsm);  // [S][kBoxRows][128]
  const unsigned all = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ncb = a.N / 128;
  const int64_t items = (a.dia_m + D::kRows - 1) / D::kRows * ncb;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), W);  // one arrival per consumer warp
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == W) {  // producer: one thread issues every window of this CTA's items
    if (lane != 0) return;
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
    int64_t use = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < items && ok; t += gridDim.x) {
      const int64_t row0 = a.dia_row0 + t / ncb * D::kRows;
      const int32_t x = (int32_t)(t % ncb) * 128;
      int d0 = 0;
      for (int q = 0; q < a.n_runs; ++q) {
        const int s = (int)(use % S);
        const int64_t j = use / S;
        if (j > 0 && !mbar_wait_hint(smem_addr(&empty_bar[s]), (uint32_t)((j - 1) & 1), a.wait_hint_ns, a.err, 5)) {
          ok = false;
          break;
        }
        const uint32_t fb = smem_addr(&full_bar[s]);
        mbar_arrive_expect_tx(fb, D::kStageBytes);
        const int32_t y = (int32_t)(row0 + a.diag_off[d0]);
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
            "[%4];" ::"r"(smem_addr(win + (size_t)s * D::kBoxRows * 128)),
            "l"(&tmap), "r"(x), "r"(y), "r"(fb)
            : "memory");
        ++use;
        d0 += a.run_len[q];
      }
    }
    // every issued window has landed before the CTA's shared memory goes away
    for (int64_t u = use > S ? use - S : 0; u < use; ++u)
      if (!mbar_wait(smem_addr(&full_bar[u % S]), (uint32_t)((u / S) & 1), a.err, 6)) break;
    return;
  }

  // consumers
  float *sv = reinterpret_cast<float *>(dsm + (size_t)S * D::kStageBytes) + warp * (kMaxDiag * 8);
  const int col = lane * 4;
  const int nv = a.n_diag * 8;  // values per warp and item, <= 256: 8 per lane
  float pv[8];
  uint32_t ppb = 0;
  auto prefetch = [&](int64_t t) {
    const int64_t i0 = t / ncb * D::kRows + warp * 8;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int idx = lane + 32 * k, d = idx >> 3, r = idx & 7;
      pv[k] = t < items && idx < nv && i0 + r < a.dia_m ? __ldg(a.dia_vals + (int64_t)d * a.dia_m + i0 + r) : 0.f;
    }
    ppb = t < items && lane < a.n_diag && i0 < a.dia_m ? __ldg(a.dia_pres + i0 / kDiaRows * a.n_diag + lane) : 0u;
  };
  prefetch(blockIdx.x);
  int64_t use = 0;
  for (int64_t t = blockIdx.x; t < items; t += gridDim.x) {
    const int64_t i0 = t / ncb * D::kRows + warp * 8;
    const int cb = (int)(t % ncb);
    __syncwarp();  // the previous item's reads of sv are done
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (lane + 32 * k < nv) sv[lane + 32 * k] = pv[k];
    const uint32_t pbyte = ppb;
    const uint32_t fullmask = __ballot_sync(all, pbyte == 0xffu);
    __syncwarp();
    prefetch(t + gridDim.x);
    float4 acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = V::zero();
    int d0 = 0;
    for (int q = 0; q < a.n_runs; ++q) {
      const int L = a.run_len[q];
      const int s = (int)(use % S);
      if (!mbar_wait_hint(smem_addr(&full_bar[s]), (uint32_t)((use / S) & 1), a.wait_hint_ns, a.err, 7)) return;
      const float *wrow = win + ((size_t)s * D::kBoxRows + warp * 8) * 128 + col;
      const uint32_t lmask = (1u << L) - 1u, eb = smem_addr(&empty_bar[s]);
      uint32_t pb[4] = {0u, 0u, 0u, 0u};
      if (((fullmask >> d0) & lmask) == lmask) {
        switch (L) {
          case 1: dia_tma_run<1, true>(wrow, sv, d0, pb, acc); break;
          case 2: dia_tma_run<2, true>(wrow, sv, d0, pb, acc); break;
          case 3: dia_tma_run<3, true>(wrow, sv, d0, pb, acc); break;
          default: dia_tma_run<4, true>(wrow, sv, d0, pb, acc); break;
        }
      } else {
#pragma unroll
        for (int l = 0; l < 4; ++l) pb[l] = __shfl_sync(all, pbyte, min(d0 + l, 31));
        switch (L) {
          case 1: dia_tma_run<1, false>(wrow, sv, d0, pb, acc); break;
          case 2: dia_tma_run<2, false>(wrow, sv, d0, pb, acc); break;
          case 3: dia_tma_run<3, false>(wrow, sv, d0, pb, acc); break;
          default: dia_tma_run<4, false>(wrow, sv, d0, pb, acc); break;
        }
      }
      __syncwarp();  // every lane's reads of the stage are done
      if (lane == 0) mbar_arrive(eb);
      ++use;
      d0 += L;
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (i0 + r >= a.dia_m) break;
      const int32_t row = (int32_t)(a.dia_row0 + i0 + r);
      float *dst = a.C + (int64_t)row * a.ldc + cb * 128 + col;
      float4 out = acc[r];
      if (accumulates<kAccum>(a, row)) V::add(out, V::ld(dst));
      V::st_stream(dst, out);
    }
  }
}

// ------------------------------------------------------------------ fixup and fills

// One warp per cut row: C[row] = (accumulating ? C[row] : 0) + sum of its partial slots,
// in order.
template <int W, bool kAccum>
__global__ void __launch_bounds__(kSpmmThreads) spmm_fixup_kernel(const SpmmArgs a) {
  using V = Vec<W>;
  using T = typename V::T;
  const int lane = threadIdx.x & 31;
  const int64_t s = ((int64_t)blockIdx.x * kSpmmThreads + threadIdx.x) >> 5;
  if (s >= a.n_split) return;
  const int32_t row = a.split_row[s];
  const int32_t p0 = a.split_ptr[s], p1 = a.split_ptr[s + 1];
  float *dst = a.C + (int64_t)row * a.ldc;
  const bool add = accumulates<kAccum>(a, row);
  for (int col = lane * W; col < a.N; col += 32 * W) {
    T r = add ? V::ld(dst + col) : V::zero();
    for (int32_t p = p0; p < p1; ++p) V::add(r, V::ld(a.partial + (int64_t)p * a.N + col));
    V::st(dst + col, r);
  }
}

__global__ void fill_dense_kernel(float *B, int64_t row0, int64_t rows, int64_t ld, int64_t ncols,
                                  uint64_t seed) {
  const int64_t total = rows * ncols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / ncols, c = i - r * ncols;
    B[r * ld + c] = dense_value(seed, row0 + r, c);
  }
}

__global__ void zero_rows_kernel(float *C, int64_t ldc, const int32_t *rows, int64_t n, int N) {
  const int lane = threadIdx.x & 31;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n;
       i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float *dst = C + (int64_t)__ldg(rows + i) * ldc;
    for (int c = lane; c < N; c += 32) __stcs(dst + c, 0.f);
  }
}

__global__ void fill_const_kernel(float *B, int64_t n, float v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    B[i] = v;
}

// ------------------------------------------------------------------ launch selection

namespace {

using KernelFn = void (*)(const SpmmArgs);

// Instantiated (lanes per row, vectors per lane) shapes. float4 path: every LPR with
// VPL = 1, and the wider per-lane shapes that let one warp work on 2-8 rows at once (fewer
// shuffles and row checks per nonzero). Scalar path: one warp per row.
#define DSP_SHAPES_W4(X) \
  X(1, 1) X(2, 1) X(4, 1) X(8, 1) X(16, 1) X(32, 1) X(4, 2) X(8, 2) X(16, 2) X(32, 2) X(2, 4) X(4, 4) X(8, 4) \
  X(16, 4) X(32, 4) X(2, 8) X(4, 8) X(8, 8) X(16, 8) X(32, 8)
#define DSP_SHAPES_W1(X) X(32, 1) X(32, 2) X(32, 4)
// 256-bit path: the same per-lane register budgets (8-64 floats) in half the vectors
#define DSP_SHAPES_W8(X) \
  X(1, 1) X(2, 1) X(4, 1) X(8, 1) X(16, 1) X(32, 1) X(2, 2) X(4, 2) X(8, 2) X(16, 2) X(32, 2) X(2, 4) X(4, 4) \
  X(8, 4) X(16, 4) X(32, 4)

bool shape_supported(int W, int LPR, int VPL) {
#define DSP_HAS(L, P) if (LPR == L && VPL == P) return true;
  if (W == 8) {
    DSP_SHAPES_W8(DSP_HAS)
  } else if (W == 4) {
    DSP_SHAPES_W4(DSP_HAS)
  } else {
    DSP_SHAPES_W1(DSP_HAS)
  }
#undef DSP_HAS
  return false;
}

template <int V, int W, bool kAccum>
KernelFn kernel_for(int LPR, int VPL) {
#define DSP_K(L, P)                                                                                   \
  if (LPR == L && VPL == P)                                                                            \
    return V == kRowSplit ? (KernelFn)spmm_rows_kernel<L, P, W, kAccum> : (KernelFn)spmm_nnz_kernel<L, P, W, kAccum>;
  if constexpr (W == 8) {
    DSP_SHAPES_W8(DSP_K)
  } else if constexpr (W == 4) {
    DSP_SHAPES_W4(DSP_K)
  } else {
    DSP_SHAPES_W1(DSP_K)
  }
#undef DSP_K
  return nullptr;
}

template <int V>
KernelFn select_width(int W, bool accum, int LPR, int VPL) {
  if (W == 8) return accum ? kernel_for<V, 8, true>(LPR, VPL) : kernel_for<V, 8, false>(LPR, VPL);
  if (W == 4) return accum ? kernel_for<V, 4, true>(LPR, VPL) : kernel_for<V, 4, false>(LPR, VPL);
  return accum ? kernel_for<V, 1, true>(LPR, VPL) : kernel_for<V, 1, false>(LPR, VPL);
}

KernelFn select_kernel(int variant, int W, bool accum, int LPR, int VPL) {
  return variant == kRowSplit ? select_width<kRowSplit>(W, accum, LPR, VPL)
                              : select_width<kNnzSplit>(W, accum, LPR, VPL);
}

bool aligned(const void *p, uintptr_t bytes) { return ((uintptr_t)p & (bytes - 1)) == 0; }

// Warp-per-chunk shapes: vectors of 4 floats per lane per 128 columns, nonzeros per step,
// and the blocks per SM the register allocation is held to (1: the compiler's choice).
#define DSP_WARP_SHAPES(X) X(1, 4, 1) X(1, 4, 5) X(1, 8, 1) X(2, 4, 1) X(2, 4, 3) X(4, 4, 1)

KernelFn warp_kernel_for(int VPL, int U, bool accum, int MB = 1) {
#define DSP_WK(P, Q, B) \
  if (VPL == P && U == Q && MB == B) return accum ? spmm_warp_kernel<P, Q, true, B> : spmm_warp_kernel<P, Q, false, B>;
  DSP_WARP_SHAPES(DSP_WK)
#undef DSP_WK
  return nullptr;
}

// The warp-per-chunk kernel's shape for a launch, or VPL = 0 when it does not apply (the
// lane-group kernels then run): N a multiple of 128, 16-byte aligned rows of B and C.
// DSP_SPMM_WARP=0 turns it off; DSP_SPMM_WARP_VPL / DSP_SPMM_WARP_U force a shape (sweeps).
struct WarpShape {
  int VPL = 0, U = 0, gy = 0, MB = 1;
};
WarpShape warp_shape(int N, const float *B, int64_t ldb, const float *C, int64_t ldc) {
  static const int env_on = [] {
    const char *e = getenv("DSP_SPMM_WARP");
    return e ? atoi(e) : 1;
  }();
  static const int env_vpl = [] {
    const char *e = getenv("DSP_SPMM_WARP_VPL");
    return e ? atoi(e) : 0;
  }();
  static const int env_u = [] {
    const char *e = getenv("DSP_SPMM_WARP_U");
    return e ? atoi(e) : 0;
  }();
  static const int env_mb = [] {
    const char *e = getenv("DSP_SPMM_WARP_MB");
    return e ? atoi(e) : 0;
  }();
  WarpShape w;
  if (!env_on || N <= 0 || N % 128 != 0 || ldb % 4 != 0 || ldb / 4 > INT32_MAX || ldc % 4 != 0 || !aligned(B, 16) ||
      !aligned(C, 16))
    return w;
  // 4 nonzeros per step. N = 128: one float4 per lane, registers held to 48 so that 5 blocks
  // (40 warps) fit an SM (R-MAT scale 20: 1.32 ms against 1.46 uncapped and 1.92 with 8
  // nonzeros per step; scale 24: 26.9 against 29.4 ms). Wider B: 2 or 4 float4 per lane
  // (one pass over A for 256 / 512 columns; scale 20: N = 256 2.38 ms against 2.66 with one
  // float4 and two column blocks, N = 512 4.97 against 5.90), blockIdx.y covering the rest.
  const int n128 = N / 128;
  const int vpl = env_vpl > 0 && n128 % env_vpl == 0 ? env_vpl : n128 % 4 == 0 ? 4 : n128 % 2 == 0 ? 2 : 1;
  const int u = env_u > 0 ? env_u : 4;
  const int dflt_mb = vpl == 1 && u == 4 ? 5 : vpl == 2 && u == 4 ? 3 : 1;
  const int mb = env_mb > 0 && warp_kernel_for(vpl, u, false, env_mb) ? env_mb : dflt_mb;
  if (!warp_kernel_for(vpl, u, false, mb)) return w;
  w.VPL = vpl;
  w.U = u;
  w.MB = mb;
  w.gy = n128 / vpl;
  return w;
}

}  // namespace

SpmmShape spmm_shape(int N, int variant, const float *B, int64_t ldb, const float *C, int64_t ldc, int max_w) {
  // Tuning knobs for sweeps: DSP_SPMM_VEC caps the vector width (4 keeps the float4
  // path), DSP_SPMM_LPR forces the lanes per row.
  static const int env_vec = [] {
    const char *e = getenv("DSP_SPMM_VEC");
    return e ? atoi(e) : 8;
  }();
  static const int forced_lpr = [] {
    const char *e = getenv("DSP_SPMM_LPR");
    return e ? atoi(e) : 0;
  }();
  const int cap = max_w < env_vec ? max_w : env_vec;
  auto fits = [&](int w, uintptr_t bytes) {
    return N % w == 0 && ldb % w == 0 && ldc % w == 0 && aligned(B, bytes) && aligned(C, bytes);
  };
  SpmmShape s;
  s.W = cap >= 8 && fits(8, 32) ? 8 : cap >= 4 && fits(4, 16) ? 4 : 1;
  const int nv = (N + s.W - 1) / s.W;  // vectors per row
  if (s.W > 1) {
    // Each nonzero costs its group a few shuffles, an address and a row check no matter
    // how many lanes share the row, so a row gets few lanes holding several vectors each
    // (one warp then advances several rows per instruction). Per-lane budgets measured on
    // B200, in floats of the output row:
    //   nnz-split: 32 floats per lane, 2-8 lanes (N = 128 -> 4 lanes x 4 float8, or
    //              4 x 8 float4; wider rows take column chunks on blockIdx.y);
    //   row-split: 16 floats per lane, up to 32 lanes (N = 128 -> 8 x 2 float8 / 8 x 4 float4).
    const int per_lane = (variant == kNnzSplit ? 32 : 16) / s.W;
    const int max_lpr = variant == kNnzSplit ? 8 : 32;
    const int max_vpl = 32 / s.W;
    int lpr = variant == kNnzSplit ? 2 : 1;
    while (lpr * per_lane < nv && lpr < max_lpr) lpr <<= 1;
    if (forced_lpr > 0) lpr = forced_lpr;
    int vpl = 1;
    while (lpr * vpl < nv && vpl < max_vpl) vpl <<= 1;
    // DSP_SPMM_COLS caps the columns one block covers (more column chunks on blockIdx.y):
    // a smaller B-row slice per block for L1 reuse on banded matrices (sweeps)
    static const int forced_cols = [] {
      const char *e = getenv("DSP_SPMM_COLS");
      return e ? atoi(e) : 0;
    }();
    if (forced_cols > 0) {
      while (lpr * vpl * s.W > forced_cols && vpl > 1) vpl >>= 1;
      while (lpr * vpl * s.W > forced_cols && lpr > 1) lpr >>= 1;
    }
    if (!shape_supported(s.W, lpr, vpl)) {  // out-of-table request: one warp per row
      lpr = nv <= 32 ? 1 : 32;
      while (lpr < nv && lpr < 32) lpr <<= 1;
      vpl = nv <= 32 ? 1 : nv <= 64 ? 2 : 4;
    }
    s.LPR = lpr;
    s.VPL = vpl;
  } else {
    s.LPR = 32;
    s.VPL = nv <= 32 ? 1 : nv <= 64 ? 2 : 4;
  }
  s.chunk_cols = s.LPR * s.VPL * s.W;
  s.chunks = (N + s.chunk_cols - 1) / s.chunk_cols;
  return s;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda)
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return (EncodeTiledFn) nullptr;
    }
    return (EncodeTiledFn)p;
  }();
  return fn;
}

// The TMA-staged diagonal kernel for a banded launch; DSP_ERR_UNSUPPORTED (nothing launched)
// when it does not apply: DSP_SPMM_DIA_TMA=0, no error word, or a B the tensor map cannot
// describe. DSP_SPMM_DIA_TMA_SHAPE picks the CTA shape (consumer warps W, stages S, CTAs per
// SM): 1 = (7, 3, 2), the default; 2 = (15, 3, 1); 3 = (6, 4, 2); 4 = (3, 5, 3).
struct DiaTmaLaunch {
  void (*k)(const SpmmArgs, const CUtensorMap);
  int W, S, MB;
};

template <int W, int S, int MB>
DiaTmaLaunch dia_tma_launch(bool accumulate) {
  return {accumulate ? spmm_dia_tma_kernel<W, S, MB, true> : spmm_dia_tma_kernel<W, S, MB, false>, W, S, MB};
}

int launch_dia_tma(const SpmmArgs &a, bool accumulate, cudaStream_t stream) {
  const char *env = getenv("DSP_SPMM_DIA_TMA");  // read per launch (tests switch it)
  if ((env && atoi(env) == 0) || !a.err || a.b_rows <= 0 || a.b_rows > INT32_MAX || a.ldb % 4 != 0 ||
      !aligned(a.B, 16))
    return DSP_ERR_UNSUPPORTED;
  EncodeTiledFn encode = encode_tiled();
  if (!encode) return DSP_ERR_UNSUPPORTED;
  const char *env_shape = getenv("DSP_SPMM_DIA_TMA_SHAPE");
  const int shape = env_shape ? atoi(env_shape) : 1;
  const DiaTmaLaunch L = shape == 2   ? dia_tma_launch<15, 3, 1>(accumulate)
                         : shape == 3 ? dia_tma_launch<6, 4, 2>(accumulate)
                         : shape == 4 ? dia_tma_launch<3, 5, 3>(accumulate)
                                      : dia_tma_launch<7, 3, 2>(accumulate);
  const int rows_per_item = 8 * L.W, box_rows = rows_per_item + 3;
  const size_t smem = (size_t)L.S * box_rows * 128 * sizeof(float) + (size_t)L.W * kMaxDiag * 8 * sizeof(float);
  CUtensorMap tmap;
  const cuuint64_t gdim[2] = {(cuuint64_t)a.N, (cuuint64_t)a.b_rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)a.ldb * sizeof(float)};
  const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  if (encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)a.B, gdim, gstride, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return DSP_ERR_UNSUPPORTED;
  int device = 0, sms = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  // all of the unified L1 / shared array as shared memory, so MB CTAs fit on an SM
  if (cudaFuncSetAttribute((const void *)L.k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess ||
      cudaFuncSetAttribute((const void *)L.k, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
    cudaGetLastError();
    return DSP_ERR_UNSUPPORTED;
  }
  const int64_t items = (a.dia_m + rows_per_item - 1) / rows_per_item * (a.N / 128);
  const int64_t grid = std::min<int64_t>(items, (int64_t)std::max(sms, 1) * L.MB);
  SpmmArgs la = a;
  const char *env_hint = getenv("DSP_SPMM_WAIT_HINT_NS");  // suspend-time hint of the waits
  la.wait_hint_ns = env_hint ? (uint32_t)std::max(0, std::min(atoi(env_hint), 1000000)) : 0u;
  L.k<<<(unsigned)grid, 32 * (L.W + 1), smem, stream>>>(la, tmap);
  return DSP_OK;
}

int launch_spmm(const SpmmArgs &a, bool accumulate, cudaStream_t stream) {
  if (a.N <= 0) return DSP_OK;
  const SpmmShape s = spmm_shape(a.N, a.variant, a.B, a.ldb, a.C, a.ldc);
  if (s.chunks > 65535) return fail(DSP_ERR_UNSUPPORTED, "spmm: N = %d too wide", a.N);
  const int64_t units = a.variant == kRowSplit ? a.n_items : a.n_chunks;
  const WarpShape ws = a.variant == kNnzSplit && a.chunk_nnz % 16 == 0 ? warp_shape(a.N, a.B, a.ldb, a.C, a.ldc)
                                                                       : WarpShape();
  // banded row-split operands: the diagonal kernel (DSP_SPMM_DIA=0 turns it off)
  static const int env_dia = [] {
    const char *e = getenv("DSP_SPMM_DIA");
    return e ? atoi(e) : 1;
  }();
  const bool dia = env_dia && a.variant == kRowSplit && a.dia_vals && a.dia_m > 0 && a.N % 128 == 0 &&
                   a.ldb % 4 == 0 && a.ldc % 4 == 0 && aligned(a.B, 16) && aligned(a.C, 16);
  if (dia && launch_dia_tma(a, accumulate, stream) == DSP_OK) {
    // launched: the TMA-staged diagonal kernel
  } else if (dia) {
    // rows per warp: 8 (each B row of a run serves up to 8 rows) or 4 (half the registers,
    // twice the warps); DSP_SPMM_DIA_ROWS picks
    const char *env_rows = getenv("DSP_SPMM_DIA_ROWS");  // read per launch (tests switch it)
    const int rb = env_rows && atoi(env_rows) == 4 ? 4 : 8;
    const int64_t warps = (a.dia_m + rb - 1) / rb;
    const int64_t gx = (warps + kSpmmThreads / 32 - 1) / (kSpmmThreads / 32);
    if (gx > INT32_MAX) return fail(DSP_ERR_UNSUPPORTED, "spmm: %lld row blocks", (long long)warps);
    KernelFn k = rb == 4 ? (accumulate ? spmm_dia_kernel<4, true> : spmm_dia_kernel<4, false>)
                         : (accumulate ? spmm_dia_kernel<8, true> : spmm_dia_kernel<8, false>);
    k<<<dim3((unsigned)gx, (unsigned)(a.N / 128)), kSpmmThreads, 0, stream>>>(a);
  } else if (units > 0 && ws.VPL > 0) {
    KernelFn k = warp_kernel_for(ws.VPL, ws.U, accumulate, ws.MB);
    const int64_t gx = (units + kSpmmThreads / 32 - 1) / (kSpmmThreads / 32);
    if (gx > INT32_MAX) return fail(DSP_ERR_UNSUPPORTED, "spmm: %lld work units", (long long)units);
    k<<<dim3((unsigned)gx, (unsigned)ws.gy), kSpmmThreads, 0, stream>>>(a);
  } else if (units > 0) {
    KernelFn k = select_kernel(a.variant, s.W, accumulate, s.LPR, s.VPL);
    const int64_t groups_per_block = kSpmmThreads / s.LPR;
    const int64_t gx = (units + groups_per_block - 1) / groups_per_block;
    if (gx > INT32_MAX) return fail(DSP_ERR_UNSUPPORTED, "spmm: %lld work units", (long long)units);
    k<<<dim3((unsigned)gx, (unsigned)s.chunks), kSpmmThreads, 0, stream>>>(a);
  } else if (!accumulate && a.zero_rows > 0) {
    // no nonzeros at all: C = 0
    cudaError_t e = cudaMemset2DAsync(a.C, sizeof(float) * (size_t)a.ldc, 0, sizeof(float) * (size_t)a.N,
                                      (size_t)a.zero_rows, stream);
    if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "spmm zero fill: %s", cudaGetErrorString(e));
  }
  if (a.n_split > 0 && !dia) {
    KernelFn f = s.W >= 4 ? (accumulate ? spmm_fixup_kernel<4, true> : spmm_fixup_kernel<4, false>)
                          : (accumulate ? spmm_fixup_kernel<1, true> : spmm_fixup_kernel<1, false>);
    const int64_t gx = (a.n_split * 32 + kSpmmThreads - 1) / kSpmmThreads;
    f<<<(unsigned)gx, kSpmmThreads, 0, stream>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "spmm launch: %s", cudaGetErrorString(e));
  return DSP_OK;
}

int launch_fill_dense(float *B, int64_t row0, int64_t rows, int64_t ld, int64_t ncols, uint64_t seed,
                      cudaStream_t stream) {
  if (rows <= 0 || ncols <= 0) return DSP_OK;
  fill_dense_kernel<<<148 * 8, 256, 0, stream>>>(B, row0, rows, ld, ncols, seed);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DSP_OK : fail(DSP_ERR_CUDA, "fill: %s", cudaGetErrorString(e));
}

int launch_zero_rows(float *C, int64_t ldc, const int32_t *rows, int64_t n, int N, cudaStream_t stream) {
  if (n <= 0 || N <= 0) return DSP_OK;
  const int64_t blocks = std::min<int64_t>((n + 7) / 8, 148 * 8);
  zero_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(C, ldc, rows, n, N);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DSP_OK : fail(DSP_ERR_CUDA, "zero rows: %s", cudaGetErrorString(e));
}

int launch_fill_const(float *B, int64_t n, float v, cudaStream_t stream) {
  if (n <= 0) return DSP_OK;
  fill_const_kernel<<<148 * 8, 256, 0, stream>>>(B, n, v);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DSP_OK : fail(DSP_ERR_CUDA, "fill: %s", cudaGetErrorString(e));
}

// ------------------------------------------------------------------ device operand

// Chunk length for an nnz-split operand: about twice default_chunk_nnz (~64K multiply-adds),
// adjusted so the chunks fill a whole number (>= 2) of waves of resident lane groups (SMs x
// blocks per SM x groups per block of the kernel a 32-byte aligned launch at `dims` picks).
// Every chunk holds the same number of nonzeros, so a partial last wave would leave SMs
// idle while it drains (a rank's phase at R-MAT 20 on 4 ranks held 1.44 waves). Measured at
// R-MAT 20, N = 128, one GPU (waves: GFLOPS): 1: 5531, 2: 5785, 3: 5664, 4: 5786, 5: 5543,
// 7: 5458, 10: 5503, 14: 5428 — fewer, longer chunks cut fewer rows (less fixup) as long
// as dynamic scheduling over a few waves absorbs the chunks' uneven cache behaviour.
int64_t wave_chunk_nnz(int device, int dims, int64_t nnz) {
  const int64_t c = 2 * default_chunk_nnz(dims, nnz);
  if (getenv("DSP_SPMM_CHUNK") || nnz <= 0) return default_chunk_nnz(dims, nnz);
  const float *aligned_ptr = reinterpret_cast<const float *>(uintptr_t(256));
  const int ld = (dims + 7) & ~7;
  const SpmmShape sh = spmm_shape(dims, kNnzSplit, aligned_ptr, ld, aligned_ptr, ld);
  const WarpShape ws = warp_shape(dims, aligned_ptr, ld, aligned_ptr, ld);
  KernelFn k = ws.VPL > 0 ? warp_kernel_for(ws.VPL, ws.U, false, ws.MB)
                          : select_kernel(kNnzSplit, sh.W, false, sh.LPR, sh.VPL);
  const int lanes = ws.VPL > 0 ? 32 : sh.LPR, col_blocks = ws.VPL > 0 ? ws.gy : sh.chunks;
  int sms = 0, per_sm = 0;
  if (!k || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kSpmmThreads, 0) != cudaSuccess || sms <= 0 ||
      per_sm <= 0) {
    cudaGetLastError();
    return c;
  }
  const int64_t resident = (int64_t)sms * per_sm * (kSpmmThreads / lanes) / std::max(col_blocks, 1);
  const int64_t waves = std::max<int64_t>(2, (nnz + c * resident - 1) / (c * resident));
  const int64_t len = std::max<int64_t>(8, (nnz + waves * resident - 1) / (waves * resident));
  return (len + 15) / 16 * 16;  // the warp-per-chunk kernel reads 4-nonzero groups at 16-byte addresses
}

// The diagonal form of listed rows [0, m) when they are consecutive output rows
// (row0 + i) and banded: at most kMaxDiag distinct offsets col - row, filling at least
// half of the m x n_diag entries, no column twice in a row. dv[d * m + i] is the value of
// (i, row0 + i + offs[d]) (0 if absent) and bit i % 8 of pres[(i / 8) * n_diag + d] says
// whether the entry exists. Returns false when the operand is not of that shape.
static bool dia_form(int64_t m, const int32_t *row_ids, const int64_t *rp, const int64_t *idx, const float *val,
                     int64_t *row0_out, std::vector<int32_t> *offs, std::vector<float> *dv,
                     std::vector<uint8_t> *pres) {
  static const int env_dia = [] {
    const char *e = getenv("DSP_SPMM_DIA");
    return e ? atoi(e) : 1;
  }();
  const int64_t nnz = m > 0 ? rp[m] : 0;
  if (!env_dia || m <= 0 || nnz <= 0) return false;
  const int64_t row0 = row_ids ? row_ids[0] : 0;
  std::atomic<bool> ok{true};
  if (row_ids)
    parallel_for(m, [&](int64_t b, int64_t e) {
      for (int64_t i = b; i < e && ok.load(std::memory_order_relaxed); ++i)
        if (row_ids[i] != row0 + i) ok = false;
    }, 1 << 16);
  if (!ok) return false;
  // distinct offsets, per host thread then merged
  std::mutex mu;
  std::vector<int64_t> all;
  parallel_for(m, [&](int64_t b, int64_t e) {
    std::vector<int64_t> mine;
    for (int64_t i = b; i < e && ok.load(std::memory_order_relaxed); ++i)
      for (int64_t j = rp[i]; j < rp[i + 1]; ++j) {
        const int64_t o = idx[j] - (row0 + i);
        if (std::find(mine.begin(), mine.end(), o) == mine.end()) {
          mine.push_back(o);
          if ((int)mine.size() > kMaxDiag) {
            ok = false;
            break;
          }
        }
      }
    std::lock_guard<std::mutex> lk(mu);
    all.insert(all.end(), mine.begin(), mine.end());
  }, 1 << 14);
  if (!ok) return false;
  std::sort(all.begin(), all.end());
  all.erase(std::unique(all.begin(), all.end()), all.end());
  const int nd = (int)all.size();
  if (nd > kMaxDiag || 2 * nnz < m * (int64_t)nd) return false;
  offs->assign(all.begin(), all.end());
  dv->assign((size_t)(m * nd), 0.f);
  const int64_t nblk = (m + kDiaRows - 1) / kDiaRows;
  pres->assign((size_t)(nblk * nd), 0);
  parallel_for(nblk, [&](int64_t b, int64_t e) {
    for (int64_t blk = b; blk < e; ++blk)
      for (int64_t i = blk * kDiaRows; i < std::min(m, (blk + 1) * kDiaRows); ++i)
        for (int64_t j = rp[i]; j < rp[i + 1]; ++j) {
          const int64_t o = idx[j] - (row0 + i);
          const int d = (int)(std::lower_bound(all.begin(), all.end(), o) - all.begin());
          uint8_t &byte = (*pres)[(size_t)(blk * nd + d)];
          const uint8_t bit = (uint8_t)(1u << (i % kDiaRows));
          if (byte & bit) ok = false;  // the same column twice in a row
          byte |= bit;
          (*dv)[(size_t)(d * m + i)] = val[j];
        }
  }, 1024);
  if (!ok) return false;
  *row0_out = row0;
  return true;
}

// Bit 31 of the stored column ids (see col_policy): set on the columns whose B rows should
// stay in L2. When the distinct columns' rows fit in half of the L2 (or DSP_SPMM_HOT=0),
// every column is hot and all B rows are read with evict_last. Otherwise the most-referenced
// columns whose rows fill half of the L2 are hot and the rest are read with evict_first:
// on a power-law matrix whose B is many times the L2 (R-MAT scale 24: 8.6 GB of B, the top
// 246 K columns, 120 MB, carry 67 % of the nonzeros) the hot rows then survive the stream
// of rows used once. Returns the number of hot columns.
static int64_t mark_hot_columns(int device, int64_t cols, int dims, int64_t nnz, int32_t *c32) {
  static const int env_hot = [] {
    const char *e = getenv("DSP_SPMM_HOT");
    return e ? atoi(e) : 1;
  }();
  int l2 = 0;
  if (cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, device) != cudaSuccess || l2 <= 0) {
    cudaGetLastError();
    l2 = 126 << 20;
  }
  const int64_t budget = std::max<int64_t>(1, (int64_t)l2 / 2 / ((int64_t)std::max(dims, 1) * 4));
  auto mark_all = [&]() {
    parallel_for(nnz, [&](int64_t b, int64_t e) {
      for (int64_t j = b; j < e; ++j) c32[j] |= INT32_MIN;
    }, 1 << 16);
    return cols;
  };
  if (!env_hot || nnz == 0 || cols <= budget) return mark_all();
  std::vector<uint32_t> cnt((size_t)cols, 0);
  parallel_for(nnz, [&](int64_t b, int64_t e) {
    for (int64_t j = b; j < e; ++j) __atomic_fetch_add(&cnt[(size_t)c32[j]], 1u, __ATOMIC_RELAXED);
  }, 1 << 16);
  int64_t distinct = 0;
  for (uint32_t x : cnt) distinct += x > 0;
  if (distinct <= budget) return mark_all();
  // the count of the budget-th most-referenced column; columns above it are hot
  std::vector<uint32_t> sorted(cnt);
  std::nth_element(sorted.begin(), sorted.begin() + (budget - 1), sorted.end(), std::greater<uint32_t>());
  const uint32_t thr = sorted[(size_t)(budget - 1)];
  int64_t hot = 0, hot_refs = 0;
  for (uint32_t x : cnt)
    if (x > thr) {
      ++hot;
      hot_refs += x;
    }
  // Only a skewed matrix gains: the hot columns must take a share of the references well
  // above their share of the columns (R-MAT scale 24: 67 % of the references on 2.8 % of the
  // columns). On flat degree distributions (stencils, uniform rows) the counts tie at the
  // threshold and evict_first would only throw away L2 reuse, so every column stays hot.
  if (hot < budget / 4 || (double)hot_refs / (double)nnz < 4.0 * (double)hot / (double)distinct) return mark_all();
  parallel_for(nnz, [&](int64_t b, int64_t e) {
    for (int64_t j = b; j < e; ++j)
      if (cnt[(size_t)c32[j]] > thr) c32[j] |= INT32_MIN;
  }, 1 << 16);
  return hot;
}

int DevOperand::upload(int device_, int64_t rows_, int64_t cols_, const int64_t *row_ptr, const int32_t *row_ids,
                       int64_t m, const int64_t *indices, const float *values, int64_t first_nz, int64_t nnz_,
                       int dims, bool include_empty, int variant_) {
  release();
  device = device_;
  rows = rows_;
  cols = cols_;
  nnz = nnz_;
  zero_rows = include_empty ? rows_ : 0;
  std::vector<int64_t> rp((size_t)m + 1);
  for (int64_t i = 0; i <= m; ++i) rp[(size_t)i] = row_ptr[i] - first_nz;
  // a banded operand runs on the diagonal kernel (with the row-split items as its fallback
  // for widths that kernel does not take), whatever its row lengths
  std::vector<int32_t> offs;
  std::vector<float> dv;
  std::vector<uint8_t> pres;
  const bool banded = variant_ != kNnzSplit &&
                      dia_form(m, row_ids, rp.data(), indices + first_nz, values + first_nz, &dia_row0, &offs, &dv, &pres);
  variant = variant_ >= 0 ? variant_ : banded ? (int)kRowSplit : choose_variant(m, rp.data(), dims);
  std::vector<int32_t> split_row, split_ptr;
  int rc;
  if (variant == kRowSplit) {
    ItemPlan plan;
    build_items(m, row_ids, rp.data(), default_piece_cap(dims), include_empty, &plan);
    n_items = (int64_t)plan.item_out.size();
    pieces = plan.pieces;
    piece_cap = plan.piece_cap;
    max_row_len = plan.max_row_len;
    split_row.swap(plan.split_row);
    split_ptr.swap(plan.split_ptr);
    if ((rc = dev_upload(&d_item_ptr, plan.item_ptr.data(), sizeof(int64_t) * plan.item_ptr.size())) ||
        (rc = dev_upload(&d_item_out, plan.item_out.data(), sizeof(int32_t) * plan.item_out.size())))
      return rc;
    if (banded) {
      n_diag = (int)offs.size();
      for (int d = 0; d < n_diag; ++d) diag_off[d] = offs[(size_t)d];
      n_runs = 0;
      for (int d = 0; d < n_diag;) {  // runs of consecutive offsets, at most 4 long
        int len = 1;
        while (d + len < n_diag && len < 4 && offs[(size_t)(d + len)] == offs[(size_t)d] + len) ++len;
        run_len[n_runs++] = (uint8_t)len;
        d += len;
      }
      n_lrows = m;
      if ((rc = dev_upload(&d_dia_vals, dv.data(), sizeof(float) * dv.size())) ||
          (rc = dev_upload(&d_dia_pres, pres.data(), pres.size())))
        return rc;
    }
  } else {
    ChunkPlan plan;
    build_chunks(m, row_ids, rp.data(), wave_chunk_nnz(device_, dims, nnz_), &plan);
    n_chunks = plan.n_chunks;
    chunk_nnz = plan.chunk_nnz;
    pieces = plan.slots;
    piece_cap = plan.chunk_nnz;
    max_row_len = plan.max_row_len;
    split_row.swap(plan.split_row);
    split_ptr.swap(plan.split_ptr);
    if ((rc = dev_upload(&d_coo_row, plan.coo_row.data(), sizeof(int32_t) * (size_t)nnz)) ||
        (rc = dev_upload(&d_chunk_slot, plan.chunk_slot.data(), sizeof(int32_t) * (size_t)(2 * n_chunks))))
      return rc;
  }
  n_split = (int64_t)split_row.size();
  // column ids (int32) and values
  const int64_t padded = std::max<int64_t>(nnz, 1);
  std::vector<int32_t> c32((size_t)padded, 0);
  std::vector<float> v32((size_t)padded, 0.f);
  parallel_for(nnz, [&](int64_t b, int64_t e) {
    for (int64_t j = b; j < e; ++j) {
      c32[(size_t)j] = (int32_t)indices[first_nz + j];
      v32[(size_t)j] = values[first_nz + j];
    }
  }, 1 << 16);
  hot_cols = mark_hot_columns(device_, cols_, dims, nnz, c32.data());
  if ((rc = dev_upload(&d_split_row, split_row.data(), sizeof(int32_t) * split_row.size())) ||
      (rc = dev_upload(&d_split_ptr, split_ptr.data(), sizeof(int32_t) * split_ptr.size())) ||
      (rc = dev_upload(&d_cols, c32.data(), sizeof(int32_t) * (size_t)padded)) ||
      (rc = dev_upload(&d_vals, v32.data(), sizeof(float) * (size_t)padded)))
    return rc;
  return DSP_OK;
}

void DevOperand::release() {
  for (void **p : {(void **)&d_item_ptr, (void **)&d_item_out, (void **)&d_coo_row, (void **)&d_chunk_slot,
                   (void **)&d_dia_vals, (void **)&d_dia_pres, (void **)&d_split_row,
                   (void **)&d_split_ptr, (void **)&d_cols, (void **)&d_vals}) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
  n_items = n_chunks = n_split = pieces = n_lrows = 0;
  n_diag = n_runs = 0;
}

int64_t DevOperand::device_bytes() const {
  const int64_t nnz_split = variant == kNnzSplit ? nnz * 4 : 0;
  const int64_t dia = d_dia_vals ? n_lrows * n_diag * 4 + (n_lrows + kDiaRows - 1) / kDiaRows * n_diag : 0;
  return n_items * 12 + 8 + n_chunks * 8 + nnz_split + n_split * 8 + 4 + nnz * 8 + dia;
}

SpmmArgs DevOperand::args(const float *B, int64_t ldb, float *C, int64_t ldc, int N, float *partial) const {
  SpmmArgs a;
  memset(&a, 0, sizeof a);
  a.variant = variant;
  a.item_ptr = d_item_ptr;
  a.item_out = d_item_out;
  a.n_items = n_items;
  a.coo_row = d_coo_row;
  a.chunk_slot = d_chunk_slot;
  a.dia_vals = d_dia_vals;
  a.dia_pres = d_dia_pres;
  a.dia_m = d_dia_vals ? n_lrows : 0;
  a.dia_row0 = dia_row0;
  a.n_diag = n_diag;
  memcpy(a.diag_off, diag_off, sizeof diag_off);
  a.n_runs = n_runs;
  memcpy(a.run_len, run_len, sizeof run_len);
  a.n_chunks = n_chunks;
  a.chunk_nnz = chunk_nnz;
  a.nnz = nnz;
  a.zero_rows = zero_rows;
  a.split_row = d_split_row;
  a.split_ptr = d_split_ptr;
  a.n_split = n_split;
  a.cols = d_cols;
  a.vals = d_vals;
  a.B = B;
  a.ldb = ldb;
  a.b_rows = cols;
  a.C = C;
  a.ldc = ldc;
  a.partial = partial;
  a.N = N;
  return a;
}

int dev_upload(void *dptr_out, const void *host, size_t bytes) {
  void **dptr = (void **)dptr_out;
  *dptr = nullptr;
  if (bytes == 0) return DSP_OK;
  cudaError_t e = cudaMalloc(dptr, bytes);
  if (e != cudaSuccess) return fail(DSP_ERR_NOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemcpy(*dptr, host, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "cudaMemcpy H2D: %s", cudaGetErrorString(e));
  return DSP_OK;
}

void prefer_l1_carveout() {
  static thread_local int done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 31 && (done_mask >> dev) & 1) return;
  for (int v = 0; v < 2; ++v)
    for (int w : {8, 4, 1})
      for (int acc = 0; acc < 2; ++acc)
        for (int lpr = 1; lpr <= 32; lpr <<= 1)
          for (int vpl = 1; vpl <= 8; vpl <<= 1)
            if (shape_supported(w, lpr, vpl))
              cudaFuncSetAttribute(select_kernel(v, w, acc != 0, lpr, vpl),
                                   cudaFuncAttributePreferredSharedMemoryCarveout, 0);
  for (int acc = 0; acc < 2; ++acc) {
#define DSP_WC(P, Q, B) \
  cudaFuncSetAttribute(warp_kernel_for(P, Q, acc != 0, B), cudaFuncAttributePreferredSharedMemoryCarveout, 0);
    DSP_WARP_SHAPES(DSP_WC)
#undef DSP_WC
  }
  cudaGetLastError();
  if (dev < 31) done_mask |= 1 << dev;
}

}  // namespace dsp

// ------------------------------------------------------------------ C ABI: single-GPU plan

struct dsp_spmm_plan {
  dsp::DevOperand op;
  float *scratch = nullptr;
  int64_t scratch_floats = 0;
  int *d_err = nullptr;  // set by a kernel whose bounded wait gave up (dsp_spmm_check_error)
};

using namespace dsp;

extern "C" int dsp_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

extern "C" int dsp_spmm_plan_create(int device, const dsp_csr *a, int dims_hint, int variant, dsp_spmm_plan **out) {
  DSP_TRY_ARG(a && out && a->indptr, "dsp_spmm_plan_create: null argument");
  DSP_TRY_ARG(a->num_cols <= INT32_MAX && a->num_rows <= INT32_MAX, "dsp_spmm_plan_create: matrix too large for int32 ids");
  *out = nullptr;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  prefer_l1_carveout();
  dsp_spmm_plan *p = new dsp_spmm_plan();
  const int dims = dims_hint > 0 ? dims_hint : 128;
  DSP_TRY_ARG(variant >= -1 && variant <= 1, "dsp_spmm_plan_create: variant %d", variant);
  int rc = p->op.upload(device, a->num_rows, a->num_cols, a->indptr, nullptr, a->num_rows, a->indices, a->values, 0,
                        a->nnz, dims, true, variant);
  if (rc == DSP_OK && p->op.pieces > 0) {
    p->scratch_floats = p->op.pieces * (int64_t)dims;
    e = cudaMalloc(&p->scratch, sizeof(float) * (size_t)p->scratch_floats);
    if (e != cudaSuccess) rc = fail(DSP_ERR_NOMEM, "spmm scratch: %s", cudaGetErrorString(e));
  }
  if (rc == DSP_OK && ((e = cudaMalloc(&p->d_err, sizeof(int))) != cudaSuccess ||
                       (e = cudaMemset(p->d_err, 0, sizeof(int))) != cudaSuccess))
    rc = fail(DSP_ERR_NOMEM, "spmm error word: %s", cudaGetErrorString(e));
  if (rc) {
    dsp_spmm_plan_destroy(p);
    return rc;
  }
  *out = p;
  return DSP_OK;
}

extern "C" void dsp_spmm_plan_destroy(dsp_spmm_plan *p) {
  if (!p) return;
  cudaSetDevice(p->op.device);
  p->op.release();
  if (p->scratch) cudaFree(p->scratch);
  if (p->d_err) cudaFree(p->d_err);
  delete p;
}

extern "C" int dsp_spmm_check_error(dsp_spmm_plan *p) {
  DSP_TRY_ARG(p, "dsp_spmm_check_error: null plan");
  cudaError_t e = cudaSetDevice(p->op.device);
  int flag = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&flag, p->d_err, sizeof flag, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && flag != 0) e = cudaMemset(p->d_err, 0, sizeof(int));
  if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "dsp_spmm_check_error: %s", cudaGetErrorString(e));
  if (flag == 0) return DSP_OK;
  return fail(DSP_ERR_TIMEOUT, "spmm: a bounded wait gave up (code %d); C is incomplete", flag);
}

extern "C" int dsp_spmm_plan_info(const dsp_spmm_plan *p, dsp_spmm_info *info) {
  DSP_TRY_ARG(p && info, "dsp_spmm_plan_info: null argument");
  info->rows = p->op.rows;
  info->cols = p->op.cols;
  info->nnz = p->op.nnz;
  info->variant = p->op.variant;
  info->items = p->op.variant == kRowSplit ? p->op.n_items : p->op.n_chunks;
  info->split_rows = p->op.n_split;
  info->pieces = p->op.pieces;
  info->piece_cap = p->op.piece_cap;
  info->max_row_len = p->op.max_row_len;
  info->scratch_bytes = p->scratch_floats * 4;
  info->device_bytes = p->op.device_bytes() + info->scratch_bytes;
  return DSP_OK;
}

extern "C" int dsp_spmm_f32(dsp_spmm_plan *p, const float *B, int64_t ldb, float *C, int64_t ldc, int N,
                            int accumulate, void *stream) {
  DSP_TRY_ARG(p, "dsp_spmm_f32: null plan");
  DSP_TRY_ARG(N >= 0 && ldb >= N && ldc >= N, "dsp_spmm_f32: N=%d ldb=%lld ldc=%lld", N, (long long)ldb,
              (long long)ldc);
  if (N == 0) return DSP_OK;  // nothing to compute; empty operands may be null
  DSP_TRY_ARG((B || p->op.nnz == 0) && (C || p->op.rows == 0), "dsp_spmm_f32: null argument");
  if (p->op.pieces > 0 && p->op.pieces * (int64_t)N > p->scratch_floats) {
    // first use with a wider B than the plan was sized for: grow the scratch (synchronous)
    cudaSetDevice(p->op.device);
    cudaStreamSynchronize((cudaStream_t)stream);
    if (p->scratch) cudaFree(p->scratch);
    p->scratch = nullptr;
    p->scratch_floats = p->op.pieces * (int64_t)N;
    cudaError_t e = cudaMalloc(&p->scratch, sizeof(float) * (size_t)p->scratch_floats);
    if (e != cudaSuccess) {
      p->scratch_floats = 0;
      return fail(DSP_ERR_NOMEM, "spmm scratch: %s", cudaGetErrorString(e));
    }
  }
  SpmmArgs a = p->op.args(B, ldb, C, ldc, N, p->scratch);
  a.err = p->d_err;
  return launch_spmm(a, accumulate != 0, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ allocation-free entry point
//
// dsp_spmm_csr_f32_noalloc: C (+)= A.B for a CSR matrix the caller already holds in device
// memory (int64 indptr / indices, fp32 values: the reference's on-disk and SparseMatrix
// layout), without allocating any device memory. It is meant for callers that cannot or
// must not call cudaMalloc: code running on a latency-critical stream next to other work
// (cudaMalloc / cudaFree can synchronise the whole device), frameworks that own all device
// memory through their own pool and forbid allocations behind their back, and steps that
// must not fail halfway with an out-of-memory error.
//
// It is the nnz-split kernel without host planning: every chunk of chunk_nnz nonzeros finds
// its first row by binary search in indptr; a row cut by chunk boundaries leaves one partial
// row per chunk it touches, in slot 2c ("cut before", the chunk's first row) or 2c + 1 ("cut
// after only", the chunk's last row), and the chunk where the row ends sums those slots in
// chunk order (deterministic). The slots are the only scratch and live in the static array
// below: kNoAllocScratchBytes on every GPU that loads this library, held until exit.
// Nothing in it has to start at zero (every slot read was written by the same call), but
// all calls on a device share it, so calls that overlap on the GPU (different streams)
// race on it.

namespace dsp {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

struct CsrChunkArgs {
  SpmmArgs base;           // B, C, N, ldb, ldc; base.partial = the slots
  const int64_t *indptr;   // [rows + 1]
  const int64_t *indices;  // [nnz]
  int64_t rows;
};

// Last row r in [lo, rows) with indptr[r] <= p (the nonempty row holding nonzero p,
// 0 <= p < nnz), given indptr[lo] <= p.
__device__ __forceinline__ int64_t row_holding(const int64_t *indptr, int64_t rows, int64_t p, int64_t lo = 0) {
  int64_t hi = rows;  // indptr[lo] <= p < indptr[hi] = nnz
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (__ldg(indptr + mid) <= p) lo = mid;
    else hi = mid;
  }
  return lo;
}

// The row holding nonzero p > the last nonzero of `row` (p < nnz): the rows a chunk moves
// into are usually adjacent, so step forward over a few rows before searching the rest.
// While r is below the holder, indptr[r + 1] <= p < nnz keeps r + 1 < rows, so every load
// is in bounds, and indptr[r] <= p holds for the search that takes over.
__device__ __forceinline__ int64_t next_row_holding(const int64_t *indptr, int64_t rows, int64_t row, int64_t p) {
  int64_t r = row + 1;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (__ldg(indptr + r + 1) > p) return r;
    ++r;
  }
  return row_holding(indptr, rows, p, r);
}

template <int LPR, int VPL, int W, bool kAccum>
__global__ void __launch_bounds__(kSpmmThreads) spmm_csr_chunks_kernel(const CsrChunkArgs ca) {
  using V = Vec<W>;
  using T = typename V::T;
  const SpmmArgs &a = ca.base;
  constexpr int U = loads_in_flight<LPR, VPL, W>();
  constexpr int K = entries_per_lane<LPR>();
  const int lane = threadIdx.x & (LPR - 1);
  const int64_t chunk = ((int64_t)blockIdx.x * kSpmmThreads + threadIdx.x) / LPR;
  if (chunk >= a.n_chunks) return;
  const unsigned gmask = group_mask<LPR>();
  const int col0 = blockIdx.y * (LPR * VPL * W) + lane * W;
  const int64_t s = chunk * a.chunk_nnz, e = min(s + a.chunk_nnz, a.nnz);
  const uint64_t pol = evict_last_policy();

  int64_t row = row_holding(ca.indptr, ca.rows, s);
  int64_t rbeg = __ldg(ca.indptr + row), rend = __ldg(ca.indptr + row + 1);
  if (!kAccum) zero_rows<LPR, VPL, W>(a, s > 0 ? row_holding(ca.indptr, ca.rows, s - 1) + 1 : 0, row, col0);
  // partial slot of the current row: cut before this chunk -> 2c, cut only after -> 2c + 1
  auto slot_of = [&](int64_t b, int64_t en) -> int32_t {
    return b < s ? (int32_t)(2 * chunk) : (en > e ? (int32_t)(2 * chunk + 1) : -1);
  };

  T acc[VPL];
#pragma unroll
  for (int w = 0; w < VPL; ++w) acc[w] = V::zero();

  for (int64_t base = s; base < e; base += LPR * K) {
    int64_t c[K];
    float v[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t p = base + k * LPR + lane;
      c[k] = p < e ? (int64_t)__ldcs((const long long *)ca.indices + p) : 0;
      v[k] = p < e ? __ldcs(a.vals + p) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t kb = base + k * LPR;
      if (kb >= e) break;
      const int n = (int)min((int64_t)LPR, e - kb);
      for (int j = 0; j < n; j += U) {
        T b[U][VPL];
        float sv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t cj = __shfl_sync(gmask, (long long)c[k], j + u, LPR);
          sv[u] = __shfl_sync(gmask, v[k], j + u, LPR);
          const float *brow = a.B + cj * a.ldb;
#pragma unroll
          for (int w = 0; w < VPL; ++w) {
            const int col = col0 + w * LPR * W;
            b[u][w] = (j + u < n && col < a.N) ? V::ldg(brow + col, pol) : V::zero();
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t p = kb + j + u;
          if (j + u < n) {
            if (p >= rend) {  // group-uniform: the chunk crosses into a later row
              flush_row<LPR, VPL, W, kAccum>(a, (int32_t)row, slot_of(rbeg, rend), col0, acc);
              const int64_t next = next_row_holding(ca.indptr, ca.rows, row, p);
              if (!kAccum) zero_rows<LPR, VPL, W>(a, row + 1, next, col0);
              row = next;
              rbeg = __ldg(ca.indptr + row);
              rend = __ldg(ca.indptr + row + 1);
#pragma unroll
              for (int w = 0; w < VPL; ++w) acc[w] = V::zero();
            }
#pragma unroll
            for (int w = 0; w < VPL; ++w) V::fma(acc[w], sv[u], b[u][w]);
          }
        }
      }
    }
  }
  flush_row<LPR, VPL, W, kAccum>(a, (int32_t)row, slot_of(rbeg, rend), col0, acc);
  if (!kAccum && chunk == a.n_chunks - 1) zero_rows<LPR, VPL, W>(a, row + 1, ca.rows, col0);
}

// One warp per chunk: if the chunk's first row began in an earlier chunk c0 and ends here,
// C[row] = (kAccum ? C[row] : 0) + slot[2 c0 + 1] + slot[2k] for k = c0+1 .. this chunk.
template <int W, bool kAccum>
__global__ void __launch_bounds__(kSpmmThreads) spmm_csr_chunks_fixup_kernel(const CsrChunkArgs ca) {
  using V = Vec<W>;
  using T = typename V::T;
  const SpmmArgs &a = ca.base;
  const int lane = threadIdx.x & 31;
  const int64_t chunk = ((int64_t)blockIdx.x * kSpmmThreads + threadIdx.x) >> 5;
  if (chunk >= a.n_chunks) return;
  const int64_t s = chunk * a.chunk_nnz, e = min(s + a.chunk_nnz, a.nnz);
  const int64_t row = row_holding(ca.indptr, ca.rows, s);
  const int64_t rbeg = __ldg(ca.indptr + row), rend = __ldg(ca.indptr + row + 1);
  if (!(rbeg < s && rend <= e)) return;  // not a cut row that ends in this chunk
  const int64_t c0 = rbeg / a.chunk_nnz;
  float *dst = a.C + row * a.ldc;
  for (int col = lane * W; col < a.N; col += 32 * W) {
    T r = kAccum ? V::ld(dst + col) : V::zero();
    V::add(r, V::ld(a.partial + (2 * c0 + 1) * (int64_t)a.N + col));
    for (int64_t k = c0 + 1; k <= chunk; ++k) V::add(r, V::ld(a.partial + (2 * k) * (int64_t)a.N + col));
    V::st(dst + col, r);
  }
}

namespace {

using CsrKernelFn = void (*)(const CsrChunkArgs);

// Every shape spmm_shape(..., max_w = 4) can return.
template <int W, bool kAccum>
CsrKernelFn csr_kernel_for(int LPR, int VPL) {
#define DSP_CK(L, P) \
  if (LPR == L && VPL == P) return spmm_csr_chunks_kernel<L, P, W, kAccum>;
  if constexpr (W == 4) {
    DSP_SHAPES_W4(DSP_CK)
  } else {
    DSP_SHAPES_W1(DSP_CK)
  }
#undef DSP_CK
  return nullptr;
}

std::mutex g_noalloc_mu;
float *g_noalloc_ptr[64] = {};

// Device address of this device's static scratch (looked up once per device, with that
// device current).
int noalloc_scratch(int dev, float **out) {
  if (dev < 0 || dev >= 64) return fail(DSP_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = (float *)p;
  }
  *out = g_noalloc_ptr[dev];
  return DSP_OK;
}

}  // namespace
}  // namespace dsp

extern "C" int dsp_spmm_csr_f32_noalloc(const int64_t *indptr, const int64_t *indices, const float *values,
                                        int64_t rows, int64_t cols, int64_t nnz, const float *B, int64_t ldb,
                                        float *C, int64_t ldc, int N, int accumulate, void *stream) {
  DSP_TRY_ARG(rows >= 0 && cols >= 0 && nnz >= 0, "dsp_spmm_csr_f32_noalloc: negative size");
  DSP_TRY_ARG(N >= 0 && ldb >= N && ldc >= N, "dsp_spmm_csr_f32_noalloc: N=%d ldb=%lld ldc=%lld", N,
              (long long)ldb, (long long)ldc);
  if (N > DSP_NOALLOC_MAX_N)
    return fail(DSP_ERR_UNSUPPORTED, "dsp_spmm_csr_f32_noalloc: N = %d exceeds the maximum %d of its %zu-byte scratch",
                N, DSP_NOALLOC_MAX_N, kNoAllocScratchBytes);
  if (rows > INT32_MAX)
    return fail(DSP_ERR_UNSUPPORTED, "dsp_spmm_csr_f32_noalloc: %lld rows exceed 2^31 - 1", (long long)rows);
  // the scratch address first, so that a call with nothing to compute (N, rows or nnz 0)
  // sets the device up ahead of latency-critical work or stream capture
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  float *slots = nullptr;
  int rc = noalloc_scratch(dev, &slots);
  if (rc) return rc;
  if (N == 0 || rows == 0) return DSP_OK;
  DSP_TRY_ARG(indptr && C && (nnz == 0 || (indices && values && B)), "dsp_spmm_csr_f32_noalloc: null argument");
  cudaStream_t st = (cudaStream_t)stream;
  if (nnz == 0) {
    if (accumulate) return DSP_OK;
    e = cudaMemset2DAsync(C, sizeof(float) * (size_t)ldc, 0, sizeof(float) * (size_t)N, (size_t)rows, st);
    return e == cudaSuccess ? DSP_OK : fail(DSP_ERR_CUDA, "zero fill: %s", cudaGetErrorString(e));
  }
  // chunk length: the usual one, grown until two slots per chunk fit the static scratch
  const int64_t max_chunks = (int64_t)(kNoAllocScratchBytes / sizeof(float)) / (2 * (int64_t)N);
  int64_t chunk = default_chunk_nnz(N, nnz);
  if ((nnz + chunk - 1) / chunk > max_chunks) chunk = ((nnz + max_chunks - 1) / max_chunks + 31) & ~int64_t(31);
  CsrChunkArgs ca;
  memset(&ca, 0, sizeof ca);
  ca.base.vals = values;
  ca.base.B = B;
  ca.base.ldb = ldb;
  ca.base.C = C;
  ca.base.ldc = ldc;
  ca.base.partial = slots;
  ca.base.N = N;
  ca.base.nnz = nnz;
  ca.base.chunk_nnz = chunk;
  ca.base.n_chunks = (nnz + chunk - 1) / chunk;
  ca.indptr = indptr;
  ca.indices = indices;
  ca.rows = rows;
  const SpmmShape s = spmm_shape(N, kNnzSplit, B, ldb, C, ldc, 4);
  CsrKernelFn k = nullptr;
  if (s.W == 4)
    k = accumulate ? csr_kernel_for<4, true>(s.LPR, s.VPL) : csr_kernel_for<4, false>(s.LPR, s.VPL);
  else
    k = accumulate ? csr_kernel_for<1, true>(s.LPR, s.VPL) : csr_kernel_for<1, false>(s.LPR, s.VPL);
  if (!k) return fail(DSP_ERR_UNSUPPORTED, "dsp_spmm_csr_f32_noalloc: no kernel for N = %d", N);
  const int64_t groups_per_block = kSpmmThreads / s.LPR;
  const int64_t gx = (ca.base.n_chunks + groups_per_block - 1) / groups_per_block;
  k<<<dim3((unsigned)gx, (unsigned)s.chunks), kSpmmThreads, 0, st>>>(ca);
  CsrKernelFn f = s.W == 4 ? (accumulate ? spmm_csr_chunks_fixup_kernel<4, true> : spmm_csr_chunks_fixup_kernel<4, false>)
                           : (accumulate ? spmm_csr_chunks_fixup_kernel<1, true> : spmm_csr_chunks_fixup_kernel<1, false>);
  f<<<(unsigned)((ca.base.n_chunks * 32 + kSpmmThreads - 1) / kSpmmThreads), kSpmmThreads, 0, st>>>(ca);
  e = cudaGetLastError();
  return e == cudaSuccess ? DSP_OK : fail(DSP_ERR_CUDA, "dsp_spmm_csr_f32_noalloc launch: %s", cudaGetErrorString(e));
}
