// spmm.cu — sm_100a CSR x dense fp32 SpMM kernels and the single-GPU plan API.
//
// C[rows x N] (+)= A[rows x cols] * B[cols x N]; A in CSR with int32 column ids, B and C
// row-major fp32. This is a gather-and-accumulate, bound by HBM / L2 bandwidth, not a
// dense contraction, so it runs on the CUDA cores:
//   * the rows are cut on the host into work items: one item per row, except rows longer
//     than `piece_cap` nonzeros, which become balanced pieces whose partial rows go to a
//     scratch buffer and are summed in piece order by a fixup kernel (deterministic; no
//     atomics);
//   * a group of LPR lanes (a warp for N >= 128) owns one item; each lane holds VPL
//     vectors of W floats of the output row, so one B row is read as LPR*W*4 contiguous
//     bytes (512 B at N = 128: 32 lanes x float4);
//   * the group loads LPR (column, value) pairs with one coalesced streaming load each,
//     broadcasts them with warp shuffles, and keeps up to 8 B-row loads in flight per lane
//     before the FMAs;
//   * B goes through the read-only path (L1-cached: rows shared by neighbouring items hit
//     in L1), A is streamed (evict-first), whole-row results are stored once.
// Replaces cusparseSpMM(COO, ALG_DEFAULT, beta = 1) of src/dist_spmm_node.cu:354-385.
#include <cuda_runtime.h>
#include <string.h>

#include "device.cuh"
#include "internal.h"

namespace dsp {

// ------------------------------------------------------------------ vector helpers
template <int W>
struct Vec;
template <>
struct Vec<4> {
  using T = float4;
  static __device__ __forceinline__ T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  static __device__ __forceinline__ T ldg(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }
  static __device__ __forceinline__ T ld(const float *p) { return *reinterpret_cast<const float4 *>(p); }
  static __device__ __forceinline__ void st(float *p, T v) { *reinterpret_cast<float4 *>(p) = v; }
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
template <>
struct Vec<1> {
  using T = float;
  static __device__ __forceinline__ T zero() { return 0.f; }
  static __device__ __forceinline__ T ldg(const float *p) { return __ldg(p); }
  static __device__ __forceinline__ T ld(const float *p) { return *p; }
  static __device__ __forceinline__ void st(float *p, T v) { *p = v; }
  static __device__ __forceinline__ void fma(T &acc, float s, T b) { acc = fmaf(s, b, acc); }
  static __device__ __forceinline__ void add(T &acc, T b) { acc += b; }
};

// ------------------------------------------------------------------ kernels

// One item per group of LPR lanes; blockIdx.y selects a chunk of LPR*VPL*W columns.
template <int LPR, int VPL, int W, bool kAccum>
__global__ void __launch_bounds__(kSpmmThreads) spmm_items_kernel(const SpmmArgs a) {
  using V = Vec<W>;
  using T = typename V::T;
  // nonzeros whose B vectors are loaded before their FMAs: 8 vectors in flight per lane
  constexpr int U = LPR < 8 ? LPR : (8 / VPL >= 2 ? 8 / VPL : 2);
  const int lane = threadIdx.x & (LPR - 1);
  const int64_t item = ((int64_t)blockIdx.x * kSpmmThreads + threadIdx.x) / LPR;
  if (item >= a.n_items) return;
  const unsigned gmask =
      LPR == 32 ? 0xffffffffu : (((1u << LPR) - 1u) << ((threadIdx.x & 31) & ~(LPR - 1)));
  const int col0 = blockIdx.y * (LPR * VPL * W) + lane * W;
  const int64_t beg = a.item_ptr[item], end = a.item_ptr[item + 1];

  T acc[VPL];
#pragma unroll
  for (int w = 0; w < VPL; ++w) acc[w] = V::zero();

  for (int64_t base = beg; base < end; base += LPR) {
    const int n = (int)min((int64_t)LPR, end - base);
    int c = 0;
    float v = 0.f;
    if (lane < n) {
      c = __ldcs(a.cols + base + lane);
      v = __ldcs(a.vals + base + lane);
    }
    for (int j = 0; j < n; j += U) {
      T b[U][VPL];
      float s[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int cj = __shfl_sync(gmask, c, j + u, LPR);
        s[u] = __shfl_sync(gmask, v, j + u, LPR);
        const float *brow = a.B + (int64_t)cj * a.ldb;
#pragma unroll
        for (int w = 0; w < VPL; ++w) {
          const int col = col0 + w * LPR * W;
          b[u][w] = (j + u < n && col < a.N) ? V::ldg(brow + col) : V::zero();
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int w = 0; w < VPL; ++w)
          if (j + u < n) V::fma(acc[w], s[u], b[u][w]);
    }
  }

  const int32_t o = a.item_out[item];
  if (o >= 0) {
    float *dst = a.C + (int64_t)o * a.ldc;
#pragma unroll
    for (int w = 0; w < VPL; ++w) {
      const int col = col0 + w * LPR * W;
      if (col < a.N) {
        T r = acc[w];
        if (kAccum) V::add(r, V::ld(dst + col));
        V::st(dst + col, r);
      }
    }
  } else {
    float *dst = a.partial + (int64_t)(-(o + 1)) * a.N;
#pragma unroll
    for (int w = 0; w < VPL; ++w) {
      const int col = col0 + w * LPR * W;
      if (col < a.N) V::st(dst + col, acc[w]);
    }
  }
}

// One warp per split row: C[row] = (kAccum ? C[row] : 0) + sum of its pieces, in order.
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
  for (int col = lane * W; col < a.N; col += 32 * W) {
    T r = kAccum ? V::ld(dst + col) : V::zero();
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

__global__ void fill_const_kernel(float *B, int64_t n, float v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    B[i] = v;
}

// ------------------------------------------------------------------ launch selection

namespace {

using KernelFn = void (*)(const SpmmArgs);

template <int W, bool kAccum>
KernelFn pick_items(int LPR, int VPL) {
  if (W == 4) {
    if (VPL == 1) {
      switch (LPR) {
        case 1: return spmm_items_kernel<1, 1, W, kAccum>;
        case 2: return spmm_items_kernel<2, 1, W, kAccum>;
        case 4: return spmm_items_kernel<4, 1, W, kAccum>;
        case 8: return spmm_items_kernel<8, 1, W, kAccum>;
        case 16: return spmm_items_kernel<16, 1, W, kAccum>;
        default: return spmm_items_kernel<32, 1, W, kAccum>;
      }
    }
  }
  if (VPL == 1) return spmm_items_kernel<32, 1, W, kAccum>;
  if (VPL == 2) return spmm_items_kernel<32, 2, W, kAccum>;
  return spmm_items_kernel<32, 4, W, kAccum>;
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

SpmmShape spmm_shape(int N, const float *B, int64_t ldb, const float *C, int64_t ldc) {
  SpmmShape s;
  const bool vec4 = N % 4 == 0 && ldb % 4 == 0 && ldc % 4 == 0 && aligned16(B) && aligned16(C);
  s.W = vec4 ? 4 : 1;
  const int nv = N / s.W;  // vectors per row
  if (vec4 && nv <= 32) {
    int lpr = 1;
    while (lpr < nv) lpr <<= 1;
    s.LPR = lpr;
    s.VPL = 1;
  } else {
    s.LPR = 32;
    s.VPL = nv <= 32 ? 1 : nv <= 64 ? 2 : 4;
  }
  s.chunk_cols = s.LPR * s.VPL * s.W;
  s.chunks = (N + s.chunk_cols - 1) / s.chunk_cols;
  return s;
}

int launch_spmm(const SpmmArgs &a, bool accumulate, cudaStream_t stream) {
  if (a.N <= 0) return DSP_OK;
  const SpmmShape s = spmm_shape(a.N, a.B, a.ldb, a.C, a.ldc);
  if (s.chunks > 65535) return fail(DSP_ERR_UNSUPPORTED, "spmm: N = %d too wide", a.N);
  if (a.n_items > 0) {
    KernelFn k;
    if (s.W == 4)
      k = accumulate ? pick_items<4, true>(s.LPR, s.VPL) : pick_items<4, false>(s.LPR, s.VPL);
    else
      k = accumulate ? pick_items<1, true>(s.LPR, s.VPL) : pick_items<1, false>(s.LPR, s.VPL);
    const int64_t groups_per_block = kSpmmThreads / s.LPR;
    const int64_t gx = (a.n_items + groups_per_block - 1) / groups_per_block;
    if (gx > INT32_MAX) return fail(DSP_ERR_UNSUPPORTED, "spmm: %lld items", (long long)a.n_items);
    k<<<dim3((unsigned)gx, (unsigned)s.chunks), kSpmmThreads, 0, stream>>>(a);
  }
  if (a.n_split > 0) {
    KernelFn f = s.W == 4 ? (accumulate ? spmm_fixup_kernel<4, true> : spmm_fixup_kernel<4, false>)
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

int launch_fill_const(float *B, int64_t n, float v, cudaStream_t stream) {
  if (n <= 0) return DSP_OK;
  fill_const_kernel<<<148 * 8, 256, 0, stream>>>(B, n, v);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DSP_OK : fail(DSP_ERR_CUDA, "fill: %s", cudaGetErrorString(e));
}

// ------------------------------------------------------------------ device operand

int DevOperand::upload(int device_, int64_t rows_, int64_t cols_, const int64_t *row_ptr, const int32_t *row_ids,
                       int64_t m, const int64_t *indices, const float *values, int64_t first_nz, int64_t nnz_,
                       int64_t piece_cap, bool include_empty) {
  release();
  device = device_;
  rows = rows_;
  cols = cols_;
  nnz = nnz_;
  ItemPlan plan;
  std::vector<int64_t> rp((size_t)m + 1);
  for (int64_t i = 0; i <= m; ++i) rp[(size_t)i] = row_ptr[i] - first_nz;
  build_items(m, row_ids, rp.data(), piece_cap, include_empty, &plan);
  n_items = (int64_t)plan.item_out.size();
  n_split = (int64_t)plan.split_row.size();
  pieces = plan.pieces;
  this->piece_cap = plan.piece_cap;
  max_row_len = plan.max_row_len;
  std::vector<int32_t> c32((size_t)std::max<int64_t>(nnz, 1));
  parallel_for(nnz, [&](int64_t b, int64_t e) {
    for (int64_t j = b; j < e; ++j) c32[(size_t)j] = (int32_t)indices[first_nz + j];
  }, 1 << 16);
  int rc;
  if ((rc = dev_upload(&d_item_ptr, plan.item_ptr.data(), sizeof(int64_t) * plan.item_ptr.size())) ||
      (rc = dev_upload(&d_item_out, plan.item_out.data(), sizeof(int32_t) * plan.item_out.size())) ||
      (rc = dev_upload(&d_split_row, plan.split_row.data(), sizeof(int32_t) * plan.split_row.size())) ||
      (rc = dev_upload(&d_split_ptr, plan.split_ptr.data(), sizeof(int32_t) * plan.split_ptr.size())) ||
      (rc = dev_upload(&d_cols, c32.data(), sizeof(int32_t) * (size_t)nnz)) ||
      (rc = dev_upload(&d_vals, values + first_nz, sizeof(float) * (size_t)nnz)))
    return rc;
  return DSP_OK;
}

void DevOperand::release() {
  for (void **p : {(void **)&d_item_ptr, (void **)&d_item_out, (void **)&d_split_row, (void **)&d_split_ptr,
                   (void **)&d_cols, (void **)&d_vals}) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
  n_items = n_split = pieces = 0;
}

int64_t DevOperand::device_bytes() const {
  return n_items * 12 + 8 + n_split * 8 + 4 + nnz * 8;
}

SpmmArgs DevOperand::args(const float *B, int64_t ldb, float *C, int64_t ldc, int N, float *partial) const {
  SpmmArgs a;
  a.item_ptr = d_item_ptr;
  a.item_out = d_item_out;
  a.n_items = n_items;
  a.split_row = d_split_row;
  a.split_ptr = d_split_ptr;
  a.n_split = n_split;
  a.cols = d_cols;
  a.vals = d_vals;
  a.B = B;
  a.ldb = ldb;
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
  const KernelFn ks[] = {
      pick_items<4, false>(1, 1),  pick_items<4, false>(2, 1),  pick_items<4, false>(4, 1),
      pick_items<4, false>(8, 1),  pick_items<4, false>(16, 1), pick_items<4, false>(32, 1),
      pick_items<4, false>(32, 2), pick_items<4, false>(32, 4), pick_items<4, true>(1, 1),
      pick_items<4, true>(2, 1),   pick_items<4, true>(4, 1),   pick_items<4, true>(8, 1),
      pick_items<4, true>(16, 1),  pick_items<4, true>(32, 1),  pick_items<4, true>(32, 2),
      pick_items<4, true>(32, 4),  pick_items<1, false>(32, 1), pick_items<1, false>(32, 2),
      pick_items<1, false>(32, 4), pick_items<1, true>(32, 1),  pick_items<1, true>(32, 2),
      pick_items<1, true>(32, 4)};
  for (KernelFn k : ks) cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 0);
  cudaGetLastError();
  if (dev < 31) done_mask |= 1 << dev;
}

}  // namespace dsp

// ------------------------------------------------------------------ C ABI: single-GPU plan

struct dsp_spmm_plan {
  dsp::DevOperand op;
  float *scratch = nullptr;
  int64_t scratch_floats = 0;
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

extern "C" int dsp_spmm_plan_create(int device, const dsp_csr *a, int dims_hint, dsp_spmm_plan **out) {
  DSP_TRY_ARG(a && out && a->indptr, "dsp_spmm_plan_create: null argument");
  DSP_TRY_ARG(a->num_cols <= INT32_MAX && a->num_rows <= INT32_MAX, "dsp_spmm_plan_create: matrix too large for int32 ids");
  *out = nullptr;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  prefer_l1_carveout();
  dsp_spmm_plan *p = new dsp_spmm_plan();
  int rc = p->op.upload(device, a->num_rows, a->num_cols, a->indptr, nullptr, a->num_rows, a->indices, a->values, 0,
                        a->nnz, default_piece_cap(dims_hint > 0 ? dims_hint : 128), true);
  if (rc == DSP_OK && p->op.pieces > 0) {
    p->scratch_floats = p->op.pieces * (int64_t)std::max(dims_hint, 1);
    e = cudaMalloc(&p->scratch, sizeof(float) * (size_t)p->scratch_floats);
    if (e != cudaSuccess) rc = fail(DSP_ERR_NOMEM, "spmm scratch: %s", cudaGetErrorString(e));
  }
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
  delete p;
}

extern "C" int dsp_spmm_plan_info(const dsp_spmm_plan *p, dsp_spmm_info *info) {
  DSP_TRY_ARG(p && info, "dsp_spmm_plan_info: null argument");
  info->rows = p->op.rows;
  info->cols = p->op.cols;
  info->nnz = p->op.nnz;
  info->items = p->op.n_items;
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
  return launch_spmm(a, accumulate != 0, (cudaStream_t)stream);
}
