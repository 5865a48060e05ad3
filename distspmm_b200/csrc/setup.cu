// setup.cu — the distributed plan's column tiling on the GPU.
//
// The reference builds every tile's needed-column set with std::unordered_set inserts, one
// per local nonzero (src/dist_spmm_node.cu:103-132), and the node union of the sets with
// more hash sets after an MPI_Allgatherv (src/utils.h:439-547); at R-MAT scale 24 that loop
// dominates set-up. Here a rank marks the columns its nonzeros touch in a byte map of the
// global columns (one store per nonzero), counts per tile, and compacts the marked columns
// into ascending tile-local lists with a two-pass block scan. The node union is the
// element-wise maximum of the ranks' byte maps (an all-reduce the caller runs, e.g.
// torch.distributed MAX over NCCL), listed by the same compaction. Results are identical to
// dsp_tile_counts / dsp_tile_needed / dsp_merge_needed (ascending lists).
#include <cuda_runtime.h>
#include <string.h>

#include <vector>

#include "device.cuh"
#include "internal.h"

namespace dsp {
namespace {

constexpr int kSetupThreads = 256;
constexpr int kColsPerThread = 16;
constexpr int kColsPerBlock = kSetupThreads * kColsPerThread;  // compaction granule
constexpr int kMaxTilesDevice = 8192;                          // shared-memory histogram

// present[c] = 1 for every column c of the nonzeros; *bad = 1 if a column is out of range
// (the store is skipped).
__global__ void presence_kernel(const int64_t *__restrict__ cols, int64_t nnz, int64_t num_cols,
                                uint8_t *__restrict__ present, int *bad) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nnz; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = cols[i];
    if (c >= 0 && c < num_cols)
      present[c] = 1;
    else
      *bad = 1;
  }
}

// counts[t] += number of nonzeros in tile t (cols / cpt), per-block shared histogram.
__global__ void tile_nnz_kernel(const int64_t *__restrict__ cols, int64_t nnz, int64_t num_cols, int64_t cpt, int T,
                                unsigned long long *counts) {
  extern __shared__ unsigned int hist[];
  for (int t = threadIdx.x; t < T; t += blockDim.x) hist[t] = 0;
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nnz; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = cols[i];
    if (c >= 0 && c < num_cols) atomicAdd(&hist[c / cpt], 1u);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += blockDim.x)
    if (hist[t]) atomicAdd(&counts[t], (unsigned long long)hist[t]);
}

// counts[t] += number of marked columns in tile t.
__global__ void tile_present_kernel(const uint8_t *__restrict__ present, int64_t num_cols, int64_t cpt, int T,
                                    unsigned long long *counts) {
  extern __shared__ unsigned int hist[];
  for (int t = threadIdx.x; t < T; t += blockDim.x) hist[t] = 0;
  __syncthreads();
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < num_cols;
       c += (int64_t)gridDim.x * blockDim.x)
    if (present[c]) atomicAdd(&hist[c / cpt], 1u);
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += blockDim.x)
    if (hist[t]) atomicAdd(&counts[t], (unsigned long long)hist[t]);
}

// Exclusive scan of one value per thread over a 256-thread block (shared memory).
__device__ __forceinline__ int block_exclusive_scan(int v, int *sh, int *total) {
  const int tid = threadIdx.x;
  sh[tid] = v;
  __syncthreads();
  for (int off = 1; off < kSetupThreads; off <<= 1) {
    const int x = tid >= off ? sh[tid - off] : 0;
    __syncthreads();
    sh[tid] += x;
    __syncthreads();
  }
  const int incl = sh[tid];
  *total = sh[kSetupThreads - 1];
  __syncthreads();
  return incl - v;
}

// Pass 1: marked columns per block of kColsPerBlock columns.
__global__ void block_count_kernel(const uint8_t *__restrict__ present, int64_t num_cols, int *block_counts) {
  __shared__ int sh[kSetupThreads];
  const int64_t c0 = (int64_t)blockIdx.x * kColsPerBlock + (int64_t)threadIdx.x * kColsPerThread;
  int n = 0;
#pragma unroll
  for (int j = 0; j < kColsPerThread; ++j) n += (c0 + j < num_cols && present[c0 + j]) ? 1 : 0;
  int total;
  block_exclusive_scan(n, sh, &total);
  if (threadIdx.x == 0) block_counts[blockIdx.x] = total;
}

// Pass 2: write the marked columns, ascending, as tile-local ids (c - t*cpt = c % cpt),
// the block starting at out + block_offsets[block].
__global__ void compact_kernel(const uint8_t *__restrict__ present, int64_t num_cols, int64_t cpt,
                               const int64_t *__restrict__ block_offsets, int32_t *__restrict__ out) {
  __shared__ int sh[kSetupThreads];
  const int64_t c0 = (int64_t)blockIdx.x * kColsPerBlock + (int64_t)threadIdx.x * kColsPerThread;
  int n = 0;
#pragma unroll
  for (int j = 0; j < kColsPerThread; ++j) n += (c0 + j < num_cols && present[c0 + j]) ? 1 : 0;
  int total;
  int64_t pos = block_offsets[blockIdx.x] + block_exclusive_scan(n, sh, &total);
#pragma unroll
  for (int j = 0; j < kColsPerThread; ++j)
    if (c0 + j < num_cols && present[c0 + j]) out[pos++] = (int32_t)((c0 + j) % cpt);
}

struct DevBuf {
  void *p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

#define SETUP_CUDA(call)                                                                         \
  do {                                                                                           \
    cudaError_t e_ = (call);                                                                     \
    if (e_ != cudaSuccess) return fail(DSP_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

}  // namespace
}  // namespace dsp

using namespace dsp;

extern "C" int dsp_col_presence(const int64_t *d_cols, int64_t nnz, int64_t num_cols, uint8_t *d_present,
                                void *stream) {
  DSP_TRY_ARG(nnz >= 0 && num_cols >= 1 && d_present && (nnz == 0 || d_cols), "dsp_col_presence: bad argument");
  cudaStream_t s = (cudaStream_t)stream;
  DevBuf bad;
  SETUP_CUDA(cudaMalloc(&bad.p, sizeof(int)));
  SETUP_CUDA(cudaMemsetAsync(bad.p, 0, sizeof(int), s));
  SETUP_CUDA(cudaMemsetAsync(d_present, 0, (size_t)num_cols, s));
  if (nnz > 0) {
    const int64_t blocks = std::min<int64_t>((nnz + kSetupThreads - 1) / kSetupThreads, 148 * 16);
    presence_kernel<<<(unsigned)blocks, kSetupThreads, 0, s>>>(d_cols, nnz, num_cols, d_present, (int *)bad.p);
    SETUP_CUDA(cudaGetLastError());
  }
  int flag = 0;
  SETUP_CUDA(cudaMemcpyAsync(&flag, bad.p, sizeof flag, cudaMemcpyDeviceToHost, s));
  SETUP_CUDA(cudaStreamSynchronize(s));
  if (flag) return fail(DSP_ERR_FORMAT, "dsp_col_presence: a column id lies outside [0, %lld)", (long long)num_cols);
  return DSP_OK;
}

extern "C" int dsp_tile_device(const int64_t *d_cols, int64_t nnz, const uint8_t *d_present, int64_t num_cols, int T,
                               int64_t *cpt_out, int32_t *n_col_list, int32_t *n_slice_list, int64_t *nnz_list,
                               int64_t *offsets, int32_t *cols, void *stream) {
  DSP_TRY_ARG(num_cols >= 1 && T >= 1 && nnz >= 0, "dsp_tile_device: bad argument");
  DSP_TRY_ARG(T <= kMaxTilesDevice, "dsp_tile_device: T = %d exceeds %d", T, kMaxTilesDevice);
  DSP_TRY_ARG(d_cols || nnz == 0, "dsp_tile_device: %lld nonzeros without column ids", (long long)nnz);
  DSP_TRY_ARG(!cols || offsets, "dsp_tile_device: cols needs offsets");
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t cpt = (num_cols + T - 1) / T;  // src/dist_spmm_node.cu:106
  if (cpt_out) *cpt_out = cpt;
  DevBuf own_present, counts;
  int rc;
  if (!d_present) {
    SETUP_CUDA(cudaMalloc(&own_present.p, (size_t)num_cols));
    if ((rc = dsp_col_presence(d_cols, nnz, num_cols, (uint8_t *)own_present.p, stream))) return rc;
    d_present = (const uint8_t *)own_present.p;
  }
  SETUP_CUDA(cudaMalloc(&counts.p, sizeof(unsigned long long) * 2 * (size_t)T));
  SETUP_CUDA(cudaMemsetAsync(counts.p, 0, sizeof(unsigned long long) * 2 * (size_t)T, s));
  unsigned long long *d_tile_cols = (unsigned long long *)counts.p, *d_tile_nnz = d_tile_cols + T;
  const size_t hist_bytes = sizeof(unsigned int) * (size_t)T;
  tile_present_kernel<<<(unsigned)std::min<int64_t>((num_cols + kSetupThreads - 1) / kSetupThreads, 148 * 8),
                        kSetupThreads, hist_bytes, s>>>(d_present, num_cols, cpt, T, d_tile_cols);
  if (d_cols && nnz > 0)
    tile_nnz_kernel<<<(unsigned)std::min<int64_t>((nnz + kSetupThreads - 1) / kSetupThreads, 148 * 8), kSetupThreads,
                      hist_bytes, s>>>(d_cols, nnz, num_cols, cpt, T, d_tile_nnz);
  SETUP_CUDA(cudaGetLastError());
  std::vector<unsigned long long> h((size_t)2 * T);
  SETUP_CUDA(cudaMemcpyAsync(h.data(), counts.p, sizeof(unsigned long long) * 2 * (size_t)T, cudaMemcpyDeviceToHost, s));
  SETUP_CUDA(cudaStreamSynchronize(s));
  for (int t = 0; t < T; ++t) {
    const int64_t lo = (int64_t)t * cpt;
    if (n_col_list) n_col_list[t] = (int32_t)h[(size_t)t];
    if (nnz_list) nnz_list[t] = (int64_t)h[(size_t)T + t];
    // assigned only for tiles holding local nonzeros (src/dist_spmm_node.cu:210-223)
    if (n_slice_list)
      n_slice_list[t] = h[(size_t)T + t] > 0 ? (int32_t)std::min<int64_t>(cpt, num_cols - lo) : 0;
  }
  if (offsets) {
    offsets[0] = 0;
    for (int t = 0; t < T; ++t) offsets[t + 1] = offsets[t] + (int64_t)h[(size_t)t];
  }
  if (!cols || !offsets || offsets[T] == 0) return DSP_OK;

  // ascending marked columns as tile-local ids: tile t's list starts at offsets[t] because
  // the global order is ascending and tiles are contiguous column ranges
  const int64_t nb = (num_cols + kColsPerBlock - 1) / kColsPerBlock;
  DevBuf bcount, boff, list;
  SETUP_CUDA(cudaMalloc(&bcount.p, sizeof(int) * (size_t)nb));
  SETUP_CUDA(cudaMalloc(&boff.p, sizeof(int64_t) * (size_t)nb));
  SETUP_CUDA(cudaMalloc(&list.p, sizeof(int32_t) * (size_t)offsets[T]));
  block_count_kernel<<<(unsigned)nb, kSetupThreads, 0, s>>>(d_present, num_cols, (int *)bcount.p);
  SETUP_CUDA(cudaGetLastError());
  std::vector<int> hc((size_t)nb);
  std::vector<int64_t> ho((size_t)nb);
  SETUP_CUDA(cudaMemcpyAsync(hc.data(), bcount.p, sizeof(int) * (size_t)nb, cudaMemcpyDeviceToHost, s));
  SETUP_CUDA(cudaStreamSynchronize(s));
  int64_t run = 0;
  for (int64_t b = 0; b < nb; ++b) {
    ho[(size_t)b] = run;
    run += hc[(size_t)b];
  }
  if (run != offsets[T]) return fail(DSP_ERR_STATE, "dsp_tile_device: %lld marked columns, %lld counted",
                                     (long long)run, (long long)offsets[T]);
  SETUP_CUDA(cudaMemcpyAsync(boff.p, ho.data(), sizeof(int64_t) * (size_t)nb, cudaMemcpyHostToDevice, s));
  compact_kernel<<<(unsigned)nb, kSetupThreads, 0, s>>>(d_present, num_cols, cpt, (const int64_t *)boff.p,
                                                          (int32_t *)list.p);
  SETUP_CUDA(cudaGetLastError());
  SETUP_CUDA(cudaMemcpyAsync(cols, list.p, sizeof(int32_t) * (size_t)offsets[T], cudaMemcpyDeviceToHost, s));
  SETUP_CUDA(cudaStreamSynchronize(s));
  return DSP_OK;
}
