// cusparse_arm.cu — the reference's local SpMM, timed beside this engine's kernels.
//
// This is a measurement arm, not part of the engine: the engine never links cuSPARSE.
// It reproduces the per-tile SpMM of DistSpMM (src/dist_spmm_node.cu:103-129 tiling,
// :206-234 descriptors, :354-385 the call):
//   - the local rows are cut into T = P * n_rolls column tiles of cpt = ceil(M / T) columns;
//   - tile t is a COO matrix (m_local x n_slice_t) with int64 row ids (ascending), int64
//     tile-local column ids (col % cpt) and fp32 values, in the local CSR's nonzero order;
//   - its B operand is the [n_slice_t x dims] row-major slice of B owned by the tile;
//   - C [m_local x dims] row-major is accumulated tile by tile with alpha = beta = 1 and
//     CUSPARSE_SPMM_ALG_DEFAULT; tiles without nonzeros are skipped (:344).
// Two deviations, both in cuSPARSE's favour: descriptors and work buffers are created once
// at set-up (the reference creates the B descriptor and allocates the buffer per tile per
// repetition inside its timed loop, :356-383), and all tiles read one resident B (no fetch).
// A second arm runs the whole local matrix as one CSR (int64 indices) with ALG_DEFAULT and
// beta = 0: the library's best single call for the same product.
#include <cuda_runtime.h>
#include <cusparse.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <vector>

namespace {

char g_err[256];

int err(const char *what, int code) {
  snprintf(g_err, sizeof g_err, "%s failed (%d)", what, code);
  return -1;
}

#define CU(x)                                                 \
  do {                                                        \
    cudaError_t e_ = (x);                                     \
    if (e_ != cudaSuccess) return err(#x, (int)e_);           \
  } while (0)
#define CS(x)                                                 \
  do {                                                        \
    cusparseStatus_t s_ = (x);                                \
    if (s_ != CUSPARSE_STATUS_SUCCESS) return err(#x, (int)s_); \
  } while (0)

}  // namespace

struct csa {
  cusparseHandle_t h = nullptr;
  int64_t m = 0, M = 0, nnz = 0, cpt = 0;
  int T = 0, dims = 0;
  struct Tile {
    int64_t nnz = 0, n_slice = 0;
    int64_t *rows = nullptr, *cols = nullptr;
    float *vals = nullptr;
    cusparseSpMatDescr_t A = nullptr;
    void *buf = nullptr;
  };
  std::vector<Tile> tiles;
  int64_t *csr_ptr = nullptr, *csr_idx = nullptr;
  float *csr_val = nullptr;
  cusparseSpMatDescr_t A_csr = nullptr;
  void *csr_buf = nullptr;
  int64_t device_bytes = 0;
};

extern "C" const char *csa_last_error(void) { return g_err; }

extern "C" void csa_destroy(csa *c) {
  if (!c) return;
  for (auto &t : c->tiles) {
    if (t.A) cusparseDestroySpMat(t.A);
    cudaFree(t.rows);
    cudaFree(t.cols);
    cudaFree(t.vals);
    cudaFree(t.buf);
  }
  if (c->A_csr) cusparseDestroySpMat(c->A_csr);
  cudaFree(c->csr_ptr);
  cudaFree(c->csr_idx);
  cudaFree(c->csr_val);
  cudaFree(c->csr_buf);
  if (c->h) cusparseDestroy(c->h);
  delete c;
}

// Build both arms for the local CSR (m rows; global column ids < M) at width dims, with B
// and C laid out as [M x dims] and [m x dims] row-major (B and C: device pointers, used
// only to size the work buffers).
extern "C" int csa_create(int64_t m, int64_t M, const int64_t *indptr, const int64_t *indices, const float *values,
                          int T, int dims, const float *B, float *C, csa **out) {
  *out = nullptr;
  if (m < 1 || M < 1 || T < 1 || dims < 1) return err("csa_create arguments", 0);
  csa *c = new csa();
  *out = c;
  c->m = m;
  c->M = M;
  c->T = T;
  c->dims = dims;
  c->nnz = indptr[m];
  c->cpt = (M + T - 1) / T;  // src/dist_spmm_node.cu:105
  CS(cusparseCreate(&c->h));
  const float alpha = 1.f, beta = 1.f, zero = 0.f;
  cusparseDnMatDescr_t dC;
  CS(cusparseCreateDnMat(&dC, m, dims, dims, C, CUDA_R_32F, CUSPARSE_ORDER_ROW));
  // per-tile COO exactly as the reference builds it (row ids ascending within a tile)
  std::vector<int64_t> cnt((size_t)T, 0);
  for (int64_t j = 0; j < c->nnz; ++j) cnt[(size_t)(indices[j] / c->cpt)]++;
  c->tiles.resize((size_t)T);
  // one pass in row order: every tile's nonzeros keep the local CSR's order
  std::vector<std::vector<int64_t>> rr((size_t)T), cc((size_t)T);
  std::vector<std::vector<float>> vv((size_t)T);
  for (int t = 0; t < T; ++t) {
    rr[(size_t)t].reserve((size_t)cnt[(size_t)t]);
    cc[(size_t)t].reserve((size_t)cnt[(size_t)t]);
    vv[(size_t)t].reserve((size_t)cnt[(size_t)t]);
  }
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = indptr[i]; j < indptr[i + 1]; ++j) {
      const size_t t = (size_t)(indices[j] / c->cpt);
      rr[t].push_back(i);
      cc[t].push_back(indices[j] % c->cpt);
      vv[t].push_back(values[j]);
    }
  for (int t = 0; t < T; ++t) {
    auto &tl = c->tiles[(size_t)t];
    tl.nnz = cnt[(size_t)t];
    tl.n_slice = std::min<int64_t>(c->cpt, M - (int64_t)t * c->cpt);
    if (tl.nnz == 0) continue;
    std::vector<int64_t> r, cl;
    std::vector<float> v;
    r.swap(rr[(size_t)t]);
    cl.swap(cc[(size_t)t]);
    v.swap(vv[(size_t)t]);
    CU(cudaMalloc(&tl.rows, 8 * (size_t)tl.nnz));
    CU(cudaMalloc(&tl.cols, 8 * (size_t)tl.nnz));
    CU(cudaMalloc(&tl.vals, 4 * (size_t)tl.nnz));
    CU(cudaMemcpy(tl.rows, r.data(), 8 * (size_t)tl.nnz, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(tl.cols, cl.data(), 8 * (size_t)tl.nnz, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(tl.vals, v.data(), 4 * (size_t)tl.nnz, cudaMemcpyHostToDevice));
    c->device_bytes += 20 * tl.nnz;
    CS(cusparseCreateCoo(&tl.A, m, tl.n_slice, tl.nnz, tl.rows, tl.cols, tl.vals, CUSPARSE_INDEX_64I,
                         CUSPARSE_INDEX_BASE_ZERO, CUDA_R_32F));
    cusparseDnMatDescr_t dB;
    CS(cusparseCreateDnMat(&dB, tl.n_slice, dims, dims, (void *)(B + (size_t)t * c->cpt * dims), CUDA_R_32F,
                           CUSPARSE_ORDER_ROW));
    size_t bytes = 0;
    CS(cusparseSpMM_bufferSize(c->h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, tl.A,
                               dB, &beta, dC, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, &bytes));
    cusparseDestroyDnMat(dB);
    if (bytes) CU(cudaMalloc(&tl.buf, bytes));
    c->device_bytes += (int64_t)bytes;
  }
  // whole-matrix CSR
  CU(cudaMalloc(&c->csr_ptr, 8 * (size_t)(m + 1)));
  CU(cudaMalloc(&c->csr_idx, 8 * (size_t)std::max<int64_t>(c->nnz, 1)));
  CU(cudaMalloc(&c->csr_val, 4 * (size_t)std::max<int64_t>(c->nnz, 1)));
  CU(cudaMemcpy(c->csr_ptr, indptr, 8 * (size_t)(m + 1), cudaMemcpyHostToDevice));
  CU(cudaMemcpy(c->csr_idx, indices, 8 * (size_t)c->nnz, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(c->csr_val, values, 4 * (size_t)c->nnz, cudaMemcpyHostToDevice));
  c->device_bytes += 8 * (m + 1) + 12 * c->nnz;
  CS(cusparseCreateCsr(&c->A_csr, m, M, c->nnz, c->csr_ptr, c->csr_idx, c->csr_val, CUSPARSE_INDEX_64I,
                       CUSPARSE_INDEX_64I, CUSPARSE_INDEX_BASE_ZERO, CUDA_R_32F));
  cusparseDnMatDescr_t dB;
  CS(cusparseCreateDnMat(&dB, M, dims, dims, (void *)B, CUDA_R_32F, CUSPARSE_ORDER_ROW));
  size_t bytes = 0;
  CS(cusparseSpMM_bufferSize(c->h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha,
                             c->A_csr, dB, &zero, dC, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, &bytes));
  cusparseDestroyDnMat(dB);
  cusparseDestroyDnMat(dC);
  if (bytes) CU(cudaMalloc(&c->csr_buf, bytes));
  c->device_bytes += (int64_t)bytes;
  return 0;
}

extern "C" int64_t csa_device_bytes(const csa *c) { return c ? c->device_bytes : 0; }

// The reference's tile loop: C += A_t . B_t for every tile with nonzeros (alpha = beta = 1).
// The caller zeroes C first, as the reference does before each repetition (:331).
extern "C" int csa_run_tiles(csa *c, const float *B, float *C, void *stream) {
  CS(cusparseSetStream(c->h, (cudaStream_t)stream));
  const float alpha = 1.f, beta = 1.f;
  cusparseDnMatDescr_t dC;
  CS(cusparseCreateDnMat(&dC, c->m, c->dims, c->dims, C, CUDA_R_32F, CUSPARSE_ORDER_ROW));
  for (int t = 0; t < c->T; ++t) {
    auto &tl = c->tiles[(size_t)t];
    if (tl.nnz == 0) continue;
    cusparseDnMatDescr_t dB;
    CS(cusparseCreateDnMat(&dB, tl.n_slice, c->dims, c->dims, (void *)(B + (size_t)t * c->cpt * c->dims), CUDA_R_32F,
                           CUSPARSE_ORDER_ROW));
    CS(cusparseSpMM(c->h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, tl.A, dB, &beta,
                    dC, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, tl.buf));
    cusparseDestroyDnMat(dB);
  }
  cusparseDestroyDnMat(dC);
  return 0;
}

// Whole local matrix as one CSR SpMM, C = A . B.
extern "C" int csa_run_csr(csa *c, const float *B, float *C, void *stream) {
  CS(cusparseSetStream(c->h, (cudaStream_t)stream));
  const float alpha = 1.f, zero = 0.f;
  cusparseDnMatDescr_t dB, dC;
  CS(cusparseCreateDnMat(&dB, c->M, c->dims, c->dims, (void *)B, CUDA_R_32F, CUSPARSE_ORDER_ROW));
  CS(cusparseCreateDnMat(&dC, c->m, c->dims, c->dims, C, CUDA_R_32F, CUSPARSE_ORDER_ROW));
  CS(cusparseSpMM(c->h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, c->A_csr, dB, &zero,
                  dC, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, c->csr_buf));
  cusparseDestroyDnMat(dB);
  cusparseDestroyDnMat(dC);
  return 0;
}
