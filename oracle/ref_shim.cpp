// ref_shim.cpp — thin extern "C" driver over the reference's own header-only code.
//
// TEST INFRASTRUCTURE ONLY (never linked into the product). Built by oracle/Makefile
// against the reference sources where they lie (REF_SRC, the reference's src/ directory)
// into oracle/_ref/libdsp_ref.so, so the oracle restatement and the golden fixtures can be
// pinned against the reference's behaviour:
//   ref_hsdma     -> hierarchical_iterative_refinement_allocation (src/h_sdma.h:78-228)
//   ref_load_csr  -> SparseMatrix<int64_t,float>::load_from_csr     (src/sparse_matrix.h:83-159)
//                    + turn_local_l_u_csr                           (src/sparse_matrix.h:178-199)
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "h_sdma.h"
#include "sparse_matrix.h"

extern "C" {

int ref_hsdma(const int32_t *demand, int P, int T, const int32_t *node_of_gpu,
              int tasks_per_gpu, int max_inter, int max_intra, int32_t *remap) {
  std::vector<std::vector<int>> D(P, std::vector<int>(T));
  for (int g = 0; g < P; ++g)
    for (int t = 0; t < T; ++t) D[g][t] = demand[(int64_t)g * T + t];
  std::vector<GpuInfo> topo;
  for (int g = 0; g < P; ++g) topo.push_back({g, node_of_gpu[g]});
  std::vector<int> out;
  hierarchical_iterative_refinement_allocation(D, topo, tasks_per_gpu, out, max_inter, max_intra,
                                               false);
  for (int t = 0; t < T; ++t) remap[t] = t < (int)out.size() ? out[t] : -2;
  return 0;
}

// Load with the reference loader and keep rows [lb, ub) (the whole matrix if lb<0).
// Sizes are returned first (call with null arrays), then the arrays are filled on a
// second call with the same arguments.
int ref_load_csr(const char *prefix, int64_t lb, int64_t ub, int64_t *num_rows, int64_t *num_cols,
                 int64_t *nnz, int64_t *indptr, int64_t *indices, float *values) {
  SparseMatrix<int64_t, float> m;
  if (!m.load_from_csr(std::string(prefix))) return -2;
  if (lb < 0) {
    lb = 0;
    ub = m.num_rows;
  }
  m.turn_local_l_u_csr(lb, ub);
  *num_rows = m.local_m;
  *num_cols = m.num_cols;
  *nnz = (int64_t)m.local_nnz;
  if (indptr) std::memcpy(indptr, m.row_ptr.data(), sizeof(int64_t) * m.row_ptr.size());
  if (indices) std::memcpy(indices, m.col_idx.data(), sizeof(int64_t) * m.col_idx.size());
  if (values) std::memcpy(values, m.values.data(), sizeof(float) * m.values.size());
  return 0;
}
}
