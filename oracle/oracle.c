/*
 * oracle.c — CPU restatement of the reference's hot-path algorithms.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the shipped library links, loads or calls this
 * file. tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * arm use it as the checker and as the timed CPU baseline; the product path never does.
 *
 * Parity status:
 *   - HSDMA (orc_hsdma) and the CSR loader are pinned against the reference's own
 *     src/h_sdma.h and src/sparse_matrix.h, compiled from the reference sources by
 *     oracle/Makefile into oracle/_ref (tests/golden/make_golden.py, tests/test_oracle.py).
 *   - Tiling, node merge, selector and traffic formulas restate code that lives inside
 *     MPI-dependent files (src/dist_spmm_node.cu, src/utils.h, src/comm_man.h) that cannot
 *     be built here; they follow the cited lines directly.
 *   - SpMM numerics: the reference delegates to cuSPARSE and never checks C (B is all
 *     ones), so C is "parity unpinned" against the reference; orc_spmm_f64 is a plain
 *     CSR x dense loop with double accumulation that also returns |A|.|B| for the
 *     elementwise tolerance max|dC| <= 1e-5 * (|A|.|B|).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ SpMM */

/* C[i,:] = sum_j A[i,j] * B[j,:] in double; Cabs[i,:] = sum_j |A[i,j]| * |B[j,:]|.
 * Plain CSR x dense loop (the operation of cusparseSpMM in src/dist_spmm_node.cu:371-383
 * summed over all tiles). Rows are independent, so the OpenMP split does not change any
 * result. */
int orc_spmm_f64(int64_t m, const int64_t *indptr, const int64_t *indices, const float *values,
                 const float *B, int64_t ldb, int64_t N, double *C, double *Cabs) {
  int64_t i;
#pragma omp parallel for schedule(dynamic, 64)
  for (i = 0; i < m; ++i) {
    double *c = C + i * N;
    double *ca = Cabs ? Cabs + i * N : NULL;
    for (int64_t k = 0; k < N; ++k) {
      c[k] = 0.0;
      if (ca) ca[k] = 0.0;
    }
    for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) {
      const double v = (double)values[p];
      const float *b = B + indices[p] * ldb;
      for (int64_t k = 0; k < N; ++k) c[k] += v * (double)b[k];
      if (ca)
        for (int64_t k = 0; k < N; ++k) ca[k] += fabs(v) * fabs((double)b[k]);
    }
  }
  return 0;
}

/* The CPU baseline: the same loop in fp32 with fp32 accumulation, OpenMP static schedule
 * over rows, `threads` host threads (0 = all). */
int orc_spmm_f32(int64_t m, const int64_t *indptr, const int64_t *indices, const float *values,
                 const float *B, int64_t ldb, int64_t N, float *C, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  int64_t i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < m; ++i) {
    float *c = C + i * N;
    for (int64_t k = 0; k < N; ++k) c[k] = 0.f;
    for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) {
      const float v = values[p];
      const float *b = B + indices[p] * ldb;
      for (int64_t k = 0; k < N; ++k) c[k] += v * b[k];
    }
  }
  return 0;
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------ partition */

/* src/dist_spmm_node.cu:85-91: m_local = ceil(M/P); lb = rank*m_local;
 * ub = min(lb+m_local, M). */
void orc_partition_bounds(int64_t M, int P, int rank, int64_t *lb, int64_t *ub) {
  int64_t m_local = (M + P - 1) / P;
  int64_t l = (int64_t)rank * m_local;
  int64_t u = l + m_local < M ? l + m_local : M;
  *lb = l;
  *ub = u;
}

/* ------------------------------------------------------------------ tiling */

/* src/dist_spmm_node.cu:105-106: col_per_tile = (N + total_tiles - 1) / total_tiles with
 * N the int64 column count. */
int64_t orc_cpt(int64_t ncols, int T) { return (ncols + T - 1) / T; }

/* src/dist_spmm_node.cu:117-129 (part_id = col / cpt, col_local = col % cpt, one set of
 * col_local per tile) and :210-223 (n_slice_list only for tiles with local nonzeros).
 * The reference's std::unordered_set is restated as a per-tile "seen" flag array; the
 * needed lists come out ascending. needed may be NULL (counts only); when given,
 * offsets[T+1] is written. */
int orc_tile(int64_t m, const int64_t *indptr, const int64_t *indices, int64_t ncols, int T,
             int32_t *n_col_list, int32_t *n_slice_list, int64_t *nnz_list, int64_t *offsets,
             int32_t *needed) {
  int64_t cpt = orc_cpt(ncols, T);
  unsigned char *seen = (unsigned char *)calloc((size_t)(cpt * T > 0 ? cpt * T : 1), 1);
  if (!seen) return -5;
  for (int t = 0; t < T; ++t) {
    n_col_list[t] = 0;
    nnz_list[t] = 0;
  }
  for (int64_t row = 0; row < m; ++row) {
    for (int64_t j = indptr[row]; j < indptr[row + 1]; ++j) {
      int64_t col_local = indices[j] % cpt;
      int64_t part_id = indices[j] / cpt;
      nnz_list[part_id]++;
      unsigned char *s = seen + part_id * cpt + col_local;
      if (!*s) {
        *s = 1;
        n_col_list[part_id]++;
      }
    }
  }
  for (int t = 0; t < T; ++t) {
    int64_t slice = cpt < ncols - (int64_t)t * cpt ? cpt : ncols - (int64_t)t * cpt;
    n_slice_list[t] = nnz_list[t] > 0 ? (int32_t)slice : 0;
  }
  if (needed) {
    int64_t pos = 0;
    for (int t = 0; t < T; ++t) {
      offsets[t] = pos;
      for (int64_t c = 0; c < cpt; ++c)
        if (seen[t * cpt + c]) needed[pos++] = (int32_t)c;
    }
    offsets[T] = pos;
  }
  free(seen);
  return 0;
}

/* ------------------------------------------------------------------ HSDMA */

/* swap_refinement, src/h_sdma.h:27-38: (D[ma][b] + D[mb][a]) - (D[ma][a] + D[mb][b]). */
static double orc_swap_gain(const double *D, int ntask, int a, int b, const int *map) {
  int ma = map[a], mb = map[b];
  return (D[(int64_t)ma * ntask + b] + D[(int64_t)mb * ntask + a]) -
         (D[(int64_t)ma * ntask + a] + D[(int64_t)mb * ntask + b]);
}

/* One refinement loop of src/h_sdma.h:129-157 / :191-220: up to `iters` times pick the
 * first strictly best swap among pairs a<b mapped to different units and apply it while
 * the gain is positive. */
static void orc_refine(const double *D, int ntask, int *map, int iters) {
  for (int it = 0; it < iters; ++it) {
    double best = 0;
    int ba = -1, bb = -1;
    for (int a = 0; a < ntask; ++a)
      for (int b = a + 1; b < ntask; ++b) {
        if (map[a] == map[b]) continue;
        double g = orc_swap_gain(D, ntask, a, b, map);
        if (g > best) {
          best = g;
          ba = a;
          bb = b;
        }
      }
    if (best > 0) {
      int t = map[ba];
      map[ba] = map[bb];
      map[bb] = t;
    } else {
      break;
    }
  }
}

/* hierarchical_iterative_refinement_allocation, src/h_sdma.h:78-228. demand is P x T
 * row-major; node_of_gpu[P]. Phase 1 (nodes > 1) refines a node map over node demand
 * sums; phase 2 refines, per node, the GPU map over that node's (sorted) tasks. */
int orc_hsdma(const int32_t *demand, int P, int T, const int32_t *node_of_gpu, int tasks_per_gpu,
              int max_inter, int max_intra, int32_t *remap) {
  if (P <= 0 || T <= 0) return 0;
  int nodes = 0;
  for (int g = 0; g < P; ++g)
    if (node_of_gpu[g] + 1 > nodes) nodes = node_of_gpu[g] + 1;
  int tasks_per_node = T / nodes;
  int gpn = P / nodes;
  int *node_map = (int *)malloc(sizeof(int) * T);
  int *list = (int *)malloc(sizeof(int) * T);
  int *cnt = (int *)calloc(nodes, sizeof(int));
  if (nodes <= 1) {
    for (int t = 0; t < T; ++t) node_map[t] = 0;
  } else {
    double *ND = (double *)calloc((size_t)nodes * T, sizeof(double));
    for (int g = 0; g < P; ++g)
      for (int t = 0; t < T; ++t) ND[(int64_t)node_of_gpu[g] * T + t] += demand[(int64_t)g * T + t];
    for (int t = 0; t < T; ++t) node_map[t] = t / tasks_per_node;
    orc_refine(ND, T, node_map, max_inter);
    free(ND);
  }
  for (int t = 0; t < T; ++t) remap[t] = -1;
  for (int node = 0; node < nodes; ++node) {
    /* tasks of this node in ascending order (src/h_sdma.h:159-173) */
    int n = 0;
    for (int t = 0; t < T; ++t)
      if (node_map[t] == node) list[n++] = t;
    if (n == 0) continue;
    double *GD = (double *)calloc((size_t)gpn * n, sizeof(double));
    for (int i = 0; i < gpn; ++i)
      for (int j = 0; j < n; ++j) GD[(int64_t)i * n + j] = demand[(int64_t)(i + node * gpn) * T + list[j]];
    int *gmap = (int *)malloc(sizeof(int) * n);
    for (int i = 0; i < n; ++i) gmap[i] = i / tasks_per_gpu;
    orc_refine(GD, n, gmap, max_intra);
    for (int i = 0; i < n; ++i) remap[list[i]] = gmap[i] + node * gpn;
    free(gmap);
    free(GD);
  }
  free(cnt);
  free(list);
  free(node_map);
  return 0;
}

/* ------------------------------------------------------------------ node merge */

/* double_level_comm_node_processing, src/utils.h:471-533: every rank's set for tile t
 * becomes the union of all node ranks' sets; n_col_list[t] = |union|. Inputs are laid out
 * as the Allgather/Allgatherv there deliver them (rank-major, tile-major per rank). */
int orc_merge(int R, int T, int64_t cpt, const int32_t *counts, const int32_t *cols,
              int32_t *n_col_merged, int64_t *offsets, int32_t *merged) {
  unsigned char *seen = (unsigned char *)calloc((size_t)(cpt * T > 0 ? cpt * T : 1), 1);
  if (!seen) return -5;
  const int32_t *p = cols;
  for (int r = 0; r < R; ++r)
    for (int t = 0; t < T; ++t) {
      int32_t c = counts[(int64_t)r * T + t];
      for (int32_t k = 0; k < c; ++k) seen[(int64_t)t * cpt + p[k]] = 1;
      p += c;
    }
  int64_t pos = 0;
  for (int t = 0; t < T; ++t) {
    if (offsets) offsets[t] = pos;
    int32_t n = 0;
    for (int64_t c = 0; c < cpt; ++c)
      if (seen[t * cpt + c]) {
        if (merged) merged[pos] = (int32_t)c;
        ++pos;
        ++n;
      }
    n_col_merged[t] = n;
  }
  if (offsets) offsets[T] = pos;
  free(seen);
  return 0;
}

/* ------------------------------------------------------------------ selector */

/* CommMan_hp::initialize_comm_model, src/comm_man.h:369-410, comm_type 2 branch:
 * k = min((float)c, (float)dims); thr = 1 / (a * pow(k, u) + b / k) in float (the
 * reference is built by nvcc, where pow(float, float) is the float overload);
 * d_i = (float)n_col / (float)(n_slice + 1); sparse iff thr > d_i. */
float orc_threshold(float a, float b, float c, float u, int dims) {
  float k = c < (float)dims ? c : (float)dims;
  float p = powf(k, u);
  float t1 = a * p;
  float t2 = b / k;
  float den = t1 + t2;
  return 1.0f / den;
}

int orc_select(int comm_type, int dims, float a, float b, float c, float u, int T,
               const int32_t *n_col, const int32_t *n_slice, uint8_t *sparse) {
  if (comm_type == 0) {
    for (int i = 0; i < T; ++i) sparse[i] = 0;
  } else if (comm_type == 1) {
    for (int i = 0; i < T; ++i) sparse[i] = 1;
  } else if (comm_type == 2) {
    float thr = orc_threshold(a, b, c, u, dims);
    for (int i = 0; i < T; ++i) {
      float d = (float)n_col[i] / (float)(n_slice[i] + 1);
      sparse[i] = thr > d;
    }
  } else {
    return -1;
  }
  return 0;
}

/* CommMan_hp::get_comm_traffic_intra, src/comm_man.h:529-542. */
int64_t orc_traffic_intra(int me, int T, const int32_t *remap, const uint8_t *sparse,
                          const int32_t *n_col, const int32_t *n_slice, int dims) {
  int64_t bytes = 0;
  for (int i = 0; i < T; ++i)
    if (remap[i] != me) bytes += (int64_t)sizeof(float) * dims * (sparse[i] ? n_col[i] : n_slice[i]);
  return bytes;
}
